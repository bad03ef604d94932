"""Generate the golden fixtures in this directory from the reference project.

Run from the repository root with the reference checkout's location:

    python tests/golden/make_golden.py --reference <path-to-triton-kernel-lab>

For every case it draws seeded inputs on the CPU and records:
* ``ref_o``/``ref_lse``/``ref_dq``/``ref_dk``/``ref_dv`` — the reference's own
  Triton kernels (``_flash_attention_forward_kernel`` and the three backward
  kernels of ``src/tklab/kernels/flash_attention.py``) executed by the Triton
  CPU interpreter (``TRITON_INTERPRET=1``), where the reference supports the
  case (float16, head_dim 64);
* ``sdpa_o``/``sdpa_dq``/``sdpa_dk``/``sdpa_dv`` — the reference's ``ref_fn``
  (fp32 ``F.scaled_dot_product_attention``) and its autograd gradient;
* ``man_dq``/``man_dk``/``man_dv`` — ``_manual_fp32_backward`` from the
  reference's ``tests/test_flash_attention_backward.py``.
RoPE attention cases (``rope_*``) add the reference's rotate-half kernels
(``src/tklab/kernels/rope.py`` ``_rope_forward_kernel`` /
``_rope_backward_kernel``, interpreter, fp16 tables, one (batch, head) slab
at a time): ``ref_qrot``/``ref_krot`` (rope of Q and K), the attention
kernels above on the rotated tensors (``ref_o``, ``ref_lse``, ``ref_dv``),
dQ and dK mapped back through the rope backward kernel (``ref_dq``,
``ref_dk``), and the same chain with the fp32 manual algebra
(``man_dq``/``man_dk``/``man_dv``).
16-bit tensors are stored as their raw uint16 bit patterns (``<name>_bits``)
with the dtype name, so tests rebuild bit-identical tensors; fp32 tensors are
stored as float32.  The fp32 config-1 case keeps the SDPA gradients (its
reference path); the others keep the manual-algebra gradients (the tighter
pin of the two).
"""

from __future__ import annotations

import argparse
import importlib.util
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (name, shape, dtype, causal, seed, run reference Triton kernels)
CASES = [
    ("f16_s129_d64_causal", (1, 2, 129, 64), "float16", True, 0, True),
    ("f16_s129_d64_noncausal", (1, 2, 129, 64), "float16", False, 1, True),
    ("f16_s1000_d64_causal", (1, 1, 1000, 64), "float16", True, 2, True),
    ("f16_s7_d64_noncausal", (1, 3, 7, 64), "float16", False, 3, True),
    ("f16_s192_d64_causal_b2", (2, 1, 192, 64), "float16", True, 4, True),
    ("c1_fp32_s256_d64_noncausal", (1, 4, 256, 64), "float32", False, 0, False),
    ("bf16_s130_d128_causal", (1, 2, 130, 128), "bfloat16", True, 5, False),
    ("bf16_s300_d128_noncausal", (1, 1, 300, 128), "bfloat16", False, 6, False),
]


# (name, shape, dtype, causal, seed): fused-RoPE attention cases.
ROPE_CASES = [
    ("rope_f16_s129_d64_causal", (1, 2, 129, 64), "float16", True, 11),
    ("rope_f16_s200_d64_noncausal", (2, 1, 200, 64), "float16", False, 12),
]


def _rope_tables(torch, seq: int, dim: int, dtype):
    """angle[p][i] = p * 10000^(-2i/dim), evaluated in float64."""
    inv = 10000.0 ** (-torch.arange(0, dim // 2, dtype=torch.float64) * 2.0 / dim)
    angles = torch.arange(seq, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(angles).to(dtype), torch.sin(angles).to(dtype)


def _ref_rope(torch, triton, rp, x, cos, sin, *, backward_of=None):
    """Reference rope over the last dim of (b, h, s, d), one slab at a time.

    With ``backward_of`` (the rope input), ``x`` is the upstream gradient and
    the result is the rope input gradient (the transpose rotation)."""
    b, h, s, d = x.shape
    out = torch.empty_like(x)
    grid = (s, triton.cdiv(d // 2, rp._BLOCK_SIZE))
    for i in range(b):
        for j in range(h):
            src = x[i, j].contiguous()
            dst = torch.empty_like(src)
            if backward_of is None:
                rp._rope_forward_kernel[grid](
                    src, cos, sin, dst, src.stride(0), cos.stride(0), sin.stride(0), dst.stride(0), d // 2,
                    BLOCK_SIZE=rp._BLOCK_SIZE,
                )
            else:
                xin = backward_of[i, j].contiguous()
                rp._rope_backward_kernel[grid](
                    src, xin, cos, sin, dst, dst, dst, src.stride(0), xin.stride(0), cos.stride(0),
                    sin.stride(0), dst.stride(0), dst.stride(0), dst.stride(0), d // 2,
                    COMPUTE_DCOS=False, COMPUTE_DSIN=False, BLOCK_SIZE=rp._BLOCK_SIZE,
                )
            out[i, j] = dst
    return out


def _rope_case(torch, triton, fa, rp, ref_tests, shape, dtype_name, causal, seed):
    dtype = getattr(torch, dtype_name)
    gen = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(shape, generator=gen).to(dtype) for _ in range(4))
    cos, sin = _rope_tables(torch, shape[2], shape[3], dtype)
    record = {"dtype": np.array(dtype_name), "causal": np.array(causal), "seed": np.array(seed)}
    for key, tensor in (("q", q), ("k", k), ("v", v), ("do", do), ("cos", cos), ("sin", sin)):
        _store(record, key, tensor)
    q_r = _ref_rope(torch, triton, rp, q, cos, sin)
    k_r = _ref_rope(torch, triton, rp, k, cos, sin)
    _store(record, "ref_qrot", q_r)
    _store(record, "ref_krot", k_r)
    o, lse, dq_r, dk_r, dv = _reference_kernels(torch, triton, fa, q_r, k_r, v, do, causal)
    dq = _ref_rope(torch, triton, rp, dq_r, cos, sin, backward_of=q)
    dk = _ref_rope(torch, triton, rp, dk_r, cos, sin, backward_of=k)
    record["ref_lse"] = lse.numpy()
    for key, tensor in (("ref_o", o), ("ref_dq", dq), ("ref_dk", dk), ("ref_dv", dv)):
        _store(record, key, tensor)
    man_dq_r, man_dk_r, man_dv = ref_tests._manual_fp32_backward(q_r, k_r, v, do, causal=causal)
    cos32, sin32 = cos.float(), sin.float()
    man_dq = _ref_rope(torch, triton, rp, man_dq_r.float(), cos32, sin32, backward_of=q.float())
    man_dk = _ref_rope(torch, triton, rp, man_dk_r.float(), cos32, sin32, backward_of=k.float())
    for key, grad in (("man_dq", man_dq), ("man_dk", man_dk), ("man_dv", man_dv)):
        record[key] = grad.float().numpy()
    return record


def _inputs(torch, shape, dtype_name, seed, c1: bool):
    dtype = getattr(torch, dtype_name)
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=gen).to(dtype)
    k = torch.randn(shape, generator=gen).to(dtype)
    v = torch.randn(shape, generator=gen).to(dtype)
    if c1:
        # Q/K/V from seed 0 in that order, dO from seed 1.
        do = torch.randn(shape, generator=torch.Generator().manual_seed(1)).to(dtype)
    else:
        do = torch.randn(shape, generator=gen).to(dtype)
    return q, k, v, do


def _store(record: dict, key: str, tensor) -> None:
    """Raw uint16 bits for 16-bit tensors, float32 otherwise."""
    import torch

    if tensor.dtype in (torch.float16, torch.bfloat16):
        record[key + "_bits"] = tensor.contiguous().view(torch.int16).numpy().view(np.uint16)
    else:
        record[key] = tensor.detach().float().numpy()


def _reference_kernels(torch, triton, fa, q, k, v, do, causal):
    b, h, s, d = q.shape
    o = torch.empty_like(q)
    lse = torch.empty((b, h, s), dtype=torch.float32)
    grid = (triton.cdiv(s, 64), b * h)
    fa._flash_attention_forward_kernel.fn[grid](
        q, k, v, o, lse, *q.stride(), *k.stride(), *v.stride(), *o.stride(), h, 1.0 / math.sqrt(d),
        N_CTX=s, HEAD_DIM=d, CAUSAL=causal, STORE_LSE=True, BLOCK_M=64, BLOCK_N=32,
    )
    delta = torch.empty((b, h, s), dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    sm_scale = 1.0 / math.sqrt(d)
    strides = q.stride()
    fa._attn_bwd_preprocess_kernel[(triton.cdiv(s, 64), b * h)](
        o, do, delta, *strides, h, N_CTX=s, HEAD_DIM=d, BLOCK_M=64
    )
    fa._attn_bwd_dkdv_kernel[(triton.cdiv(s, 64), b * h)](
        q, k, v, do, dk, dv, lse, delta, *strides, h, sm_scale, sm_scale * 1.4426950408889634,
        N_CTX=s, HEAD_DIM=d, CAUSAL=causal, BLOCK_M=64, BLOCK_N=64,
    )
    fa._attn_bwd_dq_kernel[(triton.cdiv(s, 64), b * h)](
        q, k, v, do, dq, lse, delta, *strides, h, sm_scale, sm_scale * 1.4426950408889634,
        N_CTX=s, HEAD_DIM=d, CAUSAL=causal, BLOCK_M=64, BLOCK_N=64,
    )
    return o, lse, dq, dk, dv


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, type=Path, help="triton-kernel-lab checkout")
    args = parser.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(args.reference / "src"))
    import torch
    import triton
    from tklab.kernels import flash_attention as fa
    from tklab.kernels import rope as rp

    spec = importlib.util.spec_from_file_location(
        "ref_test_backward", args.reference / "tests" / "test_flash_attention_backward.py"
    )
    ref_tests = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref_tests)

    for name, shape, dtype_name, causal, seed, run_kernels in CASES:
        q, k, v, do = _inputs(torch, shape, dtype_name, seed, c1=name.startswith("c1_"))
        record = {"dtype": np.array(dtype_name), "causal": np.array(causal), "seed": np.array(seed)}
        for key, tensor in (("q", q), ("k", k), ("v", v), ("do", do)):
            _store(record, key, tensor)
        ref_fn = fa._reference_factory(causal=causal)
        qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
        sdpa_o = ref_fn(qf, kf, vf)
        record["sdpa_o"] = sdpa_o.detach().numpy()
        if dtype_name == "float32":
            sdpa_grads = torch.autograd.grad(sdpa_o, (qf, kf, vf), grad_outputs=do.float())
            for key, grad in zip(("sdpa_dq", "sdpa_dk", "sdpa_dv"), sdpa_grads, strict=True):
                record[key] = grad.numpy()
        else:
            man = ref_tests._manual_fp32_backward(q, k, v, do, causal=causal)
            for key, grad in zip(("man_dq", "man_dk", "man_dv"), man, strict=True):
                record[key] = grad.numpy()
        if run_kernels:
            o, lse, dq, dk, dv = _reference_kernels(torch, triton, fa, q, k, v, do, causal)
            record["ref_lse"] = lse.numpy()
            for key, tensor in (("ref_o", o), ("ref_dq", dq), ("ref_dk", dk), ("ref_dv", dv)):
                _store(record, key, tensor)
        np.savez_compressed(HERE / f"{name}.npz", **record)
        print(f"wrote {name}.npz")

    for name, shape, dtype_name, causal, seed in ROPE_CASES:
        record = _rope_case(torch, triton, fa, rp, ref_tests, shape, dtype_name, causal, seed)
        np.savez_compressed(HERE / f"{name}.npz", **record)
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
