"""GPU: the forward's key-split schedule (``tk_attn_fwd_ws``).

Problems with few (batch, head) slabs and long sequences have fewer query
tiles than the device has SMs, so the longest query tile would set the
forward's time.  ``tk_attn_fwd_workspace_bytes`` reports scratch for them,
and ``tk_attn_fwd_ws`` then runs each long query tile as chunks of its key
range (fp32 partial outputs and base-2 log-sum-exps in the scratch) merged by
a second kernel.  These tests run such shapes (causal and not, fp16 and
bf16, head_dim 40 / 64 / 72 / 96 / 128, ragged sequence lengths) through the C ABI
into NaN-prefilled outputs and compare:

* with the CPU oracle (``chunked_reference``) on the first and last slabs, at
  the north-star bounds (max-abs 2e-2 for O, relative Frobenius error below
  2e-2, LSE within 1e-3 relative);
* with the unsplit ``tk_attn_fwd`` on the same inputs: O within four 16-bit
  rounding steps at |O| <= 1 (both round an fp32 value that agrees to fp32
  precision) and the LSE within 1e-4;

plus which shapes are split at all, the argument checks (scratch too small
or misaligned), the no-statistic form (lse NULL), and the public autograd
path, whose backward consumes the merged log-sum-exp.
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle.attention_oracle import chunked_reference
from tklab import _native
from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _NATIVE_DTYPE, attention_causal, attention_noncausal, check_device_status

# Status codes of include/tklab_attn.h.
TK_ERR_INVALID_ARGUMENT = 1
TK_ERR_MISALIGNED = 3

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

# (batch, heads, seq, head_dim, dtype, causal): each has too few query tiles
# for a B200's 148 SMs, so the split schedule is taken.
SPLIT_CASES = [
    (1, 2, 8192, 128, torch.bfloat16, True),
    (1, 2, 16384, 128, torch.float16, True),
    (1, 2, 16384, 64, torch.bfloat16, True),
    (1, 1, 16384, 128, torch.bfloat16, False),
    (1, 2, 8000, 96, torch.bfloat16, True),
    (1, 1, 7000, 64, torch.float16, False),
    (1, 1, 12300, 128, torch.float16, True),
    (1, 1, 7000, 40, torch.bfloat16, True),
    (1, 2, 8192, 72, torch.float16, False),
]


def _case_id(case) -> str:
    b, h, s, d, dtype, causal = case
    return f"b{b}h{h}s{s}d{d}-{'f16' if dtype == torch.float16 else 'bf16'}-{'causal' if causal else 'full'}"


def _inputs(shape, dtype, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(shape, generator=gen, device="cuda").to(dtype) for _ in range(3)]


def _fwd(lib, q, k, v, o, lse, causal, workspace=None, ws_bytes=0) -> int:
    b, h, s, d = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tk_attn_fwd_ws(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), None if lse is None else lse.data_ptr(),
        b, h, s, d, _NATIVE_DTYPE[q.dtype], int(causal), 1.0 / math.sqrt(d),
        None if workspace is None else workspace.data_ptr(), ws_bytes, stream,
    )


def _ws_bytes(lib, q, causal) -> int:
    b, h, s, d = q.shape
    return int(lib.tk_attn_fwd_workspace_bytes(b, h, s, d, _NATIVE_DTYPE[q.dtype], int(causal)))


def _slab(t: torch.Tensor, i: int) -> torch.Tensor:
    return t.reshape(-1, *t.shape[2:])[i].unsqueeze(0).unsqueeze(0).cpu()


def test_workspace_only_for_underfilled_problems() -> None:
    lib = _native.load()
    bf16 = _native.TK_DTYPE_BF16
    # The headline shape has thousands of query tiles: never split.
    assert lib.tk_attn_fwd_workspace_bytes(8, 32, 4096, 128, bf16, 1) == 0
    # Short sequences are not split (items too short to pay for it), nor
    # problems that keep the device more than half busy on average.
    assert lib.tk_attn_fwd_workspace_bytes(1, 1, 1024, 128, bf16, 1) == 0
    assert lib.tk_attn_fwd_workspace_bytes(1, 8, 4096, 128, bf16, 1) == 0
    assert lib.tk_attn_fwd_workspace_bytes(1, 4, 16384, 128, bf16, 1) == 0
    # Head widths above 128 run another kernel: no split.
    assert lib.tk_attn_fwd_workspace_bytes(1, 1, 16384, 256, bf16, 1) == 0
    # Invalid shapes report 0 instead of failing.
    assert lib.tk_attn_fwd_workspace_bytes(1, 1, 16384, 100, bf16, 1) == 0
    assert lib.tk_attn_fwd_workspace_bytes(0, 1, 16384, 128, bf16, 1) == 0
    for b, h, s, d, dtype, causal in SPLIT_CASES:
        assert lib.tk_attn_fwd_workspace_bytes(b, h, s, d, _NATIVE_DTYPE[dtype], int(causal)) > 0


@pytest.mark.parametrize("case", SPLIT_CASES, ids=[_case_id(c) for c in SPLIT_CASES])
def test_split_forward_matches_oracle_and_unsplit(case) -> None:
    b, h, s, d, dtype, causal = case
    lib = _native.load()
    q, k, v = _inputs((b, h, s, d), dtype)
    ws_bytes = _ws_bytes(lib, q, causal)
    assert ws_bytes > 0
    ws = torch.full((ws_bytes,), 0xFF, dtype=torch.uint8, device="cuda")  # NaN-filled fp32 scratch
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, s), float("nan"), device="cuda")
    assert _fwd(lib, q, k, v, o, lse, causal, ws, ws_bytes) == 0
    o_ref = torch.full_like(q, float("nan"))
    lse_ref = torch.full((b, h, s), float("nan"), device="cuda")
    assert _fwd(lib, q, k, v, o_ref, lse_ref, causal) == 0
    check_device_status()
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    if causal:
        assert torch.equal(o[:, :, 0, :], v[:, :, 0, :])
    # Against the unsplit kernel: a few 16-bit rounding steps at |O| <= 1.
    step = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    assert (o.float() - o_ref.float()).abs().max().item() <= 4 * step
    assert (lse - lse_ref).abs().max().item() <= 1e-4 * max(1.0, lse_ref.abs().max().item())
    # Against the CPU oracle.
    for i in (0, b * h - 1):
        zero = torch.zeros_like(_slab(q, i))
        ro, rl, *_ = chunked_reference(_slab(q, i), _slab(k, i), _slab(v, i), zero, causal=causal, chunk=1024)
        got_o = _slab(o, i).float()
        assert (got_o - ro).abs().max().item() <= 2e-2, ("o", i)
        assert relative_frobenius_error(got_o, ro) < 2e-2, ("o", i)
        got_l = lse.reshape(-1, s)[i].cpu()
        assert (got_l - rl.reshape(-1)).abs().max().item() <= 1e-3 * max(1.0, rl.abs().max().item()), ("lse", i)


def test_split_forward_without_statistic() -> None:
    lib = _native.load()
    q, k, v = _inputs((1, 2, 8192, 128), torch.bfloat16, seed=3)
    ws_bytes = _ws_bytes(lib, q, True)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    o = torch.full_like(q, float("nan"))
    o_ref = torch.full_like(q, float("nan"))
    assert _fwd(lib, q, k, v, o, None, True, ws, ws_bytes) == 0
    assert _fwd(lib, q, k, v, o_ref, None, True) == 0
    check_device_status()
    assert (o.float() - o_ref.float()).abs().max().item() <= 4 * 2.0 ** -8


def test_split_forward_argument_checks() -> None:
    lib = _native.load()
    q, k, v = _inputs((1, 2, 8192, 128), torch.bfloat16)
    ws_bytes = _ws_bytes(lib, q, True)
    o = torch.empty_like(q)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device="cuda")
    assert _fwd(lib, q, k, v, o, None, True, ws, ws_bytes - 256) == TK_ERR_INVALID_ARGUMENT
    misaligned = ws[16:]
    assert _fwd(lib, q, k, v, o, None, True, misaligned, ws_bytes) == TK_ERR_MISALIGNED
    check_device_status()


@pytest.mark.parametrize("causal", [True, False], ids=["causal", "full"])
def test_public_autograd_path_on_split_shape(causal) -> None:
    shape = (1, 2, 8192, 128)
    q, k, v = (t.requires_grad_() for t in _inputs(shape, torch.bfloat16, seed=5))
    gen = torch.Generator(device="cuda").manual_seed(6)
    do = torch.randn(shape, generator=gen, device="cuda").to(torch.bfloat16)
    fn = attention_causal if causal else attention_noncausal
    o = fn(q, k, v)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
    check_device_status()
    for i in (0, 1):
        ro, _, rdq, rdk, rdv = chunked_reference(
            _slab(q.detach(), i), _slab(k.detach(), i), _slab(v.detach(), i), _slab(do, i), causal=causal, chunk=1024
        )
        assert (_slab(o.detach(), i).float() - ro).abs().max().item() <= 2e-2
        for label, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            g = _slab(got, i).float()
            assert (g - want).abs().max().item() <= 5e-2, (label, i)
            assert relative_frobenius_error(g, want) < 2e-2, (label, i)
