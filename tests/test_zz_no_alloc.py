"""GPU: the allocation-free backward entry point, ``tk_attn_bwd_noalloc``.

Some callers cannot allocate device memory at the point where they run the
backward — a plugin whose host gives it no allocator, a host framework whose
pool owns every device byte, an allocation-free hot loop — so they cannot hand the regular backward its two scratch buffers
(delta and the fp32 dQ accumulator).  ``tk_attn_bwd_noalloc`` keeps that
scratch in a 64 MiB array inside the library instead.  This file checks,
through the C ABI, that two calls in a row (different inputs, so the second
one depends on the shared scratch being re-cleared) give the same dQ, dK and
dV as the regular entry points and as the CPU fp32 oracle
(``oracle.attention_oracle.manual_backward``), and that an over-capacity
problem is refused before anything is launched.  It sits in its own file,
collected last.
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle.attention_oracle import manual_backward
from tklab import _native
from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _NATIVE_DTYPE, _launch_forward, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

TK_ERR_TOO_LARGE = 8


def _inputs(shape, dtype, seed, causal):
    gen = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(shape, generator=gen).to(dtype).cuda() for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty(shape[:-1], dtype=torch.float32, device="cuda")
    _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
    return q, k, v, o, do, lse


def _regular(lib, q, k, v, o, do, lse, causal, stream):
    b, h, s, d = q.shape
    nd = _NATIVE_DTYPE[q.dtype]
    delta = torch.empty((b, h, s), dtype=torch.float32, device="cuda")
    accum = torch.empty((b, h, s, d), dtype=torch.float32, device="cuda")
    grads = [torch.empty_like(q) for _ in range(3)]
    _native.check(lib.tk_attn_bwd_pre(o.data_ptr(), do.data_ptr(), delta.data_ptr(), accum.data_ptr(),
                                      b, h, s, d, nd, stream), "tk_attn_bwd_pre")
    _native.check(lib.tk_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                  delta.data_ptr(), accum.data_ptr(), grads[0].data_ptr(), grads[1].data_ptr(),
                                  grads[2].data_ptr(), b, h, s, d, nd, int(causal), 1.0 / math.sqrt(d), stream),
                  "tk_attn_bwd")
    return grads


def _noalloc(lib, q, k, v, o, do, lse, causal, stream):
    b, h, s, d = q.shape
    grads = [torch.full_like(q, float("nan")) for _ in range(3)]
    _native.check(lib.tk_attn_bwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                          lse.data_ptr(), grads[0].data_ptr(), grads[1].data_ptr(),
                                          grads[2].data_ptr(), b, h, s, d, _NATIVE_DTYPE[q.dtype], int(causal),
                                          1.0 / math.sqrt(d), stream), "tk_attn_bwd_noalloc")
    return grads


@pytest.mark.parametrize(
    ("shape", "dtype", "causal"),
    [((1, 4, 1000, 128), torch.bfloat16, True), ((2, 3, 257, 64), torch.float16, False)],
)
def test_noalloc_backward_matches_regular_entry_point_twice(shape, dtype, causal) -> None:
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((1, 2)):
        q, k, v, o, do, lse = _inputs(shape, dtype, seed=seed + 17 * len(shape[2:]), causal=causal)
        expected = _regular(lib, q, k, v, o, do, lse, causal, stream)
        got = _noalloc(lib, q, k, v, o, do, lse, causal, stream)
        check_device_status()
        oracle = manual_backward(q, k, v, do, causal=causal)
        for name, g, e, r in zip(("dq", "dk", "dv"), got, expected, oracle, strict=True):
            g, e = g.float().cpu(), e.float().cpu()
            assert torch.isfinite(g).all(), (call, name)
            assert (g - e).abs().max().item() <= 5e-2, (call, name)
            assert relative_frobenius_error(g, e) < 2e-2, (call, name)
            # Against the CPU fp32 oracle: the gradient tolerances of the
            # parity tests (max abs 5e-2, relative Frobenius 2e-2).
            assert (g - r).abs().max().item() <= 5e-2, (call, name, "oracle")
            assert relative_frobenius_error(g, r) < 2e-2, (call, name, "oracle")


def test_noalloc_refuses_problems_beyond_its_scratch() -> None:
    lib = _native.load()
    x = torch.empty(16, dtype=torch.float16, device="cuda")
    p = x.data_ptr()
    # 1 x 32 x 4096 x (128 + 1) floats = 16.9 Mi > 16 Mi: refused before any launch.
    rc = lib.tk_attn_bwd_noalloc(p, p, p, p, p, p, p, p, p, 1, 32, 4096, 128, 1, 1, 0.088, None)
    assert rc == TK_ERR_TOO_LARGE
    assert _native.status_string(rc) == "problem size exceeds the supported range"
