"""GPU: the tcgen05 operand conventions the attention kernels rely on.

``tk_selftest_umma`` (in the test-only probe library) runs one 128 x n x 128
product per operand form used inside the kernels (K-major x K-major, TMEM A
x MN-major B, MN-major x MN-major, K-major x MN-major).  Each is compared with an fp32 matmul of the
same 16-bit inputs; the tensor core accumulates in fp32, so agreement is
tight.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_selftest_lib, selftest_status
from tklab import _native

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

DTYPES = {torch.float16: _native.TK_DTYPE_F16, torch.bfloat16: _native.TK_DTYPE_BF16}


def _run(mode: int, n: int, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    gen = torch.Generator().manual_seed(100 + 10 * mode + n)
    a = torch.randn(128, 128, generator=gen).to(dtype).cuda()
    b_cols = 128 if mode == 0 else n
    b = torch.randn(128, b_cols, generator=gen).to(dtype).cuda()
    c = torch.full((128, b_cols), float("nan"), device="cuda")
    lib = load_selftest_lib()
    status = lib.tk_selftest_umma(
        a.data_ptr(), b.data_ptr(), c.data_ptr(), mode, n, DTYPES[dtype],
        torch.cuda.current_stream().cuda_stream,
    )
    _native.check(status, "tk_selftest_umma")
    assert selftest_status(lib, torch.cuda.current_stream().cuda_stream) == 0
    af, bf = a.float(), b.float()
    if mode == 0:
        expected = af @ bf.T
    elif mode == 2:
        expected = af.T @ bf
    else:
        expected = af @ bf
    return c, expected


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize(("mode", "n"), [(0, 128), (1, 128), (1, 64), (2, 128), (2, 64), (3, 128), (3, 64)])
def test_umma_operand_forms(mode: int, n: int, dtype: torch.dtype) -> None:
    got, expected = _run(mode, n, dtype)
    assert torch.isfinite(got).all()
    err = (got - expected).abs().max().item()
    assert err <= 1e-3 * max(1.0, expected.abs().max().item()), f"mode {mode} n {n}: max err {err}"
