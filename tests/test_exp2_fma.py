"""GPU: the FMA-pipe base-2 exponential against its stated bounds.

The forward, the fused backward and the deterministic dQ kernel evaluate
part of each softmax's exponentials on the FP32 units with
``exp2_fma_pair`` (``csrc/sm100_primitives.cuh``): n = round(x), f = x - n
in [-1/2, 1/2], a fitted degree-3 polynomial for 2^f and n added to the
exponent field.  Its comment states the contract checked here, through
``tk_selftest_exp2_fma`` of the test-only probe library:

* relative error at most 7.5e-5 against the exact 2^x (fp64) wherever the
  result is a normal float, checked on a dense grid of [-125.5, 127], on
  every integer and half-integer (the rounding ties of n) and on random
  points;
* just above -126, where the result may come out subnormal, at most 1.5e-4;
* inputs below -126 (and -inf) clamp: the result lies in [0, 2^-126].
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import load_selftest_lib, selftest_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

BOUND = 7.5e-5
SUBNORMAL_EDGE_BOUND = 1.5e-4
TWO_POW_M126 = 2.0**-126


def _eval(x: torch.Tensor) -> torch.Tensor:
    lib = load_selftest_lib()
    xd = x.to(device="cuda", dtype=torch.float32).contiguous()
    y = torch.full_like(xd, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.tk_selftest_exp2_fma(xd.data_ptr(), y.data_ptr(), xd.numel(), stream) == 0
    assert selftest_status(lib, stream) == 0
    return y.cpu()


def _rel_err(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    exact = torch.exp2(x.double())
    return ((y.double() - exact) / exact).abs()


def test_relative_error_bound_on_dense_grid() -> None:
    grid = torch.linspace(-125.5, 127.0, 1 << 23, dtype=torch.float64).float()
    err = _rel_err(grid, _eval(grid))
    worst = int(err.argmax())
    assert err.max().item() <= BOUND, f"max relative error {err.max().item():.3e} at x = {grid[worst].item()!r}"


def test_relative_error_bound_at_rounding_ties_and_random_points() -> None:
    ints = torch.arange(-125, 128, dtype=torch.float32)
    halves = torch.arange(-125, 127, dtype=torch.float32) + 0.5
    gen = torch.Generator().manual_seed(0)
    rand = torch.rand(1 << 22, generator=gen, dtype=torch.float64).mul(252.5).sub(125.5).float()
    near = torch.cat([halves.nextafter(halves + 1), halves.nextafter(halves - 1)])
    x = torch.cat([ints, halves, near, rand])
    err = _rel_err(x, _eval(x))
    assert err.max().item() <= BOUND, f"max relative error {err.max().item():.3e} at x = {x[int(err.argmax())].item()!r}"


def test_subnormal_edge_just_above_the_clamp() -> None:
    x = torch.linspace(-126.0, -125.5, 1 << 16, dtype=torch.float64).float()
    err = _rel_err(x, _eval(x))
    assert err.max().item() <= SUBNORMAL_EDGE_BOUND


def test_inputs_below_minus_126_clamp() -> None:
    x = torch.tensor([-126.5, -127.0, -150.0, -1000.0, -1e30, -math.inf], dtype=torch.float32)
    y = _eval(x).double()
    assert torch.isfinite(y).all()
    assert (y >= 0).all() and (y <= TWO_POW_M126).all(), y.tolist()


def test_odd_length_and_pairing() -> None:
    """Pairs are formed as (x[2i], x[2i+1]); an odd last element is evaluated alone."""
    x = torch.tensor([0.0, 1.0, -1.0, 10.25, 3.5], dtype=torch.float32)
    y = _eval(x)
    assert _rel_err(x, y).max().item() <= BOUND
    assert _eval(x[:1]).item() == pytest.approx(1.0, rel=BOUND)
