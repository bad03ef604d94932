"""GPU: the sm_100a kernels against the reference's own outputs (golden fixtures).

Same seeded inputs (bit-identical 16-bit tensors rebuilt from the fixtures),
called through the C ABI via the public launchers.  Compared with the
reference Triton kernels' results (float16/head_dim 64 cases) and with the
reference's fp32 SDPA / manual-algebra results (every case).
"""

from __future__ import annotations

import math

import pytest
import torch
from conftest import golden_cases, load_golden

from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _launch_backward, _launch_forward, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

# The fp32 config-1 case is the CPU reference's own configuration; the
# kernels take 16-bit inputs, so it is exercised through its bf16/f16 peers.
CASES = [name for name in golden_cases() if not name.startswith("c1_")]


def _run(case: dict) -> dict[str, torch.Tensor]:
    q, k, v, do = (case[key].cuda() for key in ("q", "k", "v", "do"))
    b, h, s, _ = q.shape
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, s), float("nan"), device="cuda")
    _launch_forward(q, k, v, o, lse, causal=case["causal"], store_lse=True)
    dq, dk, dv = _launch_backward(q, k, v, o, lse, do, causal=case["causal"])
    check_device_status()
    return {"o": o.float().cpu(), "lse": lse.cpu(), "dq": dq.float().cpu(), "dk": dk.float().cpu(),
            "dv": dv.float().cpu()}


@pytest.mark.parametrize("name", CASES)
def test_against_reference_fp32(name: str) -> None:
    case = load_golden(name)
    got = _run(case)
    assert relative_frobenius_error(got["o"], case["sdpa_o"]) < 2e-2
    assert (got["o"] - case["sdpa_o"]).abs().max().item() <= 2e-2
    for key in ("dq", "dk", "dv"):
        want = case[f"man_{key}"]
        assert torch.isfinite(got[key]).all(), key
        assert relative_frobenius_error(got[key], want) < 3e-2, key
        assert (got[key] - want).abs().max().item() <= 5e-2, key


@pytest.mark.parametrize("name", [c for c in CASES if "ref_o" in load_golden(c)])
def test_against_reference_triton_kernels(name: str) -> None:
    """Agreement with the reference kernels is at the level of their own fp16 rounding."""
    case = load_golden(name)
    got = _run(case)
    assert relative_frobenius_error(got["o"], case["ref_o"].float()) < 2e-3
    assert relative_frobenius_error(got["lse"], case["ref_lse"]) < 1e-4
    for key in ("dq", "dk", "dv"):
        assert relative_frobenius_error(got[key], case[f"ref_{key}"].float()) < 3e-3, key
