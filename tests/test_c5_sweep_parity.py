"""GPU: parity for every configuration of the shape sweep.

The sweep covers causal and non-causal attention, fp16 and bf16, head_dim 64
and 128, S in {512, 1024, 2048, 4096, 8192, 16384} with B = 16384 / S and
H = 16, Q/K/V/dO drawn N(0, 1) from seed 0 — the configurations
``bench.py --sweep`` times.  Each problem runs whole on the GPU (forward with
the LSE, then the backward through ``_launch_backward``) into NaN-prefilled
outputs; the first and last (batch, head) slabs are compared with the
chunked fp32 oracle at the north-star bounds (max-abs 2e-2 for O, 5e-2 for
dQ/dK/dV; relative Frobenius error below 2e-2), the LSE at 1e-3 relative,
and the whole outputs are checked for finiteness (and, causal, for the first
output row equal to V's first row).  This follows the reference's
``tests/test_flash_attention_backward.py:72-111`` at the sweep's sizes.
"""

from __future__ import annotations

import itertools

import pytest
import torch

from oracle.attention_oracle import chunked_reference
from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _launch_backward, _launch_forward, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

TOKENS = 16384
HEADS = 16
SEQ_LENS = (512, 1024, 2048, 4096, 8192, 16384)
CASES = list(itertools.product((torch.float16, torch.bfloat16), (False, True), (64, 128), SEQ_LENS))


def _case_id(case) -> str:
    dtype, causal, d, s = case
    return f"{'f16' if dtype == torch.float16 else 'bf16'}-{'causal' if causal else 'full'}-d{d}-s{s}"


def _slab(t: torch.Tensor, i: int) -> torch.Tensor:
    return t.reshape(-1, *t.shape[2:])[i].unsqueeze(0).unsqueeze(0).cpu()


@pytest.mark.parametrize("case", CASES, ids=[_case_id(c) for c in CASES])
def test_sweep_configuration_matches_oracle(case) -> None:
    dtype, causal, d, s = case
    b = TOKENS // s
    shape = (b, HEADS, s, d)
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(shape, generator=gen, device="cuda").to(dtype) for _ in range(4))
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, HEADS, s), float("nan"), device="cuda")
    _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
    dq, dk, dv = _launch_backward(q, k, v, o, lse, do, causal=causal)
    check_device_status()
    for t in (o, lse, dq, dk, dv):
        assert torch.isfinite(t).all()
    if causal:
        assert torch.equal(o[:, :, 0, :], v[:, :, 0, :])
    chunk = 2048 if s <= 4096 else 1024
    for i in (0, b * HEADS - 1):
        ro, rl, rdq, rdk, rdv = chunked_reference(
            _slab(q, i), _slab(k, i), _slab(v, i), _slab(do, i), causal=causal, chunk=chunk
        )
        got_o = _slab(o, i).float()
        assert (got_o - ro).abs().max().item() <= 2e-2, ("o", i)
        assert relative_frobenius_error(got_o, ro) < 2e-2, ("o", i)
        got_l = lse.reshape(-1, s)[i].cpu()
        assert (got_l - rl.reshape(-1)).abs().max().item() <= 1e-3 * max(1.0, rl.abs().max().item()), ("lse", i)
        for label, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            g = _slab(got, i).float()
            assert (g - want).abs().max().item() <= 5e-2, (label, i)
            assert relative_frobenius_error(g, want) < 2e-2, (label, i)
