"""GPU: the forward's persistent schedule, including odd head dims and ragged tails.

The forward runs one persistent CTA per SM (units pairing a head's query-tile
pairs, O written from registers straight to global memory) for causal
problems and for short non-causal ones (S <= 512) once there are at least two
units per SM; otherwise one CTA per query-tile pair.  These cases have 320
(batch, head) slabs, enough units for the persistent schedule on a B200, at
ragged sequence lengths and head dims that are not 64 or 128 (the epilogue
then skips the columns past the true width).  Sampled slabs are compared
with the CPU fp32 oracle (``manual_forward_lse``) at the parity bounds
(max-abs 2e-2 for O, relative Frobenius error below 2e-2, LSE within 1e-3),
and every output element must be written (NaN-prefilled buffers).
"""

from __future__ import annotations

import itertools

import pytest
import torch

from oracle.attention_oracle import manual_forward_lse
from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _launch_forward, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

CASES = list(itertools.product((torch.float16, torch.bfloat16), (False, True), (40, 72, 128), (300, 512)))


def _case_id(case) -> str:
    dtype, causal, d, s = case
    return f"{'f16' if dtype == torch.float16 else 'bf16'}-{'causal' if causal else 'full'}-d{d}-s{s}"


@pytest.mark.parametrize("case", CASES, ids=[_case_id(c) for c in CASES])
def test_persistent_forward_matches_oracle(case) -> None:
    dtype, causal, d, s = case
    shape = (20, 16, s, d)
    gen = torch.Generator(device="cuda").manual_seed(d * 1000 + s + int(causal))
    q, k, v = (torch.randn(shape, generator=gen, device="cuda").to(dtype) for _ in range(3))
    o = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:-1], float("nan"), device="cuda")
    _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
    check_device_status()
    assert torch.isfinite(o).all()
    assert torch.isfinite(lse).all()
    flat = (q.reshape(-1, s, d), k.reshape(-1, s, d), v.reshape(-1, s, d))
    for i in (0, 161, 319):
        qi, ki, vi = (t[i].reshape(1, 1, s, d).cpu() for t in flat)
        ref_o, ref_l = manual_forward_lse(qi, ki, vi, causal=causal)
        got_o = o.reshape(-1, s, d)[i].reshape(1, 1, s, d).float().cpu()
        assert (got_o - ref_o).abs().max().item() <= 2e-2, ("o", i)
        assert relative_frobenius_error(got_o, ref_o) < 2e-2, ("o", i)
        got_l = lse.reshape(-1, s)[i].cpu()
        ref_l = ref_l.reshape(-1)
        assert (got_l - ref_l).abs().max().item() <= 1e-3 * max(1.0, ref_l.abs().max().item()), ("lse", i)
