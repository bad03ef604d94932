"""GPU: the forward for head dims 136..256 (persistent 192- and 256-column kernels, 64-key tiles)
against fp32 SDPA, and the backward's refusal of those widths.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from tklab.harness.tolerances import assert_relative_frobenius
from tklab.kernels.flash_attention import (
    _launch_forward,
    attention_causal,
    attention_noncausal,
    check_device_status,
)

gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")


def test_head_dim_above_256_rejected_before_device_work() -> None:
    q = torch.zeros(1, 1, 4, 264, dtype=torch.float16)
    with pytest.raises(ValueError):
        attention_causal(q, q, q)


def _expected_lse(q: torch.Tensor, k: torch.Tensor, causal: bool) -> torch.Tensor:
    n = q.shape[2]
    scores = q.float() @ k.float().transpose(-1, -2) / math.sqrt(q.shape[-1])
    if causal:
        scores = scores.masked_fill(torch.ones(n, n, device=q.device, dtype=torch.bool).triu(1), float("-inf"))
    return torch.logsumexp(scores, dim=-1) / math.log(2.0)


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [136, 192, 200, 256])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq", [1, 7, 64, 65, 129, 1000])
def test_wide_head_forward_matches_sdpa(dtype: torch.dtype, head_dim: int, causal: bool, seq: int) -> None:
    torch.manual_seed(13 * head_dim + seq + int(causal))
    shape = (2, 3, seq, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(3))
    output = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    assert (output.float() - reference).abs().max().item() <= 2e-2
    expected = _expected_lse(q, k, causal)
    assert (lse - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("head_dim", [176, 256])
@pytest.mark.parametrize("causal", [False, True])
def test_wide_head_forward_many_units_per_cta(head_dim: int, causal: bool) -> None:
    """Enough (batch, head) slabs that every persistent CTA walks several work units, with an odd
    number of query tiles (1100 rows: 9 tiles, the middle one an unpaired causal unit)."""
    torch.manual_seed(17 + head_dim + int(causal))
    shape = (2, 48, 1100, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    output = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    assert (output.float() - reference).abs().max().item() <= 3e-2
    expected = _expected_lse(q, k, causal)
    assert (lse - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    again = torch.empty_like(q)
    _launch_forward(q, k, v, again, lse, causal=causal, store_lse=True)
    assert torch.equal(again, output)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("causal", [False, True])
def test_wide_head_forward_growing_scores(causal: bool) -> None:
    """Scores that grow along the keys move every row's running maximum many times (the O rescale
    path), with a spread of 2^10 in base 2 across a row."""
    torch.manual_seed(5)
    seq, head_dim = 777, 256
    q = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    ramp = torch.linspace(0.2, 3.0, seq, device="cuda")[None, None, :, None]
    k = (k.float() * ramp).to(torch.bfloat16)
    v = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    output = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    assert (output.float() - reference).abs().max().item() <= 3e-2
    expected = _expected_lse(q, k, causal)
    assert (lse - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    check_device_status()


@pytest.mark.gpu
@gpu
def test_wide_head_public_api_inference_and_backward_refusal() -> None:
    torch.manual_seed(2)
    q, k, v = (torch.randn(2, 4, 300, 256, device="cuda", dtype=torch.float16) for _ in range(3))
    with torch.no_grad():
        out_c = attention_causal(q, k, v)
        out_n = attention_noncausal(q, k, v)
    for out, causal in ((out_c, True), (out_n, False)):
        ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
        assert_relative_frobenius(out, ref, max_relative_error=2e-2)
    # Bitwise reproducible.
    with torch.no_grad():
        assert torch.equal(attention_causal(q, k, v), out_c)
    # The forward runs under autograd; the backward of a 256-wide head is not built and says so.
    qg = q.clone().requires_grad_(True)
    out = attention_causal(qg, k, v)
    assert torch.equal(out.detach(), out_c)
    with pytest.raises(NotImplementedError, match="forward-only"):
        out.sum().backward()
    check_device_status()
