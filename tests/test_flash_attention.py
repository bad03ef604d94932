"""GPU: flash-attention forward (the reference's tests, plus bf16 / head_dim 128).

The first two tests are the reference's ``tests/test_flash_attention.py``
unchanged in substance (same seeds, shapes and thresholds); they run against
the sm_100a kernels through the same public names.
"""

from __future__ import annotations

import math
from collections.abc import Callable

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

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]


@pytest.mark.parametrize(
    ("causal", "kernel"),
    [(False, attention_noncausal), (True, attention_causal)],
)
@pytest.mark.parametrize("sequence_length", [128, 1000])
def test_flash_attention_matches_sdpa(
    causal: bool,
    kernel: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
    sequence_length: int,
) -> None:
    """Validate regular and partial query/key tiles against SDPA."""
    torch.manual_seed(23 + sequence_length + int(causal))
    shape = (1, 16, sequence_length, 64)
    q = torch.randn(shape, device="cuda", dtype=torch.float16)
    k = torch.randn(shape, device="cuda", dtype=torch.float16)
    v = torch.randn(shape, device="cuda", dtype=torch.float16)

    output = kernel(q, k, v)
    reference = F.scaled_dot_product_attention(q, k, v, is_causal=causal)

    assert torch.isfinite(output).all()
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    check_device_status()


@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_saved_statistic_is_base2_logsumexp(causal: bool) -> None:
    """Lock the saved statistic to normalized LSE, never the running maximum."""
    torch.manual_seed(91 + int(causal))
    shape = (1, 2, 129, 64)
    q = torch.randn(shape, device="cuda", dtype=torch.float16)
    k = torch.randn(shape, device="cuda", dtype=torch.float16)
    v = torch.randn(shape, device="cuda", dtype=torch.float16)
    output = torch.empty_like(q)
    softmax_lse = torch.empty(shape[:-1], device="cuda", dtype=torch.float32)

    _launch_forward(q, k, v, output, softmax_lse, causal=causal, store_lse=True)

    scores = (q.float() @ k.float().transpose(-2, -1)) * (shape[-1] ** -0.5)
    if causal:
        upper = torch.triu(torch.ones(shape[-2], shape[-2], device=q.device, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(upper, -torch.inf)
    expected = torch.logsumexp(scores, dim=-1) * math.log2(math.e)

    assert torch.isfinite(softmax_lse).all()
    assert_relative_frobenius(softmax_lse, expected, max_relative_error=1e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sequence_length", [1, 200, 513])
def test_widened_contract_matches_sdpa(
    dtype: torch.dtype, head_dim: int, causal: bool, sequence_length: int
) -> None:
    """bf16 and head_dim 128 (the widened contract) against fp32 SDPA."""
    torch.manual_seed(7 * sequence_length + head_dim + int(causal))
    shape = (2, 3, sequence_length, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(3))
    output = (attention_causal if causal else attention_noncausal)(q, k, v)
    reference = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    assert (output.float() - reference).abs().max().item() <= 2e-2
    check_device_status()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [8, 32, 48, 80, 96, 112])
@pytest.mark.parametrize("causal", [False, True])
def test_general_head_dim_matches_sdpa(dtype: torch.dtype, head_dim: int, causal: bool) -> None:
    """Head dims that are not a kernel width (run with the columns past head_dim zero-filled on load
    and clipped on store) against fp32 SDPA, with the base-2 LSE."""
    torch.manual_seed(11 * head_dim + int(causal))
    shape = (2, 3, 333, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(3))
    output = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)
    assert (output.float() - reference).abs().max().item() <= 2e-2
    scores = q.float() @ k.float().transpose(-1, -2) / math.sqrt(head_dim)
    if causal:
        scores = scores.masked_fill(torch.ones(333, 333, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    expected = torch.logsumexp(scores, dim=-1) / math.log(2.0)
    assert (lse - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    check_device_status()
