"""CPU: the public wrappers validate before any launch (reference ``tests/test_kernel_validation.py:185-191``)."""

from __future__ import annotations

import pytest
import torch

from tklab.kernels.flash_attention import (
    _launch_backward,
    _launch_forward,
    attention_causal,
    attention_noncausal,
)


def test_attention_rejects_shape_mismatch() -> None:
    """Reject mismatched Q/K/V metadata before requiring CUDA."""
    query = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    key = torch.zeros(1, 2, 7, 64, dtype=torch.float16)
    value = torch.zeros_like(query)
    with pytest.raises(ValueError, match="identical shapes"):
        attention_noncausal(query, key, value)


@pytest.mark.parametrize(
    ("shape", "message"),
    [((2, 8, 64), "batch, heads, sequence, dim"), ((1, 0, 8, 64), "empty dimensions")],
)
def test_attention_rejects_bad_rank_and_empty(shape, message) -> None:
    x = torch.zeros(shape, dtype=torch.float16)
    with pytest.raises(ValueError, match=message):
        attention_causal(x, x, x)


def test_attention_requires_cuda() -> None:
    x = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="requires CUDA"):
        attention_causal(x, x, x)


def test_attention_requires_cuda_on_meta_tensors() -> None:
    x = torch.empty(1, 2, 8, 64, dtype=torch.float16, device="meta")
    with pytest.raises(ValueError, match="requires CUDA"):
        _launch_forward(x, x, x, x, x, causal=False, store_lse=False)


def test_backward_rejects_mismatched_upstream_gradient() -> None:
    x = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    lse = torch.zeros(1, 2, 8)
    with pytest.raises(ValueError, match="upstream gradient"):
        _launch_backward(x, x, x, x, lse, torch.zeros(1, 2, 8, 64), causal=True)
