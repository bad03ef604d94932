"""GPU: flash-attention backward (the reference's tests, plus bf16 / head_dim 128).

The first two tests are the reference's ``tests/test_flash_attention_backward.py``
(same seeds, shapes and thresholds, including the 1e-3 pin against the
manual fp32 algebra at fp16, S=128).
"""

from __future__ import annotations

from collections.abc import Callable

import pytest
import torch
import torch.nn.functional as F

from oracle.attention_oracle import manual_backward
from tklab.harness.tolerances import assert_relative_frobenius
from tklab.kernels.flash_attention import attention_causal, attention_noncausal, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

Kernel = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _inputs(
    sequence_length: int, dtype: torch.dtype = torch.float16, head_dim: int = 64, heads: int = 16
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Create contiguous leaves and an upstream gradient."""
    shape = (1, heads, sequence_length, head_dim)
    q = torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True)
    k = torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True)
    v = torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True)
    do = torch.randn(shape, device="cuda", dtype=dtype)
    return q, k, v, do


@pytest.mark.parametrize(
    ("causal", "kernel"),
    [(False, attention_noncausal), (True, attention_causal)],
)
@pytest.mark.parametrize("sequence_length", [128, 1000])
def test_flash_attention_backward_matches_sdpa(causal: bool, kernel: Kernel, sequence_length: int) -> None:
    """Validate dQ, dK, and dV against SDPA autograd on full and partial tiles."""
    torch.manual_seed(41 + sequence_length + int(causal))
    q, k, v, do = _inputs(sequence_length)

    reference = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    dq_ref, dk_ref, dv_ref = torch.autograd.grad(reference, (q, k, v), grad_outputs=do)

    output = kernel(q, k, v)
    dq_tri, dk_tri, dv_tri = torch.autograd.grad(output, (q, k, v), grad_outputs=do)

    for grad, reference_grad in ((dq_tri, dq_ref), (dk_tri, dk_ref), (dv_tri, dv_ref)):
        assert torch.isfinite(grad).all()
        assert_relative_frobenius(grad, reference_grad, max_relative_error=3e-2)
    check_device_status()


@pytest.mark.parametrize(
    ("causal", "kernel"),
    [(False, attention_noncausal), (True, attention_causal)],
)
def test_flash_attention_backward_matches_manual_fp32_algebra(causal: bool, kernel: Kernel) -> None:
    """Cross-check dQ/dK/dV without relying on the SDPA backward implementation."""
    torch.manual_seed(79 + int(causal))
    q, k, v, do = _inputs(128)
    expected = manual_backward(q, k, v, do, causal=causal)
    output = kernel(q, k, v)
    actual = torch.autograd.grad(output, (q, k, v), grad_outputs=do)
    for grad, reference_grad in zip(actual, expected, strict=True):
        assert_relative_frobenius(grad.cpu(), reference_grad, max_relative_error=1e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sequence_length", [1, 129, 384])
def test_widened_backward_matches_manual_algebra(
    dtype: torch.dtype, head_dim: int, causal: bool, sequence_length: int
) -> None:
    """bf16 and head_dim 128 gradients against the fp32 algebra (max-abs and rel-Frobenius)."""
    torch.manual_seed(5 * sequence_length + head_dim + int(causal))
    q, k, v, do = _inputs(sequence_length, dtype=dtype, head_dim=head_dim, heads=3)
    expected = manual_backward(q, k, v, do, causal=causal)
    output = (attention_causal if causal else attention_noncausal)(q, k, v)
    actual = torch.autograd.grad(output, (q, k, v), grad_outputs=do)
    for name, grad, reference_grad in zip(("dq", "dk", "dv"), actual, expected, strict=True):
        grad = grad.float().cpu()
        assert torch.isfinite(grad).all(), name
        assert (grad - reference_grad).abs().max().item() <= 5e-2, name
        if sequence_length == 1 and name in ("dq", "dk"):
            # One key: dS = dP - delta == 0 exactly; dQ and dK are rounding noise on both sides.
            assert grad.abs().max().item() <= 1e-5
            continue
        assert_relative_frobenius(grad, reference_grad, max_relative_error=3e-2)
    check_device_status()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [8, 32, 48, 80, 96, 112])
@pytest.mark.parametrize("causal", [False, True])
def test_general_head_dim_backward_matches_manual_algebra(dtype: torch.dtype, head_dim: int, causal: bool) -> None:
    """Gradients for head dims that are not a kernel width (zero-filled loads, clipped stores and
    dQ reductions past head_dim) against the fp32 algebra."""
    torch.manual_seed(13 * head_dim + int(causal))
    q, k, v, do = _inputs(300, dtype=dtype, head_dim=head_dim, heads=3)
    expected = manual_backward(q, k, v, do, causal=causal)
    output = (attention_causal if causal else attention_noncausal)(q, k, v)
    actual = torch.autograd.grad(output, (q, k, v), grad_outputs=do)
    for name, grad, reference_grad in zip(("dq", "dk", "dv"), actual, expected, strict=True):
        grad = grad.float().cpu()
        assert grad.shape == reference_grad.shape, name
        assert torch.isfinite(grad).all(), name
        assert (grad - reference_grad).abs().max().item() <= 5e-2, name
        assert_relative_frobenius(grad, reference_grad, max_relative_error=3e-2)
    check_device_status()
