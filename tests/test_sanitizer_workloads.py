"""GPU: the reference's partial-tile workloads (``tests/test_sanitizer_workloads.py:170-199``).

The reference wrote these to run under compute-sanitizer.  Sanitizer tools
are closed on the B200 pool, so here they run as plain tests with NaN-filled
outputs (an unwritten element cannot pass) and a device-status check after
each launch.
"""

from __future__ import annotations

from collections.abc import Callable

import pytest
import torch

from tklab.kernels.flash_attention import attention_causal, attention_noncausal, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]


@pytest.mark.parametrize("kernel", [attention_noncausal, attention_causal])
def test_sanitizer_flash_attention_partial_tiles(
    kernel: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
) -> None:
    shape = (1, 16, 1000, 64)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.float16) for _ in range(3))
    output = kernel(q, k, v)
    check_device_status()
    if not torch.isfinite(output).all():
        raise AssertionError("attention workload produced non-finite output")


@pytest.mark.parametrize("kernel", [attention_noncausal, attention_causal])
def test_sanitizer_flash_attention_backward_partial_tiles(
    kernel: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
) -> None:
    shape = (1, 16, 129, 64)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.float16, requires_grad=True) for _ in range(3))
    do = torch.randn(shape, device="cuda", dtype=torch.float16)
    output = kernel(q, k, v)
    gradients = torch.autograd.grad(output, (q, k, v), grad_outputs=do)
    check_device_status()
    if not all(torch.isfinite(gradient).all() for gradient in gradients):
        raise AssertionError("attention backward workload produced non-finite gradients")
