"""GPU: registry-wide correctness (the reference's ``tests/test_correctness.py``).

Every registered entry, every dtype it declares, its correctness sizes and
its adversarial case, against the fp32 PyTorch reference on the GPU.
"""

from __future__ import annotations

import pytest
import torch

import tklab.kernels  # noqa: F401
from tklab.harness.tolerances import assert_close
from tklab.registry import REGISTRY, KernelSpec


def _assert_spec_output(spec: KernelSpec, output: torch.Tensor, reference: torch.Tensor) -> None:
    if spec.assert_fn is None:
        assert_close(output, reference, rtol=spec.rtol, atol=spec.atol)
    else:
        spec.assert_fn(output, reference)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")
@pytest.mark.parametrize("name", REGISTRY)
def test_matches_reference_on_gpu(name: str) -> None:
    spec = REGISTRY[name]
    device = torch.device("cuda")
    torch.manual_seed(0)
    for dtype in spec.dtypes:
        for size in spec.validation_sizes():
            args = spec.make_inputs(size, device, dtype)
            output = spec.triton_fn(*args)
            reference = spec.ref_fn(*(argument.float() for argument in args))
            _assert_spec_output(spec, output, reference)
    if spec.make_adversarial is not None:
        args = spec.make_adversarial(device)
        output = spec.triton_fn(*args)
        reference = spec.ref_fn(*(argument.float() for argument in args))
        _assert_spec_output(spec, output, reference)
