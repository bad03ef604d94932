"""CPU: registry invariants (the reference's ``tests/test_registry.py``, attention entries only)."""

from __future__ import annotations

from typing import Any, cast

import pytest
import torch

import tklab.kernels  # noqa: F401
from tklab.registry import REGISTRY, KernelSpec, register


def _identity(x: torch.Tensor) -> torch.Tensor:
    return x


def _launch(args: tuple[torch.Tensor, ...], output: torch.Tensor) -> None:
    output.copy_(args[0])


def _make_inputs(size: int, device: torch.device, dtype: torch.dtype) -> tuple[torch.Tensor, ...]:
    return (torch.zeros(size, device=device, dtype=dtype),)


def _make_output(args: tuple[torch.Tensor, ...]) -> torch.Tensor:
    return torch.empty_like(args[0])


def _memory_spec(**overrides: object) -> KernelSpec:
    values: dict[str, object] = {
        "name": "example_kernel",
        "description": "Example kernel used by unit tests.",
        "triton_fn": _identity,
        "launch_fn": _launch,
        "ref_fn": _identity,
        "make_inputs": _make_inputs,
        "make_output": _make_output,
        "sizes": (1, 2),
        "bound": "memory",
        "bytes_moved": lambda size, dtype: size * torch.empty((), dtype=dtype).element_size(),
    }
    values.update(overrides)
    return KernelSpec(**cast(dict[str, Any], values))


def test_registry_contains_the_attention_entries() -> None:
    assert set(REGISTRY) == {
        "attention_causal",
        "attention_noncausal",
        "attention_rope_causal",
        "attention_rope_noncausal",
    }
    for spec in REGISTRY.values():
        assert spec.bound == "compute"
        assert spec.compute_mode == "attention_fp16_fp32acc"
        assert torch.float16 in spec.dtypes and torch.bfloat16 in spec.dtypes
        assert spec.supports_interpreter is False
        assert tuple(spec.validation_sizes()) == (128, 512)


@pytest.mark.parametrize(
    ("overrides", "message"),
    [
        ({"name": ""}, "name"),
        ({"description": " "}, "description"),
        ({"sizes": ()}, "sizes"),
        ({"sizes": (1, 1)}, "duplicates"),
        ({"sizes": (True, 2)}, "positive integers"),
        ({"dtypes": (torch.float16, torch.float16)}, "dtypes"),
        ({"bytes_moved": None}, "bytes_moved"),
        ({"compute_mode": "fp16_fp32acc"}, "compute metadata"),
        ({"bound": "other", "bytes_moved": None}, "unsupported bound"),
        (
            {"bound": "compute", "bytes_moved": None, "flops": lambda size, dtype: size, "compute_mode": "other"},
            "unsupported compute mode",
        ),
    ],
)
def test_invalid_memory_specs_are_rejected(overrides: dict[str, object], message: str) -> None:
    with pytest.raises(ValueError, match=message):
        _memory_spec(**overrides)


def test_duplicate_registration_is_rejected() -> None:
    with pytest.raises(ValueError, match="duplicate kernel"):
        register(REGISTRY["attention_causal"])


def test_validation_sizes_default_to_benchmark_sizes() -> None:
    assert tuple(_memory_spec().validation_sizes()) == (1, 2)


def test_spec_normalizes_mutable_sequences_to_tuples() -> None:
    spec = _memory_spec(sizes=[1, 2], dtypes=[torch.float16])
    assert spec.sizes == (1, 2)
    assert spec.dtypes == (torch.float16,)
