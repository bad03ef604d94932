"""Kernel registry: the contract shared by correctness tests and benchmarks.

The field names, defaults, validation rules and error messages are kept
identical to the reference registry (``src/tklab/registry.py:16-186``) so
that code written against the reference's :class:`KernelSpec` and
``REGISTRY`` keeps working.  Only the attention entries are registered here.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from typing import Literal, TypeAlias

import torch

TensorArgs: TypeAlias = tuple[torch.Tensor, ...]
BenchmarkScalar: TypeAlias = str | int | float | bool
InputFn: TypeAlias = Callable[[int, torch.device, torch.dtype], TensorArgs]
AdversarialFn: TypeAlias = Callable[[torch.device], TensorArgs]
TensorFn: TypeAlias = Callable[..., torch.Tensor]
LaunchFn: TypeAlias = Callable[[TensorArgs, torch.Tensor], None]
OutputFn: TypeAlias = Callable[[TensorArgs], torch.Tensor]
CostFn: TypeAlias = Callable[[int, torch.dtype], int]
AssertFn: TypeAlias = Callable[[torch.Tensor, torch.Tensor], None]
BenchmarkMetadataFn: TypeAlias = Callable[[int, torch.dtype], Mapping[str, BenchmarkScalar]]
BenchmarkCall: TypeAlias = Callable[[], object]
BenchmarkCallFactory: TypeAlias = Callable[[TensorArgs, torch.Tensor], BenchmarkCall]
Bound: TypeAlias = Literal["memory", "compute"]
ComputeMode: TypeAlias = Literal["fp16_fp32acc", "fp16_fp16acc", "attention_fp16_fp32acc"]

_COMPUTE_MODES = frozenset({"fp16_fp32acc", "fp16_fp16acc", "attention_fp16_fp32acc"})


@dataclass(frozen=True, slots=True)
class KernelSpec:
    """Everything tests and benchmarks need to run, check and time one kernel.

    ``triton_fn`` keeps the reference's field name: it is the user-facing
    wrapper that allocates and returns the output (here a CUDA/C-ABI call).
    ``launch_fn`` is the allocation-free launcher the benchmark times and
    ``ref_fn`` the high-precision PyTorch reference.
    """

    name: str
    description: str
    triton_fn: TensorFn
    launch_fn: LaunchFn
    ref_fn: TensorFn
    make_inputs: InputFn
    make_output: OutputFn
    sizes: Sequence[int]
    bound: Bound
    bytes_moved: CostFn | None = None
    flops: CostFn | None = None
    dtypes: Sequence[torch.dtype] = field(default_factory=lambda: (torch.float16,))
    correctness_sizes: Sequence[int] | None = None
    make_adversarial: AdversarialFn | None = None
    naive_fn: TensorFn | None = None
    reference_launch_fn: LaunchFn | None = None
    assert_fn: AssertFn | None = None
    benchmark_metadata: BenchmarkMetadataFn | None = None
    benchmark_call_factory: BenchmarkCallFactory | None = None
    reference_call_factory: BenchmarkCallFactory | None = None
    naive_call_factory: BenchmarkCallFactory | None = None
    compute_mode: ComputeMode | None = None
    supports_interpreter: bool = True
    rtol: float | None = None
    atol: float | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "sizes", tuple(self.sizes))
        if self.correctness_sizes is not None:
            object.__setattr__(self, "correctness_sizes", tuple(self.correctness_sizes))
        object.__setattr__(self, "dtypes", tuple(self.dtypes))
        if not self.name or not self.name.isidentifier():
            raise ValueError("kernel name must be a non-empty Python identifier")
        if not self.description.strip():
            raise ValueError(f"{self.name}: description must not be empty")
        _check_sizes(self.sizes, "sizes")
        if self.correctness_sizes is not None:
            _check_sizes(self.correctness_sizes, "correctness_sizes")
        if not self.dtypes:
            raise ValueError(f"{self.name}: at least one dtype is required")
        if not all(isinstance(dtype, torch.dtype) for dtype in self.dtypes):
            raise ValueError(f"{self.name}: dtypes must contain torch.dtype values")
        if len(set(self.dtypes)) != len(self.dtypes):
            raise ValueError(f"{self.name}: dtypes must not contain duplicates")
        if self.bound == "memory":
            if self.bytes_moved is None:
                raise ValueError(f"{self.name}: memory-bound kernels require bytes_moved")
            if self.flops is not None or self.compute_mode is not None:
                raise ValueError(f"{self.name}: memory-bound kernels cannot define compute metadata")
        elif self.bound == "compute":
            if self.flops is None or self.compute_mode is None:
                raise ValueError(f"{self.name}: compute-bound kernels require flops and compute_mode")
            if self.compute_mode not in _COMPUTE_MODES:
                raise ValueError(f"{self.name}: unsupported compute mode {self.compute_mode!r}")
        else:
            raise ValueError(f"{self.name}: unsupported bound {self.bound!r}")

    def validation_sizes(self) -> Sequence[int]:
        """Sizes used by correctness tests (the benchmark sizes by default)."""
        return self.correctness_sizes or self.sizes


def _check_sizes(sizes: Sequence[int], field_name: str) -> None:
    valid = bool(sizes) and all(
        isinstance(size, int) and not isinstance(size, bool) and size > 0 for size in sizes
    )
    if not valid:
        raise ValueError(f"{field_name} must contain positive integers")
    if len(set(sizes)) != len(sizes):
        raise ValueError(f"{field_name} must not contain duplicates")


REGISTRY: dict[str, KernelSpec] = {}


def register(spec: KernelSpec) -> KernelSpec:
    """Add ``spec`` to :data:`REGISTRY`; names must be unique."""
    if spec.name in REGISTRY:
        raise ValueError(f"duplicate kernel: {spec.name}")
    REGISTRY[spec.name] = spec
    return spec
