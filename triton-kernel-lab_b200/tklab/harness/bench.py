"""Benchmark rows for registered kernels, in the reference's row format.

Mirrors the reference's ``src/tklab/harness/bench.py``: ``bench_spec``
(``:52-155``) times every (dtype, size) of a :class:`KernelSpec` — median
with 20th/80th percentiles — times the PyTorch reference the same way
(``:158-181``), merges the spec's tile metadata and adds the roofline
metrics (``:184-219``), validating its request with the same messages
(``:222-243``).  The reference times with ``triton.testing.do_bench``; this
package has no Triton dependency, so :func:`do_bench` is its own CUDA-event
timer with the same warm-up / repetition budget semantics and an L2 flush
before every timed call.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable, Sequence
from functools import partial
from typing import NotRequired, TypedDict, cast

import torch

from tklab.registry import KernelSpec

_L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


class BenchRow(TypedDict):
    """One serialized benchmark observation (the reference's keys)."""

    kernel: str
    dtype: str
    size: int
    ms: float
    ms_lo: float
    ms_hi: float
    torch_ms: float
    speedup: float
    gbps: NotRequired[float]
    tflops: NotRequired[float]
    pct_peak: NotRequired[float]
    naive_ms: NotRequired[float]
    speedup_vs_naive: NotRequired[float]
    reference_tflops: NotRequired[float]
    pct_cublas_same_size: NotRequired[float]
    pct_cublas_peak: NotRequired[float]
    pct_theoretical: NotRequired[float]
    block_m: NotRequired[int]
    block_n: NotRequired[int]
    num_warps: NotRequired[int]
    num_stages: NotRequired[int]
    heads: NotRequired[int]
    head_dim: NotRequired[int]
    causal: NotRequired[bool]


def do_bench(
    fn: Callable[[], object],
    *,
    warmup_ms: float = 25,
    repetition_ms: float = 100,
    quantiles: Sequence[float] | None = None,
) -> float | list[float]:
    """Time ``fn`` on the current CUDA stream.

    A first estimate from five calls sizes the warm-up and the timed
    repetitions to about ``warmup_ms`` and ``repetition_ms``; every timed
    call is preceded by a 256 MiB write that evicts L2 and is bracketed by
    its own CUDA events.  Returns the median in milliseconds, or the
    requested quantiles (linear interpolation) when ``quantiles`` is given.
    """
    flush = torch.empty(_L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(5):
        flush.zero_()
        fn()
    end.record()
    torch.cuda.synchronize()
    estimate = max(start.elapsed_time(end) / 5, 1e-3)
    n_warmup = max(1, int(warmup_ms / estimate))
    n_repeat = max(1, int(repetition_ms / estimate))
    for _ in range(n_warmup):
        fn()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_repeat)]
    for begin, finish in events:
        flush.zero_()
        begin.record()
        fn()
        finish.record()
    torch.cuda.synchronize()
    times = sorted(begin.elapsed_time(finish) for begin, finish in events)
    if quantiles is None:
        return float(statistics.median(times))
    return [_quantile(times, q) for q in quantiles]


def _quantile(sorted_times: Sequence[float], q: float) -> float:
    """Linear-interpolation quantile of an ascending sequence."""
    if not 0.0 <= q <= 1.0:
        raise ValueError("quantiles must lie in [0, 1]")
    position = q * (len(sorted_times) - 1)
    low = int(position)
    high = min(low + 1, len(sorted_times) - 1)
    return float(sorted_times[low] + (sorted_times[high] - sorted_times[low]) * (position - low))


def bench_spec(
    spec: KernelSpec,
    *,
    peak_bw_gbps: float | None,
    cublas_tflops: float | None,
    theoretical_tflops: float | None,
    device: int = 0,
    warmup_ms: int = 25,
    repetition_ms: int = 100,
    sizes: Sequence[int] | None = None,
    dtypes: Sequence[torch.dtype] | None = None,
) -> list[BenchRow]:
    """Benchmark every dtype and size of ``spec`` (or the given subsets).

    Raises:
        ValueError: If timing parameters or required baselines are invalid.
        RuntimeError: If the selected CUDA device is unavailable.
    """
    _validate_benchmark_request(device=device, warmup_ms=warmup_ms, repetition_ms=repetition_ms)
    rows: list[BenchRow] = []
    torch_device = torch.device("cuda", device)
    with torch.cuda.device(device):
        for dtype in dtypes or spec.dtypes:
            for size in sizes or spec.sizes:
                args = spec.make_inputs(size, torch_device, dtype)
                output = spec.make_output(args)
                launch = (
                    spec.benchmark_call_factory(args, output)
                    if spec.benchmark_call_factory is not None
                    else partial(spec.launch_fn, args, output)
                )
                median_ms, low_ms, high_ms = cast(
                    list[float],
                    do_bench(launch, quantiles=[0.5, 0.2, 0.8], warmup_ms=warmup_ms, repetition_ms=repetition_ms),
                )
                torch_ms = _benchmark_reference(
                    spec, args=args, output=output, warmup_ms=warmup_ms, repetition_ms=repetition_ms
                )
                row: BenchRow = {
                    "kernel": spec.name,
                    "dtype": str(dtype).removeprefix("torch."),
                    "size": size,
                    "ms": median_ms,
                    "ms_lo": low_ms,
                    "ms_hi": high_ms,
                    "torch_ms": torch_ms,
                    "speedup": torch_ms / median_ms,
                }
                if spec.benchmark_metadata is not None:
                    row.update(cast(BenchRow, dict(spec.benchmark_metadata(size, dtype))))
                naive_call: Callable[[], object] | None = None
                if spec.naive_call_factory is not None:
                    naive_call = spec.naive_call_factory(args, output)
                elif spec.naive_fn is not None:
                    naive_call = partial(spec.naive_fn, *args)
                if naive_call is not None:
                    naive_ms = cast(float, do_bench(naive_call, warmup_ms=warmup_ms, repetition_ms=repetition_ms))
                    row["naive_ms"] = naive_ms
                    row["speedup_vs_naive"] = naive_ms / median_ms
                _add_performance_metrics(
                    row,
                    spec=spec,
                    size=size,
                    dtype=dtype,
                    milliseconds=median_ms,
                    peak_bw_gbps=peak_bw_gbps,
                    cublas_tflops=cublas_tflops,
                    theoretical_tflops=theoretical_tflops,
                )
                rows.append(row)
                del args, output
    return rows


def _benchmark_reference(
    spec: KernelSpec,
    *,
    args: tuple[torch.Tensor, ...],
    output: torch.Tensor,
    warmup_ms: int,
    repetition_ms: int,
) -> float:
    """Median time of the PyTorch reference, allocation-free when the spec allows."""
    reference_call: Callable[[], object]
    if spec.reference_call_factory is not None:
        reference_call = spec.reference_call_factory(args, output)
    elif spec.reference_launch_fn is not None:
        reference_call = partial(spec.reference_launch_fn, args, output)
    else:
        reference_call = partial(spec.ref_fn, *args)
    return cast(float, do_bench(reference_call, warmup_ms=warmup_ms, repetition_ms=repetition_ms))


def _add_performance_metrics(
    row: BenchRow,
    *,
    spec: KernelSpec,
    size: int,
    dtype: torch.dtype,
    milliseconds: float,
    peak_bw_gbps: float | None,
    cublas_tflops: float | None,
    theoretical_tflops: float | None,
) -> None:
    """Add the roofline metrics of one row.

    Raises:
        ValueError: If the spec lacks its cost model or the needed baseline.
    """
    seconds = milliseconds * 1e-3
    if spec.bound == "memory":
        if spec.bytes_moved is None or peak_bw_gbps is None:
            raise ValueError(f"{spec.name}: missing memory cost model or bandwidth peak")
        gigabytes_per_second = spec.bytes_moved(size, dtype) / seconds / 1e9
        row["gbps"] = gigabytes_per_second
        row["pct_peak"] = 100.0 * gigabytes_per_second / peak_bw_gbps
        return
    if spec.flops is None or theoretical_tflops is None:
        raise ValueError(f"{spec.name}: missing compute cost model or theoretical peak")
    teraflops = spec.flops(size, dtype) / seconds / 1e12
    reference_teraflops = spec.flops(size, dtype) / (row["torch_ms"] * 1e-3) / 1e12
    row["tflops"] = teraflops
    row["reference_tflops"] = reference_teraflops
    row["pct_theoretical"] = 100.0 * teraflops / theoretical_tflops
    if cublas_tflops is not None:
        row["pct_cublas_same_size"] = 100.0 * teraflops / reference_teraflops
        row["pct_cublas_peak"] = 100.0 * teraflops / cublas_tflops


def _validate_benchmark_request(*, device: int, warmup_ms: int, repetition_ms: int) -> None:
    """Validate timing parameters and the device (the reference's messages).

    Raises:
        ValueError: If a parameter is negative or zero.
        RuntimeError: If CUDA or the device is unavailable.
    """
    if device < 0:
        raise ValueError("device index must be non-negative")
    if warmup_ms <= 0 or repetition_ms <= 0:
        raise ValueError("warmup and repetition durations must be positive")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for GPU benchmarks")
    if device >= torch.cuda.device_count():
        raise RuntimeError(f"CUDA device {device} is unavailable; found {torch.cuda.device_count()} device(s)")
