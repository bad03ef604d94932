"""Command-line interface for the registered attention benchmarks (``tklab-bench``).

Mirrors the reference's ``src/tklab/cli.py`` so that its
``benchmarks/run.py`` (``from tklab.cli import main``) runs unchanged on
this package: the same options (``parse_args``, ``:45-103``), the same GPU
preflight (``:127-135``, ``:215-231``), the same peak handling
(``load_or_measure_peaks``, ``:137-146``), one ``bench_spec`` pass per
selected kernel (``:150-160``) and the same schema-7 result file per kernel
at ``<results>/<gpu-slug>/<kernel>.json`` (``:162-172``, ``:253-291``).

Differences, each additive: ``--results-dir`` (default: the checkout's
``results/``, as the reference), ``--peaks`` to take the empirical ceilings
from a measurement file (otherwise ``TKLAB_MEASURED_PEAKS``, otherwise a
live measurement), and ``--size`` to restrict the sweep.  The speedup and
throughput PNGs need matplotlib; without it they are skipped with a note
and the JSON carries the numbers.
"""

from __future__ import annotations

import argparse
import importlib.util
import time
from dataclasses import dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

import torch

import tklab.kernels  # noqa: F401  (registers the attention specs)
from tklab.harness.bench import BenchRow, bench_spec
from tklab.harness.jsonio import write_json_atomic
from tklab.harness.results import MAX_IDLE_GPU_UTILIZATION_PCT, compute_baselines, result_payload
from tklab.harness.roofline import PeakResults, gpu_utilization_pct, load_or_measure_peaks
from tklab.registry import REGISTRY, KernelSpec

GPU_PREFLIGHT_SAMPLE_COUNT = 5
GPU_PREFLIGHT_INTERVAL_SECONDS = 1.0


@dataclass(frozen=True, slots=True)
class BenchmarkOptions:
    """Validated command-line benchmark options (the reference's fields, then the additions)."""

    device: int
    force_peaks: bool
    kernels: tuple[str, ...] | None
    warmup_ms: int
    repetition_ms: int
    list_kernels: bool
    allow_busy_gpu: bool
    results_dir: Path | None = None
    peaks: Path | None = None
    sizes: tuple[int, ...] | None = None


def parse_args(argv: list[str] | None = None) -> BenchmarkOptions:
    """Parse benchmark CLI arguments (``None`` reads ``sys.argv``)."""
    parser = argparse.ArgumentParser(
        prog="tklab-bench",
        description="Benchmark the registered attention kernels and write JSON results.",
    )
    parser.add_argument("--device", type=int, default=0, help="CUDA device index.")
    parser.add_argument("--force-peaks", action="store_true", help="Re-obtain the roofline ceilings.")
    parser.add_argument(
        "--kernel",
        action="append",
        dest="kernels",
        choices=sorted(REGISTRY),
        help="Kernel to benchmark. Repeat the option to select multiple kernels.",
    )
    parser.add_argument("--warmup-ms", type=int, default=25, help="Approximate warmup duration per observation.")
    parser.add_argument(
        "--repetition-ms", type=int, default=100, help="Approximate measurement duration per observation."
    )
    parser.add_argument("--list-kernels", action="store_true", help="Print registered kernels and exit.")
    parser.add_argument(
        "--allow-busy-gpu",
        action="store_true",
        help="Run despite pre-existing GPU utilization above 10%%.",
    )
    parser.add_argument("--results-dir", type=Path, default=None, help="Results root (default: <checkout>/results).")
    parser.add_argument("--peaks", type=Path, default=None, help="Peak-measurement JSON to take the ceilings from.")
    parser.add_argument("--size", type=int, action="append", dest="sizes", help="Restrict the sweep to these sizes.")
    namespace = parser.parse_args(argv)
    return BenchmarkOptions(
        device=namespace.device,
        force_peaks=namespace.force_peaks,
        kernels=tuple(namespace.kernels) if namespace.kernels else None,
        warmup_ms=namespace.warmup_ms,
        repetition_ms=namespace.repetition_ms,
        list_kernels=namespace.list_kernels,
        allow_busy_gpu=namespace.allow_busy_gpu,
        results_dir=namespace.results_dir,
        peaks=namespace.peaks,
        sizes=tuple(namespace.sizes) if namespace.sizes else None,
    )


def run_benchmarks(options: BenchmarkOptions, *, project_root: Path | None = None) -> dict[str, dict[str, Any]]:
    """Execute the selected benchmarks and write their result files.

    Returns:
        Mapping from kernel name to its payload (``{"rows": [...]}``, as the
        reference's plot payload) plus ``"path"``, the result file written.

    Raises:
        RuntimeError: If CUDA is unavailable or the GPU is busy (unless allowed).
        ValueError: If no selected kernel exists.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for benchmarks")
    started = datetime.now(timezone.utc).isoformat()
    utilization = _gpu_utilization_samples(options.device)
    maximum = max(utilization)
    print(f"preflight GPU utilization: {','.join(str(value) for value in utilization)}%")
    if not options.allow_busy_gpu and maximum > MAX_IDLE_GPU_UTILIZATION_PCT:
        raise RuntimeError(
            f"GPU {options.device} reached {maximum}% utilization during preflight; "
            "close GPU workloads or pass --allow-busy-gpu to accept contaminated results"
        )
    specs = _select_specs(options.kernels)
    root = project_root or Path(__file__).resolve().parents[2]
    results_root = options.results_dir or root / "results"
    peaks, peaks_path = load_or_measure_peaks(
        results_root,
        device=options.device,
        force=options.force_peaks,
        measured_peaks_path=options.peaks,
        calibration_started_at_utc=started,
        calibration_preflight_gpu_utilization_pct=utilization,
        calibration_preflight_gpu_utilization_limit_pct=MAX_IDLE_GPU_UTILIZATION_PCT,
    )
    output_dir = peaks_path.parent
    _print_peak_summary(peaks, path=peaks_path)
    payloads: dict[str, dict[str, Any]] = {}
    for spec in specs:
        cublas_tflops, theoretical_tflops = compute_baselines(spec, peaks)
        rows = bench_spec(
            spec,
            peak_bw_gbps=peaks["peak_bw_gbps"],
            cublas_tflops=cublas_tflops,
            theoretical_tflops=theoretical_tflops,
            device=options.device,
            warmup_ms=options.warmup_ms,
            repetition_ms=options.repetition_ms,
            sizes=options.sizes,
        )
        output_path = output_dir / f"{spec.name}.json"
        write_json_atomic(
            output_path,
            result_payload(
                spec,
                rows=rows,
                peaks=peaks,
                benchmark_started_at_utc=started,
                benchmark_preflight_gpu_utilization_pct=utilization,
            ),
        )
        payloads[spec.name] = {"rows": rows, "path": output_path}
        _print_result_summary(spec, rows=rows, output_path=output_path, has_cublas_baseline=cublas_tflops is not None)
    return payloads


def main(argv: list[str] | None = None) -> int:
    """Run the benchmark CLI; returns the process exit status."""
    options = parse_args(argv)
    if options.list_kernels:
        for spec in REGISTRY.values():
            print(f"{spec.name}: {spec.description}")
        return 0
    run_benchmarks(options)
    return 0


def _select_specs(kernel_names: tuple[str, ...] | None) -> list[KernelSpec]:
    """Resolve selected kernel names in registry order."""
    if kernel_names is None:
        return list(REGISTRY.values())
    names = set(kernel_names)
    specs = [spec for spec in REGISTRY.values() if spec.name in names]
    if not specs:
        raise ValueError("no kernels selected")
    return specs


def _gpu_utilization_samples(
    device: int,
    *,
    sample_count: int = GPU_PREFLIGHT_SAMPLE_COUNT,
    interval_seconds: float = GPU_PREFLIGHT_INTERVAL_SECONDS,
) -> tuple[int, ...]:
    """Sample whole-device utilization repeatedly before benchmarking."""
    if sample_count <= 0:
        raise ValueError("GPU preflight sample count must be positive")
    if interval_seconds < 0:
        raise ValueError("GPU preflight interval must be non-negative")
    samples: list[int] = []
    for index in range(sample_count):
        samples.append(gpu_utilization_pct(device))
        if index + 1 < sample_count:
            time.sleep(interval_seconds)
    return tuple(samples)


def _print_peak_summary(peaks: PeakResults, *, path: Path) -> None:
    print(f"peaks: {path}")
    print(f"measured bandwidth peak: {peaks['peak_bw_gbps']:.3f} GB/s")
    print(f"measured cuBLAS FP16/FP32-acc baseline: {peaks['cublas_tflops_fp16_fp32acc']:.3f} TFLOP/s")
    print(
        "maximum-observed-clock theoretical FP16/FP32-acc: "
        f"{peaks['theoretical_tflops_fp16_fp32acc_at_measured_clock']:.3f} TFLOP/s"
    )
    print(
        "maximum-observed-clock theoretical FP16/FP16-acc: "
        f"{peaks['theoretical_tflops_fp16_fp16acc_at_measured_clock']:.3f} TFLOP/s"
    )
    print(f"theoretical ceiling clock: {peaks['theoretical_ceiling_sm_clock_mhz']} MHz")


def _print_result_summary(
    spec: KernelSpec, *, rows: list[BenchRow], output_path: Path, has_cublas_baseline: bool
) -> None:
    if spec.bound == "memory":
        key, baseline_name = "pct_peak", "bandwidth peak"
    elif has_cublas_baseline:
        key, baseline_name = "pct_cublas_same_size", "same-size cuBLAS"
    else:
        key, baseline_name = "pct_theoretical", "theoretical"
    best = max(rows, key=lambda row: float(row.get(key, 0.0)))
    performance = best.get("gbps", best.get("tflops", 0.0))
    print(f"results: {output_path}")
    if importlib.util.find_spec("matplotlib") is None:
        print("plots: skipped (matplotlib is not installed; the JSON carries the numbers)")
    print(f"best {spec.name}: {float(best.get(key, 0.0)):.2f}% {baseline_name} ({performance:.3f})")


if __name__ == "__main__":
    raise SystemExit(main())
