"""Schema-7 benchmark result files and the attention roofline point on B200.

``python -m tklab.harness.results [--kernel NAME]... [--results-dir DIR]``
benchmarks the registered attention kernels with
:func:`tklab.harness.bench.bench_spec` and writes one
``<results-dir>/<gpu-slug>/<kernel>.json`` per kernel in the reference's
schema-7 layout (``src/tklab/cli.py:114-183`` ``run_benchmarks`` and
``:253-291`` ``_result_payload``), with the ceilings from
``MEASURED_PEAKS.json`` (:func:`tklab.harness.roofline.load_measured_peaks`).

It then prints the table the reference's ``benchmarks/plot_roofline.py``
prints under its figure (``:296-299``: kernel, throughput, percent of
ceiling, analytic intensity) for the flash-attention points, with the
results directory and the title taken from options instead of the
hard-coded RTX 4060 ones (``:30``, ``:290``).  The PNG itself needs
matplotlib, which this environment does not have; the JSON and the table
carry the same numbers.
"""

from __future__ import annotations

import argparse
import time
from collections.abc import Sequence
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, cast

import torch

import tklab.kernels  # noqa: F401  (registers the attention specs)
from tklab.harness.bench import BenchRow, bench_spec
from tklab.harness.jsonio import JsonObject, read_json_object, write_json_atomic
from tklab.harness.roofline import PeakResults, gpu_utilization_pct, load_measured_peaks, roofline_point
from tklab.registry import REGISTRY, KernelSpec

RESULT_SCHEMA_VERSION = 7
MAX_IDLE_GPU_UTILIZATION_PCT = 10
DEFAULT_RESULTS_DIR = Path("results")


def compute_baselines(spec: KernelSpec, peaks: PeakResults) -> tuple[float | None, float | None]:
    """(cuBLAS baseline, theoretical ceiling) for a spec's compute mode (``cli.py:234-250``)."""
    if spec.compute_mode == "fp16_fp32acc":
        return peaks["cublas_tflops_fp16_fp32acc"], peaks["theoretical_tflops_fp16_fp32acc_at_measured_clock"]
    if spec.compute_mode == "fp16_fp16acc":
        return None, peaks["theoretical_tflops_fp16_fp16acc_at_measured_clock"]
    if spec.compute_mode == "attention_fp16_fp32acc":
        return None, peaks["theoretical_tflops_fp16_fp32acc_at_measured_clock"]
    return None, None


def result_payload(
    spec: KernelSpec,
    *,
    rows: list[BenchRow],
    peaks: PeakResults,
    benchmark_started_at_utc: str,
    benchmark_preflight_gpu_utilization_pct: Sequence[int],
) -> JsonObject:
    """The versioned JSON object for one kernel (the reference's keys, in its order)."""
    payload: dict[str, Any] = {
        "schema_version": RESULT_SCHEMA_VERSION,
        "kernel": spec.name,
        "description": spec.description,
        "gpu": peaks["gpu_name"],
        "compute_capability": peaks["compute_capability"],
        "torch_version": peaks["torch_version"],
        "triton_version": peaks.get("triton_version"),
        "benchmark_started_at_utc": benchmark_started_at_utc,
        "benchmark_preflight_gpu_utilization_pct": list(benchmark_preflight_gpu_utilization_pct),
        "benchmark_preflight_gpu_utilization_limit_pct": MAX_IDLE_GPU_UTILIZATION_PCT,
        "peak_calibration_started_at_utc": peaks["calibration_started_at_utc"],
        "peak_calibration_preflight_gpu_utilization_pct": peaks["calibration_preflight_gpu_utilization_pct"],
        "peak_calibration_preflight_gpu_utilization_limit_pct": peaks[
            "calibration_preflight_gpu_utilization_limit_pct"
        ],
        "peak_bw_gbps": peaks["peak_bw_gbps"],
        "cublas_tflops_fp16_fp32acc": peaks["cublas_tflops_fp16_fp32acc"],
        "cublas_tflops_fp16_reduced_precision_allowed": peaks["cublas_tflops_fp16_reduced_precision_allowed"],
        "theoretical_tflops_fp16_fp32acc_at_measured_clock": peaks[
            "theoretical_tflops_fp16_fp32acc_at_measured_clock"
        ],
        "theoretical_tflops_fp16_fp16acc_at_measured_clock": peaks[
            "theoretical_tflops_fp16_fp16acc_at_measured_clock"
        ],
        "theoretical_ceiling_sm_clock_mhz": peaks["theoretical_ceiling_sm_clock_mhz"],
        "compute_mode": spec.compute_mode,
        "peaks_source": peaks.get("peaks_source"),
        "rows": rows,
    }
    return cast(JsonObject, payload)


def attention_bytes(row: BenchRow | dict[str, Any]) -> int:
    """Compulsory HBM bytes of one attention forward: Q, K, V read and O written once."""
    element = 2 if row["dtype"] in ("float16", "bfloat16") else 4
    return 4 * int(row.get("batch", 1)) * int(row["heads"]) * int(row["size"]) * int(row["head_dim"]) * element


def flash_roofline_rows(payload: JsonObject, *, label: str, size: int | None = None) -> list[dict[str, Any]]:
    """Roofline points for the rows of an attention result file.

    One point per dtype at ``size`` (default: the largest size in the file),
    against the file's theoretical ceiling and bandwidth.  Intensity is the
    spec's FLOP count over :func:`attention_bytes`: ``~N/s`` non-causal and
    ``~N/2s`` causal for ``s``-byte elements, the reference figure's
    ``"~N/2s @ N=4096"`` for its causal point.
    """
    rows = cast(list[dict[str, Any]], payload["rows"])
    target = size if size is not None else max(int(row["size"]) for row in rows)
    points = []
    for row in rows:
        if int(row["size"]) != target:
            continue
        flops = float(row["tflops"]) * 1e12 * float(row["ms"]) * 1e-3
        point = roofline_point(
            flops=flops,
            bytes_moved=attention_bytes(row),
            seconds=float(row["ms"]) * 1e-3,
            peak_tflops=float(payload["theoretical_tflops_fp16_fp32acc_at_measured_clock"]),
            peak_gbps=float(payload["peak_bw_gbps"]),
        )
        points.append({"kernel": f"{label} {row['dtype']}", "size": target, **point})
    return points


def print_roofline_table(points: Sequence[dict[str, Any]], *, title: str) -> None:
    """Print the figure's summary table for ``points``."""
    print(title)
    print(f"{'kernel':34s} {'throughput':16s} {'% ceiling':>9s} {'intensity':>10s} {'bound':>8s}")
    for point in points:
        throughput = f"{point['achieved_tflops']:.1f} TFLOP/s"
        print(
            f"{point['kernel']:34s} {throughput:16s} {point['pct_attainable']:8.1f}% "
            f"{point['intensity_flop_per_byte']:10.1f} {point['bound']:>8s}"
        )


def _utilization_samples(device: int, count: int = 5, interval_s: float = 1.0) -> tuple[int, ...]:
    """Whole-device utilization sampled before benchmarking (``cli.py:215-231``)."""
    samples = []
    for index in range(count):
        samples.append(gpu_utilization_pct(device))
        if index + 1 < count:
            time.sleep(interval_s)
    return tuple(samples)


def run(
    kernels: Sequence[str],
    *,
    results_dir: Path,
    device: int = 0,
    warmup_ms: int = 25,
    repetition_ms: int = 100,
    sizes: Sequence[int] | None = None,
    allow_busy_gpu: bool = False,
    peaks_path: Path | None = None,
) -> dict[str, Path]:
    """Benchmark ``kernels`` and write their result files; returns name -> path.

    Raises:
        RuntimeError: If CUDA is unavailable or the GPU is busy (unless allowed).
        ValueError: If a kernel name is not registered.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for benchmarks")
    unknown = sorted(set(kernels) - set(REGISTRY))
    if unknown:
        raise ValueError(f"unknown kernel(s): {', '.join(unknown)}")
    started = datetime.now(timezone.utc).isoformat()
    utilization = _utilization_samples(device)
    if not allow_busy_gpu and max(utilization) > MAX_IDLE_GPU_UTILIZATION_PCT:
        raise RuntimeError(
            f"GPU {device} reached {max(utilization)}% utilization during preflight; "
            "close GPU workloads or pass --allow-busy-gpu to accept contaminated results"
        )
    peaks = load_measured_peaks(peaks_path, device=device)
    out_dir = results_dir / peaks["gpu_slug"]
    written: dict[str, Path] = {}
    for name in kernels:
        spec = REGISTRY[name]
        cublas_tflops, theoretical_tflops = compute_baselines(spec, peaks)
        rows = bench_spec(
            spec,
            peak_bw_gbps=peaks["peak_bw_gbps"],
            cublas_tflops=cublas_tflops,
            theoretical_tflops=theoretical_tflops,
            device=device,
            warmup_ms=warmup_ms,
            repetition_ms=repetition_ms,
            sizes=sizes,
        )
        path = out_dir / f"{name}.json"
        write_json_atomic(
            path,
            result_payload(
                spec,
                rows=rows,
                peaks=peaks,
                benchmark_started_at_utc=started,
                benchmark_preflight_gpu_utilization_pct=utilization,
            ),
        )
        written[name] = path
    return written


def main(argv: Sequence[str] | None = None) -> int:
    """Command-line entry point."""
    parser = argparse.ArgumentParser(prog="python -m tklab.harness.results", description=__doc__.split("\n")[0])
    parser.add_argument("--kernel", action="append", dest="kernels", choices=sorted(REGISTRY))
    parser.add_argument("--results-dir", type=Path, default=DEFAULT_RESULTS_DIR)
    parser.add_argument("--title", default=None, help="title of the roofline table (default: from the GPU)")
    parser.add_argument("--size", type=int, action="append", dest="sizes", help="restrict to these sizes")
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--warmup-ms", type=int, default=25)
    parser.add_argument("--repetition-ms", type=int, default=100)
    parser.add_argument("--allow-busy-gpu", action="store_true")
    parser.add_argument("--peaks", type=Path, default=None, help="MEASURED_PEAKS.json to use")
    parser.add_argument("--table-only", action="store_true", help="print the table from existing result files")
    options = parser.parse_args(argv)
    kernels = options.kernels or ["attention_noncausal", "attention_causal"]
    if options.table_only:
        paths = {}
        for name in kernels:
            matches = sorted(options.results_dir.glob(f"*/{name}.json"))
            if not matches:
                raise FileNotFoundError(f"no result file for {name} under {options.results_dir}")
            paths[name] = matches[-1]
    else:
        paths = run(
            kernels,
            results_dir=options.results_dir,
            device=options.device,
            warmup_ms=options.warmup_ms,
            repetition_ms=options.repetition_ms,
            sizes=options.sizes,
            allow_busy_gpu=options.allow_busy_gpu,
            peaks_path=options.peaks,
        )
    points: list[dict[str, Any]] = []
    gpu = ""
    for name, path in paths.items():
        payload = read_json_object(path)
        gpu = str(payload["gpu"])
        print(f"wrote {path}" if not options.table_only else f"read {path}")
        points.extend(flash_roofline_rows(payload, label=name.replace("attention_", "flash_attn ")))
    print_roofline_table(points, title=options.title or f"triton-kernel-lab — roofline ({gpu})")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
