"""Schema-7 benchmark result files and the attention roofline table on B200.

The result payload (``result_payload``) and the baseline choice
(``compute_baselines``) are the reference's ``src/tklab/cli.py:253-291`` and
``:234-250``; ``tklab.cli`` (the reference's ``tklab-bench`` entry point)
writes the files with them.

``python -m tklab.harness.results [--kernel NAME]... [--results-dir DIR]
[--title TITLE] [--table-only]`` runs that benchmark (unless
``--table-only``) and prints the table the reference's
``benchmarks/plot_roofline.py`` prints under its figure (``:296-299``:
kernel, throughput, percent of ceiling, analytic intensity) for the
flash-attention points, with the results directory and the title taken
from options instead of the hard-coded RTX 4060 ones (``:30``, ``:290``).
The PNG itself needs matplotlib, which this environment does not have; the
JSON and the table carry the same numbers.
"""

from __future__ import annotations

import argparse
from collections.abc import Sequence
from pathlib import Path
from typing import Any, cast

import tklab.kernels  # noqa: F401  (registers the attention specs)
from tklab.harness.bench import BenchRow
from tklab.harness.jsonio import JsonObject, read_json_object
from tklab.harness.roofline import PeakResults, roofline_point
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
    parser.add_argument("--peaks", type=Path, default=None, help="peak-measurement JSON to take the ceilings from")
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
        from tklab.cli import BenchmarkOptions, run_benchmarks

        payloads = run_benchmarks(
            BenchmarkOptions(
                device=options.device,
                force_peaks=False,
                kernels=tuple(kernels),
                warmup_ms=options.warmup_ms,
                repetition_ms=options.repetition_ms,
                list_kernels=False,
                allow_busy_gpu=options.allow_busy_gpu,
                results_dir=options.results_dir,
                peaks=options.peaks,
                sizes=tuple(options.sizes) if options.sizes else None,
            )
        )
        paths = {name: payload["path"] for name, payload in payloads.items()}
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
