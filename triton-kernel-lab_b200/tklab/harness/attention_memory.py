"""Peak device memory of flash attention against materialized attention.

``python -m tklab.harness.attention_memory [--size N]... [--out FILE]`` is the
B200 rerun of the reference's ``benchmarks/flash_attention_memory.py``: for
each sequence length, one fresh worker process per implementation measures
the peak CUDA allocation of one non-causal forward (B=1, H=16, D=64,
float16: the reference's configuration, ``:22-26``) above the inputs, so an
out-of-memory in the quadratic path cannot disturb the next point
(``:74-145``).  The study records the log-log slope of memory against
sequence length from the first and last successful points (``:163-180``;
~1 for flash attention, ~2 for the materialized scores and probabilities),
the bytes the two quadratic fp16 buffers take per N² and the sequence length
at which they alone would fill the device (``:183-191``), and writes the
schema-1 JSON object of ``:226-268``.  The reference's PNG needs matplotlib,
absent here; the JSON carries the numbers.
"""

from __future__ import annotations

import argparse
import json
import math
import platform
import subprocess
import sys
from collections.abc import Sequence
from pathlib import Path
from typing import Any, TypedDict, cast

import torch

DEFAULT_SIZES = (512, 1024, 2048, 4096, 8192, 12288, 16384, 24576, 32768, 65536)
BATCH = 1
HEADS = 16
HEAD_DIM = 64
DTYPE = torch.float16
IMPLEMENTATIONS = ("flash", "materialized")


class WorkerResult(TypedDict):
    """One isolated-process measurement (the reference's keys)."""

    implementation: str
    sequence_length: int
    baseline_allocated_bytes: int
    peak_allocated_bytes: int | None
    peak_increment_bytes: int | None
    output_finite: bool | None
    oom: bool
    error: str | None


def materialized_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Attention that keeps the N x N scores and probabilities alive."""
    scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(q.shape[-1]))
    probabilities = torch.softmax(scores, dim=-1)
    return torch.matmul(probabilities, v)


def worker(implementation: str, sequence_length: int, device: int) -> WorkerResult:
    """Measure one implementation at one length in this (fresh) process."""
    from tklab.kernels.flash_attention import attention_noncausal

    torch.cuda.set_device(device)
    torch.manual_seed(31)
    shape = (BATCH, HEADS, sequence_length, HEAD_DIM)
    q, k, v = (torch.randn(shape, device="cuda", dtype=DTYPE) for _ in range(3))
    if implementation == "flash":
        # Load the library and build the tensor maps once before measuring.
        del_me = attention_noncausal(q, k, v)
        torch.cuda.synchronize()
        del del_me
    torch.cuda.synchronize()
    baseline = torch.cuda.memory_allocated(device)
    torch.cuda.reset_peak_memory_stats(device)
    try:
        output = attention_noncausal(q, k, v) if implementation == "flash" else materialized_attention(q, k, v)
        torch.cuda.synchronize()
        peak = torch.cuda.max_memory_allocated(device)
        return {
            "implementation": implementation,
            "sequence_length": sequence_length,
            "baseline_allocated_bytes": baseline,
            "peak_allocated_bytes": peak,
            "peak_increment_bytes": peak - baseline,
            "output_finite": bool(torch.isfinite(output).all().item()),
            "oom": False,
            "error": None,
        }
    except torch.OutOfMemoryError as error:
        return {
            "implementation": implementation,
            "sequence_length": sequence_length,
            "baseline_allocated_bytes": baseline,
            "peak_allocated_bytes": None,
            "peak_increment_bytes": None,
            "output_finite": None,
            "oom": True,
            "error": type(error).__name__,
        }


def run_worker(implementation: str, sequence_length: int, device: int, *, timeout_s: int = 600) -> WorkerResult:
    """Run :func:`worker` in a child interpreter and parse its last stdout line."""
    completed = subprocess.run(
        [
            sys.executable,
            "-m",
            "tklab.harness.attention_memory",
            "--worker",
            "--implementation",
            implementation,
            "--worker-size",
            str(sequence_length),
            "--device",
            str(device),
        ],
        check=True,
        capture_output=True,
        text=True,
        timeout=timeout_s,
        cwd=Path(__file__).resolve().parents[2],
    )
    return cast(WorkerResult, json.loads(completed.stdout.strip().splitlines()[-1]))


def empirical_slope(rows: Sequence[WorkerResult]) -> float | None:
    """log(memory ratio) / log(length ratio) between the first and last successful rows."""
    ok = [row for row in rows if not row["oom"] and row["peak_increment_bytes"]]
    if len(ok) < 2:
        return None
    first, last = ok[0], ok[-1]
    return math.log(cast(int, last["peak_increment_bytes"]) / cast(int, first["peak_increment_bytes"])) / math.log(
        last["sequence_length"] / first["sequence_length"]
    )


def quadratic_bytes_per_n_squared() -> int:
    """Bytes per N² of the two fp16 N x N buffers the materialized path keeps."""
    return 2 * BATCH * HEADS * torch.empty((), dtype=DTYPE).element_size()


def dedicated_memory_crossing(total_memory_bytes: int) -> float:
    """Sequence length at which the two quadratic buffers alone fill the device."""
    if total_memory_bytes <= 0:
        raise ValueError("total_memory_bytes must be positive")
    return math.sqrt(total_memory_bytes / quadratic_bytes_per_n_squared())


def study_payload(
    measurements: Sequence[WorkerResult],
    *,
    gpu: str,
    compute_capability: str,
    total_memory_bytes: int,
    driver: dict[str, Any],
) -> dict[str, Any]:
    """The schema-1 study object."""
    by_impl = {name: [row for row in measurements if row["implementation"] == name] for name in IMPLEMENTATIONS}
    return {
        "schema_version": 1,
        "study": "flash_attention_memory",
        "gpu": gpu,
        "compute_capability": compute_capability,
        "torch_version": torch.__version__,
        "triton_version": None,
        "platform": {
            "system": platform.system(),
            "release": platform.release(),
            "is_wsl": "microsoft" in platform.release().lower(),
            **driver,
            "torch_device_total_memory_bytes": total_memory_bytes,
        },
        "batch": BATCH,
        "heads": HEADS,
        "head_dim": HEAD_DIM,
        "dtype": str(DTYPE).removeprefix("torch."),
        "measurements": list(measurements),
        "empirical_log_log_slope": {name: empirical_slope(rows) for name, rows in by_impl.items()},
        "analytical_context": {
            "materialized_quadratic_buffers": 2,
            "quadratic_element_dtype": str(DTYPE).removeprefix("torch."),
            "quadratic_bytes_per_n_squared": quadratic_bytes_per_n_squared(),
            "quadratic_only_dedicated_memory_crossing_sequence_length": dedicated_memory_crossing(total_memory_bytes),
        },
    }


def _driver_metadata(device: int) -> dict[str, Any]:
    """Driver version and reported memory from ``nvidia-smi`` (empty if unavailable)."""
    try:
        completed = subprocess.run(
            ["nvidia-smi", f"--id={device}", "--query-gpu=driver_version,memory.total", "--format=csv,noheader,nounits"],
            check=True,
            capture_output=True,
            text=True,
            timeout=30,
        )
        version, memory_mib = (field.strip() for field in completed.stdout.strip().split(","))
        return {"driver_version": version, "reported_dedicated_memory_mib": int(memory_mib)}
    except (FileNotFoundError, subprocess.CalledProcessError, subprocess.TimeoutExpired, ValueError):
        return {}


def main(argv: Sequence[str] | None = None) -> int:
    """Run the workers and write the study JSON."""
    parser = argparse.ArgumentParser(prog="python -m tklab.harness.attention_memory", description=__doc__.split("\n")[0])
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--size", type=int, action="append", dest="sizes")
    parser.add_argument("--out", type=Path, default=None, help="study JSON (default: results/<gpu-slug>/...)")
    parser.add_argument("--worker", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--implementation", choices=IMPLEMENTATIONS, help=argparse.SUPPRESS)
    parser.add_argument("--worker-size", type=int, help=argparse.SUPPRESS)
    options = parser.parse_args(argv)
    if options.worker:
        if options.implementation is None or options.worker_size is None:
            raise ValueError("worker mode requires implementation and size")
        print(json.dumps(worker(options.implementation, options.worker_size, options.device), separators=(",", ":")))
        return 0
    from tklab.harness.jsonio import write_json_atomic
    from tklab.harness.roofline import slug_for_name

    sizes = tuple(options.sizes or DEFAULT_SIZES)
    if any(size <= 0 for size in sizes):
        raise ValueError("sequence lengths must be positive")
    total_memory = torch.cuda.get_device_properties(options.device).total_memory
    measurements: list[WorkerResult] = []
    for implementation in IMPLEMENTATIONS:
        for size in sizes:
            if implementation == "materialized" and quadratic_bytes_per_n_squared() * size * size > total_memory // 2:
                # Not attempted: on a shared machine the sweep stays well
                # inside device memory instead of probing for the OOM point.
                result: WorkerResult = {
                    "implementation": implementation,
                    "sequence_length": size,
                    "baseline_allocated_bytes": 0,
                    "peak_allocated_bytes": None,
                    "peak_increment_bytes": None,
                    "output_finite": None,
                    "oom": False,
                    "error": "not run: the two N x N buffers would exceed half of device memory",
                }
                measurements.append(result)
                print(f"{implementation} N={size}: not run (quadratic buffers > half of device memory)", flush=True)
                continue
            result = run_worker(implementation, size, options.device)
            measurements.append(result)
            status = "OOM" if result["oom"] else f"{cast(int, result['peak_increment_bytes']) / 2**20:.2f} MiB"
            print(f"{implementation} N={size}: {status}", flush=True)
    gpu = torch.cuda.get_device_name(options.device)
    major, minor = torch.cuda.get_device_capability(options.device)
    payload = study_payload(
        measurements,
        gpu=gpu,
        compute_capability=f"{major}.{minor}",
        total_memory_bytes=total_memory,
        driver=_driver_metadata(options.device),
    )
    out = options.out or Path("results") / slug_for_name(gpu) / "flash_attention_memory.json"
    write_json_atomic(out, payload)
    print(f"slopes: {payload['empirical_log_log_slope']}; wrote {out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
