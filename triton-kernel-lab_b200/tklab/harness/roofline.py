"""Roofline ceilings for the attention benchmarks, with a B200 profile.

Follows the parts of the reference's ``src/tklab/harness/roofline.py`` that
the attention benchmark rows and the roofline figure consume:

* :class:`GpuTheoreticalProfile` (``:39-62``) and the audited profile table
  (``:64-73``) with the lookup that refuses unknown GPUs (``:609-621``).
  The reference table only knows its RTX 4060; this one adds B200.  The
  reference derives the FP16-accumulate ceiling as twice the
  FP32-accumulate one, which is a GeForce property; data-center Blackwell
  runs both at the same rate, so the profile carries that ratio.
* The schema-7 peak payload (``PeakResults``, ``:110-144``) that result files
  embed, and :func:`load_or_measure_peaks` (``:354-405``): a compatible
  ``<results>/<gpu-slug>/peaks.json`` is reused; otherwise the ceilings come
  from a measurement file named explicitly (argument, or the
  ``TKLAB_MEASURED_PEAKS`` environment variable: a device-copy bandwidth and
  a cuBLAS bf16 GEMM rate measured on the same machines) or are measured
  live (:func:`measure_peaks`), then written to ``peaks.json``.
"""

from __future__ import annotations

import os
import re
import subprocess
import threading
import time
from collections.abc import Mapping
from dataclasses import dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, TypedDict, cast

import torch

from tklab.harness.jsonio import JsonObject, read_json_object, write_json_atomic

PEAKS_SCHEMA_VERSION = 7
MEASURED_PEAKS_ENV = "TKLAB_MEASURED_PEAKS"


@dataclass(frozen=True, slots=True)
class GpuTheoreticalProfile:
    """Hardware facts from which clock-scaled tensor-core ceilings follow.

    ``fp16acc_rate_multiplier`` is how much faster FP16-accumulate MMAs run
    than FP32-accumulate ones (2 on GeForce Ada, 1 on B200).
    """

    model_substring: str
    rated_boost_mhz: int
    streaming_multiprocessors: int
    tensor_cores_per_sm: int
    fp16_fp32acc_flops_per_clock_per_tensor_core: int
    product_spec_url: str
    architecture_whitepaper_url: str
    fp16acc_rate_multiplier: float = 2.0

    def fp16_fp32acc_tflops(self, clock_mhz: int) -> float:
        """Dense FP16-input / FP32-accumulate TFLOP/s at ``clock_mhz``."""
        return (
            self.streaming_multiprocessors
            * self.tensor_cores_per_sm
            * self.fp16_fp32acc_flops_per_clock_per_tensor_core
            * clock_mhz
            / 1e6
        )

    def fp16_fp16acc_tflops(self, clock_mhz: int) -> float:
        """Dense FP16-input / FP16-accumulate TFLOP/s at ``clock_mhz``."""
        return self.fp16acc_rate_multiplier * self.fp16_fp32acc_tflops(clock_mhz)


# The reference's audited RTX 4060 entry, kept so result files written on
# that part still resolve.
RTX4060_PROFILE = GpuTheoreticalProfile(
    model_substring="RTX 4060",
    rated_boost_mhz=2460,
    streaming_multiprocessors=24,
    tensor_cores_per_sm=4,
    fp16_fp32acc_flops_per_clock_per_tensor_core=128,
    product_spec_url="https://www.nvidia.com/en-us/geforce/graphics-cards/40-series/rtx-4060-4060ti/",
    architecture_whitepaper_url=(
        "https://images.nvidia.com/aem-dam/Solutions/geforce/ada/nvidia-ada-gpu-architecture.pdf"
    ),
)

# B200 (sm_100): 148 SMs, four tensor cores each.  One tcgen05.mma kind::f16
# of M=128, N=128, K=16 (524,288 FLOP) completes every 64 SM cycles with
# fp32 accumulation, i.e. 8,192 FLOP per clock per SM, 2,048 per tensor
# core; fp16 accumulation does not go faster.  1,965 MHz is the part's
# `clocks.max.sm`.  At that clock the ceiling is 2,383 TFLOP/s, against
# NVIDIA's 2.25 PFLOP/s dense FP16/BF16 figure per GPU (the HGX B200
# product page, 36 PFLOP/s per 8 GPUs with sparsity); the SM count and the
# tensor-core generation are in the Blackwell architecture technical brief.
B200_PROFILE = GpuTheoreticalProfile(
    model_substring="B200",
    rated_boost_mhz=1965,
    streaming_multiprocessors=148,
    tensor_cores_per_sm=4,
    fp16_fp32acc_flops_per_clock_per_tensor_core=2048,
    product_spec_url="https://www.nvidia.com/en-us/data-center/hgx/",
    architecture_whitepaper_url="https://resources.nvidia.com/en-us-blackwell-architecture",
    fp16acc_rate_multiplier=1.0,
)

_GPU_PROFILES = (RTX4060_PROFILE, B200_PROFILE)


class PeakResults(TypedDict, total=False):
    """Schema-7 roofline ceilings embedded in every result file."""

    schema_version: int
    gpu_name: str
    gpu_slug: str
    compute_capability: str
    torch_version: str
    triton_version: str | None
    calibration_started_at_utc: str
    calibration_preflight_gpu_utilization_pct: list[int]
    calibration_preflight_gpu_utilization_limit_pct: int
    peak_bw_gbps: float
    cublas_tflops_fp16_fp32acc: float
    cublas_tflops_fp16_reduced_precision_allowed: float
    theoretical_tflops_fp16_fp32acc_rated: float
    theoretical_tflops_fp16_fp32acc_at_measured_clock: float
    theoretical_tflops_fp16_fp16acc_rated: float
    theoretical_tflops_fp16_fp16acc_at_measured_clock: float
    theoretical_ceiling_sm_clock_mhz: int
    cublas_tflops_sustained: float
    peaks_source: str
    peaks_method: str
    theoretical_provenance: dict[str, Any]


def profile_for(gpu_name: str) -> GpuTheoreticalProfile:
    """Return the audited profile whose model substring occurs in ``gpu_name``.

    Raises:
        ValueError: If no profile matches (the reference's message).
    """
    for profile in _GPU_PROFILES:
        if profile.model_substring in gpu_name:
            return profile
    raise ValueError(
        f"no theoretical compute profile for {gpu_name!r}; "
        "add an audited GpuTheoreticalProfile before benchmarking compute kernels"
    )


_profile_for = profile_for


def theoretical_tflops_fp16_fp32acc(sm_clock_mhz: int, *, profile: GpuTheoreticalProfile = B200_PROFILE) -> float:
    """Theoretical dense FP16/FP32-accumulate ceiling at ``sm_clock_mhz``."""
    return profile.fp16_fp32acc_tflops(sm_clock_mhz)


def theoretical_tflops_fp16_fp16acc(sm_clock_mhz: int, *, profile: GpuTheoreticalProfile = B200_PROFILE) -> float:
    """Theoretical dense FP16/FP16-accumulate ceiling at ``sm_clock_mhz``."""
    return profile.fp16_fp16acc_tflops(sm_clock_mhz)


def slug_for_name(gpu_name: str) -> str:
    """Filesystem-safe lowercase slug of a device name (``NVIDIA B200`` -> ``nvidia_b200``)."""
    return re.sub(r"[^a-z0-9]+", "_", gpu_name.lower()).strip("_")


def gpu_slug(device: int = 0) -> str:
    """Slug of CUDA device ``device``'s name.

    Raises:
        RuntimeError: If CUDA or the device is unavailable.
    """
    _validate_cuda_device(device)
    return slug_for_name(torch.cuda.get_device_name(device))


def gpu_utilization_pct(device: int = 0) -> int:
    """Whole-device utilization in percent, read from ``nvidia-smi``.

    Raises:
        RuntimeError: If ``nvidia-smi`` cannot provide the value.
    """
    try:
        completed = subprocess.run(
            ["nvidia-smi", f"--id={device}", "--query-gpu=utilization.gpu", "--format=csv,noheader,nounits"],
            check=True,
            capture_output=True,
            text=True,
            timeout=30,
        )
        return int(completed.stdout.strip().splitlines()[0])
    except (FileNotFoundError, subprocess.CalledProcessError, subprocess.TimeoutExpired, IndexError, ValueError) as error:
        raise RuntimeError("unable to query GPU utilization with nvidia-smi") from error


def peaks_from_measurement(
    measured: Mapping[str, Any],
    *,
    gpu_name: str,
    compute_capability: str,
    torch_version: str,
    source: str,
) -> PeakResults:
    """Build the schema-7 ceilings from a ``MEASURED_PEAKS.json`` record.

    ``measured`` holds ``hbm_gbs`` (device copy, read + write bytes),
    ``bf16_tflops`` (cuBLAS burst), optionally ``bf16_tflops_sustained``,
    and ``sm_max_mhz``; the theoretical ceiling is taken at that clock.

    Raises:
        ValueError: If a required field is missing or not positive, or the
            GPU has no profile.
    """
    profile = profile_for(gpu_name)
    values: dict[str, float] = {}
    for key in ("hbm_gbs", "bf16_tflops", "sm_max_mhz"):
        value = measured.get(key)
        if not isinstance(value, (int, float)) or value <= 0:
            raise ValueError(f"measured peaks: {key!r} must be a positive number")
        values[key] = float(value)
    clock = int(round(values["sm_max_mhz"]))
    peaks: PeakResults = {
        "schema_version": PEAKS_SCHEMA_VERSION,
        "gpu_name": gpu_name,
        "gpu_slug": slug_for_name(gpu_name),
        "compute_capability": compute_capability,
        "torch_version": torch_version,
        "triton_version": None,
        "calibration_started_at_utc": str(measured.get("when", "")),
        "calibration_preflight_gpu_utilization_pct": [],
        "calibration_preflight_gpu_utilization_limit_pct": 10,
        "peak_bw_gbps": values["hbm_gbs"],
        "cublas_tflops_fp16_fp32acc": values["bf16_tflops"],
        "cublas_tflops_fp16_reduced_precision_allowed": values["bf16_tflops"],
        "theoretical_tflops_fp16_fp32acc_rated": profile.fp16_fp32acc_tflops(profile.rated_boost_mhz),
        "theoretical_tflops_fp16_fp32acc_at_measured_clock": profile.fp16_fp32acc_tflops(clock),
        "theoretical_tflops_fp16_fp16acc_rated": profile.fp16_fp16acc_tflops(profile.rated_boost_mhz),
        "theoretical_tflops_fp16_fp16acc_at_measured_clock": profile.fp16_fp16acc_tflops(clock),
        "theoretical_ceiling_sm_clock_mhz": clock,
        "peaks_source": source,
        "peaks_method": str(measured.get("how", "")),
        "theoretical_provenance": {
            "model": profile.model_substring,
            "rated_boost_clock_mhz": profile.rated_boost_mhz,
            "streaming_multiprocessors": profile.streaming_multiprocessors,
            "tensor_cores_per_sm": profile.tensor_cores_per_sm,
            "fp16_fp32acc_flops_per_clock_per_tensor_core": profile.fp16_fp32acc_flops_per_clock_per_tensor_core,
            "fp16acc_rate_multiplier": profile.fp16acc_rate_multiplier,
            "ceiling_clock_policy": "maximum SM clock of the measured part",
            "product_spec_url": profile.product_spec_url,
            "architecture_whitepaper_url": profile.architecture_whitepaper_url,
        },
    }
    sustained = measured.get("bf16_tflops_sustained")
    if isinstance(sustained, (int, float)) and sustained > 0:
        peaks["cublas_tflops_sustained"] = float(sustained)
    return peaks


def load_measured_peaks(path: Path | None = None, *, device: int = 0) -> PeakResults:
    """Read a peak-measurement file and return the ceilings for CUDA device ``device``.

    ``path`` defaults to the file named by the ``TKLAB_MEASURED_PEAKS``
    environment variable.  The file's ``gpu_name`` must match the device (a
    file measured on another part is refused).

    Raises:
        FileNotFoundError: If no file is named or it is missing.
        ValueError: If it does not describe this device.
        RuntimeError: If CUDA or the device is unavailable.
    """
    _validate_cuda_device(device)
    if path is None:
        env = os.environ.get(MEASURED_PEAKS_ENV)
        if not env:
            raise FileNotFoundError(f"no peak-measurement file given and {MEASURED_PEAKS_ENV} is not set")
        path = Path(env)
    measured = read_json_object(path)
    gpu_name = torch.cuda.get_device_name(device)
    recorded = str(measured.get("gpu_name", ""))
    if recorded and recorded != gpu_name:
        raise ValueError(f"{path}: measured on {recorded!r}, not on {gpu_name!r}")
    major, minor = torch.cuda.get_device_capability(device)
    return peaks_from_measurement(
        measured,
        gpu_name=gpu_name,
        compute_capability=f"{major}.{minor}",
        torch_version=torch.__version__,
        source=str(path),
    )


def _sample_max_sm_clock(device: int, stop: threading.Event, out: list[int]) -> None:
    """Poll ``clocks.sm`` with nvidia-smi until ``stop`` is set (reads only)."""
    while not stop.is_set():
        try:
            completed = subprocess.run(
                ["nvidia-smi", f"--id={device}", "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"],
                check=True,
                capture_output=True,
                text=True,
                timeout=10,
            )
            out.append(int(completed.stdout.strip().splitlines()[0]))
        except (FileNotFoundError, subprocess.CalledProcessError, subprocess.TimeoutExpired, IndexError, ValueError):
            return
        stop.wait(0.2)


def _event_ms(fn, reps: int) -> list[float]:
    times = []
    for _ in range(reps):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    return times


def measure_peaks(
    device: int,
    *,
    calibration_started_at_utc: str,
    calibration_preflight_gpu_utilization_pct: tuple[int, ...],
    calibration_preflight_gpu_utilization_limit_pct: int,
    copy_elements: tuple[int, ...] = (1 << 27, 1 << 29),
    gemm_sizes: tuple[int, ...] = (4096, 8192),
    repetitions: int = 10,
) -> PeakResults:
    """Measure the empirical ceilings on ``device`` (``roofline.py:296-352`` of the reference).

    Device-copy bandwidth (``b.copy_(a)`` of 16-bit buffers, read + write
    bytes) and the cuBLAS fp16 GEMM rate with fp32 accumulation (``2 n^3``
    FLOP), each the best of ``repetitions`` CUDA-event timings over a size
    sweep; the theoretical ceilings are taken at the highest SM clock that
    ``nvidia-smi`` reported during the GEMMs (the rated clock if it could
    not be read).  Every sample is kept in the payload.
    """
    _validate_cuda_device(device)
    gpu_name = torch.cuda.get_device_name(device)
    profile = profile_for(gpu_name)
    with torch.cuda.device(device):
        bandwidth_samples = []
        for n in copy_elements:
            a = torch.empty(n, dtype=torch.float16, device="cuda").normal_()
            b = torch.empty_like(a)
            b.copy_(a)
            best = min(_event_ms(lambda a=a, b=b: b.copy_(a), repetitions))
            bandwidth_samples.append({"elements": n, "gbps": 2 * n * 2 / (best * 1e-3) / 1e9})
            del a, b
        clocks: list[int] = []
        stop = threading.Event()
        sampler = threading.Thread(target=_sample_max_sm_clock, args=(device, stop, clocks), daemon=True)
        sampler.start()
        gemm_samples = []
        reduced = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
        try:
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
            for n in gemm_sizes:
                x = torch.randn(n, n, dtype=torch.float16, device="cuda")
                y = torch.randn(n, n, dtype=torch.float16, device="cuda")
                torch.matmul(x, y)
                best = min(_event_ms(lambda x=x, y=y: torch.matmul(x, y), repetitions))
                gemm_samples.append({"n": n, "tflops": 2 * n**3 / (best * 1e-3) / 1e12})
                del x, y
            time.sleep(0.3)
        finally:
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = reduced
            stop.set()
            sampler.join(timeout=15)
    clock = max(clocks) if clocks else profile.rated_boost_mhz
    major, minor = torch.cuda.get_device_capability(device)
    measured = {
        "hbm_gbs": max(sample["gbps"] for sample in bandwidth_samples),
        "bf16_tflops": max(sample["tflops"] for sample in gemm_samples),
        "sm_max_mhz": clock,
        "when": calibration_started_at_utc,
        "how": "b.copy_(a) fp16 (read + write bytes) and torch.matmul fp16 with fp32 accumulation, best of "
        f"{repetitions} CUDA-event timings per size",
    }
    peaks = peaks_from_measurement(
        measured,
        gpu_name=gpu_name,
        compute_capability=f"{major}.{minor}",
        torch_version=torch.__version__,
        source="measured live",
    )
    peaks["calibration_preflight_gpu_utilization_pct"] = list(calibration_preflight_gpu_utilization_pct)
    peaks["calibration_preflight_gpu_utilization_limit_pct"] = calibration_preflight_gpu_utilization_limit_pct
    peaks["theoretical_provenance"]["bandwidth_samples"] = bandwidth_samples
    peaks["theoretical_provenance"]["gemm_samples"] = gemm_samples
    peaks["theoretical_provenance"]["sm_clock_samples_mhz"] = clocks
    return peaks


def load_or_measure_peaks(
    results_root: Path,
    *,
    device: int = 0,
    force: bool = False,
    measured_peaks_path: Path | None = None,
    calibration_started_at_utc: str | None = None,
    calibration_preflight_gpu_utilization_pct: tuple[int, ...] = (),
    calibration_preflight_gpu_utilization_limit_pct: int = 10,
) -> tuple[PeakResults, Path]:
    """Reuse a compatible ``<results_root>/<gpu-slug>/peaks.json`` or obtain and persist new ceilings.

    New ceilings come from ``measured_peaks_path`` (or the file the
    ``TKLAB_MEASURED_PEAKS`` environment variable names) when one is given,
    otherwise from :func:`measure_peaks`.  A stored file is reused only when
    it has this schema and describes this GPU, compute capability and torch
    version.

    Returns:
        The ceilings and the path of ``peaks.json``.
    """
    _validate_cuda_device(device)
    output_path = results_root / gpu_slug(device) / "peaks.json"
    major, minor = torch.cuda.get_device_capability(device)
    if output_path.exists() and not force:
        stored = read_json_object(output_path)
        expected = {
            "schema_version": PEAKS_SCHEMA_VERSION,
            "gpu_name": torch.cuda.get_device_name(device),
            "compute_capability": f"{major}.{minor}",
            "torch_version": torch.__version__,
        }
        if all(stored.get(key) == value for key, value in expected.items()):
            return cast(PeakResults, stored), output_path
    started = calibration_started_at_utc or datetime.now(timezone.utc).isoformat()
    named = measured_peaks_path or (Path(os.environ[MEASURED_PEAKS_ENV]) if os.environ.get(MEASURED_PEAKS_ENV) else None)
    if named is not None:
        peaks = load_measured_peaks(named, device=device)
        peaks["calibration_preflight_gpu_utilization_pct"] = list(calibration_preflight_gpu_utilization_pct)
        peaks["calibration_preflight_gpu_utilization_limit_pct"] = calibration_preflight_gpu_utilization_limit_pct
    else:
        peaks = measure_peaks(
            device,
            calibration_started_at_utc=started,
            calibration_preflight_gpu_utilization_pct=calibration_preflight_gpu_utilization_pct,
            calibration_preflight_gpu_utilization_limit_pct=calibration_preflight_gpu_utilization_limit_pct,
        )
    write_json_atomic(output_path, cast(JsonObject, peaks))
    return peaks, output_path


class RooflinePoint(TypedDict):
    """One kernel on the roofline."""

    intensity_flop_per_byte: float
    achieved_tflops: float
    attainable_tflops: float
    pct_attainable: float
    bound: str


def roofline_point(
    *, flops: float, bytes_moved: float, seconds: float, peak_tflops: float, peak_gbps: float
) -> RooflinePoint:
    """Place a measured kernel on the roofline ``min(peak, intensity x bandwidth)``.

    Raises:
        ValueError: If any quantity is not positive.
    """
    if min(flops, bytes_moved, seconds, peak_tflops, peak_gbps) <= 0:
        raise ValueError("roofline quantities must be positive")
    intensity = flops / bytes_moved
    memory_roof = intensity * peak_gbps / 1e3
    attainable = min(peak_tflops, memory_roof)
    achieved = flops / seconds / 1e12
    return {
        "intensity_flop_per_byte": intensity,
        "achieved_tflops": achieved,
        "attainable_tflops": attainable,
        "pct_attainable": 100.0 * achieved / attainable,
        "bound": "compute" if peak_tflops <= memory_roof else "memory",
    }


def _validate_cuda_device(device: int) -> None:
    """Check that ``device`` can be selected (the reference's checks and messages)."""
    if device < 0:
        raise ValueError("device index must be non-negative")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable")
    if device >= torch.cuda.device_count():
        raise RuntimeError(f"CUDA device {device} is unavailable; found {torch.cuda.device_count()} device(s)")
