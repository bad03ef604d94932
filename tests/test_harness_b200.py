"""Benchmark / artifact plumbing for B200: roofline profile, schema-7 result
files, the roofline table and the attention memory study.

CPU tests check the arithmetic and the file layouts against the reference's
(``src/tklab/harness/roofline.py``, ``src/tklab/cli.py``,
``benchmarks/plot_roofline.py``, ``benchmarks/flash_attention_memory.py``);
GPU tests run the benchmark and the memory worker on the real kernels.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import pytest
import torch

import tklab.kernels  # noqa: F401  (registers the attention specs)
from tklab import cli
from tklab.harness import attention_memory, bench, results, roofline
from tklab.harness.jsonio import write_json_atomic
from tklab.registry import REGISTRY

MEASURED = {
    "hbm_gbs": 6543.7,
    "bf16_tflops": 1616.1,
    "bf16_tflops_sustained": 1390.4,
    "sm_max_mhz": 1965.0,
    "gpu_name": "NVIDIA B200",
    "when": "2026-12-01T19:36:59Z",
    "how": "device copy and cuBLAS bf16 GEMM",
}

# The reference's schema-7 result keys, in its order (cli.py:253-291).
REFERENCE_RESULT_KEYS = [
    "schema_version",
    "kernel",
    "description",
    "gpu",
    "compute_capability",
    "torch_version",
    "triton_version",
    "benchmark_started_at_utc",
    "benchmark_preflight_gpu_utilization_pct",
    "benchmark_preflight_gpu_utilization_limit_pct",
    "peak_calibration_started_at_utc",
    "peak_calibration_preflight_gpu_utilization_pct",
    "peak_calibration_preflight_gpu_utilization_limit_pct",
    "peak_bw_gbps",
    "cublas_tflops_fp16_fp32acc",
    "cublas_tflops_fp16_reduced_precision_allowed",
    "theoretical_tflops_fp16_fp32acc_at_measured_clock",
    "theoretical_tflops_fp16_fp16acc_at_measured_clock",
    "theoretical_ceiling_sm_clock_mhz",
    "compute_mode",
    "rows",
]


def _peaks() -> roofline.PeakResults:
    return roofline.peaks_from_measurement(
        MEASURED, gpu_name="NVIDIA B200", compute_capability="10.0", torch_version="t", source="MEASURED_PEAKS.json"
    )


def test_b200_profile_ceilings() -> None:
    profile = roofline.profile_for("NVIDIA B200")
    assert profile is roofline.B200_PROFILE
    # 148 SMs x 8192 FLOP/clk/SM (one 128x128x16 MMA per 64 cycles) x 1965 MHz.
    assert profile.fp16_fp32acc_tflops(1965) == pytest.approx(148 * 8192 * 1965e6 / 1e12)
    assert profile.fp16_fp16acc_tflops(1965) == pytest.approx(profile.fp16_fp32acc_tflops(1965))
    assert roofline.theoretical_tflops_fp16_fp32acc(1000) == pytest.approx(148 * 8192 * 1e9 / 1e12)


def test_reference_profile_kept_with_its_fp16acc_doubling() -> None:
    profile = roofline.profile_for("NVIDIA GeForce RTX 4060")
    assert profile is roofline.RTX4060_PROFILE
    assert profile.fp16_fp32acc_tflops(2460) == pytest.approx(24 * 4 * 128 * 2460 / 1e6)
    assert profile.fp16_fp16acc_tflops(2460) == pytest.approx(2 * profile.fp16_fp32acc_tflops(2460))


def test_unknown_gpu_is_refused() -> None:
    with pytest.raises(ValueError, match="no theoretical compute profile for 'NVIDIA H100'"):
        roofline.profile_for("NVIDIA H100")


def test_slug() -> None:
    assert roofline.slug_for_name("NVIDIA B200") == "nvidia_b200"
    assert roofline.slug_for_name("NVIDIA GeForce RTX 4060") == "nvidia_geforce_rtx_4060"


def test_peaks_from_measurement() -> None:
    peaks = _peaks()
    assert peaks["schema_version"] == roofline.PEAKS_SCHEMA_VERSION == 7
    assert peaks["peak_bw_gbps"] == 6543.7
    assert peaks["cublas_tflops_fp16_fp32acc"] == 1616.1
    assert peaks["cublas_tflops_sustained"] == 1390.4
    assert peaks["theoretical_ceiling_sm_clock_mhz"] == 1965
    assert peaks["theoretical_tflops_fp16_fp32acc_at_measured_clock"] == pytest.approx(2382.397, rel=1e-6)
    assert peaks["gpu_slug"] == "nvidia_b200"
    bad = dict(MEASURED, hbm_gbs=0)
    with pytest.raises(ValueError, match="hbm_gbs"):
        roofline.peaks_from_measurement(
            bad, gpu_name="NVIDIA B200", compute_capability="10.0", torch_version="t", source="x"
        )


def test_b200_profile_is_sourced() -> None:
    """Theoretical ceilings come only from a profile with primary-source URLs (reference docs/benchmarking.md:60-62)."""
    for profile in (roofline.B200_PROFILE, roofline.RTX4060_PROFILE):
        assert profile.product_spec_url.startswith("https://www.nvidia.com/")
        assert profile.architecture_whitepaper_url.startswith("https://")


def test_peaks_file_is_named_explicitly_never_found_in_the_checkout() -> None:
    assert not hasattr(roofline, "DEFAULT_MEASURED_PEAKS")
    assert roofline.MEASURED_PEAKS_ENV == "TKLAB_MEASURED_PEAKS"


def test_roofline_point() -> None:
    # Intensity 1000 FLOP/B at 6.5 TB/s -> 6.5 PF memory roof: compute bound.
    point = roofline.roofline_point(flops=1e12, bytes_moved=1e9, seconds=1e-3, peak_tflops=2000, peak_gbps=6500)
    assert point["bound"] == "compute"
    assert point["achieved_tflops"] == pytest.approx(1000)
    assert point["pct_attainable"] == pytest.approx(50)
    low = roofline.roofline_point(flops=1e9, bytes_moved=1e9, seconds=1e-3, peak_tflops=2000, peak_gbps=6500)
    assert low["bound"] == "memory" and low["attainable_tflops"] == pytest.approx(6.5)
    with pytest.raises(ValueError):
        roofline.roofline_point(flops=0, bytes_moved=1, seconds=1, peak_tflops=1, peak_gbps=1)


def _row(size: int, ms: float, dtype: str = "float16") -> bench.BenchRow:
    spec = REGISTRY["attention_causal"]
    tflops = spec.flops(size, torch.float16) / (ms * 1e-3) / 1e12
    row: bench.BenchRow = {
        "kernel": spec.name,
        "dtype": dtype,
        "size": size,
        "ms": ms,
        "ms_lo": ms * 0.9,
        "ms_hi": ms * 1.1,
        "torch_ms": ms * 3,
        "speedup": 3.0,
        "tflops": tflops,
    }
    row.update(spec.benchmark_metadata(size, torch.float16))  # type: ignore[misc, typeddict-item]
    return row


def test_result_payload_has_the_reference_keys_in_order() -> None:
    spec = REGISTRY["attention_causal"]
    payload = results.result_payload(
        spec, rows=[_row(512, 0.02)], peaks=_peaks(), benchmark_started_at_utc="now", benchmark_preflight_gpu_utilization_pct=(0, 1)
    )
    keys = [key for key in payload if key != "peaks_source"]
    assert keys == REFERENCE_RESULT_KEYS
    assert payload["schema_version"] == 7
    assert payload["compute_mode"] == "attention_fp16_fp32acc"
    assert results.compute_baselines(spec, _peaks()) == (None, pytest.approx(2382.397, rel=1e-6))
    for key in ("block_m", "block_n", "num_warps", "num_stages", "heads", "head_dim", "causal"):
        assert key in payload["rows"][0]


def test_flash_roofline_rows_and_intensity() -> None:
    spec = REGISTRY["attention_causal"]
    rows = [_row(4096, 0.05), _row(8192, 0.15), _row(8192, 0.2, dtype="bfloat16")]
    payload = results.result_payload(
        spec, rows=rows, peaks=_peaks(), benchmark_started_at_utc="now", benchmark_preflight_gpu_utilization_pct=()
    )
    points = results.flash_roofline_rows(payload, label="flash_attn causal")
    assert [p["kernel"] for p in points] == ["flash_attn causal float16", "flash_attn causal bfloat16"]
    # Causal intensity ~ N / (2 s): 4 H N(N+1)/2 D / (4 H N D s) = (N+1)/(2s).
    assert points[0]["intensity_flop_per_byte"] == pytest.approx((8192 + 1) / 4)
    assert points[0]["bound"] == "compute"
    assert points[0]["achieved_tflops"] == pytest.approx(rows[1]["tflops"])


def test_results_table_only_reads_existing_files(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    for name in ("attention_noncausal", "attention_causal"):
        spec = REGISTRY[name]
        payload = results.result_payload(
            spec, rows=[_row(2048, 0.05)], peaks=_peaks(), benchmark_started_at_utc="now", benchmark_preflight_gpu_utilization_pct=()
        )
        write_json_atomic(tmp_path / "nvidia_b200" / f"{name}.json", payload)
    assert results.main(["--table-only", "--results-dir", str(tmp_path), "--title", "B200 roofline"]) == 0
    out = capsys.readouterr().out
    assert "B200 roofline" in out and "flash_attn causal float16" in out and "% ceiling" in out


def test_quantile() -> None:
    assert bench._quantile([1.0, 2.0, 3.0, 4.0, 5.0], 0.5) == 3.0
    assert bench._quantile([1.0, 2.0, 3.0, 4.0, 5.0], 0.2) == pytest.approx(1.8)
    with pytest.raises(ValueError):
        bench._quantile([1.0], 1.5)


def test_bench_spec_request_validation() -> None:
    spec = REGISTRY["attention_causal"]
    with pytest.raises(ValueError, match="warmup and repetition durations must be positive"):
        bench.bench_spec(spec, peak_bw_gbps=1, cublas_tflops=None, theoretical_tflops=1, warmup_ms=0)
    with pytest.raises(ValueError, match="device index must be non-negative"):
        bench.bench_spec(spec, peak_bw_gbps=1, cublas_tflops=None, theoretical_tflops=1, device=-1)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="CUDA is required for GPU benchmarks"):
            bench.bench_spec(spec, peak_bw_gbps=1, cublas_tflops=None, theoretical_tflops=1)


def _mem_row(impl: str, n: int, increment: int | None, oom: bool = False) -> attention_memory.WorkerResult:
    return {
        "implementation": impl,
        "sequence_length": n,
        "baseline_allocated_bytes": 0,
        "peak_allocated_bytes": increment,
        "peak_increment_bytes": increment,
        "output_finite": None if increment is None else True,
        "oom": oom,
        "error": "OutOfMemoryError" if oom else None,
    }


def test_memory_study_arithmetic() -> None:
    linear = [_mem_row("flash", n, 100 * n) for n in (512, 1024, 4096)]
    quadratic = [_mem_row("materialized", n, n * n) for n in (512, 2048)] + [_mem_row("materialized", 65536, None, True)]
    assert attention_memory.empirical_slope(linear) == pytest.approx(1.0)
    assert attention_memory.empirical_slope(quadratic) == pytest.approx(2.0)
    assert attention_memory.empirical_slope(linear[:1]) is None
    assert attention_memory.quadratic_bytes_per_n_squared() == 2 * 1 * 16 * 2
    assert attention_memory.dedicated_memory_crossing(64 * 1000**2) == pytest.approx(1000)
    payload = attention_memory.study_payload(
        linear + quadratic, gpu="NVIDIA B200", compute_capability="10.0", total_memory_bytes=2**30, driver={}
    )
    assert payload["schema_version"] == 1 and payload["study"] == "flash_attention_memory"
    assert payload["empirical_log_log_slope"]["flash"] == pytest.approx(1.0)
    assert payload["analytical_context"]["materialized_quadratic_buffers"] == 2


# ---------------------------------------------------------------- GPU
gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")


@pytest.mark.gpu
@gpu
def test_bench_spec_rows_on_b200() -> None:
    spec = REGISTRY["attention_causal"]
    rows = bench.bench_spec(
        spec,
        peak_bw_gbps=6500.0,
        cublas_tflops=None,
        theoretical_tflops=2382.0,
        warmup_ms=5,
        repetition_ms=20,
        sizes=(1024,),
        dtypes=(torch.float16,),
    )
    assert len(rows) == 1
    row = rows[0]
    assert row["kernel"] == "attention_causal" and row["size"] == 1024 and row["dtype"] == "float16"
    assert 0 < row["ms_lo"] <= row["ms"] <= row["ms_hi"]
    assert row["tflops"] > 0 and row["speedup"] > 0
    assert row["pct_theoretical"] == pytest.approx(100 * row["tflops"] / 2382.0)
    assert row["block_m"] == 128 and row["causal"] is True


def _peaks_file() -> Path | None:
    """The driver-measured peaks of this pool when the checkout carries them (else a live measurement)."""
    path = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    return path if path.exists() else None


@pytest.mark.gpu
@gpu
def test_cli_run_benchmarks_writes_schema7_file(tmp_path: Path) -> None:
    options = cli.BenchmarkOptions(
        device=0, force_peaks=False, kernels=("attention_noncausal",), warmup_ms=5, repetition_ms=20,
        list_kernels=False, allow_busy_gpu=True, results_dir=tmp_path, peaks=_peaks_file(), sizes=(1024,),
    )
    payloads = cli.run_benchmarks(options)
    path = payloads["attention_noncausal"]["path"]
    payload = json.loads(path.read_text())
    assert [key for key in payload if key != "peaks_source"] == REFERENCE_RESULT_KEYS
    assert payload["gpu"] == torch.cuda.get_device_name(0)
    assert {row["dtype"] for row in payload["rows"]} == {"float16", "bfloat16"}
    assert path.parent.name == roofline.gpu_slug(0)
    assert (path.parent / "peaks.json").exists()


@pytest.mark.gpu
@gpu
def test_cli_main_as_the_reference_benchmark_script_calls_it(tmp_path: Path) -> None:
    """``benchmarks/run.py`` of the reference is ``raise SystemExit(main())`` over ``tklab.cli.main``."""
    argv = ["--kernel", "attention_causal", "--size", "512", "--warmup-ms", "5", "--repetition-ms", "20",
            "--allow-busy-gpu", "--results-dir", str(tmp_path)]
    peaks = _peaks_file()
    if peaks is not None:
        argv += ["--peaks", str(peaks)]
    assert cli.main(argv) == 0
    payload = json.loads((tmp_path / roofline.gpu_slug(0) / "attention_causal.json").read_text())
    assert payload["schema_version"] == 7 and payload["kernel"] == "attention_causal"
    assert all(row["size"] == 512 and row["tflops"] > 0 for row in payload["rows"])


@pytest.mark.gpu
@gpu
def test_flash_attention_memory_is_linear() -> None:
    small = attention_memory.worker("flash", 2048, 0)
    large = attention_memory.worker("flash", 16384, 0)
    assert not small["oom"] and small["output_finite"] and large["output_finite"]
    slope = attention_memory.empirical_slope([small, large])
    assert slope is not None and slope == pytest.approx(1.0, abs=0.1)
    # The output alone: B*H*N*D fp16 bytes (plus at most allocator rounding).
    expected = 1 * 16 * 16384 * 64 * 2
    assert expected <= large["peak_increment_bytes"] <= 2 * expected
    dense_small = attention_memory.worker("materialized", 2048, 0)
    dense_large = attention_memory.worker("materialized", 8192, 0)
    dense_slope = attention_memory.empirical_slope([dense_small, dense_large])
    assert dense_slope is not None and dense_slope > 1.8
    assert math.isfinite(dense_slope)


def test_cli_options_mirror_the_reference() -> None:
    options = cli.parse_args([])
    assert options == cli.BenchmarkOptions(
        device=0, force_peaks=False, kernels=None, warmup_ms=25, repetition_ms=100, list_kernels=False,
        allow_busy_gpu=False,
    )
    chosen = cli.parse_args(["--kernel", "attention_causal", "--kernel", "attention_noncausal", "--device", "1"])
    assert chosen.kernels == ("attention_causal", "attention_noncausal") and chosen.device == 1
    with pytest.raises(SystemExit):
        cli.parse_args(["--kernel", "matmul_fp32acc"])
    with pytest.raises(ValueError, match="no kernels selected"):
        cli._select_specs(("not-registered",))
    assert [spec.name for spec in cli._select_specs(("attention_causal", "attention_noncausal"))] == [
        name for name in REGISTRY if name in ("attention_causal", "attention_noncausal")
    ]


def test_cli_list_kernels(capsys: pytest.CaptureFixture[str]) -> None:
    assert cli.main(["--list-kernels"]) == 0
    out = capsys.readouterr().out
    assert "attention_causal:" in out and "attention_noncausal:" in out


def test_cli_requires_cuda_before_anything_else(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="CUDA is required for benchmarks"):
        cli.run_benchmarks(cli.parse_args([]))


REFERENCE_RUN_PY = Path("/root/reference/benchmarks/run.py")


@pytest.mark.skipif(not REFERENCE_RUN_PY.exists(), reason="the reference checkout is not present on this machine")
def test_reference_benchmark_script_runs_unchanged_on_this_package() -> None:
    """The reference's own ``benchmarks/run.py`` (``from tklab.cli import main``), unmodified, on this package."""
    import subprocess
    import sys

    package_dir = Path(__file__).resolve().parents[1] / "triton-kernel-lab_b200"
    proc = subprocess.run(
        [sys.executable, str(REFERENCE_RUN_PY), "--list-kernels"],
        env={"PYTHONPATH": str(package_dir), "PATH": "/usr/bin:/bin"},
        capture_output=True,
        text=True,
        timeout=300,
        check=False,
    )
    assert proc.returncode == 0, proc.stderr
    assert "attention_causal:" in proc.stdout and "attention_noncausal:" in proc.stdout
