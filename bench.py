"""Benchmark of the attention hot path: causal bf16 fwd + bwd, B=8 H=32 S=4096 D=128.

One step = forward (with LSE) + backward (delta/clear, fused recompute
kernel, dQ conversion) over this rank's (batch*head) slab of the BASELINE
config-3 problem.  With N GPUs (torchrun, one process per GPU) the 256
(batch, head) slabs are split evenly, with no collective on the data path
("strong" scaling: the total problem is fixed).  Timing: per-step CUDA
events on the launching stream after an L2 flush, K timed steps between a
barrier + synchronize on both sides, max over ranks.

``--impl reference`` times the reference's CPU path instead (fp32
``F.scaled_dot_product_attention`` forward + autograd backward on the host
cores, the reference's ``ref_fn``) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _entry in (ROOT / "triton-kernel-lab_b200", ROOT):
    if str(_entry) not in sys.path:
        sys.path.insert(0, str(_entry))

import torch  # noqa: E402

CONFIGS = {
    # name: (batch, heads, seq, head_dim, dtype, causal, qk_std)
    "c3": (8, 32, 4096, 128, torch.bfloat16, True, 1.0),
    "c2": (4, 16, 1024, 64, torch.float16, False, 1.0),
    "c4": (1, 32, 16384, 128, torch.bfloat16, True, 1.5),
}
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (read + write) per (batch, head) slab of the C3 shape for one
# launch of the fused backward kernel, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of the 64-slab case:
# 404.8 MB + 223.9 MB over 64 slabs.  Traffic grows in proportion to the
# slab count.
BWD_DRAM_BYTES_PER_SLAB_C3 = 629.63e6 / 64
THROTTLE_REASONS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
}


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"bf16_tflops": data["bf16_tflops"], "bf16_tflops_sustained": data["bf16_tflops_sustained"],
                "hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def fwd_flops(b: int, h: int, s: int, d: int, causal: bool) -> int:
    """Reference FLOP model: 4 * B * H * pairs * D (flash_attention.py:737-747)."""
    pairs = s * (s + 1) // 2 if causal else s * s
    return 4 * b * h * pairs * d


def bwd_flops(b: int, h: int, s: int, d: int, causal: bool) -> int:
    """Algorithmic backward: 5 GEMMs = 2.5x the forward (recompute not credited)."""
    return fwd_flops(b, h, s, d, causal) * 5 // 2


class ClockSampler:
    """Streams ``nvidia-smi -lms 20`` clock / throttle-reason samples, each
    stamped with the host monotonic clock, so that the samples falling inside
    a timed window can be picked out afterwards."""

    def __init__(self, index: int, interval_ms: int = 20) -> None:
        self.index = index
        self.interval_ms = interval_ms
        self.samples: list[tuple[float, float, float, int]] = []
        self._proc: subprocess.Popen | None = None
        self._thread = threading.Thread(target=self._read, daemon=True)

    def _read(self) -> None:
        assert self._proc is not None and self._proc.stdout is not None
        for line in self._proc.stdout:
            try:
                sm, sm_max, reasons = (x.strip() for x in line.split(","))
                self.samples.append((time.monotonic(), float(sm), float(sm_max), int(reasons, 16)))
            except ValueError:
                continue

    def __enter__(self) -> ClockSampler:
        query = "clocks.sm,clocks.max.sm,clocks_event_reasons.active"
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={query}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self._thread.start()
        except OSError:
            self._proc = None
        return self

    def wait_first(self, timeout_s: float = 5.0) -> None:
        """Block until the first sample has arrived (nvidia-smi takes a moment to start)."""
        deadline = time.monotonic() + timeout_s
        while self._proc is not None and not self.samples and time.monotonic() < deadline:
            time.sleep(0.01)

    def __exit__(self, *exc: object) -> None:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._thread.join(timeout=5)

    def summary(self, t0: float | None = None, t1: float | None = None) -> dict:
        """Summary of the samples taken in [t0, t1] (all samples when no window is given).
        A window shorter than the sampling interval may hold none: then the
        first samples after t0, within two intervals of t1, are used."""
        picked = list(self.samples)
        if t0 is not None and t1 is not None:
            inside = [x for x in self.samples if t0 <= x[0] <= t1]
            if not inside:
                slack = 2 * self.interval_ms / 1000.0
                inside = [x for x in self.samples if t0 <= x[0] <= t1 + slack][:2]
            picked = inside
        if not picked:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        mask = 0
        for _, _, _, r in picked:
            mask |= r
        reasons = [name for bit, name in THROTTLE_REASONS.items() if mask & bit and bit != 0x1]
        return {
            "sm_mhz": statistics.median(s for _, s, _, _ in picked),
            "sm_max_mhz": max(m for _, _, m, _ in picked),
            "reasons": reasons,
            "samples": len(picked),
        }


def _dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _make_inputs(shape: tuple[int, ...], dtype: torch.dtype, qk_std: float, seed: int, device) -> list[torch.Tensor]:
    """Seeded synthetic Q, K, V, dO drawn on the device (no host round trip at this size)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(shape, generator=gen, device=device) * qk_std).to(dtype)
    k = (torch.randn(shape, generator=gen, device=device) * qk_std).to(dtype)
    v = torch.randn(shape, generator=gen, device=device).to(dtype)
    do = torch.randn(shape, generator=gen, device=device).to(dtype)
    return [q, k, v, do]


def _metric_and_config(config: str, world: int, bh_total: int | None = None) -> tuple[str, dict]:
    """The metric name and the ``config`` object of a run of ``config`` on ``world`` GPUs.

    Both arms (ours and ``--impl reference``) print exactly these, so the two
    lines describe the same workload."""
    b, h, s, d, dtype, causal, _ = CONFIGS[config]
    bh_total = b * h if bh_total is None else bh_total
    dtype_name = "bf16" if dtype == torch.bfloat16 else "fp16"
    metric = (f"attention fwd+bwd TFLOP/s ({'causal' if causal else 'non-causal'} {dtype_name} "
              f"B={b} H={h} S={s} D={d}), aggregate over GPUs")
    per_rank = -(-bh_total // world)
    cfg = {
        "workload": f"{config}: causal={causal} B={b} H={h} S={s} D={d} {str(dtype).split('.')[-1]}",
        "global_batch": b,
        "seq_len": s,
        "heads": h,
        "head_dim": d,
        "parallelism": f"(batch*head) slabs {per_rank}/rank x {world} ranks, no collective",
        "bh_total": bh_total,
        "l2": "flushed: 256 MiB write before every timed step (outside its events)",
    }
    return metric, cfg


def run_ours(args: argparse.Namespace) -> None:
    from tklab import _native
    from tklab.kernels.flash_attention import _NATIVE_DTYPE, attention_causal, attention_noncausal

    rank, world, local_rank = _dist_env()
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    from tklab.sharding import slab_range

    b, h, s, d, dtype, causal, qk_std = CONFIGS[args.config]
    bh_total = b * h
    if args.bh is not None:
        # Profiling mode: a smaller problem of the same per-slab shape.
        bh_total = args.bh * world
    start_bh, stop_bh = slab_range(bh_total, world, rank)
    slab = stop_bh - start_bh
    shape = (1, slab, s, d)  # this rank's contiguous slab of the flattened (B*H) axis
    lib = _native.load()
    q, k, v, do = _make_inputs(shape, dtype, qk_std, seed=args.seed + rank, device=device)
    o = torch.empty_like(q)
    lse = torch.empty((1, slab, s), dtype=torch.float32, device=device)
    delta = torch.empty_like(lse)
    dq_accum = torch.empty(shape, dtype=torch.float32, device=device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    sp = int(stream.cuda_stream)
    nd = _NATIVE_DTYPE[dtype]
    scale = 1.0 / math.sqrt(d)
    numel = q.numel()
    # Scratch of the forward's key-split schedule (0 when this rank's slab
    # count fills the device): allocated once, outside the timed region.
    fwd_ws_bytes = int(lib.tk_attn_fwd_workspace_bytes(1, slab, s, d, nd, int(causal)))
    fwd_ws = torch.empty(max(fwd_ws_bytes, 1), dtype=torch.uint8, device=device)
    fwd_ws_ptr = fwd_ws.data_ptr() if fwd_ws_bytes else None

    def step(ev: list[torch.cuda.Event] | None) -> None:
        def mark(i: int) -> None:
            if ev is not None:
                ev[i].record(stream)

        mark(0)
        _native.check(lib.tk_attn_fwd_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                         1, slab, s, d, nd, int(causal), scale, fwd_ws_ptr, fwd_ws_bytes, sp), "fwd")
        mark(1)
        _native.check(lib.tk_attn_bwd_pre(o.data_ptr(), do.data_ptr(), delta.data_ptr(), dq_accum.data_ptr(),
                                          1, slab, s, d, nd, sp), "bwd_pre")
        mark(2)
        _native.check(lib.tk_attn_bwd_fused(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                            lse.data_ptr(), delta.data_ptr(), dq_accum.data_ptr(),
                                            dk.data_ptr(), dv.data_ptr(), 1, slab, s, d, nd, int(causal),
                                            scale, sp), "bwd")
        mark(3)
        _native.check(lib.tk_attn_dq_convert(dq_accum.data_ptr(), dq.data_ptr(), numel, nd, sp), "dq_convert")
        mark(4)

    # Every rank samples its own GPU's clocks, from before the warm-up so
    # that the samples cover the whole timed region, however short.
    sampler = ClockSampler(local_rank)
    sampler.__enter__()
    sampler.wait_first()
    liveness = None
    if world > 1:
        from tklab.sharding import check_ranks_alive, liveness_group

        liveness = liveness_group()
    try:
        for _ in range(args.warmup):
            flush.zero_()
            step(None)
        torch.cuda.synchronize(device)
        status = _native.device_status(sp)
        if status:
            _native.check(status, "warm-up device status")

        events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
        if world > 1:
            # Between warm-up and timing, with nothing in flight: a rank that
            # has gone is reported here instead of blocking the barrier.
            check_ranks_alive(liveness, timeout_s=60.0)
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        t_start = time.monotonic()
        for i in range(args.steps):
            flush.zero_()  # write > L2 (126 MB) between timed steps, outside the step's events
            step(events[i])
        torch.cuda.synchronize(device)
        t_end = time.monotonic()
        time.sleep(2 * sampler.interval_ms / 1000.0)
    finally:
        sampler.__exit__()
    if world > 1:
        torch.distributed.barrier()
    status = _native.device_status(sp)
    if status:
        _native.check(status, "timed-region device status")

    per_kernel = [0.0] * 4
    total_ms = 0.0
    for ev in events:
        for j in range(4):
            per_kernel[j] += ev[j].elapsed_time(ev[j + 1])
        total_ms += ev[0].elapsed_time(ev[4])
    my_clocks = sampler.summary(t_start, t_end)
    reason_mask = sum(bit for bit, name in THROTTLE_REASONS.items() if name in my_clocks["reasons"])
    mine = [total_ms] + per_kernel + [my_clocks["sm_mhz"] or 0.0, my_clocks["sm_max_mhz"] or 0.0,
                                      float(reason_mask), float(my_clocks["samples"])]
    if world > 1:
        gathered = [torch.zeros(len(mine), dtype=torch.float64, device=device) for _ in range(world)]
        torch.distributed.all_gather(gathered, torch.tensor(mine, dtype=torch.float64, device=device))
        rows = [g.tolist() for g in gathered]
    else:
        rows = [mine]
    # Whole-job time = the slowest rank's (max over ranks, per column).
    total_ms, k_fwd, k_pre, k_bwd, k_cvt = (max(r[j] for r in rows) for j in range(5))
    per_rank = [
        {
            "rank": i,
            "ms_per_step": round(r[0] / args.steps, 4),
            "kernel_ms_per_step": {name: round(r[1 + j] / args.steps, 4)
                                   for j, name in enumerate(("attn_fwd", "attn_bwd_pre", "attn_bwd_fused",
                                                             "dq_convert"))},
            "sm_mhz": r[5] or None,
            "sm_max_mhz": r[6] or None,
            "reasons": [name for bit, name in THROTTLE_REASONS.items() if int(r[7]) & bit],
            "clock_samples": int(r[8]),
            # time x clock: comparable across ranks whose clocks differ
            "ms_x_ghz": round(r[0] / args.steps * (r[5] or 0.0) / 1000.0, 4),
        }
        for i, r in enumerate(rows)
    ]

    # End-to-end through the public autograd API with host buffers.
    e2e = None
    if not args.no_e2e:
        e2e = _e2e(args, attention_causal if causal else attention_noncausal, shape, dtype, qk_std, device, rank, world)

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(args.config, seconds=args.cpu_seconds)

    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        peaks = _peaks()
        steps = args.steps
        ff = fwd_flops(1, bh_total, s, d, causal)
        bf = bwd_flops(1, bh_total, s, d, causal)
        ms_per_step = total_ms / steps
        value = (ff + bf) / (ms_per_step * 1e-3) / 1e12
        # Dominant kernel: the one with the largest share of the step.
        kernels = {"attn_fwd": (k_fwd / steps, ff / world), "attn_bwd_fused": (k_bwd / steps, bf / world)}
        dom = max(kernels, key=lambda n: kernels[n][0])
        dom_ms, dom_flops = kernels[dom]
        achieved = dom_flops / (dom_ms * 1e-3) / 1e12
        clocks = dict(my_clocks)
        clocks["reasons"] = sorted({name for r in per_rank for name in r["reasons"]})
        clocks["sm_mhz_min_over_ranks"] = min((r["sm_mhz"] or 0.0) for r in per_rank)
        metric, config = _metric_and_config(args.config, world, bh_total)
        line = {
            "metric": metric,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16" if dtype == torch.bfloat16 else "f16",
            "data": "synthetic (seeded randn; Q,K std %.1f)" % qk_std,
            "config": config,
            "fwd_tflops_per_gpu": round(ff / world / (k_fwd / steps * 1e-3) / 1e12, 2),
            "bwd_tflops_per_gpu": round(bf / world / ((k_pre + k_bwd + k_cvt) / steps * 1e-3) / 1e12, 2),
            "pct_peak_fwd": round(100 * ff / world / (k_fwd / steps * 1e-3) / 1e12 / peaks["bf16_tflops"], 2),
            "pct_peak_bwd": round(
                100 * bf / world / ((k_pre + k_bwd + k_cvt) / steps * 1e-3) / 1e12 / peaks["bf16_tflops"], 2),
            "kernel_ms_per_step": {"attn_fwd": round(k_fwd / steps, 4), "attn_bwd_pre": round(k_pre / steps, 4),
                                   "attn_bwd_fused": round(k_bwd / steps, 4), "dq_convert": round(k_cvt / steps, 4)},
            "roofline": {
                "kernel": dom,
                "bound": "tensor",
                "achieved": round(achieved, 2),
                "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops"], 4),
                "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
                "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                "traffic": args.traffic_bytes if args.traffic_bytes is not None else (
                    round(BWD_DRAM_BYTES_PER_SLAB_C3 * slab) if (args.config == "c3" and dom == "attn_bwd_fused")
                    else None),
                "traffic_source": "ncu dram bytes of one 64-slab launch scaled by slabs/rank",
            },
            "gpu_launches": (5 if fwd_ws_bytes else 4) * steps,
            "gpu_launches_note": ("per rank: fwd, " + ("fwd_combine, " if fwd_ws_bytes else "")
                                  + "bwd_pre, bwd_fused, dq_convert per step"),
            "clocks": clocks,
            "per_rank": per_rank,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def _e2e(args, attn, shape, dtype, qk_std, device, rank, world) -> dict | None:
    """Public API, pinned host buffers in, results (O, dQ, dK, dV) back to the host, every step.

    The copies of consecutive steps overlap, as in a streaming pipeline: step
    k's inputs go up on a copy stream into one of two device input sets (a set
    is reused once the compute that read it has finished), the public call
    runs on the compute stream, and step k's results come down on a third
    stream while step k+1 computes and step k+2 uploads.  Every step still
    moves its full inputs in and its full results out inside the timed region.
    """
    b, h, s, d, _, causal, _ = CONFIGS[args.config]
    host_in = [t.cpu().pin_memory() for t in _make_inputs(shape, dtype, qk_std, seed=args.seed + 100 + rank,
                                                           device=device)]
    host_out = [torch.empty(shape, dtype=dtype).pin_memory() for _ in range(4)]
    dev_in = [[torch.empty(shape, dtype=dtype, device=device) for _ in range(4)] for _ in range(2)]
    compute = torch.cuda.current_stream(device)
    up = torch.cuda.Stream(device)
    down = torch.cuda.Stream(device)
    in_free = [torch.cuda.Event() for _ in range(2)]
    for ev in in_free:
        ev.record(compute)

    def one(step: int) -> torch.cuda.Event:
        slot = dev_in[step % 2]
        up.wait_event(in_free[step % 2])
        with torch.cuda.stream(up):
            for dst, src in zip(slot, host_in, strict=True):
                dst.copy_(src, non_blocking=True)
        uploaded = torch.cuda.Event()
        uploaded.record(up)
        compute.wait_event(uploaded)
        q, k, v = (t.detach().requires_grad_(True) for t in slot[:3])
        out = attn(q, k, v)
        grads = torch.autograd.grad(out, (q, k, v), grad_outputs=slot[3])
        in_free[step % 2].record(compute)
        down.wait_stream(compute)
        with torch.cuda.stream(down):
            for dst, src in zip(host_out, (out, *grads), strict=True):
                dst.copy_(src.detach(), non_blocking=True)
        for t in (out, *grads):
            t.record_stream(down)
        downloaded = torch.cuda.Event()
        downloaded.record(down)
        return downloaded

    for i in range(max(1, args.warmup)):
        one(i)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    up.wait_stream(compute)
    last = None
    for i in range(args.e2e_steps):
        last = one(i)
    compute.wait_event(last)
    end.record(compute)
    torch.cuda.synchronize(device)
    ms = torch.tensor([start.elapsed_time(end) / args.e2e_steps], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms_step = float(ms.item())
    flops = fwd_flops(b, h, s, d, causal) + bwd_flops(b, h, s, d, causal)
    per_rank_bytes = 4 * math.prod(shape) * torch.empty((), dtype=dtype).element_size()
    return {
        "value": round(flops / (ms_step * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms_step, 3),
        "h2d_bytes_per_step": per_rank_bytes * world,
        "d2h_bytes_per_step": per_rank_bytes * world,
        "path": "tklab.kernels.flash_attention.attention_causal + torch.autograd.grad, pinned host buffers; "
                "uploads, compute and downloads of consecutive steps overlap on three streams",
        "steps": args.e2e_steps,
    }


def _cpu_slab_step(shape, dtype, causal, qk_std, seed) -> float:
    from oracle.attention_oracle import sdpa_backward

    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(shape, generator=gen) * qk_std).to(dtype)
    k = (torch.randn(shape, generator=gen) * qk_std).to(dtype)
    v = torch.randn(shape, generator=gen).to(dtype)
    do = torch.randn(shape, generator=gen).to(dtype)
    t0 = time.perf_counter()
    sdpa_backward(q, k, v, do, causal=causal)
    return time.perf_counter() - t0


def _cpu_baseline(config: str, seconds: float) -> dict:
    """The reference's CPU path (fp32 SDPA fwd + autograd bwd) on a bounded sample: one (b, h) slab per rep."""
    b, h, s, d, dtype, causal, qk_std = CONFIGS[config]
    torch.set_num_threads(os.cpu_count() or 1)
    shape = (1, 1, s, d)
    _cpu_slab_step(shape, dtype, causal, qk_std, 0)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 3:
        times.append(_cpu_slab_step(shape, dtype, causal, qk_std, len(times) + 1))
    per_slab = statistics.median(times)
    flops = (fwd_flops(1, 1, s, d, causal) + bwd_flops(1, 1, s, d, causal))
    return {
        "value": round(flops / per_slab / 1e12, 4),
        "unit": "TFLOP/s",
        "cores": torch.get_num_threads(),
        "kind": "reference",
        "sample": f"{len(times)} reps of one (b,h) slab ({s}x{d}, causal={causal}) fwd+bwd; median {per_slab:.3f} s",
    }


def run_reference(args: argparse.Namespace) -> None:
    rank, world, _ = _dist_env()
    if rank != 0:
        return
    b, h, s, d, dtype, causal, qk_std = CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count() or 1)
    shape = (1, 1, s, d)
    for i in range(args.warmup):
        _cpu_slab_step(shape, dtype, causal, qk_std, 1000 + i)
    total = 0.0
    for i in range(args.steps):
        total += _cpu_slab_step(shape, dtype, causal, qk_std, i)
    per_step = total / args.steps
    flops = fwd_flops(1, 1, s, d, causal) + bwd_flops(1, 1, s, d, causal)
    value = flops / per_step / 1e12
    metric, config = _metric_and_config(args.config, world)
    line = {
        "impl": "reference",
        "metric": metric,
        "value": round(value, 4),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded randn)",
        "config": config,
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "reference",
                         "sample": f"one (b,h) slab ({s}x{d}) of the workload per step: fp32 SDPA fwd + "
                                   "autograd bwd on the host cores"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_sweep(args: argparse.Namespace) -> None:
    """C5 sweep: fp16 and bf16, causal and non-causal, D in {64, 128},
    S in {512, ..., 16384} with B = 16384 / S and H = 16 (seeded N(0,1)
    inputs).  Forward (with LSE) and backward (preprocess + fused kernel +
    dQ conversion) are timed separately with CUDA events after an L2 flush;
    the (batch*head) slabs are split over the ranks as in the main benchmark
    and the time is the max over ranks.  Rank 0 prints one JSON line per
    configuration (these lines are not the benchmark's headline line)."""
    from tklab import _native
    from tklab.kernels.flash_attention import _NATIVE_DTYPE
    from tklab.sharding import slab_range

    rank, world, local_rank = _dist_env()
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    lib = _native.load()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    sp = int(stream.cuda_stream)
    for dtype in (torch.float16, torch.bfloat16):
        for causal in (False, True):
            for d in (64, 128):
                for s in (512, 1024, 2048, 4096, 8192, 16384):
                    b, h = 16384 // s, 16
                    start_bh, stop_bh = slab_range(b * h, world, rank)
                    slab = stop_bh - start_bh
                    shape = (1, slab, s, d)
                    q, k, v, do = _make_inputs(shape, dtype, 1.0, seed=args.seed + rank, device=device)
                    o = torch.empty_like(q)
                    lse = torch.empty((1, slab, s), dtype=torch.float32, device=device)
                    delta = torch.empty_like(lse)
                    acc = torch.empty(shape, dtype=torch.float32, device=device)
                    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
                    nd = _NATIVE_DTYPE[dtype]
                    scale = 1.0 / math.sqrt(d)

                    ws_bytes = int(lib.tk_attn_fwd_workspace_bytes(1, slab, s, d, nd, int(causal)))
                    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
                    ws_ptr = ws.data_ptr() if ws_bytes else None

                    def fwd() -> None:
                        _native.check(lib.tk_attn_fwd_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                         lse.data_ptr(), 1, slab, s, d, nd, int(causal), scale,
                                                         ws_ptr, ws_bytes, sp), "fwd")

                    def bwd() -> None:
                        _native.check(lib.tk_attn_bwd_pre(o.data_ptr(), do.data_ptr(), delta.data_ptr(),
                                                          acc.data_ptr(), 1, slab, s, d, nd, sp), "bwd_pre")
                        _native.check(lib.tk_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                                      lse.data_ptr(), delta.data_ptr(), acc.data_ptr(), dq.data_ptr(),
                                                      dk.data_ptr(), dv.data_ptr(), 1, slab, s, d, nd, int(causal),
                                                      scale, sp), "bwd")

                    times = {}
                    for name, fn in (("fwd", fwd), ("bwd", bwd)):
                        for _ in range(args.warmup):
                            fn()
                        samples = []
                        for _ in range(args.steps):
                            flush.zero_()
                            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            e0.record(stream)
                            fn()
                            e1.record(stream)
                            torch.cuda.synchronize(device)
                            samples.append(e0.elapsed_time(e1))
                        t = torch.tensor([statistics.median(samples)], dtype=torch.float64, device=device)
                        if world > 1:
                            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                        times[name] = float(t.item())
                    if rank == 0:
                        ff, bf = fwd_flops(b, h, s, d, causal), bwd_flops(b, h, s, d, causal)
                        print(json.dumps({
                            "sweep": "c5", "dtype": str(dtype).replace("torch.", ""), "causal": causal, "D": d,
                            "S": s, "B": b, "H": h, "n_gpus": world, "fwd_ms": round(times["fwd"], 4),
                            "bwd_ms": round(times["bwd"], 4),
                            "fwd_tflops": round(ff / times["fwd"] / 1e9, 1),
                            "bwd_tflops": round(bf / times["bwd"] / 1e9, 1),
                            "fwd_key_split": bool(ws_bytes),
                            "bwd_timed": "tk_attn_bwd_pre + tk_attn_bwd (fused kernel + dQ conversion)",
                            "l2": "flushed before every timed call"}), flush=True)
                    del q, k, v, do, o, lse, delta, acc, dq, dk, dv
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_rope(args: argparse.Namespace) -> None:
    """Fused rotate-half RoPE attention at the configured shape (1 GPU).

    Times, with CUDA events after an L2 flush: the plain forward, the fused
    RoPE forward (K rotated once into a workspace, Q rotated in shared memory
    inside the kernel), the same result unfused (Q and K rotated in device
    memory by the elementwise kernel, then the plain forward) and the RoPE
    backward (rotate Q and K, delta + clear, fused backward, dQ conversion
    with the transpose rotation, dK rotated back).  Prints one JSON line per measurement (not the
    benchmark's headline line)."""
    from tklab import _native
    from tklab.kernels.flash_attention import _NATIVE_DTYPE
    from tklab.kernels.rope_attention import _launch_backward_rope, rope_tables, rotate

    b, h, s, d, dtype, causal, std = CONFIGS[args.config]
    bh = args.bh if args.bh is not None else b * h
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    shape = (1, bh, s, d)
    q, k, v, do = _make_inputs(shape, dtype, std, seed=args.seed, device=device)
    cos, sin = rope_tables(s, d, device=device)
    o = torch.empty_like(q)
    lse = torch.empty((1, bh, s), dtype=torch.float32, device=device)
    q_r, k_r = torch.empty_like(q), torch.empty_like(k)
    lib = _native.load()
    nd = _NATIVE_DTYPE[dtype]
    scale = 1.0 / math.sqrt(d)
    sp = int(torch.cuda.current_stream(device).cuda_stream)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    def plain() -> None:
        _native.check(lib.tk_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                      1, bh, s, d, nd, int(causal), scale, sp), "fwd")

    def fused() -> None:
        _native.check(lib.tk_attn_fwd_rope(q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                           k_r.data_ptr(), o.data_ptr(), lse.data_ptr(), 1, bh, s, d, nd,
                                           int(causal), scale, sp),
                      "fwd_rope")

    def unfused() -> None:
        rotate(q, cos, sin, out=q_r)
        rotate(k, cos, sin, out=k_r)
        _native.check(lib.tk_attn_fwd(q_r.data_ptr(), k_r.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                      1, bh, s, d, nd, int(causal), scale, sp), "fwd")

    def backward() -> None:
        _launch_backward_rope(q, k, v, o, lse, do, cos, sin, causal=causal)

    results = {}
    for name, fn in (("fwd_plain", plain), ("fwd_rope_fused", fused), ("fwd_rope_unfused", unfused),
                     ("bwd_rope", backward)):
        for _ in range(args.warmup):
            fn()
        samples = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(device)
            samples.append(e0.elapsed_time(e1))
        results[name] = statistics.median(samples)
    ff, bf = fwd_flops(1, bh, s, d, causal), bwd_flops(1, bh, s, d, causal)
    for name, ms in results.items():
        flops = bf if name.startswith("bwd") else ff
        print(json.dumps({
            "rope": name, "config": args.config, "bh": bh, "S": s, "D": d, "causal": causal,
            "dtype": str(dtype).replace("torch.", ""), "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
            "vs_fwd_plain": round(ms / results["fwd_plain"], 3) if name.startswith("fwd") else None,
            "l2": "flushed before every timed call"}), flush=True)


def run_decode(args: argparse.Namespace) -> None:
    """GQA decode (``tk_gqa_decode``) at the reference model's numerical point
    (B=1, Hq=32, Hkv=8, Dh=128, L=4096, fp16) and larger batch / context
    shapes, 1 GPU.  Each shape is timed with CUDA events in the two cache
    states the model asks to keep apart: "controlled cache-thrashing" (a
    256 MiB write evicts L2 before every call) and warm (back-to-back calls).
    Reported against the model's minimum traffic (unique KV + Q + O bytes)
    and the measured HBM copy bandwidth; one JSON line per shape."""
    from tklab.kernels.gqa_decode import decode_model, gqa_decode, set_decode_path

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peaks = _peaks()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    shapes = [(1, 32, 8, 128, 4096), (1, 32, 8, 128, 131072), (32, 32, 8, 128, 4096), (64, 32, 8, 128, 8192),
              (16, 64, 8, 128, 16384), (16, 128, 8, 128, 16384), (16, 64, 8, 64, 16384)]
    if args.shape:
        if len(args.shape) != 5:
            raise SystemExit("--decode --shape takes B,Hq,Hkv,Dh,L")
        shapes = [tuple(args.shape)]
    for batch, hq, hkv, d, seq in shapes:
        g = torch.Generator(device=device).manual_seed(args.seed)
        q = torch.randn((batch, hq, d), generator=g, device=device).to(torch.float16)
        k = torch.randn((batch, hkv, seq, d), generator=g, device=device).to(torch.float16)
        v = torch.randn((batch, hkv, seq, d), generator=g, device=device).to(torch.float16)
        model = decode_model(batch, hq, hkv, d, seq)
        tensor_cores = d in (64, 128) and hq // hkv in (4, 8, 16)
        # Both kernels where the tensor-core one applies, interleaved call by
        # call so that clock and power drift hit them alike.  Each kernel's
        # call is also captured in a CUDA graph: replaying it times the
        # device work alone (decode steps run from graphs in serving), while
        # the eager call includes the host-side argument checks, allocation
        # and tensor-map encoding.
        paths = ("auto", "cuda_cores") if tensor_cores else ("cuda_cores",)
        graphs = {}
        for path in paths:
            set_decode_path(path)
            side = torch.cuda.Stream(device)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                for _ in range(args.warmup):
                    gqa_decode(q, k, v)
            torch.cuda.current_stream(device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                gqa_decode(q, k, v)
            graphs[path] = graph
        runs = {"graph": lambda path: graphs[path].replay(), "call": lambda path: gqa_decode(q, k, v)}
        samples = {(p, r, st): [] for p in paths for r in runs for st in ("l2_flushed", "warm")}
        for state in ("l2_flushed", "warm"):
            for path in paths:
                set_decode_path(path)
                for _ in range(args.warmup):
                    gqa_decode(q, k, v)
                    graphs[path].replay()
            for _ in range(args.steps):
                for path in paths:
                    set_decode_path(path)
                    for run_name, run in runs.items():
                        if state == "l2_flushed":
                            flush.zero_()
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        run(path)
                        e1.record()
                        torch.cuda.synchronize(device)
                        samples[(path, run_name, state)].append(e0.elapsed_time(e1))
        set_decode_path("auto")
        del graphs
        for path in paths:
            med = {key[1:]: statistics.median(v) for key, v in samples.items() if key[0] == path}
            ms = med[("graph", "l2_flushed")]
            gbs = model.bytes_min / (ms * 1e-3) / 1e9
            kernel = "tensor cores (tcgen05)" if path == "auto" else "CUDA cores"
            print(json.dumps({
                "decode": "gqa", "kernel": kernel, "B": batch, "Hq": hq, "Hkv": hkv, "G": hq // hkv, "Dh": d,
                "L": seq,
                "dtype": "float16", "ms_l2_flushed": round(ms, 4), "ms_warm": round(med[("graph", "warm")], 4),
                "ms_call_l2_flushed": round(med[("call", "l2_flushed")], 4),
                "ms_call_warm": round(med[("call", "warm")], 4),
                "bytes_min": model.bytes_min, "gbs_of_bytes_min": round(gbs, 1),
                "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 3) if peaks.get("hbm_gbs") else None,
                "useful_tflops": round(model.flops_useful / (ms * 1e-3) / 1e12, 2),
                "intensity_min": round(model.intensity_min, 4),
                "timing": "CUDA events, median; ms_*: replay of a CUDA graph holding the public call (split + "
                          "combine kernels), ms_call_*: the eager public call (host work included)",
            }), flush=True)
        del q, k, v


def run_wide(args: argparse.Namespace) -> None:
    """Forward and backward for head dims above 128, 1 GPU, bf16.
    Each shape: ``--warmup`` calls, then ``--steps`` back-to-back calls timed
    with CUDA events on the launching stream (Q, K and V are 134-268 MB each,
    larger than L2).  FLOPs are the reference's model, 4·D per attended pair
    forward and 10·D backward; the backward is ``tk_attn_bwd_pre`` +
    ``tk_attn_bwd_fused`` + ``tk_attn_dq_convert`` with each kernel timed on
    its own; one JSON line per shape."""
    from tklab import _native
    from tklab.kernels.flash_attention import _NATIVE_DTYPE, _launch_forward, check_device_status

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak = _peaks().get("bf16_tflops")
    shapes = [(4, 16, 4096, 256), (2, 16, 8192, 256), (4, 16, 4096, 192)]
    causal_modes = (True, False)
    if args.shape:
        if len(args.shape) != 4:
            raise SystemExit("--wide --shape takes B,H,S,D")
        shapes, causal_modes = [tuple(args.shape)], (True,)
    for batch, heads, seq, d in shapes:
        for causal in causal_modes:
            q, k, v, _ = _make_inputs((batch, heads, seq, d), torch.bfloat16, 1.0, args.seed, device)
            o = torch.empty_like(q)
            lse = torch.empty((batch, heads, seq), dtype=torch.float32, device=device)
            for _ in range(args.warmup):
                _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
            e1.record()
            torch.cuda.synchronize(device)
            ms = e0.elapsed_time(e1) / args.steps
            tflops = fwd_flops(batch, heads, seq, d, causal) / (ms * 1e-3) / 1e12
            # Backward: three launches per call, each bracketed by events.
            lib = _native.load()
            do = torch.randn_like(q)
            delta = torch.empty_like(lse)
            dq_accum = torch.empty(q.shape, dtype=torch.float32, device=device)
            dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
            sp = int(torch.cuda.current_stream(device).cuda_stream)
            nd, scale, numel = _NATIVE_DTYPE[q.dtype], 1.0 / math.sqrt(d), q.numel()

            def backward(ev=None) -> None:
                if ev is not None:
                    ev[0].record()
                _native.check(lib.tk_attn_bwd_pre(o.data_ptr(), do.data_ptr(), delta.data_ptr(), dq_accum.data_ptr(),
                                                  batch, heads, seq, d, nd, sp), "bwd_pre")
                if ev is not None:
                    ev[1].record()
                _native.check(lib.tk_attn_bwd_fused(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                                    lse.data_ptr(), delta.data_ptr(), dq_accum.data_ptr(),
                                                    dk.data_ptr(), dv.data_ptr(), batch, heads, seq, d, nd,
                                                    int(causal), scale, sp), "bwd_fused")
                if ev is not None:
                    ev[2].record()
                _native.check(lib.tk_attn_dq_convert(dq_accum.data_ptr(), dq.data_ptr(), numel, nd, sp), "convert")
                if ev is not None:
                    ev[3].record()

            for _ in range(args.warmup):
                backward()
            torch.cuda.synchronize(device)
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
            for ev in evs:
                backward(ev)
            torch.cuda.synchronize(device)
            parts = [sum(ev[j].elapsed_time(ev[j + 1]) for ev in evs) / args.steps for j in range(3)]
            bwd_ms = sum(parts)
            bf = bwd_flops(batch, heads, seq, d, causal)
            print(json.dumps({
                "wide_head": True, "B": batch, "H": heads, "S": seq, "D": d, "causal": causal,
                "dtype": "bf16", "ms": round(ms, 4), "tflops": round(tflops, 1),
                "frac_of_measured_bf16": round(tflops / peak, 3) if peak else None,
                "kernel": "attn_fwd_d256_kernel (%d columns; D below it zero-filled)" % (192 if d <= 192 else 256),
                "bwd_ms": round(bwd_ms, 4), "bwd_tflops": round(bf / (bwd_ms * 1e-3) / 1e12, 1),
                "bwd_kernel_ms": {"attn_bwd_pre": round(parts[0], 4), "attn_bwd_d256": round(parts[1], 4),
                                  "dq_convert": round(parts[2], 4)},
                "bwd_fused_tflops": round(bf / (parts[1] * 1e-3) / 1e12, 1),
                "bwd_fused_frac_of_measured_bf16": round(bf / (parts[1] * 1e-3) / 1e12 / peak, 3) if peak else None,
            }), flush=True)
            del q, k, v, o, lse, do, delta, dq_accum, dq, dk, dv
    check_device_status()


def run_compare_sdpa(args: argparse.Namespace) -> None:
    """Context, not a target: torch's own SDPA (cuDNN's fused attention on
    this part) beside this library on the same inputs, 1 GPU.  For C3 and
    C2, and the reference's registered benchmark shape (B=1, H=16, D=64,
    fp16, S 2048 and 8192): forward and forward+backward through the public
    autograd API of each, CUDA events around each call after an L2 flush,
    medians of ``--steps`` calls; TFLOP/s under the reference's FLOP model.
    One JSON line per shape."""
    import torch.nn.functional as F

    from tklab.kernels.flash_attention import attention_causal, attention_noncausal, check_device_status

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    shapes = [("c3", CONFIGS["c3"]), ("c2", CONFIGS["c2"]),
              ("registered S=2048", (1, 16, 2048, 64, torch.float16, True, 1.0)),
              ("registered S=8192", (1, 16, 8192, 64, torch.float16, False, 1.0))]
    for name, (b, h, s, d, dtype, causal, qk_std) in shapes:
        q, k, v, do = _make_inputs((b, h, s, d), dtype, qk_std, args.seed, device)
        ours = attention_causal if causal else attention_noncausal

        def sdpa(x, y, z):
            return F.scaled_dot_product_attention(x, y, z, is_causal=causal)

        row = {"compare_sdpa": name, "B": b, "H": h, "S": s, "D": d, "causal": causal,
               "dtype": str(dtype).replace("torch.", "")}
        for label, fn in (("ours", ours), ("torch_sdpa", sdpa)):
            for mode in ("fwd", "fwd_bwd"):
                def call() -> None:
                    if mode == "fwd":
                        with torch.no_grad():
                            fn(q, k, v)
                    else:
                        qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))
                        out = fn(qg, kg, vg)
                        torch.autograd.grad(out, (qg, kg, vg), grad_outputs=do)

                for _ in range(args.warmup):
                    call()
                samples = []
                for _ in range(args.steps):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    call()
                    e1.record()
                    torch.cuda.synchronize(device)
                    samples.append(e0.elapsed_time(e1))
                ms = statistics.median(samples)
                flops = fwd_flops(b, h, s, d, causal) + (bwd_flops(b, h, s, d, causal) if mode == "fwd_bwd" else 0)
                row[f"{label}_{mode}_ms"] = round(ms, 4)
                row[f"{label}_{mode}_tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
        row["sdpa_backend_note"] = "torch F.scaled_dot_product_attention (cuDNN fused attention on B200)"
        print(json.dumps(row), flush=True)
        del q, k, v, do
    check_device_status()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=30)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--config", choices=tuple(CONFIGS), default="c3")
    parser.add_argument("--seed", type=int, default=0)
    # Enough timed steps that the pipeline's fill and drain (one extra
    # upload and download) weigh little against the steady-state rate.
    parser.add_argument("--e2e-steps", type=int, default=30)
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--bh", type=int, default=None,
                        help="(batch*head) slabs per rank instead of the config's (profiling only)")
    parser.add_argument("--traffic-bytes", type=float, default=None,
                        help="ncu dram bytes per launch of the dominant kernel, if captured")
    parser.add_argument("--sweep", action="store_true",
                        help="C5 sweep (fwd and bwd per dtype/causal/D/S), one JSON line per configuration")
    parser.add_argument("--decode", action="store_true",
                        help="GQA decode at the reference model's shapes, one JSON line per shape (1 GPU)")
    parser.add_argument("--rope", action="store_true",
                        help="fused RoPE attention vs plain and unfused, one JSON line per measurement (1 GPU)")
    parser.add_argument("--wide", action="store_true",
                        help="forward for head_dim 192/256 (the 256-column kernel), one JSON line per shape (1 GPU)")
    parser.add_argument("--compare-sdpa", action="store_true",
                        help="torch SDPA (cuDNN) beside this library at C3, C2 and the registered shape (1 GPU)")
    parser.add_argument("--shape", type=lambda t: [int(x) for x in t.split(",")], default=None,
                        help="one shape instead of the mode's list: --wide B,H,S,D (causal); --decode B,Hq,Hkv,Dh,L")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.sweep:
        run_sweep(args)
    elif args.rope:
        run_rope(args)
    elif args.decode:
        run_decode(args)
    elif args.wide:
        run_wide(args)
    elif args.compare_sdpa:
        run_compare_sdpa(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
