"""CPU: the multi-rank host logic of the sharded attention path (gloo).

Each rank takes its (batch*head) slab, computes attention on it (the CPU
oracle stands in for the kernels here), and the gathered slabs must equal
the unsharded result; the timing reduction is the MAX over ranks.  A
failure test makes one rank leave between steps (it exits without another
collective) and checks that the survivors' liveness check names it within a
bounded time and that the parent sees every process end.
"""

from __future__ import annotations

import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tklab.sharding import check_ranks_alive, slab_range, slab_view


def test_slab_ranges_tile_the_axis() -> None:
    for total in (1, 7, 256, 257):
        for world in (1, 2, 3, 8):
            ranges = [slab_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        slab_range(8, 2, 2)


def test_slab_view_is_zero_copy() -> None:
    x = torch.arange(2 * 4 * 3 * 2, dtype=torch.float32).reshape(2, 4, 3, 2)
    v = slab_view(x, 2, 1)
    assert v.shape == (1, 4, 3, 2)
    assert v.data_ptr() == x.reshape(8, 3, 2)[4].data_ptr()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, root: str, out: dict) -> None:
    sys.path[:0] = [str(Path(root) / "triton-kernel-lab_b200"), root]
    from oracle.attention_oracle import manual_forward_lse
    from tklab.sharding import slab_view as view

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(3)
        q, k, v = (torch.randn(2, 3, 40, 64, generator=gen) for _ in range(3))
        o, _ = manual_forward_lse(view(q, world, rank), view(k, world, rank), view(v, world, rank), causal=True)
        pieces = [None] * world
        dist.all_gather_object(pieces, o)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full, _ = manual_forward_lse(q, k, v, causal=True)
            gathered = torch.cat([p.squeeze(0) for p in pieces], dim=0).reshape(full.shape)
            out["max_err"] = float((gathered - full).abs().max())
            out["t_max"] = float(t.item())
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shards_match_unsharded() -> None:
    root = str(Path(__file__).resolve().parents[1])
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_worker, args=(2, _free_port(), root, out), nprocs=2, start_method="spawn")
        assert out["max_err"] == 0.0
        assert out["t_max"] == 2.0


def _leaving_worker(rank: int, world: int, port: int, root: str, leaver: int, out: dict) -> None:
    sys.path[:0] = [str(Path(root) / "triton-kernel-lab_b200"), root]
    from tklab.sharding import check_ranks_alive as alive

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    # Step 1: everybody present.
    alive(timeout_s=5.0)
    t = torch.tensor([float(rank)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == leaver:
        out[f"left{rank}"] = True
        os._exit(0)  # leaves between steps: nothing of this rank in flight
    # Step 2: the survivors must learn of the departure before launching anything.
    start = time.monotonic()
    try:
        alive(timeout_s=2.0)
        out[f"rank{rank}"] = "no error"
    except RuntimeError as error:
        out[f"rank{rank}"] = str(error)
    out[f"seconds{rank}"] = time.monotonic() - start
    os._exit(0)


def test_a_rank_that_leaves_between_steps_is_reported_not_waited_for() -> None:
    root = str(Path(__file__).resolve().parents[1])
    world, leaver = 3, 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_leaving_worker, args=(rank, world, port, root, leaver, out)) for rank in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive_procs = [p for p in procs if p.is_alive()]
        for p in alive_procs:
            p.kill()
        assert not alive_procs, "a survivor blocked instead of reporting the missing rank"
        assert out.get(f"left{leaver}") is True
        assert "2" in out["rank0"] and "liveness check failed on rank 0" in out["rank0"], out["rank0"]
        assert out["rank1"].startswith("rank liveness check failed on rank 1"), out["rank1"]
        assert out["seconds0"] < 30 and out["seconds1"] < 30


def test_liveness_check_passes_with_every_rank_present() -> None:
    root = str(Path(__file__).resolve().parents[1])
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_leaving_worker, args=(rank, 2, port, root, -1, out)) for rank in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(not p.is_alive() for p in procs)
        assert out["rank0"] == "no error" and out["rank1"] == "no error"


def test_liveness_timeout_must_be_positive() -> None:
    with pytest.raises(ValueError):
        check_ranks_alive(timeout_s=0)
