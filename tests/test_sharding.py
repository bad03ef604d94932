"""CPU: the multi-rank host logic of the sharded attention path (gloo, world_size 2).

Each rank takes its (batch*head) slab, computes attention on it (the CPU
oracle stands in for the kernels here), and the gathered slabs must equal
the unsharded result; the timing reduction is the MAX over ranks.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tklab.sharding import slab_range, slab_view


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
