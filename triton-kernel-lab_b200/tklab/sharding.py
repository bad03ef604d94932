"""(batch, head) sharding of the attention path across ranks.

Every (batch, head) pair is independent in the forward and the backward, so
N ranks split the flattened ``B*H`` axis into contiguous slabs and run the
kernels on their own slab with no collective on the data path.  Contiguous
slabs of a contiguous ``(B, H, S, D)`` tensor are contiguous in memory, so a
slab is a zero-copy view.

Failure detection is host-side: between steps, :func:`check_ranks_alive`
has every rank report in on a gloo group within a short timeout, so a rank
that raised, exited or never joined is named by the survivors (as a
``RuntimeError``) before their next launch instead of leaving them blocked
in a collective.  The reference has no multi-rank path; its only liveness
check is the single-GPU busy preflight (``src/tklab/cli.py:127-135``).
"""

from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist


def slab_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Half-open range of flattened (batch*head) indices owned by ``rank``.

    The first ``total % world`` ranks take one extra slab, so any ``total``
    splits and the ranges tile ``[0, total)`` in rank order.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if total < 0:
        raise ValueError("total must be non-negative")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def slab_view(tensor: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's slab of a contiguous (B, H, ...) tensor, as a (1, slab, ...) view."""
    if not tensor.is_contiguous():
        raise ValueError("slab_view needs a contiguous tensor")
    flat = tensor.reshape(tensor.shape[0] * tensor.shape[1], *tensor.shape[2:])
    start, stop = slab_range(flat.shape[0], world, rank)
    return flat[start:stop].unsqueeze(0)


def liveness_group() -> dist.ProcessGroup | None:
    """A gloo group over all ranks for :func:`check_ranks_alive` (collective: every rank calls it).

    Returns ``None`` when the default group already uses gloo (it is used
    directly then).
    """
    if dist.get_backend() == "gloo":
        return None
    return dist.new_group(backend="gloo")


def check_ranks_alive(group: dist.ProcessGroup | None = None, timeout_s: float = 10.0) -> None:
    """Every rank of ``group`` reports in within ``timeout_s`` seconds, or this raises.

    Call it between steps, with no kernel or collective of this rank in
    flight; every rank must call it at the same point.  Rank 0 waits for the
    others and raises ``RuntimeError`` naming every rank that did not
    report; the other ranks raise once rank 0 has not answered in time.

    Raises:
        RuntimeError: If a rank is missing (the message lists it).
    """
    if timeout_s <= 0:
        raise ValueError("timeout_s must be positive")
    try:
        dist.monitored_barrier(group=group, timeout=timedelta(seconds=timeout_s), wait_all_ranks=True)
    except RuntimeError as error:
        raise RuntimeError(f"rank liveness check failed on rank {dist.get_rank()}: {error}") from error
