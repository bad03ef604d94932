"""(batch, head) sharding of the attention path across ranks.

Every (batch, head) pair is independent in the forward and the backward, so
N ranks split the flattened ``B*H`` axis into contiguous slabs and run the
kernels on their own slab with no collective on the data path.  Contiguous
slabs of a contiguous ``(B, H, S, D)`` tensor are contiguous in memory, so a
slab is a zero-copy view.
"""

from __future__ import annotations

import torch


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
