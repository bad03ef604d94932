"""Signed-int32 offset guard for attention launchers.

The reference rejects any tensor whose largest element offset does not fit a
signed 32-bit integer (``src/tklab/harness/addressing.py:14-48``) because its
Triton kernels index with int32 arithmetic.  The sm_100a kernels address
through TMA coordinates and 64-bit offsets, but the same guard and message are
kept so the drop-in rejects exactly what the reference rejects.
"""

from __future__ import annotations

import torch

MAX_INT32_OFFSET = 2**31 - 1


def max_relative_offset(tensor: torch.Tensor) -> int:
    """Largest element displacement reachable inside ``tensor``.

    Computed as the sum over dimensions of ``(size - 1) * |stride|``; an empty
    tensor has no reachable element and reports 0.
    """
    if tensor.numel() == 0:
        return 0
    total = 0
    for size, stride in zip(tensor.shape, tensor.stride(), strict=True):
        total += (size - 1) * abs(stride)
    return total


def assert_int32_addressable(tensor: torch.Tensor, *, name: str) -> None:
    """Raise ``ValueError`` when ``tensor`` spans more than ``MAX_INT32_OFFSET``."""
    # A contiguous tensor's largest displacement is numel - 1 (the same sum).
    reach = tensor.numel() - 1 if tensor.is_contiguous() and tensor.numel() > 0 else max_relative_offset(tensor)
    if reach > MAX_INT32_OFFSET:
        raise ValueError(f"{name} strides exceed the signed int32 offset range")
