"""CPU: the FLOP model and benchmark metadata (reference ``tests/test_bench.py:46-56``)."""

from __future__ import annotations

import torch

from tklab.kernels.flash_attention import ATTENTION_CAUSAL, ATTENTION_NONCAUSAL, attention_pairs


def test_attention_flops_use_full_and_lower_triangular_pair_counts() -> None:
    assert ATTENTION_NONCAUSAL.flops is not None
    assert ATTENTION_CAUSAL.flops is not None
    sequence_length = 8
    fixed_factor = 4 * 1 * 16 * 64
    assert ATTENTION_NONCAUSAL.flops(sequence_length, torch.float16) == fixed_factor * sequence_length**2
    assert ATTENTION_CAUSAL.flops(sequence_length, torch.float16) == fixed_factor * 36


def test_pairs() -> None:
    assert attention_pairs(4096, causal=True) == 4096 * 4097 // 2
    assert attention_pairs(4096, causal=False) == 4096**2


def test_metadata_keys_match_the_reference_rows() -> None:
    assert ATTENTION_CAUSAL.benchmark_metadata is not None
    meta = ATTENTION_CAUSAL.benchmark_metadata(1024, torch.float16)
    assert set(meta) == {"block_m", "block_n", "num_warps", "num_stages", "heads", "head_dim", "causal"}
    assert meta["causal"] is True and meta["block_m"] == 128
