"""CPU: the host side of the forward's key-split schedule.

The attention library's launcher counts the units (CTAs) of a split forward
from its plan, and each CTA of the kernel decodes its own unit index into
(slab, query-tile group, chunk).  Both run the code of
``csrc/attn_fwd_split_plan.h``, which the test-only self-test library
compiles too and exposes on the host (``tk_selftest_fwd_split_plan``,
``tk_selftest_fwd_split_decode``).  These tests walk every unit of many
plans on the CPU and check that the walk enumerates each chunk of each
query-tile group exactly once, that the chunks of a group tile its key range
``[0, n_a)`` (tile A's key tiles: ``kT * ct + 1`` under a causal mask, all of
them otherwise), that the merge kernel's first row is the first row of a
group with several chunks, and that the workspace size matches the layout
the kernel writes.  No GPU is used.
"""

from __future__ import annotations

import ctypes
import itertools
import random

import pytest

from conftest import load_selftest_lib

SMS = 148  # B200
TILE = 128


@pytest.fixture(scope="module")
def lib():
    return load_selftest_lib()


def _plan(lib, bh, s, d, causal, sms=SMS):
    out = (ctypes.c_int64 * 6)()
    if not lib.tk_selftest_fwd_split_plan(bh, s, d, int(causal), sms, out):
        return None
    split_l, cmax, units, row0, nbytes, kt = (int(x) for x in out)
    return {"L": split_l, "cmax": cmax, "units": units, "row0": row0, "bytes": nbytes, "kT": kt}


def _decode(lib, u, bh, n_ctiles, causal, kt, split_l):
    out = (ctypes.c_int * 3)()
    lib.tk_selftest_fwd_split_decode(u, bh, n_ctiles, int(causal), kt, split_l, out)
    return tuple(int(x) for x in out)


def _check_plan(lib, bh, s, d, causal, plan) -> None:
    kt, L, cmax = plan["kT"], plan["L"], plan["cmax"]
    width = 64 if d <= 64 else 128
    assert kt == (1 if d <= 64 else 2)
    n_ctiles = -(-s // (kt * TILE))
    n_ntiles = -(-s // TILE)

    def n_a(ct):
        return min(kt * ct + 1, n_ntiles) if causal else n_ntiles

    assert 2 <= cmax <= 32 and L >= 12
    assert cmax == -(-max(n_a(ct) for ct in range(n_ctiles)) // L)
    seen = set()
    for u in range(plan["units"]):
        b, ct, c = _decode(lib, u, bh, n_ctiles, causal, kt, L)
        assert 0 <= b < bh and 0 <= ct < n_ctiles and 0 <= c < cmax, (u, b, ct, c)
        assert c * L < n_a(ct), ("empty chunk", u, b, ct, c)
        assert (b, ct, c) not in seen, ("unit decoded twice", u, b, ct, c)
        seen.add((b, ct, c))
    # Every group's chunks are exactly 0 .. ceil(n_a / L) - 1: together they
    # cover [0, n_a) once.
    expected = {(b, ct, c) for b in range(bh) for ct in range(n_ctiles) for c in range(-(-n_a(ct) // L))}
    assert seen == expected
    # The merge starts at the first row of the first group with two chunks.
    multi = [ct for ct in range(n_ctiles) if n_a(ct) > L]
    assert multi and plan["row0"] == multi[0] * kt * TILE
    assert all(n_a(ct) <= L for ct in range(multi[0]))
    part = bh * cmax * s * width * 4
    assert plan["bytes"] == -(-part // 256) * 256 + bh * cmax * s * 4


# The shapes tests/test_forward_split.py runs on the GPU, which must split.
GPU_SPLIT_CASES = [
    (2, 8192, 128, True), (2, 16384, 128, True), (2, 16384, 64, True), (1, 16384, 128, False),
    (2, 8000, 96, True), (1, 7000, 64, False), (1, 12300, 128, True), (1, 7000, 40, True), (2, 8192, 72, False),
]


@pytest.mark.parametrize("case", GPU_SPLIT_CASES, ids=lambda c: "bh{}-s{}-d{}-{}".format(*c[:3], "causal" if c[3] else "full"))
def test_gpu_test_shapes_split_and_enumerate(lib, case) -> None:
    bh, s, d, causal = case
    plan = _plan(lib, bh, s, d, causal)
    assert plan is not None
    _check_plan(lib, bh, s, d, causal, plan)


@pytest.mark.parametrize(
    "case",
    [
        (256, 4096, 128, True),   # C3: thousands of query tiles
        (32, 16384, 128, True),   # C4 on one GPU
        (4, 16384, 128, True),    # C4's 4 heads per GPU: only mildly underfilled
        (8, 4096, 128, True),     # longest item 31 key tiles
        (1, 1024, 128, True),     # short sequence
        (64, 1024, 64, False),    # C2
        (16, 16384, 128, True),   # C5 S=16384 on one GPU
    ],
    ids=lambda c: "bh{}-s{}-d{}-{}".format(*c[:3], "causal" if c[3] else "full"),
)
def test_filled_problems_are_not_split(lib, case) -> None:
    assert _plan(lib, *case) is None


def test_head_dim_above_128_is_not_split(lib) -> None:
    assert _plan(lib, 1, 16384, 192, True) is None
    assert _plan(lib, 1, 16384, 256, True) is None


def test_random_shapes_enumerate_every_chunk_once(lib) -> None:
    rng = random.Random(0)
    checked = 0
    for _ in range(400):
        bh = rng.choice([1, 1, 2, 2, 3, 4, 6, 8])
        s = rng.randrange(1, 48) * 512 + rng.randrange(0, 128)
        d = rng.choice([8, 40, 64, 72, 96, 128])
        causal = rng.random() < 0.6
        plan = _plan(lib, bh, s, d, causal)
        if plan is not None:
            _check_plan(lib, bh, s, d, causal, plan)
            checked += 1
    assert checked >= 50


def test_other_sm_counts(lib) -> None:
    for sms, (bh, s, d, causal) in itertools.product((132, 148, 160), GPU_SPLIT_CASES[:4]):
        plan = _plan(lib, bh, s, d, causal, sms=sms)
        if plan is not None:
            _check_plan(lib, bh, s, d, causal, plan)
