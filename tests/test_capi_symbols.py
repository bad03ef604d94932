"""CPU: the C-ABI library loads and exports every entry point of include/tklab_attn.h.

Only calls that return before touching a GPU are made here (argument
validation and pure size arithmetic).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tklab import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "tklab_attn.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^TK_API\s+[\w\s\*]+?\b(tk_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_documented_entry_points() -> None:
    declared = _declared()
    assert {"tk_attn_fwd", "tk_attn_bwd_pre", "tk_attn_bwd"} <= declared
    assert declared == set(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol() -> None:
    lib = _native.load()
    for name in _declared():
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr), name


def test_workspace_size_arithmetic() -> None:
    lib = _native.load()
    assert lib.tk_attn_bwd_workspace_bytes(8, 32, 4096, 128) == 8 * 32 * 4096 * 128 * 4
    assert lib.tk_attn_bwd_workspace_bytes(0, 32, 4096, 128) == 0


@pytest.mark.parametrize(
    ("kwargs", "status"),
    [
        ({"q": None}, 1),
        ({"head_dim": 100}, 2),
        ({"head_dim": 260}, 2),
        ({"head_dim": 264}, 2),
        ({"dtype": 7}, 2),
        ({"seq": 0}, 1),
        ({"batch": -1}, 1),
        ({"scale": 0.0}, 1),
        ({"q": 0x1008}, 3),
    ],
)
def test_forward_rejects_bad_arguments_before_launch(kwargs: dict, status: int) -> None:
    args = {"q": 0x1000, "k": 0x2000, "v": 0x3000, "o": 0x4000, "lse": None, "batch": 1, "heads": 2,
            "seq": 128, "head_dim": 64, "dtype": 0, "causal": 0, "scale": 0.125, "stream": None}
    args.update(kwargs)
    assert _native.load().tk_attn_fwd(*args.values()) == status


@pytest.mark.parametrize(
    ("kwargs", "status"),
    [
        ({"q": None}, 1),
        ({"head_dim": 100}, 2),
        ({"scale": float("nan")}, 1),
        ({"o": 0x4004}, 3),
        ({"workspace": 0x5010, "ws_bytes": 4096}, 3),  # scratch must be 256-byte aligned
    ],
)
def test_forward_with_scratch_rejects_bad_arguments_before_launch(kwargs: dict, status: int) -> None:
    args = {"q": 0x1000, "k": 0x2000, "v": 0x3000, "o": 0x4000, "lse": None, "batch": 1, "heads": 2,
            "seq": 128, "head_dim": 64, "dtype": 0, "causal": 0, "scale": 0.125, "workspace": None,
            "ws_bytes": 0, "stream": None}
    args.update(kwargs)
    assert _native.load().tk_attn_fwd_ws(*args.values()) == status


def test_forward_scratch_size_of_invalid_shapes_is_zero() -> None:
    lib = _native.load()
    assert lib.tk_attn_fwd_workspace_bytes(0, 2, 8192, 128, 1, 1) == 0
    assert lib.tk_attn_fwd_workspace_bytes(1, 2, 8192, 100, 1, 1) == 0
    assert lib.tk_attn_fwd_workspace_bytes(1, 2, 8192, 128, 7, 1) == 0


@pytest.mark.parametrize("head_dim", [136, 256])
def test_deterministic_backward_rejects_wide_heads(head_dim: int) -> None:
    """136..256 have a default backward only: the deterministic entries refuse them as unsupported."""
    lib = _native.load()
    p = 0x1000
    assert lib.tk_attn_bwd_deterministic(p, p, p, p, p, p, p, p, p, p, 1, 2, 128, head_dim, 0, 0, 0.125, None) == 2
    assert lib.tk_attn_bwd_dkdv(p, p, p, p, p, p, p, p, 1, 2, 128, head_dim, 0, 0, 0.125, None) == 2
    assert lib.tk_attn_bwd_dq(p, p, p, p, p, p, p, 1, 2, 128, head_dim, 0, 0, 0.125, None) == 2


@pytest.mark.parametrize("head_dim", [100, 264])
def test_backward_rejects_unsupported_widths(head_dim: int) -> None:
    lib = _native.load()
    p = 0x1000
    assert lib.tk_attn_bwd_pre(p, p, p, p, 1, 2, 128, head_dim, 0, None) == 2
    assert lib.tk_attn_bwd(p, p, p, p, p, p, p, p, p, p, 1, 2, 128, head_dim, 0, 0, 0.125, None) == 2


def test_backward_rejects_missing_workspace() -> None:
    lib = _native.load()
    rc = lib.tk_attn_bwd(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000, None, 0x7000, 0x8000, 0x9000,
                         1, 2, 128, 64, 0, 1, 0.125, None)
    assert rc == 1


def test_status_strings() -> None:
    assert _native.status_string(0) == "ok"
    assert _native.status_string(6) == "device wait timed out"
    assert _native.status_string(6 | (3 << 8)) == "device wait timed out"
    with pytest.raises(RuntimeError, match="wait site 3"):
        _native.check(6 | (3 << 8), "probe")


@pytest.mark.parametrize(
    ("kwargs", "status"),
    [
        ({"dq": 0x9008}, 3),
        ({"q": 0x1004}, 3),
        ({"lse": 0x6002}, 3),
        ({"scale": float("nan")}, 1),
        ({"scale": -1.0}, 1),
        ({"dtype": 5}, 2),
        ({"head_dim": 96}, 2),
        ({"dv": None}, 1),
        ({"seq": 1 << 20, "heads": 32}, 8),
    ],
)
def test_noalloc_backward_checks_every_argument_before_touching_the_device(kwargs: dict, status: int) -> None:
    """Refusals come back from host checks alone (no GPU here), so a refused
    call can never launch work or disturb the shared scratch of a call still
    running."""
    args = {"q": 0x1000, "k": 0x2000, "v": 0x3000, "o": 0x4000, "do": 0x5000, "lse": 0x6000, "dq": 0x7000,
            "dk": 0x8000, "dv": 0x9000, "batch": 1, "heads": 2, "seq": 128, "head_dim": 64, "dtype": 0,
            "causal": 1, "scale": 0.125, "stream": None}
    args.update(kwargs)
    assert _native.load().tk_attn_bwd_noalloc(*args.values()) == status


def test_out_of_memory_status_string() -> None:
    assert _native.status_string(9) == "device memory could not be committed"
