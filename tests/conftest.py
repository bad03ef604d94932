"""Shared pytest configuration.

Puts the package directory (``triton-kernel-lab_b200``, holding ``tklab``) and
the repository root (holding ``oracle``) on ``sys.path`` — the equivalent of
the reference's ``pythonpath = ["src", "."]`` — and registers the markers.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for entry in (ROOT / "triton-kernel-lab_b200", ROOT):
    if str(entry) not in sys.path:
        sys.path.insert(0, str(entry))

GOLDEN_DIR = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: requires a CUDA GPU (B200, sm_100a)")


SELFTEST_LIB = ROOT / "triton-kernel-lab_b200" / "tklab" / "_lib" / "libtklab_selftest.so"


def load_selftest_lib():
    """ctypes handle of the test-only probe library (declared in csrc/selftest/tklab_selftest.h)."""
    import ctypes

    if not SELFTEST_LIB.exists():
        raise RuntimeError(f"{SELFTEST_LIB.name} is not built: run triton-kernel-lab_b200/build_native.py")
    lib = ctypes.CDLL(str(SELFTEST_LIB))
    vp, c_int = ctypes.c_void_p, ctypes.c_int
    lib.tk_selftest_umma.restype = c_int
    lib.tk_selftest_umma.argtypes = [vp, vp, vp, c_int, c_int, c_int, vp]
    lib.tk_selftest_exp2_fma.restype = c_int
    lib.tk_selftest_exp2_fma.argtypes = [vp, vp, ctypes.c_int64, vp]
    lib.tk_selftest_status.restype = c_int
    lib.tk_selftest_status.argtypes = [ctypes.POINTER(c_int), vp]
    i64 = ctypes.c_int64
    lib.tk_selftest_fwd_split_plan.restype = c_int
    lib.tk_selftest_fwd_split_plan.argtypes = [i64, i64, i64, c_int, c_int, ctypes.POINTER(i64)]
    lib.tk_selftest_fwd_split_decode.restype = None
    lib.tk_selftest_fwd_split_decode.argtypes = [c_int, c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)]
    return lib


def selftest_status(lib, stream: int) -> int:
    """Synchronise ``stream`` and read-and-clear the probe library's device status word."""
    import ctypes

    out = ctypes.c_int(0)
    rc = lib.tk_selftest_status(ctypes.byref(out), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"tk_selftest_status failed with status {rc}")
    return int(out.value)


def golden_cases(*, rope: bool = False) -> list[str]:
    """Names of the committed golden fixtures: plain attention, or (``rope``) the fused-RoPE cases."""
    names = sorted(path.stem for path in GOLDEN_DIR.glob("*.npz"))
    return [name for name in names if name.startswith("rope_") == rope]


def load_golden(name: str) -> dict[str, object]:
    """Load one fixture: 16-bit tensors are rebuilt bit-exactly from their stored bits."""
    import torch

    with np.load(GOLDEN_DIR / f"{name}.npz") as data:
        raw = {key: data[key] for key in data.files}
    dtype = getattr(torch, str(raw.pop("dtype")))
    out: dict[str, object] = {
        "dtype": dtype,
        "causal": bool(raw.pop("causal")),
        "seed": int(raw.pop("seed")),
    }
    for key, value in raw.items():
        if key.endswith("_bits"):
            base = key[: -len("_bits")]
            bits = torch.from_numpy(value.view(np.int16).copy())
            tensor_dtype = dtype if base in ("q", "k", "v", "do") else torch.float16
            out[base] = bits.view(tensor_dtype)
        else:
            out[key] = torch.from_numpy(value.copy())
    return out
