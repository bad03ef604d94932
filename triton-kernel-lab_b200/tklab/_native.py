"""ctypes binding of ``libtklab_attn.so`` (the C ABI in ``include/tklab_attn.h``).

The library is loaded once per process.  There is no fallback: if the shared
object is missing every attention call raises, so a GPU run can never pass on
some other implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtklab_attn.so"

TK_DTYPE_F16 = 0
TK_DTYPE_BF16 = 1

TK_OK = 0
TK_ERR_DEVICE_TIMEOUT = 6

# Every symbol declared in include/tklab_attn.h, with (restype, argtypes).
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tk_attn_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp],
    ),
    "tk_attn_fwd_ws": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            _vp, ctypes.c_size_t, _vp,
        ],
    ),
    "tk_attn_fwd_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int]),
    "tk_attn_bwd_pre": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, _vp],
    ),
    "tk_attn_bwd": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp,
        ],
    ),
    "tk_attn_bwd_fused": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp,
        ],
    ),
    "tk_attn_dq_convert": (ctypes.c_int, [_vp, _vp, _i64, ctypes.c_int, _vp]),
    "tk_attn_bwd_noalloc": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp,
        ],
    ),
    "tk_attn_bwd_dkdv": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp],
    ),
    "tk_attn_bwd_dq": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp],
    ),
    "tk_attn_bwd_deterministic": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp,
        ],
    ),
    "tk_attn_fwd_rope": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp],
    ),
    "tk_rope_rotate": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tk_attn_dq_convert_rope": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int, _vp],
    ),
    "tk_gqa_decode_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64]),
    "tk_gqa_decode": (
        ctypes.c_int,
        [
            _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t,
            _i64, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_float, _vp,
        ],
    ),
    "tk_gqa_decode_set_path": (ctypes.c_int, [ctypes.c_int]),
    "tk_attn_bwd_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64]),
    "tk_attn_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), _vp]),
    "tk_attn_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_ulonglong]),
    "tk_attn_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_ulonglong, _vp]),
    "tk_attn_status_string": (ctypes.c_char_p, [ctypes.c_int]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library (once) and declare every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built: run `python triton-kernel-lab_b200/build_native.py` "
                "(or __graft_entry__.build()) before using the attention kernels"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def status_string(status: int) -> str:
    """Return the library's name for a status code."""
    raw = load().tk_attn_status_string(int(status))
    return raw.decode() if raw else "unknown status"


def check(status: int, what: str) -> None:
    """Raise ``RuntimeError`` for a non-zero status returned by ``what``."""
    if status != TK_OK:
        site = status >> 8
        where = f", wait site {site}" if site else ""
        raise RuntimeError(f"{what} failed: {status_string(status)} (status {status}{where})")


def device_status(stream: int) -> int:
    """Synchronise ``stream`` and read-and-clear the device status word."""
    out = ctypes.c_int(0)
    check(load().tk_attn_device_status(ctypes.byref(out), ctypes.c_void_p(stream)), "tk_attn_device_status")
    return int(out.value)
