"""Build ``libtklab_attn.so`` (the sm_100a attention kernels and their C ABI).

The library is compiled in-tree with nvcc for ``sm_100a`` only and placed at
``tklab/_lib/libtklab_attn.so`` next to the Python package that loads it, so
it travels with the source tree.  Run ``python build_native.py`` or call
:func:`build`.  Rebuilds only when a source or header is newer than the
library unless ``force`` is set.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD_DIR = ROOT / "_build"
LIB_DIR = ROOT / "tklab" / "_lib"
LIB_PATH = LIB_DIR / "libtklab_attn.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def _nvcc() -> str:
    nvcc = shutil.which("nvcc")
    if nvcc is None:
        cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
        candidate = Path(cuda_home) / "bin" / "nvcc"
        if not candidate.exists():
            raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
        nvcc = str(candidate)
    return nvcc


def sources() -> list[Path]:
    """Return every CUDA translation unit of the library."""
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(dep.stat().st_mtime > lib_mtime for dep in _deps())


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link the library; return its path."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *CXX_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        return obj, _run(cmd, verbose)

    with ThreadPoolExecutor(max_workers=min(8, len(sources()))) as pool:
        results = list(pool.map(compile_one, sources()))
    if ptxas_info:
        for _, log in results:
            print(log)
    objs = [str(obj) for obj, _ in results]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs], verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = parser.parse_args()
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)


if __name__ == "__main__":
    main()
