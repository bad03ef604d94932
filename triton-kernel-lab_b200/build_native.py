"""Build ``libtklab_attn.so`` (the sm_100a attention kernels and their C ABI).

The library is compiled in-tree with nvcc for ``sm_100a`` only and placed at
``tklab/_lib/libtklab_attn.so`` next to the Python package that loads it, so
it travels with the source tree.  A second, test-only library,
``tklab/_lib/libtklab_selftest.so`` (``csrc/selftest/``: probes of the
tcgen05 operand forms and of the FMA-pipe exponential), is built beside it;
only the tests load it.  Run ``python build_native.py`` or call
:func:`build`.  Each library is rebuilt only when one of its sources or
headers is newer than it, unless ``force`` is set.
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
SELFTEST_DIR = CSRC / "selftest"
SELFTEST_LIB_PATH = LIB_DIR / "libtklab_selftest.so"

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


def sources(src_dir: Path = CSRC) -> list[Path]:
    """Return every CUDA translation unit of the library built from ``src_dir``."""
    return sorted(src_dir.glob("*.cu"))


def _deps(src_dir: Path) -> list[Path]:
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    if src_dir != CSRC:
        headers += sorted(src_dir.glob("*.h"))
    return sources(src_dir) + headers


def _stale(src_dir: Path, lib_path: Path) -> bool:
    if not lib_path.exists():
        return True
    lib_mtime = lib_path.stat().st_mtime
    return any(dep.stat().st_mtime > lib_mtime for dep in _deps(src_dir))


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def _build_one(src_dir: Path, lib_path: Path, obj_dir: Path, force: bool, verbose: bool, ptxas_info: bool) -> Path:
    if not force and not _stale(src_dir, lib_path):
        return lib_path
    nvcc = _nvcc()
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    srcs = sources(src_dir)

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *CXX_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        return obj, _run(cmd, verbose)

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        results = list(pool.map(compile_one, srcs))
    if ptxas_info:
        for _, log in results:
            print(log)
    objs = [str(obj) for obj, _ in results]
    tmp = lib_path.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs], verbose)
    os.replace(tmp, lib_path)
    return lib_path


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link the attention library and the test-only library; return the former's path."""
    _build_one(CSRC, LIB_PATH, BUILD_DIR, force, verbose, ptxas_info)
    _build_one(SELFTEST_DIR, SELFTEST_LIB_PATH, BUILD_DIR / "selftest", force, verbose, ptxas_info)
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
