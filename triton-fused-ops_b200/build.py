"""Builds the sm_100a shared library ``triton_ops/_lib/libtfo_b200.so``.

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` only (no PTX
fallback, no other architecture) and linked into one shared library that
exports the C ABI declared in ``include/tfo_b200.h``. Objects are rebuilt only
when a source or header is newer than the library.

Usage: ``python build.py [--force] [--jobs N]``
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ_DIR = HERE / "_build"
LIB_DIR = HERE / "triton_ops" / "_lib"
LIB_PATH = LIB_DIR / "libtfo_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin/ on PATH")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _needs_build(force: bool) -> bool:
    if force or not LIB_PATH.exists():
        return True
    lib_m = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_m for p in _sources() + _headers() + [Path(__file__)])


def _compile(nvcc: str, src: Path, log_dir: Path) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    (log_dir / (src.stem + ".ptxas.txt")).write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr[-6000:]}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compiles and links the library if it is out of date; returns its path."""
    if not _needs_build(force):
        return LIB_PATH
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, OBJ_DIR), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        for s in srcs:
            print((OBJ_DIR / (s.stem + ".ptxas.txt")).read_text())
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    path = build(force=a.force, jobs=a.jobs, verbose=a.verbose)
    print(path)
    sys.exit(0)
