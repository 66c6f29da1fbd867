"""Builds the sm_100a shared library ``triton_ops/_lib/libtfo_b200.so`` and its PyTorch extension.

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` only (no PTX
fallback, no other architecture) and linked into one shared library that
exports the C ABI declared in ``include/tfo_b200.h``. ``csrc_ext/tfo_ext.cpp``
is then compiled against torch's headers into ``triton_ops/_lib/_tfo_ext*.so``
(linked to the library), the fast entry points for launch-latency-bound calls.
Each is rebuilt only when a source or header is newer than it.

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


EXT_SRC = HERE / "csrc_ext" / "tfo_ext.cpp"


def _ext_path() -> Path:
    import sysconfig

    return LIB_DIR / ("_tfo_ext" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False) -> Path:
    """Compiles the PyTorch extension (``_tfo_ext``) over the C ABI, linked to the library."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    out = _ext_path()
    deps = [EXT_SRC, LIB_PATH, INCLUDE / "tfo_b200.h", Path(__file__)]
    if not force and out.exists() and all(p.stat().st_mtime <= out.stat().st_mtime for p in deps):
        return out
    try:
        inc = ce.include_paths(device_type="cuda")
    except TypeError:  # older torch
        inc = ce.include_paths(cuda=True)
    torch_lib = ce.library_paths()[0]
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_tfo_ext", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for i in [*inc, sysconfig.get_paths()["include"], str(INCLUDE)]:
        cmd += ["-I", i]
    tmp = out.with_suffix(".tmp")
    cmd += [str(EXT_SRC), "-o", str(tmp), "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-ltorch_python", "-L", str(LIB_DIR), "-ltfo_b200", "-Wl,-rpath,$ORIGIN",
            f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"extension build failed:\n{res.stderr[-6000:]}")
    os.replace(tmp, out)
    return out


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compiles and links the library (and then the extension) if out of date; returns the library's path."""
    _build_lib(force, jobs, verbose)
    build_ext(force)
    return LIB_PATH


def _build_lib(force: bool, jobs: int | None, verbose: bool) -> Path:
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
