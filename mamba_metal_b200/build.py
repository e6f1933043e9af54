"""Builds libmamba_b200.so (all CUDA sources under csrc/) for sm_100a, in-tree.

Run as ``python -m mamba_metal_b200.build`` or call :func:`build`. The shared library is written to
``mamba_metal_b200/_lib/libmamba_b200.so`` so that it travels with the source tree; nothing is
installed into site-packages and no JIT cache is used.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
BUILD_DIR = PKG / "_build"
LIB_NAME = "libmamba_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libmamba_b200")


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), PKG.parent / "include" / "mamba_b200.h", Path(__file__)]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps if d.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every csrc/*.cu (in parallel) and links libmamba_b200.so; returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    objs = [BUILD_DIR / (s.stem + ".o") for s in sources]

    def compile_one(src: Path, obj: Path) -> str:
        if not force and not _stale(obj, src):
            return ""
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(PKG.parent / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for log in ex.map(compile_one, sources, objs):
            if verbose and log:
                print(log, file=sys.stderr)
    lib = lib_path()
    if force or not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
               *map(str, objs), "-o", str(tmp)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
