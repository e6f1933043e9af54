"""Compiles the C oracle (oracle/scan_ref.c) into oracle/_build/libscanref.so with gcc + OpenMP.

TEST INFRASTRUCTURE ONLY. The reference itself (Python + Metal Shading Language, run through MLX) has
no C/C++ path that could be compiled here, so there is no oracle/_ref build: this restatement is the
compiled oracle.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "scan_ref.c"
OUT = HERE / "_build" / "libscanref.so"


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if force or not OUT.exists() or SRC.stat().st_mtime > OUT.stat().st_mtime:
        cmd = ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11", str(SRC), "-o", str(OUT), "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"gcc failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force=True))
