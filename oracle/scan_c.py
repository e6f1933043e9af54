"""ctypes binding of the C oracle scan (oracle/scan_ref.c). TEST INFRASTRUCTURE ONLY."""

from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle.build import build

_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        f = _lib.mm_ref_selective_scan
        f.restype = None
        f.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int]
        _lib.mm_ref_max_threads.restype = ctypes.c_int
    return _lib


def max_threads() -> int:
    return int(_load().mm_ref_max_threads())


def selective_scan_c(u, delta, A, B, C, D=None, z=None, delta_softplus=False, threads=0):
    """Returns (y, last_state) as float32 arrays; inputs are converted to contiguous float32."""
    lib = _load()
    f32 = lambda a: None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u, delta, A, B, C, D, z = map(f32, (u, delta, A, B, C, D, z))
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    assert dstate <= 64
    y = np.empty_like(u)
    last = np.empty((batch, dim, dstate), dtype=np.float32)
    ptr = lambda a: None if a is None else a.ctypes.data
    lib.mm_ref_selective_scan(ptr(u), ptr(delta), ptr(A), ptr(B), ptr(C), ptr(D), ptr(z), ptr(y), ptr(last),
                              batch, dim, dstate, seqlen, int(bool(delta_softplus)),
                              int(threads or os.cpu_count() or 1))
    return y, last
