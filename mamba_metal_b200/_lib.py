"""ctypes binding of libmamba_b200.so (the C-ABI declared in include/mamba_b200.h).

The library is built in-tree by ``mamba_metal_b200.build`` (``mamba_metal_b200/_lib/libmamba_b200.so``).
There is no CPU or PyTorch fallback: a missing library, a CPU tensor or a non-zero status code raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

# MAMBA_B200_LIB selects another build of the same library (e.g. a variant compiled with different
# launch bounds); by default the in-tree build is loaded.
LIB_PATH = Path(os.environ.get("MAMBA_B200_LIB", Path(__file__).resolve().parent / "_lib" / "libmamba_b200.so"))
HEADER_PATH = Path(__file__).resolve().parents[1] / "include" / "mamba_b200.h"

MM_F32, MM_F16, MM_BF16 = 0, 1, 2
DTYPE_CODE = {torch.float32: MM_F32, torch.float16: MM_F16, torch.bfloat16: MM_BF16}

ERROR_NAMES = {
    0: "MM_OK", -1: "MM_ERR_ARG", -2: "MM_ERR_SHAPE", -3: "MM_ERR_DTYPE",
    -4: "MM_ERR_WORKSPACE", -5: "MM_ERR_LAUNCH", -6: "MM_ERR_TIMEOUT", -7: "MM_ERR_TOO_LARGE",
}
MM_SCAN_NOALLOC_SCRATCH_BYTES = 16 << 20

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


class MMScanArgs(ctypes.Structure):
    _fields_ = [
        ("u", _p), ("delta", _p), ("A", _p), ("B", _p), ("C", _p), ("D", _p), ("z", _p), ("y", _p),
        ("state_out", _p), ("dtype", _i64), ("batch", _i64), ("dim", _i64), ("dstate", _i64), ("seqlen", _i64),
        ("u_stride", _i64 * 3), ("delta_stride", _i64 * 3), ("z_stride", _i64 * 3), ("y_stride", _i64 * 3),
        ("B_stride", _i64 * 3), ("C_stride", _i64 * 3), ("A_stride", _i64 * 2),
        ("delta_softplus", _i64), ("piece_tiles", _i64), ("options", _i64), ("delta_bias", _p),
    ]


class MMConvArgs(ctypes.Structure):
    _fields_ = [
        ("x", _p), ("weight", _p), ("bias", _p), ("out", _p), ("conv_state", _p), ("dtype", _i64),
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("width", _i64),
        ("x_stride", _i64 * 3), ("out_stride", _i64 * 3), ("silu", _i64),
    ]


class MMConvStepArgs(ctypes.Structure):
    _fields_ = [
        ("x", _p), ("conv_state", _p), ("weight", _p), ("bias", _p), ("out", _p), ("dtype", _i64),
        ("batch", _i64), ("dim", _i64), ("width", _i64), ("x_stride_b", _i64), ("out_stride_b", _i64),
        ("silu", _i64), ("early_state", _i64),
    ]


class MMSSMStepArgs(ctypes.Structure):
    _fields_ = [
        ("x", _p), ("dt", _p), ("z", _p), ("B", _p), ("C", _p), ("A", _p), ("D", _p), ("ssm_state", _p),
        ("y", _p), ("dtype", _i64), ("batch", _i64), ("dim", _i64), ("dstate", _i64),
        ("x_stride_b", _i64), ("dt_stride_b", _i64), ("z_stride_b", _i64), ("B_stride_b", _i64),
        ("C_stride_b", _i64), ("y_stride_b", _i64), ("dt_softplus", _i64), ("early_state", _i64),
        ("dt_in", _p), ("dt_w", _p), ("dt_bias", _p), ("dt_rank", _i64), ("dt_in_stride_b", _i64),
        ("dt_w_stride", _i64),
    ]


class MMAddNormArgs(ctypes.Structure):
    _fields_ = [
        ("residual", _p), ("delta", _p), ("weight", _p), ("out", _p), ("dtype", _i64), ("rows", _i64),
        ("dim", _i64), ("delta_stride_r", _i64), ("out_stride_r", _i64), ("eps", ctypes.c_double),
    ]


MM_MAX_TP = 8
MM_PEER_MAX_BLOCKS = 64
MM_PEER_FLAGS, MM_PEER_LL = 0, 1


class MMPeerReduceArgs(ctypes.Structure):
    _fields_ = [
        ("slots", _p * MM_MAX_TP), ("signals", _p * MM_MAX_TP), ("counters", _p), ("out", _p),
        ("dtype", _i64), ("n", _i64), ("stride", _i64), ("world", _i64), ("rank", _i64), ("nblocks", _i64),
        ("protocol", _i64),
    ]


class MMPeerAddNormArgs(ctypes.Structure):
    _fields_ = [
        ("reduce", MMPeerReduceArgs), ("residual", _p), ("weight", _p), ("out", _p), ("rows", _i64),
        ("dim", _i64), ("out_stride_r", _i64), ("eps", ctypes.c_double),
    ]


class MMLinearArgs(ctypes.Structure):
    _fields_ = [
        ("x", _p), ("w", _p), ("bias", _p), ("y", _p), ("ldx", _i64), ("ldw", _i64), ("ldy", _i64),
        ("y_dtype", _i64), ("M", _i64), ("N", _i64), ("K", _i64), ("splits", _i64),
    ]


_SIGNATURES = {
    "mm_selective_scan_workspace_size": ([ctypes.POINTER(MMScanArgs), ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "mm_selective_scan_fwd": ([ctypes.POINTER(MMScanArgs), _p, ctypes.c_size_t, _p], ctypes.c_int),
    "mm_selective_scan_fwd_noalloc": ([ctypes.POINTER(MMScanArgs), _p], ctypes.c_int),
    "mm_selective_scan_status": ([_p, _p], ctypes.c_int),
    "mm_selective_scan_stats": ([_p, ctypes.POINTER(ctypes.c_ulonglong), _p], ctypes.c_int),
    "mm_causal_conv1d_fwd": ([ctypes.POINTER(MMConvArgs), _p], ctypes.c_int),
    "mm_causal_conv1d_step": ([ctypes.POINTER(MMConvStepArgs), _p], ctypes.c_int),
    "mm_ssm_decode_step": ([ctypes.POINTER(MMSSMStepArgs), _p], ctypes.c_int),
    "mm_add_rmsnorm": ([ctypes.POINTER(MMAddNormArgs), _p], ctypes.c_int),
    "mm_peer_allreduce": ([ctypes.POINTER(MMPeerReduceArgs), _p], ctypes.c_int),
    "mm_peer_allreduce_add_rmsnorm": ([ctypes.POINTER(MMPeerAddNormArgs), _p], ctypes.c_int),
    "mm_exp2_check": ([_p, _p, _p, _i64, _p], ctypes.c_int),
    "mm_linear_workspace_size": ([ctypes.POINTER(MMLinearArgs), ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "mm_linear_fwd": ([ctypes.POINTER(MMLinearArgs), _p, ctypes.c_size_t, _p], ctypes.c_int),
    "mm_linear_status": ([_p, _p], ctypes.c_int),
    "mm_version": ([], ctypes.c_char_p),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libmamba_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"libmamba_b200.so is not built ({LIB_PATH}); run `python -m mamba_metal_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with {ERROR_NAMES.get(rc, rc)}")


def require_cuda(*tensors) -> torch.device:
    """All given tensors (None skipped) must be CUDA tensors on one device; returns it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("mamba_metal_b200 runs on CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def strides3(t, default=(0, 0, 0)):
    return (_i64 * 3)(*(t.stride() if t is not None else default))


def header_functions() -> list[str]:
    """Names of the entry points declared in include/mamba_b200.h."""
    import re

    text = HEADER_PATH.read_text()
    return re.findall(r"^\s*(?:int|const char\*)\s+(mm_\w+)\s*\(", text, flags=re.M)
