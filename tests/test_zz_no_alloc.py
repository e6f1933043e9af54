"""The allocation-free scan entry point, mm_selective_scan_fwd_noalloc.

Some callers cannot allocate device memory once they are running -- a service that hands all device
memory to another allocator at start-up, or an FFI host whose policy forbids allocation in its serving
loop -- so this entry point takes no workspace and uses the library's own fixed scratch buffer. These
tests call it through the C-ABI (ctypes, no torch wrapper in between), twice in a row, and compare its
outputs with those of the workspace-taking entry point mm_selective_scan_fwd on the same inputs, at the
tolerances the other scan tests use. The file is named so that pytest collects it last, and it passes
both on its own in a fresh process and after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from mamba_metal_b200 import _lib
from mamba_metal_b200.selective_scan import selective_scan_into
from oracle import scan_ref as R
from tests.helpers import RTOL, assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _args(u, delta, A, Bm, Cm, D, z, y, state, softplus=True):
    a = _lib.MMScanArgs()
    a.u, a.delta, a.A, a.B, a.C = (t.data_ptr() for t in (u, delta, A, Bm, Cm))
    a.D, a.z, a.y, a.state_out = D.data_ptr(), z.data_ptr(), y.data_ptr(), state.data_ptr()
    a.dtype = _lib.DTYPE_CODE[u.dtype]
    a.batch, a.dim, a.dstate, a.seqlen = u.shape[0], u.shape[1], A.shape[1], u.shape[2]
    a.u_stride, a.delta_stride, a.z_stride = _lib.strides3(u), _lib.strides3(delta), _lib.strides3(z)
    a.y_stride, a.B_stride, a.C_stride = _lib.strides3(y), _lib.strides3(Bm), _lib.strides3(Cm)
    a.A_stride = (ctypes.c_int64 * 2)(*A.stride())
    a.delta_softplus = int(softplus)
    return a


def _run_both(shape, dtype, seed):
    """Runs the workspace entry point once and the no-alloc entry point twice in a row on the same
    inputs; checks both no-alloc calls against the workspace call and returns the inputs (fp32, as the
    kernel saw them after rounding to `dtype`) with the last no-alloc outputs."""
    b, d, n, L = shape
    inp = R.make_baseline_inputs(b, d, n, L, seed=seed)
    t = {k: torch.as_tensor(v).to(DEV, dtype if k in ("u", "delta", "z", "B", "C") else torch.float32)
         for k, v in inp.items()}
    y_ref = torch.empty_like(t["u"])
    h_ref = torch.empty((b, d, n), device=DEV)
    selective_scan_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"], y_ref, h_ref, True)
    lib = _lib.lib()
    stream = _lib.stream_handle(DEV)
    name = str(dtype).split(".")[-1]
    for call in range(2):  # the shared buffer keeps the previous call's contents: both must be right
        y = torch.full_like(t["u"], float("nan"))
        h = torch.full((b, d, n), float("nan"), device=DEV)
        a = _args(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"], y, h)
        with torch.cuda.device(DEV):
            rc = lib.mm_selective_scan_fwd_noalloc(ctypes.byref(a), stream)
        assert rc == 0, _lib.ERROR_NAMES.get(rc, rc)
        torch.cuda.synchronize()
        assert_close(y, y_ref, RTOL[name], f"no-alloc call {call} y")
        assert_close(h, h_ref, RTOL["float32"], f"no-alloc call {call} state")
    return {k: v.float().cpu().numpy() for k, v in t.items()}, y, h


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_noalloc_matches_workspace_entry_point(dtype):
    x, y, h = _run_both((2, 200, 16, 3000), dtype, seed=21)
    # and against the sequential oracle on the same (rounded) inputs
    y_o, h_o = R.selective_scan_vec(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                                    delta_softplus=True, return_state=True)
    assert_close(y, y_o, RTOL[str(dtype).split(".")[-1]], "no-alloc y vs oracle")
    assert_close(h, h_o, RTOL["float32"], "no-alloc state vs oracle")


def test_noalloc_fits_large_state_by_longer_pieces():
    """dstate 64, bf16, (1, 2048, 4096): the library's default split (one piece per resident warp)
    would need about 17 MB of workspace, more than the fixed buffer; the no-alloc entry point lengthens
    the pieces until the workspace fits instead of refusing the call."""
    a = _lib.MMScanArgs()
    a.dtype, a.batch, a.dim, a.dstate, a.seqlen = _lib.DTYPE_CODE[torch.bfloat16], 1, 2048, 64, 4096
    need = ctypes.c_size_t(0)
    with torch.cuda.device(DEV):
        assert _lib.lib().mm_selective_scan_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0
    assert need.value > _lib.MM_SCAN_NOALLOC_SCRATCH_BYTES
    x, y, h = _run_both((1, 2048, 64, 4096), torch.bfloat16, seed=5)
    from oracle.scan_c import selective_scan_c

    y_o, h_o = selective_scan_c(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], delta_softplus=True)
    assert_close(y, y_o, RTOL["bfloat16"], "no-alloc dstate-64 y vs oracle")
    assert_close(h, h_o, RTOL["float32"], "no-alloc dstate-64 state vs oracle")


def test_noalloc_rejects_too_large():
    """A call whose workspace would not fit the fixed buffer is refused before anything runs."""
    a = _lib.MMScanArgs()
    a.dtype, a.batch, a.dim, a.dstate, a.seqlen, a.piece_tiles = 1, 64, 8192, 64, 1 << 16, 1
    need = ctypes.c_size_t(0)
    assert _lib.lib().mm_selective_scan_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0
    assert need.value > _lib.MM_SCAN_NOALLOC_SCRATCH_BYTES
    dummy = torch.empty(16, device=DEV)
    for f in ("u", "delta", "A", "B", "C", "y"):
        setattr(a, f, dummy.data_ptr())
    with torch.cuda.device(DEV):
        rc = _lib.lib().mm_selective_scan_fwd_noalloc(ctypes.byref(a), _lib.stream_handle(DEV))
    assert rc == -7  # MM_ERR_TOO_LARGE
