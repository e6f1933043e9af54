"""``selective_scan`` -- the drop-in for mamba_metal/selective_scan.py:23-80, on CUDA tensors.

Same signature, shape checks (AssertionError, as the reference's asserts), optional D / z, softplus
flag, output dtype (= u.dtype) and fp32 last-state return. The work runs in the sm_100a kernel of
libmamba_b200.so (``mm_selective_scan_fwd``); there is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch

from mamba_metal_b200 import _lib

MAX_DSTATE = 64  # mamba_metal/selective_scan.py:9


def _scan_dtype(*ts) -> torch.dtype:
    """Common element type for u, delta, z, B, C. The kernel reads one activation dtype; mixed inputs
    (allowed by the reference, whose Metal kernel upcasts each input to float) run in float32."""
    dts = {t.dtype for t in ts if t is not None}
    if len(dts) == 1:
        (dt,) = dts
        if dt in _lib.DTYPE_CODE:
            return dt
    return torch.float32


def selective_scan_into(u, delta, A, B, C, D, z, y, state_out, delta_softplus: bool, piece_tiles: int = 0,
                        use_tma: bool = True, delta_bias=None):
    """Runs the scan kernel on given (possibly strided) views and writes into ``y`` / ``state_out``.

    u, delta, z, y: (batch, dim, seqlen) views with any strides (channel-first and channels-last both
    work); B, C: (batch, dstate, seqlen) views; A: (dim, dstate) float32; D: (dim,) float32 or None;
    state_out: contiguous float32 (batch, dim, dstate) or None. All activation views share one dtype.
    ``piece_tiles`` (0 = automatic) sets the timestep tiles per warp; ``use_tma=False`` stages tiles with
    cp.async / plain loads even where TMA applies. ``delta_bias`` (dim,) float32, optional, is added to
    delta before softplus (a Mamba block's dt_proj bias). Returns the workspace tensor (for status queries).
    """
    dev = _lib.require_cuda(u, delta, A, B, C, D, z, y, state_out, delta_bias)
    lib = _lib.lib()
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    args = _lib.MMScanArgs()
    args.u, args.delta, args.A, args.B, args.C = (_lib.ptr(t) for t in (u, delta, A, B, C))
    args.D, args.z, args.y, args.state_out = _lib.ptr(D), _lib.ptr(z), _lib.ptr(y), _lib.ptr(state_out)
    args.dtype = _lib.DTYPE_CODE[u.dtype]
    args.batch, args.dim, args.dstate, args.seqlen = batch, dim, dstate, seqlen
    args.u_stride = _lib.strides3(u)
    args.delta_stride = _lib.strides3(delta)
    args.z_stride = _lib.strides3(z)
    args.y_stride = _lib.strides3(y)
    args.B_stride = _lib.strides3(B)
    args.C_stride = _lib.strides3(C)
    args.A_stride = (ctypes.c_int64 * 2)(*A.stride())
    args.delta_softplus = int(bool(delta_softplus))
    args.piece_tiles = int(piece_tiles)
    args.options = 0 if use_tma else 1
    if delta_bias is not None:
        assert delta_bias.dtype == torch.float32 and delta_bias.is_contiguous() and delta_bias.numel() == dim
    args.delta_bias = _lib.ptr(delta_bias)
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.mm_selective_scan_workspace_size(ctypes.byref(args), ctypes.byref(nbytes)),
               "mm_selective_scan_workspace_size")
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.mm_selective_scan_fwd(ctypes.byref(args), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
    _lib.check(rc, "mm_selective_scan_fwd")
    return ws


def selective_scan(
    u: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    *,
    D: torch.Tensor | None = None,
    z: torch.Tensor | None = None,
    delta_softplus: bool = False,
    return_state: bool = False,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """Mamba selective scan with optional D / z / softplus.

    Shapes (mamba_metal/selective_scan.py:37-44):
      u, delta: (batch, dim, seqlen)
      A: (dim, dstate)
      B, C: (batch, dstate, seqlen)
      D: (dim,) -- additive skip coefficient (optional)
      z: (batch, dim, seqlen) -- gate, applied as SiLU(z) (optional)
      delta_softplus: map delta through softplus (with the >20 cutoff) before use
    Returns y: (batch, dim, seqlen) of u.dtype, or (y, last_state) with last_state (batch, dim, dstate)
    float32 = h at position seqlen-1 (the prefill -> decode hand-off).
    """
    batch, dim, seqlen = u.shape
    _, dstate = A.shape
    assert delta.shape == u.shape
    assert tuple(B.shape) == (batch, dstate, seqlen) == tuple(C.shape)
    assert dstate <= MAX_DSTATE
    if z is not None:
        assert z.shape == u.shape
    if D is not None:
        assert tuple(D.shape) == (dim,)
    _lib.require_cuda(u, delta, A, B, C, D, z)

    cdt = _scan_dtype(u, delta, B, C, z)
    cast = lambda t: None if t is None else (t if t.dtype == cdt else t.to(cdt))
    uc, dc, Bc, Cc, zc = map(cast, (u, delta, B, C, z))
    Af = A if A.dtype == torch.float32 else A.float()
    Df = None if D is None else (D if D.dtype == torch.float32 else D.float())
    y = torch.empty((batch, dim, seqlen), dtype=cdt, device=u.device)
    state = torch.empty((batch, dim, dstate), dtype=torch.float32, device=u.device)
    selective_scan_into(uc, dc, Af, Bc, Cc, Df, zc, y, state, delta_softplus)
    if y.dtype != u.dtype:
        y = y.to(u.dtype)
    if return_state:
        return y, state
    return y
