"""Torch-facing wrappers of the conv1d, decode-step and residual-norm kernels of libmamba_b200.so.

Each function passes device pointers, strides and the current stream of the tensors' device to the
C-ABI (include/mamba_b200.h) and raises on a non-zero status. There is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch

from mamba_metal_b200 import _lib

D_CONV = 4


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, silu: bool = True,
                  out: torch.Tensor | None = None, conv_state_out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal depthwise conv1d, width 4, as MLX nn.Conv1d(groups=dim, padding=3)[:, :L] + SiLU
    (mamba_metal/mamba_block.py:45-52, :129-130).

    x: (batch, dim, seqlen) view with any strides (channel-first and channels-last views both run on
    vector paths); weight: (dim, 1, 4) or (dim, 4) float32; bias: (dim,) float32. ``out`` (same shape,
    any strides) defaults to a new channel-first tensor of x.dtype. ``conv_state_out``, when given, is
    a contiguous float32 (batch, dim, 4) tensor that receives the last 4 pre-conv inputs
    (mamba_block.py:118-127).
    """
    batch, dim, seqlen = x.shape
    w = weight.reshape(dim, -1)
    assert w.shape[1] == D_CONV, "only d_conv == 4 is implemented"
    dev = _lib.require_cuda(x, w, bias, out, conv_state_out)
    if x.dtype not in _lib.DTYPE_CODE:
        raise TypeError(f"unsupported dtype {x.dtype}")
    w = w.float().contiguous()
    b = None if bias is None else bias.float().contiguous()
    if out is None:
        out = torch.empty((batch, dim, seqlen), dtype=x.dtype, device=dev)
    assert out.shape == x.shape and out.dtype == x.dtype
    if conv_state_out is not None:
        assert conv_state_out.is_contiguous() and conv_state_out.dtype == torch.float32
        assert tuple(conv_state_out.shape) == (batch, dim, D_CONV)
    a = _lib.MMConvArgs()
    a.x, a.weight, a.bias, a.out, a.conv_state = x.data_ptr(), w.data_ptr(), _lib.ptr(b), out.data_ptr(), \
        _lib.ptr(conv_state_out)
    a.dtype = _lib.DTYPE_CODE[x.dtype]
    a.batch, a.dim, a.seqlen, a.width = batch, dim, seqlen, D_CONV
    a.x_stride = _lib.strides3(x)
    a.out_stride = _lib.strides3(out)
    a.silu = int(bool(silu))
    with torch.cuda.device(dev):
        rc = _lib.lib().mm_causal_conv1d_fwd(ctypes.byref(a), _lib.stream_handle(dev))
    _lib.check(rc, "mm_causal_conv1d_fwd")
    return out


def causal_conv1d_step(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                       *, silu: bool = True, out: torch.Tensor | None = None, early_state: bool = False) -> torch.Tensor:
    """One decode step of the conv, updating ``conv_state`` (float32 (batch, dim, 4), contiguous) in
    place: window shift + append, dot with the weight, + bias, SiLU (mamba_block.py:171-177).
    x: (batch, dim) with unit inner stride (row stride free). Returns out (batch, dim) of x.dtype.
    ``early_state``: the caller guarantees that the kernel issued just before this call did not write
    ``conv_state``; the step then starts loading the state while that kernel finishes."""
    batch, dim = x.shape
    assert x.stride(1) == 1
    assert conv_state.is_contiguous() and conv_state.dtype == torch.float32
    assert tuple(conv_state.shape) == (batch, dim, D_CONV)
    dev = _lib.require_cuda(x, conv_state, weight, bias, out)
    w = weight.reshape(dim, -1)
    w = w if (w.dtype == torch.float32 and w.is_contiguous()) else w.float().contiguous()
    b = None if bias is None else (bias if bias.dtype == torch.float32 else bias.float())
    if out is None:
        out = torch.empty((batch, dim), dtype=x.dtype, device=dev)
    a = _lib.MMConvStepArgs()
    a.x, a.conv_state, a.weight, a.bias, a.out = x.data_ptr(), conv_state.data_ptr(), w.data_ptr(), _lib.ptr(b), \
        out.data_ptr()
    a.dtype = _lib.DTYPE_CODE[x.dtype]
    a.batch, a.dim, a.width = batch, dim, D_CONV
    a.x_stride_b, a.out_stride_b = x.stride(0), out.stride(0)
    a.silu = int(bool(silu))
    a.early_state = int(bool(early_state))
    with torch.cuda.device(dev):
        rc = _lib.lib().mm_causal_conv1d_step(ctypes.byref(a), _lib.stream_handle(dev))
    _lib.check(rc, "mm_causal_conv1d_step")
    return out


# Largest dt_rank whose fused dt projection runs in the dstate-16 step kernel (kDtMaxRank in mm_step.cu);
# larger or odd ranks, and float32, take the one-thread-per-channel kernel.
SSM_STEP_FUSED_DT_MAX_RANK = 160


def ssm_decode_step(x, dt, z, B, C, A, D, ssm_state, *, dt_softplus: bool = True, out=None,
                    early_state: bool = False, dt_in=None, dt_weight=None, dt_bias=None) -> torch.Tensor:
    """One decode step of the SSM, updating ``ssm_state`` (float32 (batch, dim, dstate), contiguous) in
    place (mamba_block.py:183-195). x, dt, z: (batch, dim); B, C: (batch, dstate) (row strides free,
    unit inner stride); A: (dim, dstate) float32 contiguous; D: (dim,) float32 or None.
    ``early_state``: the caller guarantees that the kernel issued just before this call did not write
    ``ssm_state``; the step then streams the state in while that kernel finishes.
    With ``dt_weight`` (dt_proj.weight, (dim, dt_rank)) the step computes dt itself (mamba_block.py:181):
    dt = dt_in @ dt_weight.T + dt_bias in float32, from ``dt_in`` (batch, dt_rank) (x_proj's first
    dt_rank columns) and ``dt_bias`` ((dim,) float32 or None); ``dt`` is then not used (pass None)."""
    batch, dim = x.shape
    dstate = A.shape[1]
    fused = dt_weight is not None
    if fused:
        assert dt_in is not None and dt_in.dim() == 2 and dt_in.shape[0] == batch
        assert dt_weight.dim() == 2 and dt_weight.shape == (dim, dt_in.shape[1])
        assert dt_bias is None or (dt_bias.shape == (dim,) and dt_bias.dtype == torch.float32
                                   and dt_bias.is_contiguous())
    else:
        assert dt is not None
    for t in (x, None if fused else dt, z, B, C, dt_in if fused else None, dt_weight):
        if t is not None:
            assert t.stride(-1) == 1 and t.dtype == x.dtype
    assert ssm_state.is_contiguous() and ssm_state.dtype == torch.float32
    assert A.is_contiguous() and A.dtype == torch.float32
    dev = _lib.require_cuda(x, dt, z, B, C, A, D, ssm_state, out, dt_in, dt_weight, dt_bias)
    if out is None:
        out = torch.empty((batch, dim), dtype=x.dtype, device=dev)
    a = _lib.MMSSMStepArgs()
    a.x, a.dt, a.z, a.B, a.C, a.A, a.D = (_lib.ptr(t) for t in (x, None if fused else dt, z, B, C, A, D))
    a.ssm_state, a.y = ssm_state.data_ptr(), out.data_ptr()
    a.dtype = _lib.DTYPE_CODE[x.dtype]
    a.batch, a.dim, a.dstate = batch, dim, dstate
    a.x_stride_b = x.stride(0)
    a.dt_stride_b = 0 if fused else dt.stride(0)
    a.z_stride_b = z.stride(0) if z is not None else 0
    a.B_stride_b, a.C_stride_b, a.y_stride_b = B.stride(0), C.stride(0), out.stride(0)
    a.dt_softplus = int(bool(dt_softplus))
    a.early_state = int(bool(early_state))
    if fused:
        a.dt_in, a.dt_w, a.dt_bias = _lib.ptr(dt_in), _lib.ptr(dt_weight), _lib.ptr(dt_bias)
        a.dt_rank, a.dt_in_stride_b, a.dt_w_stride = dt_in.shape[1], dt_in.stride(0), dt_weight.stride(0)
    with torch.cuda.device(dev):
        rc = _lib.lib().mm_ssm_decode_step(ctypes.byref(a), _lib.stream_handle(dev))
    _lib.check(rc, "mm_ssm_decode_step")
    return out


def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float,
                out_dtype: torch.dtype, out: torch.Tensor | None = None) -> torch.Tensor:
    """residual (float32, contiguous (..., dim)) += delta; returns RMSNorm(residual) * weight in
    ``out_dtype`` (mamba_model.py:49-58 with nn.RMSNorm)."""
    dim = residual.shape[-1]
    rows = residual.numel() // dim
    assert residual.is_contiguous() and residual.dtype == torch.float32
    dev = _lib.require_cuda(residual, delta, weight, out)
    w = weight if weight.dtype == torch.float32 else weight.float()
    if delta is not None:
        assert delta.shape == residual.shape and delta.dtype == out_dtype and delta.stride(-1) == 1
        d2 = delta.reshape(rows, dim)
    if out is None:
        out = torch.empty(residual.shape, dtype=out_dtype, device=dev)
    a = _lib.MMAddNormArgs()
    a.residual, a.delta, a.weight, a.out = residual.data_ptr(), _lib.ptr(delta), w.data_ptr(), out.data_ptr()
    a.dtype = _lib.DTYPE_CODE[out_dtype]
    a.rows, a.dim = rows, dim
    a.delta_stride_r = d2.stride(0) if delta is not None else 0
    a.out_stride_r = out.reshape(rows, dim).stride(0)
    a.eps = float(eps)
    with torch.cuda.device(dev):
        rc = _lib.lib().mm_add_rmsnorm(ctypes.byref(a), _lib.stream_handle(dev))
    _lib.check(rc, "mm_add_rmsnorm")
    return out


_LINEAR_WS: dict[int, torch.Tensor] = {}


def _linear_workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-filled workspace of mm_linear_fwd for this device (every call leaves it zeroed again); grown
    when a larger call needs it. Grow it before capturing a CUDA graph (an eager call of the same shapes
    does that)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _LINEAR_WS.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _LINEAR_WS[idx] = ws
    return ws


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, *, out_dtype: torch.dtype | None = None,
           out: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """y = x @ w.T (+ bias) for bf16 x (M, K) and w (N, K) (nn.Linear layout), fp32 accumulation, on the
    tcgen05 decode GEMM of libmamba_b200.so (mm_linear_fwd). The decode step's projections
    (mamba_metal/mamba_block.py:167, :179, :181, :197) go through here. out_dtype: bfloat16 (default) or
    float32; ``out`` may be a (M, N) view with unit inner stride."""
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    assert x.stride(1) == 1 and w.stride(1) == 1
    dev = _lib.require_cuda(x, w, bias, out)
    odt = out_dtype or (out.dtype if out is not None else torch.bfloat16)
    if out is None:
        out = torch.empty((M, N), dtype=odt, device=dev)
    assert out.shape == (M, N) and out.dtype == odt and out.stride(1) == 1
    b = None if bias is None else (bias if bias.dtype == torch.float32 and bias.is_contiguous() else
                                   bias.float().contiguous())
    a = _lib.MMLinearArgs()
    a.x, a.w, a.bias, a.y = x.data_ptr(), w.data_ptr(), _lib.ptr(b), out.data_ptr()
    a.ldx, a.ldw, a.ldy = x.stride(0), w.stride(0), out.stride(0)
    a.y_dtype = _lib.DTYPE_CODE[odt]
    a.M, a.N, a.K, a.splits = M, N, K, int(splits)
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.mm_linear_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)), "mm_linear_workspace_size")
    ws = _linear_workspace(dev, int(nbytes.value))
    with torch.cuda.device(dev):
        rc = lib.mm_linear_fwd(ctypes.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
    _lib.check(rc, "mm_linear_fwd")
    return out


def linear_status(device: torch.device | int | None = None) -> int:
    """Status word of the device's linear workspace: 0, or MM_ERR_TIMEOUT after a pipeline wait ran out."""
    dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _LINEAR_WS.get(idx)
    if ws is None:
        return 0
    with torch.cuda.device(dev):
        return _lib.lib().mm_linear_status(ws.data_ptr(), _lib.stream_handle(dev))
