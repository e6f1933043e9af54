"""One Mamba block (mixer) on the sm_100a kernels -- drop-in for mamba_metal/mamba_block.py:27-198.

Layout and semantics follow the reference block (in_proj -> causal depthwise conv + SiLU -> x_proj ->
dt_proj -> selective scan with A = -exp(A_log), D, z gate and softplus -> out_proj), with the same
constructor, ``__call__`` / ``prefill`` / ``step`` and HF parameter names (in_proj, conv1d, x_proj,
dt_proj, A_log, D, out_proj). Differences, all deliberate:

- The parallel pass (forward / prefill) lays activations out as (channels, tokens): every projection is
  one GEMM over all tokens whose output rows are channels, so the conv and the scan read t-contiguous
  rows and the four transposes of mamba_block.py:90-100 do not exist here; dt_proj's bias is applied
  inside the scan. Sequence lengths whose rows would not be 16-byte aligned use (tokens, channels)
  strided views instead.
- ``conv1d.weight`` has PyTorch/HF's (d_inner, 1, d_conv) layout (the reference transposes HF weights
  to MLX's (d_inner, d_conv, 1) at load_hf.py:46-50).
- ``step`` returns new state tensors like the reference by default; ``step(..., inplace=True)``
  updates the given conv / SSM state tensors in place (O(1) memory), which generation uses.
- The dense projections are cuBLAS GEMMs through torch; those of the decode step (``step``) can run on
  the library's tcgen05 small-batch GEMM (``ops.linear``) instead (``USE_DECODE_GEMM``); everything
  else runs in libmamba_b200.so.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from mamba_metal_b200 import ops
from mamba_metal_b200.selective_scan import selective_scan_into

# With USE_DECODE_GEMM, decode-step projections of bf16 weights with at most DECODE_GEMM_MAX_ROWS token
# rows use ops.linear (tcgen05, weight-streaming, split-K) instead of cuBLAS. Off by default: measured on
# B200 at configs[3] (batch 64) the cuBLAS projections are faster (53.5 vs 73.1 us per layer).
USE_DECODE_GEMM = False
DECODE_GEMM_MAX_ROWS = 256
# With FUSED_DT_STEP, the decode step's dt_proj (a (batch, dt_rank) x (dt_rank, d_inner) product) runs inside
# the SSM step kernel (a tensor-core tile per CTA) instead of as its own GEMM launch, for steps of at most
# FUSED_DT_MAX_ELEMS (batch rows x channels of this rank). Off by default: measured on B200 with the 2.8b
# shape (dt_rank 160, bf16, batch 64, CUDA graph), the whole decode step at 2 GPUs (2560 channels per rank)
# is slower with it, 3.00 vs 2.80 ms per step, although two-kernel measurements (x_proj GEMM, then the step,
# 64 layers) gave it 3.1-4.1 us per layer at 2560-640 channels x 64 rows (one wave of the fused kernel) and
# nothing at 5120 x 64 (two waves: each CTA waits for its dt_proj rows and the MMA before its first state row).
FUSED_DT_STEP = False
FUSED_DT_MAX_ELEMS = 2560 * 64


def decode_linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, bias32: torch.Tensor | None = None) -> torch.Tensor:
    """x @ w.T (+ bias) for a decode step's (rows, K) activation: the library's small-batch GEMM when it
    applies (bf16, 16-byte aligned rows), cuBLAS otherwise. ``bias32`` is the bias in float32 for the
    library path (converted from ``bias`` when not given)."""
    if (USE_DECODE_GEMM and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and x.shape[0] <= DECODE_GEMM_MAX_ROWS and x.stride(1) == 1 and w.stride(1) == 1
            and x.stride(0) % 8 == 0 and w.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0):
        return ops.linear(x, w, bias32 if bias32 is not None else bias, out=out)
    if out is None:
        return F.linear(x, w, bias)
    torch.matmul(x, w.t(), out=out)
    if bias is not None:
        out += bias
    return out


class MambaBlock(nn.Module):
    def __init__(self, d_model: int, d_state: int = 16, d_conv: int = 4, expand: int = 2,
                 dt_rank: int | None = None, dtype: torch.dtype = torch.float32, device=None, tp_world: int = 1):
        super().__init__()
        if d_conv != 4:
            raise ValueError("only d_conv == 4 is implemented by the conv kernels")
        if (expand * d_model) % tp_world:
            raise ValueError("d_inner must be divisible by the tensor-parallel size")
        self.d_model = d_model
        self.d_state = d_state
        self.d_conv = d_conv
        # with tensor parallelism (mamba_metal_b200.parallel) this block holds 1/tp_world of the channels
        self.d_inner = expand * d_model // tp_world
        self.tp_reduce = None  # set by mamba_metal_b200.parallel.tp_model: sums row-parallel partials
        self.tp_sites = (0, 1)  # this block's call sites (x_proj, out_proj) in the peer all-reduce
        self.dt_rank = math.ceil(d_model / 16) if dt_rank is None else dt_rank
        kw = dict(dtype=dtype, device=device)
        self.in_proj = nn.Linear(d_model, self.d_inner * 2, bias=False, **kw)
        self.conv1d = nn.Conv1d(self.d_inner, self.d_inner, kernel_size=d_conv, groups=self.d_inner,
                                padding=d_conv - 1, bias=True, dtype=torch.float32, device=device)
        self.x_proj = nn.Linear(self.d_inner, self.dt_rank + 2 * d_state, bias=False, **kw)
        self.dt_proj = nn.Linear(self.dt_rank, self.d_inner, bias=True, **kw)
        A_init = torch.arange(1, d_state + 1, dtype=torch.float32, device=device).expand(self.d_inner, d_state)
        self.A_log = nn.Parameter(torch.log(A_init).contiguous())
        self.D = nn.Parameter(torch.ones(self.d_inner, dtype=torch.float32, device=device))
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False, **kw)
        self._A_cache = None

    def _project(self, x: torch.Tensor, w: torch.Tensor, site: int) -> torch.Tensor:
        """x @ w.T; for a tensor-parallel block (x_proj, out_proj are row-parallel) the partial products
        are all-reduced over the group (site 0: x_proj, 1: out_proj)."""
        if self.tp_reduce is None:
            return decode_linear(x, w) if x.dim() == 2 else F.linear(x, w)
        return self.tp_reduce(x, w, self.tp_sites[site])

    # A = -exp(A_log) (mamba_block.py:87, :138), cached until A_log changes
    def _A(self) -> torch.Tensor:
        key = (self.A_log.data_ptr(), self.A_log._version, self.A_log.device)
        if self._A_cache is None or self._A_cache[0] != key:
            self._A_cache = (key, (-torch.exp(self.A_log.float())).contiguous())
        return self._A_cache[1]

    # dt_proj's bias in float32 (the scan's delta_bias, the decode step's fused dt projection), cached until
    # the parameter changes
    def _dt_bias32(self) -> torch.Tensor:
        b = self.dt_proj.bias
        key = (b.data_ptr(), b._version, b.device)
        if getattr(self, "_dt_bias_cache", None) is None or self._dt_bias_cache[0] != key:
            self._dt_bias_cache = (key, b.detach().float().contiguous())
        return self._dt_bias_cache[1]

    def _fused_dt_step(self, batch: int) -> bool:
        """The decode step computes dt_proj inside the SSM step kernel where that kernel's tensor-core dt tile
        applies (16-bit weights, dt_rank a multiple of 16 up to ops.SSM_STEP_FUSED_DT_MAX_RANK, d_state 16,
        d_inner a multiple of 8) and the step is small enough to gain (FUSED_DT_MAX_ELEMS); otherwise dt_proj
        stays a separate GEMM."""
        w = self.dt_proj.weight
        return (FUSED_DT_STEP and w.dtype in (torch.float16, torch.bfloat16) and w.stride(1) == 1
                and self.dt_rank % 16 == 0 and self.dt_rank <= ops.SSM_STEP_FUSED_DT_MAX_RANK
                and self.d_state == 16 and self.d_inner % 8 == 0 and batch * self.d_inner <= FUSED_DT_MAX_ELEMS)

    def _run(self, x: torch.Tensor, want_state: bool):
        bsz, L, _ = x.shape
        if (L * self.in_proj.weight.dtype.itemsize) % 16 == 0:
            return self._run_channel_first(x, want_state)
        return self._run_channels_last(x, want_state)

    def _run_channel_first(self, x: torch.Tensor, want_state: bool):
        """Parallel pass with every activation laid out (channels, tokens): each projection is one GEMM over
        all B*L tokens whose output rows are channels, so the conv and the scan read and write
        t-contiguous rows (the scan's TMA path) and no transpose is materialised. dt_proj's bias is added
        inside the scan (delta_bias)."""
        bsz, L, D = x.shape
        E, N, R = self.d_inner, self.d_state, self.dt_rank
        dt_ = self.in_proj.weight.dtype
        T = bsz * L
        cf = lambda m, c: m.view(c, bsz, L).permute(1, 0, 2)                # (c, B*L) -> (B, c, L) view
        xz_t = torch.matmul(self.in_proj.weight, x.to(dt_).reshape(T, D).t())  # (2E, B*L)
        xc_t = torch.empty((E, T), dtype=dt_, device=x.device)
        conv_state = torch.empty((bsz, E, self.d_conv), dtype=torch.float32, device=x.device) if want_state else None
        ops.causal_conv1d(cf(xz_t[:E], E), self.conv1d.weight, self.conv1d.bias, silu=True, out=cf(xc_t, E),
                          conv_state_out=conv_state)
        xdbl_t = self._project_t(self.x_proj.weight, xc_t, 0)               # (R + 2N, B*L)
        dt_t = torch.matmul(self.dt_proj.weight, xdbl_t[:R])                # (E, B*L), bias added in the scan
        y_t = torch.empty((E, T), dtype=dt_, device=x.device)
        ssm_state = torch.empty((bsz, E, N), dtype=torch.float32, device=x.device) if want_state else None
        Df = self.D if self.D.dtype == torch.float32 else self.D.float()
        selective_scan_into(cf(xc_t, E), cf(dt_t, E), self._A(), cf(xdbl_t[R:R + N], N), cf(xdbl_t[R + N:], N),
                            Df, cf(xz_t[E:], E), cf(y_t, E), ssm_state, delta_softplus=True,
                            delta_bias=self._dt_bias32())
        out = self._project(y_t.t(), self.out_proj.weight, 1)             # (B*L, d_model)
        return out.view(bsz, L, -1), conv_state, ssm_state

    def _project_t(self, w: torch.Tensor, x_t: torch.Tensor, site: int) -> torch.Tensor:
        """w @ x_t for a (K, tokens) activation -> (out_features, tokens); all-reduced over the group for a
        tensor-parallel block (row-parallel x_proj)."""
        if self.tp_reduce is None:
            return torch.matmul(w, x_t)
        return self.tp_reduce.transposed(w, x_t, self.tp_sites[site])

    def _run_channels_last(self, x: torch.Tensor, want_state: bool):
        """Parallel pass on (B, L, channels) activations, for sequence lengths whose channel-first rows
        would not be 16-byte aligned: the conv and the scan read strided views of the GEMM outputs."""
        bsz, L, _ = x.shape
        E, N, R = self.d_inner, self.d_state, self.dt_rank
        dt_ = self.in_proj.weight.dtype
        xz = F.linear(x.to(dt_), self.in_proj.weight)                    # (B, L, 2E)
        x_in = xz[..., :E].transpose(1, 2)                               # (B, E, L) view
        z = xz[..., E:].transpose(1, 2)
        xc = torch.empty((bsz, L, E), dtype=dt_, device=x.device)
        conv_state = torch.empty((bsz, E, self.d_conv), dtype=torch.float32, device=x.device) if want_state else None
        ops.causal_conv1d(x_in, self.conv1d.weight, self.conv1d.bias, silu=True, out=xc.transpose(1, 2),
                          conv_state_out=conv_state)
        x_dbl = self._project(xc, self.x_proj.weight, 0)                    # (B, L, R + 2N)
        dt = F.linear(x_dbl[..., :R], self.dt_proj.weight, self.dt_proj.bias)  # (B, L, E), bias included
        Bm = x_dbl[..., R:R + N].transpose(1, 2)                         # (B, N, L) view
        Cm = x_dbl[..., R + N:].transpose(1, 2)
        y = torch.empty((bsz, L, E), dtype=dt_, device=x.device)
        ssm_state = torch.empty((bsz, E, N), dtype=torch.float32, device=x.device) if want_state else None
        Df = self.D if self.D.dtype == torch.float32 else self.D.float()
        selective_scan_into(xc.transpose(1, 2), dt.transpose(1, 2), self._A(), Bm, Cm, Df, z,
                            y.transpose(1, 2), ssm_state, delta_softplus=True)
        out = self._project(y, self.out_proj.weight, 1)
        return out, conv_state, ssm_state

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: (B, L, d_model) -> (B, L, d_model) (mamba_block.py:68-102)."""
        return self._run(x, want_state=False)[0]

    def prefill(self, x: torch.Tensor):
        """Returns (y (B, L, d_model), conv_state (B, d_inner, d_conv) fp32, ssm_state (B, d_inner,
        d_state) fp32) -- mamba_block.py:104-153."""
        return self._run(x, want_state=True)

    def step(self, x_token: torch.Tensor, conv_state: torch.Tensor, ssm_state: torch.Tensor, inplace: bool = False,
             defer_out: bool = False):
        """O(1) per-token forward (mamba_block.py:155-198). x_token: (B, 1, d_model).
        Returns (y (B, 1, d_model), new_conv_state, new_ssm_state). With defer_out=True on a
        tensor-parallel block whose out_proj partial fits the peer all-reduce, y is instead a pending
        reduction whose add_rmsnorm(residual, weight, eps, dtype) finishes it (MambaModel does this)."""
        E, N, R = self.d_inner, self.d_state, self.dt_rank
        dt_ = self.in_proj.weight.dtype
        if not inplace or conv_state.dtype != torch.float32 or not conv_state.is_contiguous():
            conv_state = conv_state.to(torch.float32, copy=True).contiguous()
        if not inplace or ssm_state.dtype != torch.float32 or not ssm_state.is_contiguous():
            ssm_state = ssm_state.to(torch.float32, copy=True).contiguous()
        xz = decode_linear(x_token[:, 0].to(dt_), self.in_proj.weight)  # (B, 2E)
        # early_state: the kernel just before each of the two step kernels is a projection GEMM, which does
        # not write the state they update, so they may start loading it while the GEMM finishes
        xc = ops.causal_conv1d_step(xz[:, :E], conv_state, self.conv1d.weight, self.conv1d.bias, silu=True,
                                    early_state=True)
        x_dbl = self._project(xc, self.x_proj.weight, 0)                    # (B, R + 2N)
        Df = self.D if self.D.dtype == torch.float32 else self.D.float()
        if self._fused_dt_step(xc.shape[0]):
            # dt = dt_proj(x_dbl[:, :R]) computed inside the step kernel (fp32, bias included)
            y = ops.ssm_decode_step(xc, None, xz[:, E:], x_dbl[:, R:R + N], x_dbl[:, R + N:], self._A(), Df,
                                    ssm_state, dt_softplus=True, early_state=True, dt_in=x_dbl[:, :R],
                                    dt_weight=self.dt_proj.weight, dt_bias=self._dt_bias32())
        else:
            dt = decode_linear(x_dbl[:, :R], self.dt_proj.weight, self.dt_proj.bias, bias32=self._dt_bias32())
            y = ops.ssm_decode_step(xc, dt, xz[:, E:], x_dbl[:, R:R + N], x_dbl[:, R + N:], self._A(), Df,
                                    ssm_state, dt_softplus=True, early_state=True)
        if defer_out and self.tp_reduce is not None and hasattr(self.tp_reduce, "partial"):
            # tensor parallel: leave out_proj's all-reduce to the caller's fused residual add + RMSNorm
            pending = self.tp_reduce.partial(y, self.out_proj.weight, self.tp_sites[1])
            if pending is not None:
                return pending, conv_state, ssm_state
        return self._project(y, self.out_proj.weight, 1)[:, None, :], conv_state, ssm_state
