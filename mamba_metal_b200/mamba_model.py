"""Stacked Mamba causal LM on the sm_100a kernels -- drop-in for mamba_metal/mamba_model.py:23-127.

``MambaConfig`` keeps the reference's fields (mamba_model.py:23-32). ``MambaModel`` keeps the
reference's attribute layout (embeddings, layers.{i}.norm / layers.{i}.mixer, norm_f), which is HF's
``state-spaces/mamba-*-hf`` layout without the ``backbone.`` prefix, and its ``__call__`` / ``init_state`` /
``prefill`` / ``step`` API. The residual stream is kept in float32 and every "residual += mixer output;
RMSNorm" pair runs as one fused kernel (mm_add_rmsnorm); the LM head is tied to the embeddings
(mamba_model.py:76-78).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from mamba_metal_b200 import ops
from mamba_metal_b200.mamba_block import MambaBlock


@dataclass
class MambaConfig:
    d_model: int = 768
    n_layer: int = 24
    vocab_size: int = 50280
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    dt_rank: int | None = None  # auto = ceil(d_model / 16) if None
    rms_norm_eps: float = 1e-5


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight (MLX nn.RMSNorm, mamba_model.py:40). Weight kept in float32."""

    def __init__(self, dim: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.float32, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        res = x.float().contiguous()
        return ops.add_rmsnorm(res, None, self.weight, self.eps, x.dtype)


class MambaResidualBlock(nn.Module):
    """Pre-norm + residual wrapper around a MambaBlock (mamba_model.py:35-58)."""

    def __init__(self, cfg: MambaConfig, dtype: torch.dtype = torch.float32, device=None, tp_world: int = 1):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, eps=cfg.rms_norm_eps, device=device)
        self.mixer = MambaBlock(cfg.d_model, cfg.d_state, cfg.d_conv, cfg.expand, cfg.dt_rank, dtype=dtype,
                                device=device, tp_world=tp_world)

    def forward(self, x):
        return x + self.mixer(self.norm(x))

    def prefill(self, x):
        y, conv_state, ssm_state = self.mixer.prefill(self.norm(x))
        return x + y, conv_state, ssm_state

    def step(self, x_token, conv_state, ssm_state, inplace: bool = False):
        y, cs, ss = self.mixer.step(self.norm(x_token), conv_state, ssm_state, inplace=inplace)
        return x_token + y, cs, ss


class MambaModel(nn.Module):
    """Stack of MambaResidualBlocks with a tied LM head (mamba_model.py:61-127)."""

    def __init__(self, cfg: MambaConfig, dtype: torch.dtype = torch.float32, device=None, tp_world: int = 1):
        super().__init__()
        self.cfg = cfg
        self.dtype = dtype
        self.tp_world = tp_world
        self.embeddings = nn.Embedding(cfg.vocab_size, cfg.d_model, dtype=dtype, device=device)
        self.layers = nn.ModuleList([MambaResidualBlock(cfg, dtype=dtype, device=device, tp_world=tp_world)
                                     for _ in range(cfg.n_layer)])
        self.norm_f = RMSNorm(cfg.d_model, eps=cfg.rms_norm_eps, device=device)

    @property
    def d_inner(self) -> int:
        """Inner channels held by this model (all of them, or this rank's slice under tensor parallelism)."""
        return self.cfg.expand * self.cfg.d_model // self.tp_world

    def _norm_weight(self, i: int) -> torch.Tensor:
        return self.layers[i].norm.weight if i < len(self.layers) else self.norm_f.weight

    def _stack(self, input_ids: torch.Tensor, mode: str, conv_states=None, ssm_states=None, inplace=False,
               last_only=False):
        eps = self.cfg.rms_norm_eps
        x = self.embeddings(input_ids)                          # (B, L, d_model)
        residual = x.float().contiguous()
        h = ops.add_rmsnorm(residual, None, self._norm_weight(0), eps, self.dtype)
        new_conv, new_ssm = [], []
        for i, layer in enumerate(self.layers):
            if mode == "forward":
                y = layer.mixer(h)
            elif mode == "prefill":
                y, cs, ss = layer.mixer.prefill(h)
                new_conv.append(cs)
                new_ssm.append(ss)
            else:
                y, cs, ss = layer.mixer.step(h, conv_states[i], ssm_states[i], inplace=inplace, defer_out=True)
                new_conv.append(cs)
                new_ssm.append(ss)
            if hasattr(y, "add_rmsnorm"):  # tensor-parallel out_proj partial: all-reduce + add + norm fused
                h = y.add_rmsnorm(residual, self._norm_weight(i + 1), eps, self.dtype)
            else:
                h = ops.add_rmsnorm(residual, y, self._norm_weight(i + 1), eps, self.dtype)
        if last_only:
            h = h[:, -1:, :]
        logits = F.linear(h, self.embeddings.weight)            # tied head (mamba_model.py:76-78)
        return logits, new_conv, new_ssm

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """input_ids: (B, L) -> logits (B, L, vocab_size)."""
        return self._stack(input_ids, "forward")[0]

    def init_state(self, batch_size: int = 1):
        """Zero float32 conv and SSM state per layer (mamba_model.py:80-91)."""
        dev = self.embeddings.weight.device
        conv = [torch.zeros((batch_size, self.d_inner, self.cfg.d_conv), dtype=torch.float32, device=dev)
                for _ in self.layers]
        ssm = [torch.zeros((batch_size, self.d_inner, self.cfg.d_state), dtype=torch.float32, device=dev)
               for _ in self.layers]
        return conv, ssm

    def prefill(self, input_ids: torch.Tensor, last_only: bool = False):
        """Parallel prompt pass (mamba_model.py:93-110). Returns (logits (B, L, vocab) -- (B, 1, vocab)
        with last_only --, conv_states, ssm_states)."""
        return self._stack(input_ids, "prefill", last_only=last_only)

    def step(self, input_ids: torch.Tensor, conv_states, ssm_states, inplace: bool = False):
        """One token per sequence, carrying state (mamba_model.py:112-127). input_ids: (B, 1).
        Returns (logits (B, 1, vocab), new_conv_states, new_ssm_states); with inplace=True the given
        state tensors are updated and returned."""
        return self._stack(input_ids, "step", conv_states, ssm_states, inplace=inplace)


# ---------------------------------------------------------------------------------------------------
# Seeded random initialisation (no checkpoints are available offline)
# ---------------------------------------------------------------------------------------------------

@torch.no_grad()
def init_weights_(model: MambaModel, seed: int = 0, dt_min: float = 1e-3, dt_max: float = 1e-1) -> MambaModel:
    """Deterministic random init on the model's device, in a fixed parameter order.

    Distributions follow MLX's layer defaults used by the reference (nn.Linear U(+-1/sqrt(fan_in)),
    nn.Embedding N(0, 1/d_model), nn.Conv1d weight U(+-1/sqrt(k)) with zero bias, RMSNorm ones), the
    reference block's A_log = log(1..N) and D = 1 (mamba_block.py:59-64), and BASELINE's dt_proj bias:
    softplus(bias) ~ logUniform(dt_min, dt_max).
    """
    dev = model.embeddings.weight.device
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def uniform_(p, bound):
        p.copy_((torch.rand(p.shape, generator=g, device=dev, dtype=torch.float32) * 2 - 1) * bound)

    d = model.cfg.d_model
    model.embeddings.weight.copy_(torch.randn(model.embeddings.weight.shape, generator=g, device=dev) / math.sqrt(d))
    for layer in model.layers:
        m = layer.mixer
        layer.norm.weight.fill_(1.0)
        uniform_(m.in_proj.weight, 1 / math.sqrt(m.d_model))
        uniform_(m.conv1d.weight, 1 / math.sqrt(m.d_conv))
        m.conv1d.bias.zero_()
        uniform_(m.x_proj.weight, 1 / math.sqrt(m.d_inner))
        uniform_(m.dt_proj.weight, 1 / math.sqrt(m.dt_rank))
        u = torch.rand(m.d_inner, generator=g, device=dev, dtype=torch.float32)
        dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        m.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))      # inverse softplus
        A = torch.arange(1, m.d_state + 1, dtype=torch.float32, device=dev).expand(m.d_inner, m.d_state)
        m.A_log.copy_(torch.log(A))
        m.D.fill_(1.0)
        uniform_(m.out_proj.weight, 1 / math.sqrt(m.d_inner))
    model.norm_f.weight.fill_(1.0)
    return model
