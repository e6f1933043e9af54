"""Float32 PyTorch restatement of the reference model, built from plain tensor ops (no custom kernels).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Runs on CPU (or, for shapes too large for the
host, on a GPU with TF32 disabled -- still plain PyTorch ops, never libmamba_b200).

Restates mamba_metal/mamba_block.py:68-198 (forward, prefill, step), mamba_metal/mamba_model.py:35-127
(pre-RMSNorm residual stack, tied head, init_state / prefill / step) and mamba_metal/generate.py:65-110
(greedy prefill -> step hand-off), reading parameters from a ``MambaModel.state_dict()`` (HF names:
layers.{i}.mixer.in_proj.weight, ..., with conv1d.weight in PyTorch's (d_inner, 1, d_conv) layout).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _silu(x):
    return x / (1.0 + torch.exp(-x))


def _softplus_cut(x):
    """softplus with the >20 cutoff (selective_scan_chunked.metal:60-65)."""
    return torch.where(x <= 20.0, torch.log1p(torch.exp(torch.clamp(x, max=20.0))), x)


def rmsnorm(x, w, eps):
    return x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps) * w


def scan_seq(u, delta, A, B, C, D, z, delta_softplus=True):
    """Sequential scan, vectorised over (batch, channel, state). u, delta, z: (b, d, L); B, C: (b, n, L).
    Returns (y (b, d, L), last state (b, d, n))."""
    if delta_softplus:
        delta = _softplus_cut(delta)
    b, d, L = u.shape
    h = torch.zeros((b, d, A.shape[1]), dtype=u.dtype, device=u.device)
    y = torch.empty_like(u)
    for t in range(L):
        dt = delta[:, :, t, None]
        h = torch.exp(dt * A[None]) * h + (dt * u[:, :, t, None]) * B[:, None, :, t]
        y[:, :, t] = (h * C[:, None, :, t]).sum(-1)
    if D is not None:
        y = y + D[None, :, None] * u
    if z is not None:
        y = y * _silu(z)
    return y, h


def _identity(x):
    return x


def rounder(act_dtype):
    """Rounding of an activation to the dtype the reference stores it in. With bf16 / fp16 weights MLX
    keeps every layer output in the weights' dtype (matmul, conv and elementwise ops return their input
    dtype, accumulating internally in float32); the oracle then computes in float32 and rounds each such
    output to ``act_dtype``. None (or float32) = no rounding."""
    if act_dtype is None or act_dtype == torch.float32:
        return _identity
    return lambda x: x.to(act_dtype).to(torch.float32)


class RefMixer:
    def __init__(self, sd: dict, prefix: str, d_state: int, dt_rank: int, dtype=torch.float32, act_dtype=None):
        self.q = rounder(act_dtype)
        g = lambda k: sd[prefix + k].to(dtype)
        self.W_in, self.W_x, self.W_dt, self.b_dt = g("in_proj.weight"), g("x_proj.weight"), g("dt_proj.weight"), \
            g("dt_proj.bias")
        self.W_out = g("out_proj.weight")
        self.conv_w = g("conv1d.weight").reshape(self.W_dt.shape[0], -1)   # (d_inner, d_conv)
        self.conv_b = g("conv1d.bias")
        self.A = -torch.exp(g("A_log"))
        self.D = g("D")
        self.N, self.R = d_state, dt_rank
        self.E = self.W_dt.shape[0]

    def _conv(self, x):  # x: (B, L, E) channels-last; MLX Conv1d(padding=3)[:, :L] (mamba_block.py:77)
        L = x.shape[1]
        k = self.conv_w.shape[1]
        xp = F.pad(x, (0, 0, k - 1, 0))
        out = sum(self.conv_w[None, None, :, j] * xp[:, j:j + L, :] for j in range(k))
        return out + self.conv_b

    def _core(self, x):
        E, N, R, q = self.E, self.N, self.R, self.q
        xz = q(x @ self.W_in.T)
        xm, z = xz[..., :E], xz[..., E:]
        xc = q(_silu(self._conv(xm)))
        x_dbl = q(xc @ self.W_x.T)
        dt = q(x_dbl[..., :R] @ self.W_dt.T + self.b_dt)
        Bm, Cm = x_dbl[..., R:R + N], x_dbl[..., R + N:]
        y, h = scan_seq(xc.transpose(1, 2), dt.transpose(1, 2), self.A, Bm.transpose(1, 2), Cm.transpose(1, 2),
                        self.D, z.transpose(1, 2), delta_softplus=True)
        return q(q(y.transpose(1, 2)) @ self.W_out.T), xm, h

    def forward(self, x):
        return self._core(x)[0]

    def prefill(self, x):
        """mamba_block.py:104-153: conv_state = last d_conv pre-conv inputs, zero-left-padded."""
        y, xm, h = self._core(x)
        L, k = xm.shape[1], self.conv_w.shape[1]
        cs = xm[:, L - k:L, :] if L >= k else torch.cat([xm.new_zeros(xm.shape[0], k - L, xm.shape[2]), xm], 1)
        return y, cs.transpose(1, 2).contiguous(), h

    def step(self, x_tok, conv_state, ssm_state):
        """mamba_block.py:155-198 (softplus without cutoff, as nn.softplus)."""
        E, N, R, q = self.E, self.N, self.R, self.q
        xz = q(x_tok[:, 0] @ self.W_in.T)
        xm, z = xz[:, :E], xz[:, E:]
        new_conv = torch.cat([conv_state[:, :, 1:], xm[:, :, None]], dim=2)
        xc = q(_silu((new_conv * self.conv_w[None]).sum(-1) + self.conv_b))
        x_dbl = q(xc @ self.W_x.T)
        dt = F.softplus(q(x_dbl[:, :R] @ self.W_dt.T + self.b_dt))
        Bm, Cm = x_dbl[:, R:R + N], x_dbl[:, R + N:]
        new_ssm = torch.exp(dt[:, :, None] * self.A[None]) * ssm_state + (dt * xc)[:, :, None] * Bm[:, None, :]
        y = (new_ssm * Cm[:, None, :]).sum(-1) + self.D * xc
        y = q(y * _silu(z))
        return q(y @ self.W_out.T)[:, None, :], new_conv, new_ssm


class RefModel:
    """Reference model over a MambaModel state_dict (float32)."""

    def __init__(self, sd: dict, cfg, dtype=torch.float32, device="cpu", act_dtype=None):
        """``act_dtype`` (e.g. torch.bfloat16): round every projection, conv, scan and RMSNorm output to it,
        as the reference does for a model whose weights are in that dtype (see ``rounder``); the residual
        stream stays float32."""
        sd = {k: v.to(device) for k, v in sd.items()}
        dt_rank = cfg.dt_rank if cfg.dt_rank is not None else -(-cfg.d_model // 16)
        self.cfg = cfg
        self.q = rounder(act_dtype)
        self.emb = sd["embeddings.weight"].to(dtype)
        self.norms = [sd[f"layers.{i}.norm.weight"].to(dtype) for i in range(cfg.n_layer)]
        self.mixers = [RefMixer(sd, f"layers.{i}.mixer.", cfg.d_state, dt_rank, dtype, act_dtype)
                       for i in range(cfg.n_layer)]
        self.norm_f = sd["norm_f.weight"].to(dtype)
        self.eps = cfg.rms_norm_eps

    def set_act_dtype(self, act_dtype):
        """Switches the activation rounding (see ``rounder``) of the model and of every mixer."""
        self.q = rounder(act_dtype)
        for m in self.mixers:
            m.q = self.q

    def _head(self, x):
        """Final RMSNorm and tied head (mamba_model.py:76-78)."""
        return self.q(self.q(rmsnorm(x, self.norm_f, self.eps)) @ self.emb.T)

    def forward(self, ids):
        x = self.emb[ids]
        for w, m in zip(self.norms, self.mixers):
            x = x + m.forward(self.q(rmsnorm(x, w, self.eps)))
        return self._head(x)

    def prefill(self, ids, last_only=False):
        x = self.emb[ids]
        convs, ssms = [], []
        for w, m in zip(self.norms, self.mixers):
            y, cs, ss = m.prefill(self.q(rmsnorm(x, w, self.eps)))
            x = x + y
            convs.append(cs)
            ssms.append(ss)
        if last_only:
            x = x[:, -1:]
        return self._head(x), convs, ssms

    def step(self, ids, convs, ssms):
        x = self.emb[ids]
        nc, ns = [], []
        for w, m, cs, ss in zip(self.norms, self.mixers, convs, ssms):
            y, c2, s2 = m.step(self.q(rmsnorm(x, w, self.eps)), cs, ss)
            x = x + y
            nc.append(c2)
            ns.append(s2)
        return self._head(x), nc, ns

    def greedy(self, ids, n_new, forced=None, prefilled=None):
        """Greedy prefill -> step loop (generate.py:82-108). If ``forced`` (B, n_new) is given the loop is
        teacher-forced with those tokens, so one near-tie does not cascade; returns (tokens, per-step
        logits) with tokens the argmax at each step. ``prefilled`` = the (logits, convs, ssms) of an
        earlier ``prefill(ids, last_only=True)`` skips the prefill (steps never modify those states)."""
        logits, convs, ssms = prefilled if prefilled is not None else self.prefill(ids, last_only=True)
        nxt = logits[:, -1]
        toks, all_logits = [], []
        for i in range(n_new):
            all_logits.append(nxt)
            tok = torch.argmax(nxt, dim=-1)
            toks.append(tok)
            feed = tok if forced is None else forced[:, i]
            lg, convs, ssms = self.step(feed[:, None], convs, ssms)
            nxt = lg[:, 0]
        return torch.stack(toks, 1), torch.stack(all_logits, 1)


def sampling_probs(next_logits, temperature):
    """Distribution of the sampled next id at temperature T > 0: mx.random.categorical(logits / T)
    (generate.py:42-44, :92-93) draws index k with probability softmax(logits / T)_k. float64."""
    x = next_logits.double() / temperature
    x = x - x.max(dim=-1, keepdim=True).values
    e = torch.exp(x)
    return e / e.sum(dim=-1, keepdim=True)

