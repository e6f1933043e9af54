"""NumPy restatement of the reference's CPU semantics for the scan, conv1d and decode step.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Every function names the reference lines it restates. The literal functions (``*_literal``) keep the
reference's loop structure and float32 arithmetic so that golden vectors produced by the reference's
own functions reproduce to rounding; the vectorised ones loop over time only and are used for larger
shapes.
"""

from __future__ import annotations

import numpy as np


# ---------------------------------------------------------------------------------------------
# Elementwise pieces
# ---------------------------------------------------------------------------------------------

def softplus_safe(x: np.ndarray) -> np.ndarray:
    """softplus with the >20 cutoff: experiments/09-features/test_features.py:13-16 (and
    mamba_metal/kernels/selective_scan_chunked.metal:60-65)."""
    out = np.where(x <= 20.0, np.log1p(np.exp(np.clip(x, None, 20.0))), x)
    return out.astype(x.dtype)


def silu(x: np.ndarray) -> np.ndarray:
    """x / (1 + exp(-x)): experiments/09-features/test_features.py:19-20."""
    return x / (1.0 + np.exp(-x))


# ---------------------------------------------------------------------------------------------
# Selective scan
# ---------------------------------------------------------------------------------------------

def selective_scan_literal(u, delta, A, B, C, D=None, z=None, delta_softplus=False, return_state=False):
    """Sequential reference scan, per (batch, channel), in float32.

    Restates experiments/09-features/test_features.py:23-43 (y), with the float32 upcast of
    experiments/10-fp16/test_fp16.py:28-36 and the final state of
    experiments/18-prefill/verify_state_out.py:13-26. Shapes: u, delta, z (batch, dim, seqlen);
    A (dim, dstate); B, C (batch, dstate, seqlen); D (dim,).
    """
    u = np.asarray(u, dtype=np.float32)
    delta = np.asarray(delta, dtype=np.float32)
    A = np.asarray(A, dtype=np.float32)
    B = np.asarray(B, dtype=np.float32)
    C = np.asarray(C, dtype=np.float32)
    if D is not None:
        D = np.asarray(D, dtype=np.float32)
    if z is not None:
        z = np.asarray(z, dtype=np.float32)
    batch, dim, seqlen = u.shape
    _, dstate = A.shape
    if delta_softplus:
        delta = softplus_safe(delta)
    y = np.zeros_like(u)
    last = np.zeros((batch, dim, dstate), dtype=np.float32)
    for bi in range(batch):
        for di in range(dim):
            h = np.zeros(dstate, dtype=np.float32)
            for t in range(seqlen):
                a_t = np.exp(delta[bi, di, t] * A[di])
                b_t = delta[bi, di, t] * u[bi, di, t] * B[bi, :, t]
                h = a_t * h + b_t
                y[bi, di, t] = np.dot(h, C[bi, :, t])
            last[bi, di] = h
    if D is not None:
        y = y + D[None, :, None] * u
    if z is not None:
        y = y * silu(z)
    y = y.astype(np.float32)
    return (y, last) if return_state else y


def selective_scan_vec(u, delta, A, B, C, D=None, z=None, delta_softplus=False, return_state=False,
                       dtype=np.float32):
    """The same scan, vectorised over (batch, channel, state) with a loop over time.

    Same operation order as ``selective_scan_literal`` per element (a = exp(delta*A), b = delta*u*B,
    h = a*h + b, y = sum_n h*C, then + D*u, then * silu(z)); the sum over states is a pairwise NumPy
    reduction instead of ``np.dot``, which changes rounding only. ``dtype=np.float64`` gives a
    higher-precision oracle.
    """
    u = np.asarray(u, dtype=dtype)
    delta = np.asarray(delta, dtype=dtype)
    A = np.asarray(A, dtype=dtype)
    B = np.asarray(B, dtype=dtype)
    C = np.asarray(C, dtype=dtype)
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    if delta_softplus:
        delta = softplus_safe(delta)
    h = np.zeros((batch, dim, dstate), dtype=dtype)
    y = np.empty((batch, dim, seqlen), dtype=dtype)
    for t in range(seqlen):
        dt = delta[:, :, t][:, :, None]
        a = np.exp(dt * A[None])
        b = dt * u[:, :, t][:, :, None] * B[:, None, :, t]
        h = a * h + b
        y[:, :, t] = np.einsum("bdn,bn->bd", h, C[:, :, t])
    if D is not None:
        y = y + np.asarray(D, dtype=dtype)[None, :, None] * u
    if z is not None:
        y = y * silu(np.asarray(z, dtype=dtype))
    return (y, h) if return_state else y


def pair_scan_literal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """h_i = a_i h_{i-1} + b_i, h_{-1} = 0: experiments/05-pair-scan/pair_scan.py:36-42."""
    h = np.zeros_like(a)
    s = 0.0
    for i in range(a.size):
        s = a[i] * s + b[i]
        h[i] = s
    return h


# ---------------------------------------------------------------------------------------------
# Causal depthwise conv1d and the decode step
# ---------------------------------------------------------------------------------------------

def causal_conv1d_ref(x, weight, bias=None, silu_act=True, dtype=np.float32):
    """Depthwise causal conv, channel-first x (batch, dim, seqlen), weight (dim, width).

    MLX nn.Conv1d with groups=dim and padding=width-1 on both sides, output sliced to the first
    seqlen positions (mamba_metal/mamba_block.py:45-52, :77-78, :129-130): out[t] = bias +
    sum_k w[k] * x[t - (width-1) + k] with zeros before t = 0; then SiLU (mamba_block.py:78).
    """
    x = np.asarray(x, dtype=dtype)
    w = np.asarray(weight, dtype=dtype).reshape(x.shape[1], -1)
    width = w.shape[1]
    batch, dim, seqlen = x.shape
    xp = np.concatenate([np.zeros((batch, dim, width - 1), dtype=dtype), x], axis=2)
    out = np.zeros_like(x)
    for k in range(width):
        out += w[None, :, k, None] * xp[:, :, k:k + seqlen]
    if bias is not None:
        out += np.asarray(bias, dtype=dtype)[None, :, None]
    return silu(out) if silu_act else out


def conv_state_ref(x, width=4):
    """Last `width` pre-conv inputs, zero-left-padded: mamba_metal/mamba_block.py:118-127 (channel-first
    x (batch, dim, seqlen) -> (batch, dim, width))."""
    x = np.asarray(x, dtype=np.float32)
    batch, dim, seqlen = x.shape
    if seqlen >= width:
        return x[:, :, seqlen - width:].copy()
    return np.concatenate([np.zeros((batch, dim, width - seqlen), np.float32), x], axis=2)


def conv_step_ref(x_new, conv_state, weight, bias=None, silu_act=True):
    """Decode conv: shift the window, append x, dot with w, + bias, SiLU (mamba_block.py:171-177).
    x_new (batch, dim), conv_state (batch, dim, width). Returns (out, new_state)."""
    st = np.concatenate([conv_state[:, :, 1:], np.asarray(x_new, np.float32)[:, :, None]], axis=2)
    w = np.asarray(weight, np.float32).reshape(st.shape[1], -1)
    out = (st * w[None]).sum(axis=-1)
    if bias is not None:
        out = out + np.asarray(bias, np.float32)[None]
    return (silu(out) if silu_act else out), st


def ssm_step_ref(x, dt, z, B, C, A, D, ssm_state, dt_softplus=True):
    """Decode SSM step (mamba_block.py:183-195): dt = softplus(dt); h = exp(dt*A) h + (dt*x) B;
    y = sum_n h*C + D*x; y *= silu(z). Shapes: x, dt, z (batch, dim); B, C (batch, dstate);
    A (dim, dstate); D (dim,); ssm_state (batch, dim, dstate). Returns (y, new_state)."""
    x = np.asarray(x, np.float32)
    dt = np.asarray(dt, np.float32)
    if dt_softplus:
        dt = softplus_safe(dt)
    a = np.exp(dt[:, :, None] * np.asarray(A, np.float32)[None])
    b = (dt * x)[:, :, None] * np.asarray(B, np.float32)[:, None, :]
    h = a * ssm_state + b
    y = (h * np.asarray(C, np.float32)[:, None, :]).sum(axis=-1)
    if D is not None:
        y = y + np.asarray(D, np.float32)[None] * x
    if z is not None:
        y = y * silu(np.asarray(z, np.float32))
    return y, h


def rmsnorm_ref(x, weight, eps=1e-5):
    """x * rsqrt(mean(x^2) + eps) * weight over the last axis (MLX nn.RMSNorm, mamba_model.py:40)."""
    x = np.asarray(x, np.float32)
    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * np.asarray(weight, np.float32)


# ---------------------------------------------------------------------------------------------
# Seeded inputs
# ---------------------------------------------------------------------------------------------

def make_baseline_inputs(batch, dim, dstate, seqlen, seed=0):
    """Inputs with the BASELINE distributions (configs[0]/[1]/[4]), drawn from
    np.random.default_rng(seed) in the order u, delta, B, C, D, z (the draw order of
    experiments/09-features/test_features.py:46-56): u ~ N(0,1); delta ~ N(0,1)*0.5 (raw, used with
    delta_softplus=True); A[d,n] = -(n+1); B, C ~ N(0,1) (batch, dstate, seqlen); D ~ N(0,1) (dim,);
    z ~ N(0,1). Returned in float32."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((batch, dim, seqlen), dtype=np.float32)
    delta = rng.standard_normal((batch, dim, seqlen), dtype=np.float32) * np.float32(0.5)
    B = rng.standard_normal((batch, dstate, seqlen), dtype=np.float32)
    C = rng.standard_normal((batch, dstate, seqlen), dtype=np.float32)
    D = rng.standard_normal((dim,), dtype=np.float32)
    z = rng.standard_normal((batch, dim, seqlen), dtype=np.float32)
    A = -np.broadcast_to(np.arange(1, dstate + 1, dtype=np.float32), (dim, dstate)).copy()
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z)


def make_features_inputs(batch, dim, dstate, seqlen, seed=0):
    """experiments/09-features/test_features.py:46-56: u ~ N(0,1), delta ~ U(-1, 2),
    A ~ -U(0.1, 2), B, C ~ N(0,1), D ~ N(0,1), z ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((batch, dim, seqlen)).astype(np.float32)
    delta = rng.uniform(-1.0, 2.0, size=(batch, dim, seqlen)).astype(np.float32)
    A = -rng.uniform(0.1, 2.0, size=(dim, dstate)).astype(np.float32)
    B = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32)
    C = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32)
    D = rng.standard_normal((dim,)).astype(np.float32)
    z = rng.standard_normal((batch, dim, seqlen)).astype(np.float32)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z)


def make_fp16_inputs(batch, dim, dstate, seqlen, seed=0):
    """experiments/10-fp16/test_fp16.py:58-67: u, B, C ~ N(0,1)*0.5, delta ~ U(0.01, 0.1),
    A ~ -U(0.1, 2), D ~ N(0,1), z ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((batch, dim, seqlen)).astype(np.float32) * 0.5
    delta = rng.uniform(0.01, 0.1, size=(batch, dim, seqlen)).astype(np.float32)
    A = -rng.uniform(0.1, 2.0, size=(dim, dstate)).astype(np.float32)
    B = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32) * 0.5
    C = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32) * 0.5
    D = rng.standard_normal((dim,)).astype(np.float32)
    z = rng.standard_normal((batch, dim, seqlen)).astype(np.float32)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z)


def make_chunked_inputs(batch, dim, dstate, seqlen, seed=0):
    """experiments/07-chunked/selective_scan_chunked.py:29-35 (also 08-benchmark/bench.py:38-48):
    u ~ N(0,1), delta ~ U(0.01, 0.1), A ~ -U(0.1, 2), B, C ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((batch, dim, seqlen)).astype(np.float32)
    delta = rng.uniform(0.01, 0.1, size=(batch, dim, seqlen)).astype(np.float32)
    A = -rng.uniform(0.1, 2.0, size=(dim, dstate)).astype(np.float32)
    B = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32)
    C = rng.standard_normal((batch, dstate, seqlen)).astype(np.float32)
    return dict(u=u, delta=delta, A=A, B=B, C=C)


def make_conv_inputs(batch, dim, seqlen, width=4, seed=0):
    """configs[1] conv inputs: x ~ N(0,1) (batch, dim, seqlen), weight ~ U(-0.5, 0.5) (dim, width),
    bias ~ U(-0.1, 0.1) (dim,)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, dim, seqlen), dtype=np.float32)
    w = rng.uniform(-0.5, 0.5, size=(dim, width)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, size=(dim,)).astype(np.float32)
    return dict(x=x, weight=w, bias=b)
