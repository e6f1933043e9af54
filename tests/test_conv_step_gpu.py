"""Conv1d (prefill + decode step), SSM decode step and residual RMSNorm kernels vs the CPU oracle (GPU)."""

import numpy as np
import pytest
import torch

from mamba_metal_b200 import add_rmsnorm, causal_conv1d, causal_conv1d_step, ssm_decode_step
from oracle import scan_ref as R
from tests.helpers import RTOL, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def name(dt):
    return str(dt).split(".")[-1]


def q(a, dt):  # round through dt, back to float32 numpy
    return torch.as_tensor(a).to(dt).float().numpy()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("layout", ["channel_first", "channels_last", "strided"])
@pytest.mark.parametrize("shape", [(1, 5, 1), (2, 8, 3), (2, 24, 37), (1, 264, 300), (3, 16, 1025)])
def test_conv_prefill(dtype, layout, shape):
    b, d, L = shape
    inp = R.make_conv_inputs(b, d, L, seed=L)
    x = torch.as_tensor(inp["x"]).to(DEV, dtype)
    if layout == "channels_last":
        x = x.transpose(1, 2).contiguous().transpose(1, 2)
        out = torch.empty((b, L, d), dtype=dtype, device=DEV).transpose(1, 2)
    elif layout == "strided":  # every other channel of a wider buffer, as the in_proj split views are
        wide = torch.zeros((b, L, 2 * d), dtype=dtype, device=DEV)
        wide[..., :d] = x.transpose(1, 2)
        x = wide[..., :d].transpose(1, 2)
        out = torch.empty((b, d, L), dtype=dtype, device=DEV)
    else:
        out = None
    cs = torch.full((b, d, 4), 7.0, device=DEV)
    w = torch.as_tensor(inp["weight"]).to(DEV)[:, None, :]
    y = causal_conv1d(x, w, torch.as_tensor(inp["bias"]).to(DEV), silu=True, out=out, conv_state_out=cs)
    torch.cuda.synchronize()
    xr = q(inp["x"], dtype)
    assert_close(y, R.causal_conv1d_ref(xr, inp["weight"], inp["bias"]), RTOL[name(dtype)], f"{layout} {shape}")
    assert_close(cs, R.conv_state_ref(xr), 1e-6, "conv state")


def test_conv_config1_no_silu():
    """BASELINE configs[1] conv: (8, 1536, 4096) fp16, w ~ U(-.5,.5), bias ~ U(-.1,.1)."""
    inp = R.make_conv_inputs(8, 1536, 4096, seed=0)
    x = torch.as_tensor(inp["x"]).to(DEV, torch.float16)
    y = causal_conv1d(x, torch.as_tensor(inp["weight"]).to(DEV), torch.as_tensor(inp["bias"]).to(DEV), silu=False)
    ref = R.causal_conv1d_ref(q(inp["x"], torch.float16), inp["weight"], inp["bias"], silu_act=False)
    assert_close(y, ref, RTOL["float16"], "config1 conv")


@pytest.mark.parametrize("dtype", DTYPES)
def test_conv_step_matches_prefill(dtype):
    b, d, L = 3, 40, 11
    inp = R.make_conv_inputs(b, d, L, seed=1)
    w = torch.as_tensor(inp["weight"]).to(DEV)
    bias = torch.as_tensor(inp["bias"]).to(DEV)
    xs = torch.as_tensor(inp["x"]).to(DEV, dtype)
    full = causal_conv1d(xs, w, bias)
    st = torch.zeros((b, d, 4), device=DEV)
    wide = torch.zeros((b, 2 * d), dtype=dtype, device=DEV)  # row stride 2d, like the in_proj output
    for t in range(L):
        wide[:, :d] = xs[:, :, t]
        o = causal_conv1d_step(wide[:, :d], st, w, bias)
        assert_close(o, full[:, :, t], RTOL[name(dtype)], f"step {t}")
    assert_close(st, R.conv_state_ref(q(inp["x"], dtype)), 1e-6, "state")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [16, 8, 5])
@pytest.mark.parametrize("b,d", [(3, 50), (9, 136)])
def test_ssm_step_chain_matches_scan(dtype, n, b, d):
    """A chain of decode steps equals the scan (dstate 16 with dim % 8 == 0 takes the coalesced
    4-threads-per-channel kernel; the other shapes the one-thread-per-channel kernel)."""
    L = 20
    inp = R.make_features_inputs(b, d, n, L, seed=n)
    qq = {k: (q(v, dtype) if k in ("u", "delta", "B", "C", "z") else v) for k, v in inp.items()}
    yr, hr = R.selective_scan_vec(**qq, delta_softplus=True, return_state=True, dtype=np.float64)
    h = torch.zeros((b, d, n), device=DEV)
    A = torch.as_tensor(inp["A"]).to(DEV)
    D = torch.as_tensor(inp["D"]).to(DEV)
    g = lambda k, t: torch.as_tensor(np.ascontiguousarray(inp[k][:, :, t])).to(DEV, dtype)
    for t in range(L):
        y = ssm_decode_step(g("u", t), g("delta", t), g("z", t), g("B", t), g("C", t), A, D, h, dt_softplus=True)
        assert_close(y, yr[:, :, t], RTOL[name(dtype)] * 2, f"t={t}")
    assert_close(h, hr, 1e-4 if dtype == torch.float32 else 1e-2, "state")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b,d,rank,bias", [(64, 256, 160, True),   # the 2.8b shape's dt_rank (bf16 rows 320 B)
                                           (9, 136, 48, True),     # the 130m dt_rank
                                           (5, 64, 8, False),      # no bias
                                           (3, 50, 48, True),      # dim % 8 != 0: one thread per channel
                                           (4, 64, 12, True),      # rows not whole 16-byte chunks in 16-bit types
                                           (4, 64, 200, True)])    # rows beyond the register-held limit
def test_ssm_step_fused_dt_projection(dtype, b, d, rank, bias):
    """dt = dt_in @ dt_w.T + dt_bias computed inside the step (mamba_block.py:181) equals the scan of the
    same delta (float64 oracle) over a chain of steps; dt is never rounded to the element type."""
    n, L = 16, 12
    g = torch.Generator().manual_seed(rank * 7 + d)
    inp = R.make_features_inputs(b, d, n, L, seed=rank)
    qq = {k: (q(v, dtype) if k in ("u", "B", "C", "z") else v) for k, v in inp.items()}
    dt_in = (torch.randn(b, rank, L, generator=g) * 0.5).to(dtype)
    w = (torch.randn(d, rank, generator=g) / rank ** 0.5).to(dtype)
    bvec = torch.randn(d, generator=g) - 2.0 if bias else None
    delta = torch.einsum("bkl,dk->bdl", dt_in.double(), w.double())
    if bias:
        delta = delta + bvec.double()[None, :, None]
    qq["delta"] = delta.numpy()
    yr, hr = R.selective_scan_vec(**qq, delta_softplus=True, return_state=True, dtype=np.float64)
    h = torch.zeros((b, d, n), device=DEV)
    A = torch.as_tensor(inp["A"]).to(DEV)
    D = torch.as_tensor(inp["D"]).to(DEV)
    wd = w.to(DEV)
    bd = bvec.to(DEV) if bias else None
    gt = lambda k, t: torch.as_tensor(np.ascontiguousarray(qq[k][:, :, t])).to(DEV, dtype)
    for t in range(L):
        xin = dt_in[:, :, t].contiguous().to(DEV)
        y = ssm_decode_step(gt("u", t), None, gt("z", t), gt("B", t), gt("C", t), A, D, h, dt_softplus=True,
                            dt_in=xin, dt_weight=wd, dt_bias=bd)
        assert_close(y, yr[:, :, t], RTOL[name(dtype)] * 2, f"t={t}")
    assert_close(h, hr, 1e-4 if dtype == torch.float32 else 1e-2, "state")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,dim", [(1, 768), (64, 2560), (7, 100)])
def test_add_rmsnorm(dtype, rows, dim):
    g = torch.Generator().manual_seed(rows)
    res = torch.randn(rows, dim, generator=g)
    delta = torch.randn(rows, dim, generator=g).to(dtype)
    w = torch.rand(dim, generator=g) + 0.5
    r = res.to(DEV)
    out = add_rmsnorm(r, delta.to(DEV), w.to(DEV), 1e-5, dtype)
    ref_res = res + delta.float()
    ref = R.rmsnorm_ref(ref_res.numpy(), w.numpy(), 1e-5)
    assert_close(r, ref_res, 1e-6, "residual")
    assert_close(out, ref, RTOL[name(dtype)], "norm")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_early_state_launch_is_bit_identical(dtype):
    """early_state=True (programmatic dependent launch: the state is loaded while the preceding kernel,
    here a GEMM that does not touch the state, finishes) gives bit-identical outputs and states to the
    plain stream-ordered launch, over a chain of steps each preceded by the GEMM producing its input."""
    g = torch.Generator(device="cuda:0").manual_seed(3)
    b, d, n = 64, 1024, 16
    dev = "cuda:0"
    w_in = (torch.randn((2 * d, 256), generator=g, device=dev) * 0.05).to(dtype)
    xs = [torch.randn((b, 256), generator=g, device=dev).to(dtype) for _ in range(6)]
    cw = torch.randn((d, 4), generator=g, device=dev) * 0.3
    cb = torch.randn((d,), generator=g, device=dev) * 0.1
    A = -torch.rand((d, n), generator=g, device=dev) - 0.2
    D = torch.randn((d,), generator=g, device=dev)
    Bm = torch.randn((b, n), generator=g, device=dev).to(dtype)
    Cm = torch.randn((b, n), generator=g, device=dev).to(dtype)
    outs = {}
    for early in (False, True):
        conv = torch.zeros((b, d, 4), device=dev)
        ssm = torch.zeros((b, d, n), device=dev)
        ys = []
        for x in xs:
            xz = x @ w_in.T                      # the kernel just before the conv step
            xc = causal_conv1d_step(xz[:, :d], conv, cw, cb, silu=True, early_state=early)
            dt = xz[:, :d] @ torch.eye(d, device=dev, dtype=dtype)  # a GEMM just before the SSM step
            ys.append(ssm_decode_step(xc, dt, xz[:, d:], Bm, Cm, A, D, ssm, early_state=early))
        torch.cuda.synchronize()
        outs[early] = (torch.stack(ys), conv.clone(), ssm.clone())
    for a, c in zip(outs[False], outs[True]):
        assert torch.equal(a, c)
