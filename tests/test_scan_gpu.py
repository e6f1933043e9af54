"""Selective-scan kernel parity against the CPU oracle (GPU). The kernel is reached through the public
``selective_scan`` API or ``selective_scan_into`` (both call mm_selective_scan_fwd in libmamba_b200.so)."""

import ctypes

import numpy as np
import pytest
import torch

from mamba_metal_b200 import _lib, selective_scan
from mamba_metal_b200.selective_scan import selective_scan_into
from oracle import scan_ref as R
from oracle.scan_c import selective_scan_c
from tests.helpers import RTOL, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
COMBOS = {"baseline": (0, 0, 0), "D": (1, 0, 0), "softplus": (0, 0, 1), "z": (0, 1, 0), "D+z": (1, 1, 0),
          "D+softplus": (1, 0, 1), "all": (1, 1, 1)}


def T(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.asarray(a)).to(DEV, dtype)


def run(inp, dtype=torch.float32, D=True, z=True, sp=True, state=True, **kw):
    y = selective_scan(T(inp["u"], dtype), T(inp["delta"], dtype), T(inp["A"]), T(inp["B"], dtype),
                       T(inp["C"], dtype), D=T(inp.get("D")) if D else None, z=T(inp.get("z"), dtype) if z else None,
                       delta_softplus=sp, return_state=state, **kw)
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("tag", ["T1024", "T4096"])
def test_feature_matrix_fp32_golden(golden_dir, tag):
    """All D / z / softplus combinations of experiments/09-features/test_features.py, vs the reference."""
    g = dict(np.load(golden_dir / f"features_{tag}.npz"))
    for name, (ud, uz, sp) in COMBOS.items():
        if f"y_{name}" not in g:
            continue
        inp = dict(g, delta=g["delta"] if sp else g["delta_sp"])
        y, _ = run(inp, D=ud, z=uz, sp=bool(sp))
        assert y.dtype == torch.float32
        assert_close(y, g[f"y_{name}"], RTOL["float32"], f"features {tag} {name}")


@pytest.mark.parametrize("tag", ["T1024", "T4096"])
def test_fp16_golden(golden_dir, tag):
    """experiments/10-fp16/test_fp16.py: fp16 u/delta/B/C/z, fp32 A/D, output dtype fp16."""
    g = dict(np.load(golden_dir / f"fp16_{tag}.npz"))
    for name, (ud, uz, sp) in COMBOS.items():
        if f"y_{name}" not in g:
            continue
        y, _ = run(g, torch.float16, D=ud, z=uz, sp=bool(sp))
        assert y.dtype == torch.float16
        # against the oracle on the fp16-rounded inputs (kernel error only) ...
        r16 = {k: (np.asarray(v, np.float16).astype(np.float32) if k in ("u", "delta", "B", "C", "z") else v)
               for k, v in g.items()}
        ref = R.selective_scan_literal(r16["u"], r16["delta"], r16["A"], r16["B"], r16["C"],
                                       D=r16["D"] if ud else None, z=r16["z"] if uz else None, delta_softplus=bool(sp))
        assert_close(y, ref, RTOL["float16"], f"fp16 {tag} {name}")
        # ... and against the reference's fp32 golden on the unrounded inputs, as the reference test does
        # (test_fp16.py:98-101 prints the error with |ref| > 1e-2, "~1e-3 typical"). That error is set by
        # rounding the inputs to fp16 (2^-11 each), not by the kernel: bound it in absolute terms on the
        # data's scale, and the median relative error at the reference's "typical" level.
        gold = g[f"y_{name}"]
        yy = y.float().cpu().numpy()
        mask = np.abs(gold) > 1e-2
        assert np.median(np.abs(yy[mask] - gold[mask]) / np.abs(gold[mask])) < 2e-3
        assert np.max(np.abs(yy - gold)) < 1e-2 * max(1.0, np.abs(gold).max())


def test_final_state_golden(golden_dir):
    """experiments/18-prefill/verify_state_out.py shapes."""
    g = dict(np.load(golden_dir / "state.npz"))
    for i in range(3):
        inp = {k: g[f"{k}{i}"] for k in ("u", "delta", "A", "B", "C")}
        y, h = run(inp, D=False, z=False, sp=False)
        assert_close(h, g[f"h{i}"], RTOL["float32"], f"state case {i}")


def test_chunk_boundaries_golden(golden_dir):
    """experiments/07-chunked shapes incl. seqlen 1025 (one past a 1024 chunk)."""
    g = dict(np.load(golden_dir / "chunked.npz"))
    for i in range(4):
        inp = {k: g[f"{k}{i}"] for k in ("u", "delta", "A", "B", "C")}
        y, _ = run(inp, D=False, z=False, sp=False)
        assert_close(y, g[f"y{i}"], RTOL["float32"], f"chunked case {i}")


def test_config0_golden(golden_dir):
    """fp32 (1,16,2048), N=16, D, z, softplus; y and last state."""
    g = dict(np.load(golden_dir / "config0.npz"))
    y, h = run(g)
    assert_close(y, g["y"], RTOL["float32"], "config0 y")
    assert_close(h, g["h"], RTOL["float32"], "config0 state")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1, 1), (1, 3, 7), (2, 5, 31), (1, 33, 33), (3, 40, 1023), (1, 64, 1025),
                                   (2, 17, 4097), (2, 48, 4096)])
@pytest.mark.parametrize("use_tma", [True, False])
def test_odd_shapes(dtype, shape, use_tma):
    b, d, L = shape
    inp = R.make_baseline_inputs(b, d, 16, L, seed=L + d)
    y, h = _into(inp, dtype, use_tma=use_tma)
    q = {k: (torch.as_tensor(v).to(dtype).float().numpy() if k in ("u", "delta", "B", "C", "z") else v)
         for k, v in inp.items()}
    yr, hr = R.selective_scan_vec(q["u"], q["delta"], q["A"], q["B"], q["C"], q["D"], q["z"], delta_softplus=True,
                                  return_state=True, dtype=np.float64)
    name = str(dtype).split(".")[-1]
    assert_close(y, yr, RTOL[name], f"{shape} {name} y")
    assert_close(h, hr, RTOL["float32"] if dtype == torch.float32 else 1e-3, f"{shape} {name} state")


@pytest.mark.parametrize("piece_tiles", [1, 2, 3, 5, 16])
@pytest.mark.parametrize("general_A", [False, True])
@pytest.mark.parametrize("use_tma", [True, False])
def test_small_pieces_lookback(piece_tiles, general_A, use_tma):
    """Forces many warps per sequence, so carries pass through long look-back chains (TMA and
    cp.async staging)."""
    inp = R.make_baseline_inputs(2, 70, 16, 2000, seed=7)
    if general_A:
        inp["A"] = -np.random.default_rng(1).uniform(0.1, 2.0, size=(70, 16)).astype(np.float32)
    out = _into(inp, torch.float32, piece_tiles, use_tma=use_tma)
    yr, hr = R.selective_scan_vec(**inp, delta_softplus=True, return_state=True, dtype=np.float64)
    assert_close(out[0], yr, RTOL["float32"], f"pieces={piece_tiles} general={general_A} y")
    assert_close(out[1], hr, RTOL["float32"], f"pieces={piece_tiles} general={general_A} state")


def _into(inp, dtype, piece_tiles=0, sp=True, channels_last=False, use_tma=True):
    b, d, L = inp["u"].shape
    n = inp["A"].shape[1]
    t = lambda k: T(inp[k], dtype)
    if channels_last:
        cl = lambda k: T(np.ascontiguousarray(np.transpose(inp[k], (0, 2, 1))), dtype).transpose(1, 2)
        u, de, z, Bm, Cm = cl("u"), cl("delta"), cl("z"), cl("B"), cl("C")
        y = torch.empty((b, L, d), dtype=dtype, device=DEV).transpose(1, 2)
    else:
        u, de, z, Bm, Cm = t("u"), t("delta"), t("z"), t("B"), t("C")
        y = torch.empty((b, d, L), dtype=dtype, device=DEV)
    h = torch.empty((b, d, n), dtype=torch.float32, device=DEV)
    ws = selective_scan_into(u, de, T(inp["A"]), Bm, Cm, T(inp["D"]), z, y, h, sp, piece_tiles=piece_tiles,
                             use_tma=use_tma)
    rc = _lib.lib().mm_selective_scan_status(ws.data_ptr(), _lib.stream_handle(torch.device(DEV)))
    assert rc == 0, f"carry hand-off status {rc}"
    return y, h


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_channels_last_views(dtype):
    """Strided (channels-last) u/delta/z/y and B/C views, as the model passes them."""
    inp = R.make_baseline_inputs(2, 96, 16, 777, seed=11)
    y, h = _into(inp, dtype, channels_last=True)
    q = {k: (torch.as_tensor(v).to(dtype).float().numpy() if k in ("u", "delta", "B", "C", "z") else v)
         for k, v in inp.items()}
    yr, hr = R.selective_scan_vec(**q, delta_softplus=True, return_state=True, dtype=np.float64)
    name = str(dtype).split(".")[-1]
    assert_close(y, yr, RTOL[name], "channels-last y")
    assert_close(h, hr, RTOL["float32"] if dtype == torch.float32 else 1e-3, "channels-last state")


def test_negative_delta_without_softplus_and_growing_states():
    """No softplus with negative deltas (decay bound not monotone) and A >= 0 for some states: the
    carry recompute must run to the end of every piece."""
    inp = R.make_features_inputs(1, 40, 16, 1500, seed=3)   # delta ~ U(-1, 2), used raw
    inp["delta"] = inp["delta"] * 0.05
    inp["A"][:, 3] = 0.0
    inp["A"][:5, 7] = 0.01
    y, h = _into(inp, torch.float32, piece_tiles=8, sp=False)
    yr, hr = R.selective_scan_vec(**inp, delta_softplus=False, return_state=True, dtype=np.float64)
    assert_close(y, yr, RTOL["float32"], "y")
    assert_close(h, hr, RTOL["float32"], "state")


@pytest.mark.parametrize("n", [1, 4, 8, 12, 16, 17, 33, 64])
def test_dstate_range(n):
    inp = R.make_features_inputs(2, 9, n, 300, seed=n)
    y, h = run(inp)
    yr, hr = R.selective_scan_vec(**inp, delta_softplus=True, return_state=True, dtype=np.float64)
    assert_close(y, yr, RTOL["float32"], f"dstate {n} y")
    assert_close(h, hr, RTOL["float32"], f"dstate {n} state")


def test_structured_A_near_exact_log_init():
    """A = -exp(log(1..N)) in fp32 (the model's A_log init) is within a few ulp of (n+1)*A[0] and takes
    the multiply-chain path; results must match the general formula."""
    inp = R.make_baseline_inputs(1, 64, 16, 1200, seed=5)
    inp["A"] = -np.exp(np.log(np.arange(1, 17, dtype=np.float32)))[None].repeat(64, 0).astype(np.float32)
    y, h = run(inp)
    yr, hr = R.selective_scan_vec(**inp, delta_softplus=True, return_state=True, dtype=np.float64)
    assert_close(y, yr, RTOL["float32"], "y")
    assert_close(h, hr, RTOL["float32"], "state")


def test_empty_and_mixed_dtype():
    u = torch.zeros((2, 3, 0), device=DEV)
    y, h = selective_scan(u, u, torch.zeros(3, 16, device=DEV), torch.zeros(2, 16, 0, device=DEV),
                          torch.zeros(2, 16, 0, device=DEV), return_state=True)
    assert y.shape == (2, 3, 0) and torch.count_nonzero(h) == 0
    inp = R.make_baseline_inputs(1, 8, 16, 100, seed=2)
    # fp16 u with fp32 delta: computed in fp32, output in u's dtype
    y = selective_scan(T(inp["u"], torch.float16), T(inp["delta"]), T(inp["A"]), T(inp["B"]), T(inp["C"]),
                       D=T(inp["D"], torch.float16), z=T(inp["z"]), delta_softplus=True)
    assert y.dtype == torch.float16
    q = dict(inp, u=np.asarray(inp["u"], np.float16).astype(np.float32))
    assert_close(y, R.selective_scan_vec(**q, delta_softplus=True), RTOL["float16"], "mixed")


def test_config1_full_size_vs_c_oracle():
    """BASELINE configs[1] scan at full size (fp16 (8,1536,4096), N=16, D, z, softplus) against the C
    oracle on the fp16-rounded inputs: y (all elements) and final state."""
    inp = R.make_baseline_inputs(8, 1536, 16, 4096, seed=0)
    q = {k: (np.asarray(v, np.float16).astype(np.float32) if k in ("u", "delta", "B", "C", "z") else v)
         for k, v in inp.items()}
    y, h = run(inp, torch.float16)
    yr, hr = selective_scan_c(**q, delta_softplus=True)
    assert_close(y, yr, RTOL["float16"], "config1 y")
    assert_close(h, hr, 1e-3, "config1 state")


def test_config1_full_size_general_A_vs_c_oracle():
    """configs[1] shape and distributions with a trained-checkpoint-like A instead of -(n+1): A = -exp(A_log),
    A_log ~ U(log 0.5, log 16) per (channel, state), so the kernel takes its general-A path (one exp2 per
    state and step, part of them on the FMA pipe). Same checks as the structured case."""
    inp = R.make_baseline_inputs(8, 1536, 16, 4096, seed=0)
    rng = np.random.default_rng(7)
    inp["A"] = (-np.exp(rng.uniform(np.log(0.5), np.log(16.0), size=(1536, 16)))).astype(np.float32)
    q = {k: (np.asarray(v, np.float16).astype(np.float32) if k in ("u", "delta", "B", "C", "z") else v)
         for k, v in inp.items()}
    y, h = run(inp, torch.float16)
    yr, hr = selective_scan_c(**q, delta_softplus=True)
    assert_close(y, yr, RTOL["float16"], "config1 general-A y")
    assert_close(h, hr, 1e-3, "config1 general-A state")


def test_deterministic_and_l2_independent():
    inp = R.make_baseline_inputs(4, 256, 16, 3000, seed=9)
    y1, h1 = run(inp, torch.float16)
    y2, h2 = run(inp, torch.float16)
    assert torch.equal(y1, y2) and torch.equal(h1, h2)


def test_config4_long_context_final_state():
    """fp16 (4, 5120, 131072), N 16, D / z / softplus, the inputs bench.py's `long`
    workload times (on-device seeded generators). Six sampled (batch, channel) rows -- all 131,072 outputs
    and the final state -- against the C oracle on the same fp16-rounded inputs, in fp32."""
    import bench
    from oracle.scan_c import selective_scan_c

    dev = torch.device(DEV)
    d = bench.make_long_inputs(dev, 0, bench.LONG["dim"])
    y, h = selective_scan(d["u"], d["delta"], d["A"], d["B"], d["C"], D=d["D"], z=d["z"], delta_softplus=True,
                          return_state=True)
    for b, c in [(0, 0), (1, 777), (2, 2560), (3, 5119), (0, 4001), (3, 1234)]:
        row = lambda t: np.ascontiguousarray(t[b:b + 1, c:c + 1].float().cpu().numpy())
        yr, hr = selective_scan_c(row(d["u"]), row(d["delta"]), d["A"][c:c + 1].cpu().numpy(),
                                  d["B"][b:b + 1].float().cpu().numpy(), d["C"][b:b + 1].float().cpu().numpy(),
                                  d["D"][c:c + 1].cpu().numpy(), row(d["z"]), delta_softplus=True)
        assert_close(h[b, c], hr[0, 0], 2e-3, f"final state ({b},{c})")
        assert_close(y[b, c].float(), yr[0, 0], 2e-3, f"y ({b},{c})")
    del d, y, h
    torch.cuda.empty_cache()


def test_exp2_poly_accuracy():
    """The FMA-pipe 2^x that carries part of the general-A scan's exponentials: relative error within
    2.5e-7 of the exact value over the decay range (x in [-125, 0], plus a few positive arguments), no
    worse than 2x the hardware ex2.approx's own error on the same points."""
    import ctypes

    from mamba_metal_b200 import _lib

    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.linspace(-125.0, 0.0, 1_000_001), -torch.rand(1_000_000, generator=g) * 40,
                   torch.rand(1000, generator=g) * 8, torch.tensor([0.0, -0.5, 0.5, -1.0, -124.99])])
    xd = x.to(DEV)
    yp, ym = torch.empty_like(xd), torch.empty_like(xd)
    with torch.cuda.device(DEV):
        rc = _lib.lib().mm_exp2_check(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(yp.data_ptr()),
                                      ctypes.c_void_p(ym.data_ptr()), x.numel(), _lib.stream_handle(torch.device(DEV)))
    assert rc == 0
    exact = torch.exp2(x.double())
    ep = ((yp.cpu().double() - exact).abs() / exact).max().item()
    em = ((ym.cpu().double() - exact).abs() / exact).max().item()
    print(f"exp2 max relative error: polynomial {ep:.3g}, ex2.approx {em:.3g}")
    assert ep <= 2.5e-7 and ep <= 2 * max(em, 1.2e-7)


@pytest.mark.parametrize("use_tma", [True, False])
def test_delta_bias_equals_biased_delta(use_tma):
    """delta_bias (a Mamba block's dt_proj bias, added inside the scan before softplus) gives bit-identical
    outputs to passing delta + bias (added in float32 beforehand) -- with one piece per row, so that no
    carry hand-off is involved (the look-back may combine a predecessor's published prefix or walk its
    aggregates, which round differently) -- and, with the library's own piece plan, matches the oracle.
    The layout is the model's channel-first prefill one: (B, c, L) views of (c, B*L) buffers."""
    b, d, n, L = 3, 80, 16, 520
    inp = R.make_baseline_inputs(b, d, n, L, seed=21)
    bias = np.random.default_rng(5).normal(size=(d,)).astype(np.float32) - 3.0
    cf = lambda a: T(np.ascontiguousarray(np.transpose(a, (1, 0, 2))).reshape(a.shape[1], -1)).view(
        a.shape[1], b, L).permute(1, 0, 2)
    u, de, z, Bm, Cm = (cf(inp[k]) for k in ("u", "delta", "z", "B", "C"))
    de_b = cf(inp["delta"] + bias[None, :, None])
    outs = []
    whole_rows = (L + 7) // 8  # fp32 tiles of 8 steps per row
    for delta, db, pieces in ((de, T(bias), whole_rows), (de_b, None, whole_rows), (de, T(bias), 0)):
        y = torch.empty((d, b * L), device=DEV).view(d, b, L).permute(1, 0, 2)
        h = torch.empty((b, d, n), device=DEV)
        selective_scan_into(u, delta, T(inp["A"]), Bm, Cm, T(inp["D"]), z, y, h, True, use_tma=use_tma,
                            delta_bias=db, piece_tiles=pieces)
        outs.append((y, h))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    q = dict(inp)
    q["delta"] = inp["delta"] + bias[None, :, None]
    yr, hr = R.selective_scan_vec(**q, delta_softplus=True, return_state=True, dtype=np.float64)
    for y, h in (outs[0], outs[2]):
        assert_close(y, yr, RTOL["float32"], "delta_bias y")
        assert_close(h, hr, RTOL["float32"], "delta_bias state")
