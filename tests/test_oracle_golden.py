"""Pins the CPU oracle to golden vectors produced by the reference's own NumPy functions
(tests/golden/make_golden.py), and the C oracle to the NumPy oracle. CPU only."""

import json

import numpy as np
import pytest

from oracle import scan_ref as R
from oracle.scan_c import selective_scan_c

COMBOS = {"baseline": (0, 0, 0), "D": (1, 0, 0), "softplus": (0, 0, 1), "z": (0, 1, 0), "D+z": (1, 1, 0),
          "D+softplus": (1, 0, 1), "all": (1, 1, 1)}


def _load(golden_dir, name):
    return dict(np.load(golden_dir / f"{name}.npz"))


def test_manifest_hashes(golden_dir):
    import hashlib

    man = json.loads((golden_dir / "MANIFEST.json").read_text())
    for fname, meta in man["files"].items():
        assert hashlib.sha256((golden_dir / fname).read_bytes()).hexdigest() == meta["sha256"], fname


@pytest.mark.parametrize("tag", ["T1024", "T4096"])
def test_features_literal_matches_reference(golden_dir, tag):
    g = _load(golden_dir, f"features_{tag}")
    for name, (ud, uz, sp) in COMBOS.items():
        if f"y_{name}" not in g:
            continue
        y = R.selective_scan_literal(g["u"], g["delta"] if sp else g["delta_sp"], g["A"], g["B"], g["C"],
                                     D=g["D"] if ud else None, z=g["z"] if uz else None, delta_softplus=bool(sp))
        # same NumPy operations in the same order: equal up to the last bits of float32
        np.testing.assert_allclose(y, g[f"y_{name}"], rtol=1e-6, atol=1e-6, err_msg=name)


@pytest.mark.parametrize("tag", ["T1024", "T4096"])
def test_fp16_reference_inputs(golden_dir, tag):
    g = _load(golden_dir, f"fp16_{tag}")
    for name, (ud, uz, sp) in COMBOS.items():
        if f"y_{name}" not in g:
            continue
        y = R.selective_scan_literal(g["u"], g["delta"], g["A"], g["B"], g["C"], D=g["D"] if ud else None,
                                     z=g["z"] if uz else None, delta_softplus=bool(sp))
        np.testing.assert_allclose(y, g[f"y_{name}"], rtol=1e-6, atol=1e-6, err_msg=name)


def test_final_state_matches_reference(golden_dir):
    g = _load(golden_dir, "state")
    for i in range(3):
        _, h = R.selective_scan_literal(g[f"u{i}"], g[f"delta{i}"], g[f"A{i}"], g[f"B{i}"], g[f"C{i}"],
                                        return_state=True)
        np.testing.assert_allclose(h, g[f"h{i}"], rtol=1e-6, atol=1e-6)


def test_chunk_boundaries_match_reference(golden_dir):
    g = _load(golden_dir, "chunked")
    for i in range(4):
        y = R.selective_scan_literal(g[f"u{i}"], g[f"delta{i}"], g[f"A{i}"], g[f"B{i}"], g[f"C{i}"])
        np.testing.assert_allclose(y, g[f"y{i}"], rtol=1e-6, atol=1e-6)


def test_pair_scan_known_answers(golden_dir):
    g = _load(golden_dir, "pair_scan")
    for i in range(6):
        np.testing.assert_allclose(R.pair_scan_literal(g[f"a{i}"], g[f"b{i}"]), g[f"h{i}"], rtol=1e-6, atol=1e-6)
    # pair_scan.py:57-60: a = 0.5, b = 1 converges to 2
    assert abs(g["h0"][-1] - 2.0) < 1e-6


def test_config0_and_generator(golden_dir):
    g = _load(golden_dir, "config0")
    inp = R.make_baseline_inputs(1, 16, 16, 2048, seed=0)
    for k in ("u", "delta", "A", "B", "C", "D", "z"):
        np.testing.assert_array_equal(inp[k], g[k], err_msg=f"generator drift in {k}")
    y, h = R.selective_scan_literal(**inp, delta_softplus=True, return_state=True)
    np.testing.assert_allclose(y, g["y"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(h, g["h"], rtol=1e-6, atol=1e-6)


def test_c_oracle_matches_numpy(golden_dir):
    g = _load(golden_dir, "config0")
    y, h = selective_scan_c(g["u"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], delta_softplus=True)
    np.testing.assert_allclose(y, g["y"], rtol=1e-4, atol=1e-4 * np.sqrt(np.mean(g["y"] ** 2)))
    np.testing.assert_allclose(h, g["h"], rtol=1e-4, atol=1e-5)
    g = _load(golden_dir, "features_T1024")
    y, _ = selective_scan_c(g["u"], g["delta"], g["A"], g["B"], g["C"], None, None, delta_softplus=True)
    np.testing.assert_allclose(y, g["y_softplus"], rtol=1e-4, atol=1e-4 * np.sqrt(np.mean(g["y_softplus"] ** 2)))


def test_vectorised_oracle_matches_literal(golden_dir):
    g = _load(golden_dir, "config0")
    y, h = R.selective_scan_vec(g["u"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], delta_softplus=True,
                                return_state=True)
    np.testing.assert_allclose(y, g["y"], rtol=1e-4, atol=1e-4 * np.sqrt(np.mean(g["y"] ** 2)))
    np.testing.assert_allclose(h, g["h"], rtol=1e-4, atol=1e-5)


def test_conv_ref_matches_torch_conv1d():
    import torch

    inp = R.make_conv_inputs(2, 5, 37, seed=3)
    ref = R.causal_conv1d_ref(inp["x"], inp["weight"], inp["bias"], silu_act=False)
    t = torch.nn.functional.conv1d(torch.from_numpy(inp["x"]), torch.from_numpy(inp["weight"])[:, None, :],
                                   torch.from_numpy(inp["bias"]), padding=3, groups=5)[..., :37]
    np.testing.assert_allclose(ref, t.numpy(), rtol=1e-5, atol=1e-6)


def test_step_refs_agree_with_scan_and_conv():
    """Running the decode-step formulas token by token reproduces the parallel conv and scan."""
    rng = np.random.default_rng(5)
    b, d, n, L = 2, 3, 4, 9
    x = rng.standard_normal((b, d, L)).astype(np.float32)
    w = rng.uniform(-0.5, 0.5, (d, 4)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, d).astype(np.float32)
    conv = R.causal_conv1d_ref(x, w, bias)
    st = np.zeros((b, d, 4), np.float32)
    for t in range(L):
        out, st = R.conv_step_ref(x[:, :, t], st, w, bias)
        np.testing.assert_allclose(out, conv[:, :, t], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st, R.conv_state_ref(x), rtol=0, atol=0)
    inp = R.make_features_inputs(b, d, n, L, seed=1)
    y, hT = R.selective_scan_literal(**inp, delta_softplus=True, return_state=True)
    h = np.zeros((b, d, n), np.float32)
    for t in range(L):
        yt, h = R.ssm_step_ref(inp["u"][:, :, t], inp["delta"][:, :, t], inp["z"][:, :, t], inp["B"][:, :, t],
                               inp["C"][:, :, t], inp["A"], inp["D"], h)
        np.testing.assert_allclose(yt, y[:, :, t], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(h, hT, rtol=1e-4, atol=1e-6)
