"""The exp2 polynomial coefficients in mm_common.cuh are the ones the committed Remez derivation
(mamba_metal_b200/csrc/exp2_poly.py) produces, and their float32 Horner evaluation stays within the
error the source states (2.2e-7 relative on [-1/2, 1/2]). CPU only."""

import importlib.util
import re
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "mamba_metal_b200" / "csrc"


def _derivation():
    spec = importlib.util.spec_from_file_location("exp2_poly", CSRC / "exp2_poly.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _source_coefficients():
    src = (CSRC / "mm_common.cuh").read_text()
    body = src[src.index("MM_DEV f2_t exp2_poly2"):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"f2_pack\(([0-9.e+-]+)f, \1f\)", body)]
    return vals[::-1][:6]  # Horner order is c5 .. c0 -> c0 .. c5


def test_coefficients_match_remez_derivation():
    c = _derivation().remez(5).astype(np.float32)
    src = np.array(_source_coefficients(), dtype=np.float32)
    assert src.shape == (6,)
    np.testing.assert_allclose(src, c, rtol=2e-7)


def test_float32_evaluation_error_bound():
    c = np.array(_source_coefficients(), dtype=np.float32)
    f = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    p = np.full_like(f, c[5])
    for k in range(4, -1, -1):
        p = (p.astype(np.float64) * f + np.float64(c[k])).astype(np.float32)
    rel = np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1)
    assert rel.max() < 2.2e-7
