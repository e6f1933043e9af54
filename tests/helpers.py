"""Shared comparison helpers for the parity tests."""

from __future__ import annotations

import numpy as np

# Tolerances from the north-star: rtol 1e-4 for fp32, 2e-3 with fp16 inputs (bf16 keeps 8 bits of
# mantissa, so its activations are compared at 1e-2). The absolute floor is the same relative factor
# times the RMS of the reference, so elements that happen to sit near zero are judged on the scale of
# the data rather than on their own magnitude.
RTOL = {"float32": 1e-4, "float16": 2e-3, "bfloat16": 1e-2}


def to_np(x):
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().float().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float32)


def assert_close(got, ref, rtol, what="", atol_scale=1.0):
    got, ref = to_np(got).astype(np.float64), to_np(ref).astype(np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    scale = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    atol = rtol * atol_scale * scale
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    if bad.any():
        i = np.unravel_index(np.argmax(err - (atol + rtol * np.abs(ref))), err.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} / {bad.size} elements outside rtol={rtol} atol={atol:.3g}; worst at {i}: "
            f"got {got[i]:.7g} ref {ref[i]:.7g} (max abs err {err.max():.3g}, ref rms {scale:.3g})")
