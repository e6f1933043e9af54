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


def assert_close_lowp(got, ref, what="", rel_l2=1e-2, axis=None, slice_rel_l2=5e-2):
    """Comparison for bf16-stored activations: relative L2 error at most ``rel_l2`` over the whole tensor
    and at most ``slice_rel_l2`` over every slice along ``axis`` (e.g. per channel), so that a wrong
    channel, token or row cannot hide in the bulk. Element-wise bounds do not fit bf16 storage: two
    computations that round the same float32 values to bf16 differ where accumulation order moves a value
    across a rounding boundary, which moves that value by one bf16 ulp (2^-8 relative; up to 2^-5 for
    delta = softplus(dt) with dt in [-8, -4), where bf16 spacing is 2^-5) and everything computed from it,
    and a sum with cancellation (a state element near zero) can turn that into a large relative error of
    a single element. Returns the whole-tensor relative L2 error."""
    got, ref = to_np(got).astype(np.float64), to_np(ref).astype(np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    assert rel <= rel_l2, f"{what}: relative L2 error {rel:.3g} > {rel_l2}"
    if axis is not None:
        other = tuple(i for i in range(ref.ndim) if i != axis % ref.ndim)
        num = np.sqrt(np.sum((got - ref) ** 2, axis=other))
        den = np.maximum(np.sqrt(np.sum(ref ** 2, axis=other)), 1e-30)
        worst = int(np.argmax(num / den))
        assert num[worst] / den[worst] <= slice_rel_l2, (
            f"{what}: slice {worst} along axis {axis} has relative L2 error {num[worst] / den[worst]:.3g} > "
            f"{slice_rel_l2}")
    return rel
