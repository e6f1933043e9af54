"""The tcgen05 decode GEMM (mm_linear_fwd): y = x @ w.T (+ bias) for the decode step's projections.

Shapes are the Mamba-2.8b decode projections at batch 64 (in_proj, x_proj, dt_proj, out_proj of
mamba_metal/mamba_block.py:167-197) at tensor-parallel widths 1 and 8, plus ragged ones (M, N, K not
multiples of the tile). The reference is the same product in float64 on the bf16-rounded operands; the
kernel accumulates in fp32, so the bound is a few fp32 ulps of the sum of |x||w| terms.
"""

import pytest
import torch

from mamba_metal_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")

SHAPES = [
    # (M, N, K): 2.8b decode at TP 1
    (64, 10240, 2560), (64, 192, 5120), (64, 5120, 160), (64, 2560, 5120),
    # TP 8 slices
    (64, 1280, 2560), (64, 192, 640), (64, 640, 160), (64, 2560, 640),
    # ragged
    (1, 100, 64), (7, 129, 200), (63, 300, 1000), (100, 256, 512), (130, 64, 72),
]


def _check(x, w, bias, y, out_dtype):
    ref = x.double() @ w.double().T
    if bias is not None:
        ref = ref + bias.double()
    mag = x.double().abs() @ w.double().abs().T + 1e-30
    err = (y.double() - ref).abs()
    if out_dtype == torch.float32:
        bound = 1e-5 * mag + 1e-6
    else:
        bound = 1e-5 * mag + ref.abs() * 2.0 ** -8 + 1e-6
    bad = err > bound
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} outside the bound; max err {float(err.max()):.3e}"


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_linear_matches_float64(shape, out_dtype):
    M, N, K = shape
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N * 3 + K)
    x = torch.randn((M, K), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g, device=DEV) * K ** -0.5).to(torch.bfloat16)
    bias = torch.randn((N,), generator=g, device=DEV) if N % 2 == 0 else None
    y = ops.linear(x, w, bias, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert ops.linear_status(DEV) == 0
    _check(x, w, bias, y, out_dtype)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 40])
def test_linear_split_counts_agree(splits):
    """Every split count gives the same sums up to fp32 reassociation (split partials are added in arrival
    order), on repeated calls too: each call must leave the workspace's sum tiles and counters at zero."""
    M, N, K = 64, 384, 2560
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((M, K), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    for _ in range(3):
        y = ops.linear(x, w, out_dtype=torch.float32, splits=splits)
        torch.cuda.synchronize()
        _check(x, w, None, y, torch.float32)
    if splits == 1:
        assert torch.equal(y, ops.linear(x, w, out_dtype=torch.float32, splits=1))


def test_linear_strided_views():
    """x and out as column slices of wider row-major buffers (the decode step's x_dbl[:, :dt_rank] and
    xz[:, :d_inner] views)."""
    g = torch.Generator(device=DEV).manual_seed(11)
    big = torch.randn((64, 192), generator=g, device=DEV).to(torch.bfloat16)
    x = big[:, :160]
    w = torch.randn((512, 160), generator=g, device=DEV).to(torch.bfloat16)
    outbuf = torch.zeros((64, 1024), dtype=torch.bfloat16, device=DEV)
    y = ops.linear(x, w, out=outbuf[:, 256:768])
    torch.cuda.synchronize()
    _check(x, w, None, y, torch.bfloat16)
    assert torch.all(outbuf[:, :256] == 0) and torch.all(outbuf[:, 768:] == 0)
