"""The C-ABI library loads and exports every entry point include/mamba_b200.h declares; argument
validation that needs no GPU returns the documented status codes. CPU only (no compute calls)."""

import ctypes

import pytest

from mamba_metal_b200 import _lib


def test_header_declares_entry_points():
    names = _lib.header_functions()
    assert set(names) >= {"mm_selective_scan_workspace_size", "mm_selective_scan_fwd", "mm_selective_scan_status",
                          "mm_causal_conv1d_fwd", "mm_causal_conv1d_step", "mm_ssm_decode_step",
                          "mm_add_rmsnorm", "mm_version"}


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _lib.header_functions():
        assert hasattr(lib, name), f"{name} declared in include/mamba_b200.h but not exported"
    assert b"sm_100a" in lib.mm_version()


def test_struct_layouts_are_padding_free():
    # all fields are 8 bytes wide, so sizeof == 8 * field count on every FFI
    for s, n in ((_lib.MMScanArgs, 9 + 5 + 6 * 3 + 2 + 3 + 1), (_lib.MMConvArgs, 5 + 4 + 1 + 6 + 1),
                 (_lib.MMConvStepArgs, 5 + 1 + 3 + 2 + 1 + 1), (_lib.MMSSMStepArgs, 9 + 1 + 3 + 6 + 1 + 1 + 3 + 3),
                 (_lib.MMAddNormArgs, 4 + 1 + 2 + 2 + 1), (_lib.MMLinearArgs, 4 + 3 + 1 + 3 + 1)):
        assert ctypes.sizeof(s) == 8 * n, s.__name__


def _scan_args(**kw):
    a = _lib.MMScanArgs()
    a.dtype, a.batch, a.dim, a.dstate, a.seqlen, a.piece_tiles = 1, 2, 64, 16, 1000, 4
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_size_and_validation():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.mm_selective_scan_workspace_size(ctypes.byref(_scan_args()), ctypes.byref(n)) == 0
    assert n.value >= 256 and n.value % 256 == 0
    assert lib.mm_selective_scan_workspace_size(ctypes.byref(_scan_args(dstate=65)), ctypes.byref(n)) == -2
    assert lib.mm_selective_scan_workspace_size(ctypes.byref(_scan_args(dtype=7)), ctypes.byref(n)) == -3
    assert lib.mm_selective_scan_workspace_size(ctypes.byref(_scan_args(seqlen=-1)), ctypes.byref(n)) == -2
    assert lib.mm_selective_scan_workspace_size(None, ctypes.byref(n)) == -1
    # fwd rejects missing tensors / workspace before touching the device
    a = _scan_args()
    assert lib.mm_selective_scan_fwd(ctypes.byref(a), None, 0, None) == -1


def test_conv_and_step_validation():
    lib = _lib.lib()
    c = _lib.MMConvArgs()
    c.dtype, c.batch, c.dim, c.seqlen, c.width = 1, 1, 8, 16, 3
    assert lib.mm_causal_conv1d_fwd(ctypes.byref(c), None) == -2  # width must be 4
    c.width, c.dtype = 4, 9
    assert lib.mm_causal_conv1d_fwd(ctypes.byref(c), None) == -3
    c.dtype = 0
    assert lib.mm_causal_conv1d_fwd(ctypes.byref(c), None) == -1  # null pointers
    s = _lib.MMSSMStepArgs()
    s.dtype, s.batch, s.dim, s.dstate = 0, 1, 8, 65
    assert lib.mm_ssm_decode_step(ctypes.byref(s), None) == -2
    s.dstate, s.dt_w, s.dt_rank = 16, 16, 0  # fused dt projection (dt_w set, never dereferenced) without a rank
    assert lib.mm_ssm_decode_step(ctypes.byref(s), None) == -2
    r = _lib.MMAddNormArgs()
    r.dtype, r.rows, r.dim = 0, 1, 0
    assert lib.mm_add_rmsnorm(ctypes.byref(r), None) == -2


def test_cpu_tensors_fail_loudly():
    import torch

    from mamba_metal_b200 import selective_scan

    u = torch.zeros(1, 2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan(u, u, torch.zeros(2, 4), torch.zeros(1, 4, 8), torch.zeros(1, 4, 8))
    with pytest.raises(AssertionError):
        selective_scan(u, torch.zeros(1, 2, 9), torch.zeros(2, 4), torch.zeros(1, 4, 8), torch.zeros(1, 4, 8))


def test_ssm_step_fused_dt_argument_checks():
    """Host-side checks of the fused dt projection arguments (ops.ssm_decode_step), which run before any
    device work, and the loud failure on CPU tensors."""
    import torch

    from mamba_metal_b200 import ops

    bf = torch.bfloat16
    x = torch.zeros(2, 8, dtype=bf)
    B = C = torch.zeros(2, 16, dtype=bf)
    A, st = torch.zeros(8, 16), torch.zeros(2, 8, 16)
    dt_in, w = torch.zeros(2, 16, dtype=bf), torch.zeros(8, 16, dtype=bf)
    with pytest.raises(AssertionError):  # neither dt nor dt_weight
        ops.ssm_decode_step(x, None, None, B, C, A, None, st)
    with pytest.raises(AssertionError):  # dt_weight's rank differs from dt_in's
        ops.ssm_decode_step(x, None, None, B, C, A, None, st, dt_in=dt_in, dt_weight=torch.zeros(8, 32, dtype=bf))
    with pytest.raises(AssertionError):  # dt_weight rows must be the channels
        ops.ssm_decode_step(x, None, None, B, C, A, None, st, dt_in=dt_in, dt_weight=torch.zeros(4, 16, dtype=bf))
    with pytest.raises(AssertionError):  # the bias is float32
        ops.ssm_decode_step(x, None, None, B, C, A, None, st, dt_in=dt_in, dt_weight=w,
                            dt_bias=torch.zeros(8, dtype=bf))
    with pytest.raises(AssertionError):  # dt_in of another dtype than x
        ops.ssm_decode_step(x, None, None, B, C, A, None, st, dt_in=dt_in.float(), dt_weight=w)
    with pytest.raises(RuntimeError, match="CUDA"):  # valid arguments, CPU tensors: no CPU path
        ops.ssm_decode_step(x, None, None, B, C, A, None, st, dt_in=dt_in, dt_weight=w, dt_bias=torch.zeros(8))


def test_linear_workspace_plan():
    """mm_linear_workspace_size: the host-side plan of the small-batch GEMM (128-row weight tiles, 64-row
    activation tiles, 64-wide K blocks): a fixed 256-byte header plus 4096 tile counters, and one fp32
    128 x 64 partial tile per output tile when K is split. Without a device the SM count is taken as 148
    (two CTAs each: a 296-CTA wave)."""
    lib = _lib.lib()
    head = 256 + 4096 * 4
    tile = 128 * 64 * 4

    def ws(M, N, K, splits, y_dtype=2):
        a = _lib.MMLinearArgs()
        a.M, a.N, a.K, a.splits, a.y_dtype = M, N, K, splits, y_dtype
        n = ctypes.c_size_t(0)
        rc = lib.mm_linear_workspace_size(ctypes.byref(a), ctypes.byref(n))
        return rc, n.value

    assert ws(64, 192, 5120, 1) == (0, head)                 # unsplit: no partial tiles
    assert ws(64, 192, 5120, 4) == (0, head + 2 * tile)      # x_proj: 2 weight tiles x 1 batch tile, split
    assert ws(64, 192, 64, 8) == (0, head)                   # one K block: the split is clamped to 1
    assert ws(64 * 4097, 128, 5120, 4) == (0, head)          # more tiles than counter slots: not split
    assert ws(64, 10240, 2560, 0) == (0, head + 80 * tile)   # in_proj, library's choice: 80 tiles split 3 ways
    assert ws(64, 192, 5120, 0, y_dtype=0) == (0, head + 2 * tile)  # fp32 output, split up to 16 ways
    assert ws(0, 192, 5120, 0)[0] == -2                      # empty shapes are refused
    assert ws(64, 192, 5120, 0, y_dtype=1)[0] == -3          # fp16 output is not offered
    assert lib.mm_linear_workspace_size(None, ctypes.byref(ctypes.c_size_t(0))) == -1


def test_scan_work_plan():
    """The scan's work plan, read back through mm_selective_scan_workspace_size: a 256-byte header, then
    (each part 256-byte aligned) one 128-byte carry flag line, one aggregate (NM + 1 rows of 32 floats) and
    one prefix (NM rows of 32 floats) per warp, so the size gives the warp count. Without a device the plan
    targets 148 SMs x 3 CTAs x 4 warps = 1776 resident warps. Tiles are 32 bytes of time per row."""
    lib = _lib.lib()

    def a256(x):
        return (x + 255) // 256 * 256

    def size_for(n_warps, nm=16):
        return 256 + a256(128 * max(n_warps, 1)) + a256(4 * n_warps * (nm + 1) * 32) + a256(4 * n_warps * nm * 32)

    def ws(**kw):
        a = _scan_args(piece_tiles=0)
        for k, v in kw.items():
            setattr(a, k, v)
        n = ctypes.c_size_t(0)
        assert lib.mm_selective_scan_workspace_size(ctypes.byref(a), ctypes.byref(n)) == 0
        return n.value

    # configs[1] (fp16 8 x 1536 x 4096): 98304 tiles in pieces of ceil(98304 / 1776) = 56 tiles, cut inside rows
    assert ws(dtype=1, batch=8, dim=1536, seqlen=4096) == size_for(-(-98304 // 56))
    # configs[3] prefill (bf16 64 x 5120 x 2048): 10240 rows >= 1776 warps, whole rows (6 x 128 tiles) per
    # warp -- no carry hand-off -- since 768 tiles is within 9/8 of the split plan's 739
    assert ws(dtype=2, batch=64, dim=5120, seqlen=2048) == size_for(-(-1310720 // 768))
    # configs[2] prefill (fp32 1 x 1536 x 5601): rows of 701 tiles cut into pieces of 19 tiles (~37 per row)
    assert ws(dtype=0, batch=1, dim=1536, seqlen=5601) == size_for(-(-33648 // 19))
    # short sequences: pieces never shorter than two 32-step heads (4 fp16 tiles)
    assert ws(dtype=1, batch=1, dim=64, seqlen=4096) == size_for(-(-512 // 4))
    # an explicit piece length is kept, and dstate > 16 uses the 64-state layout
    assert ws(dtype=1, batch=8, dim=1536, seqlen=4096, piece_tiles=256) == size_for(384)
    assert ws(dtype=1, batch=2, dim=64, seqlen=1000, dstate=17, piece_tiles=4) == size_for(-(-252 // 4), nm=64)
