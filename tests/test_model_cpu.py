"""Model structure (no kernels): HF parameter names, parameter count, seeded init, and the reference
model restatement's causality and prefill/step consistency. CPU only."""

import torch

from mamba_metal_b200 import MambaConfig, MambaModel, init_weights_
from oracle.model_ref import RefModel

# experiments/13-mamba-model/test_model.py:15-31
HF_EXPECTED_LAYER_NAMES = {
    "norm.weight", "mixer.A_log", "mixer.D", "mixer.conv1d.bias", "mixer.conv1d.weight", "mixer.dt_proj.bias",
    "mixer.dt_proj.weight", "mixer.in_proj.weight", "mixer.out_proj.weight", "mixer.x_proj.weight",
}
HF_EXPECTED_TOP_NAMES = {"embeddings.weight", "norm_f.weight"}


def test_param_names_match_hf():
    model = MambaModel(MambaConfig(d_model=64, n_layer=1, vocab_size=128))
    names = set(dict(model.named_parameters()))
    layer = {n.removeprefix("layers.0.") for n in names if n.startswith("layers.0.")}
    assert layer == HF_EXPECTED_LAYER_NAMES
    assert {n for n in names if "layers." not in n} == HF_EXPECTED_TOP_NAMES
    assert tuple(model.layers[0].mixer.conv1d.weight.shape) == (128, 1, 4)  # HF / PyTorch layout


def test_130m_parameter_count():
    cfg = MambaConfig(d_model=768, n_layer=24, vocab_size=50280, d_state=16, d_conv=4, expand=2, dt_rank=48)
    with torch.device("meta"):
        model = MambaModel(cfg)
    total = sum(p.numel() for p in model.parameters())
    assert 125e6 < total < 135e6, total


def _small(seed=0, n_layer=2):
    cfg = MambaConfig(d_model=32, n_layer=n_layer, vocab_size=97, dt_rank=4)
    return cfg, init_weights_(MambaModel(cfg), seed=seed)


def test_seeded_init_is_deterministic():
    _, a = _small(3)
    _, b = _small(3)
    _, c = _small(4)
    for (k, va), vb, vc in zip(a.state_dict().items(), b.state_dict().values(), c.state_dict().values()):
        assert torch.equal(va, vb), k
    assert not torch.equal(a.embeddings.weight, c.embeddings.weight)
    sp = torch.nn.functional.softplus(a.layers[0].mixer.dt_proj.bias)
    assert sp.min() >= 1e-3 * 0.999 and sp.max() <= 1e-1 * 1.001


def test_reference_model_causality():
    """experiments/11-mamba-block/test_block.py:42-61 on the oracle model."""
    cfg, m = _small(1)
    ref = RefModel(m.state_dict(), cfg)
    g = torch.Generator().manual_seed(42)
    ids1 = torch.randint(0, cfg.vocab_size, (1, 64), generator=g)
    ids2 = ids1.clone()
    ids2[:, 32:] = torch.randint(0, cfg.vocab_size, (1, 32), generator=g)
    y1, y2 = ref.forward(ids1), ref.forward(ids2)
    assert (y1[:, :32] - y2[:, :32]).abs().max() < 1e-4
    assert (y1[:, 32:] - y2[:, 32:]).abs().max() > 1e-3


def test_reference_prefill_step_handoff():
    """prefill(L) then step(token L) equals prefill(L+1) at the last position (generate.py:82-108)."""
    cfg, m = _small(2)
    ref = RefModel(m.state_dict(), cfg)
    ids = torch.randint(0, cfg.vocab_size, (2, 13), generator=torch.Generator().manual_seed(0))
    full, _, _ = ref.prefill(ids)
    lg, convs, ssms = ref.prefill(ids[:, :12])
    st, _, _ = ref.step(ids[:, 12:13], convs, ssms)
    torch.testing.assert_close(st[:, 0], full[:, 12], rtol=1e-4, atol=1e-4)
    for L in (1, 2, 3):  # prompts shorter than d_conv: zero-left-padded conv state
        lg, convs, ssms = ref.prefill(ids[:, :L])
        st, _, _ = ref.step(ids[:, L:L + 1], convs, ssms)
        full, _, _ = ref.prefill(ids[:, :L + 1])
        torch.testing.assert_close(st[:, 0], full[:, L], rtol=1e-4, atol=1e-4)


def test_fused_dt_step_gate():
    """Which decode steps compute dt_proj inside the SSM step kernel (MambaBlock._fused_dt_step): only with
    FUSED_DT_STEP set, 16-bit weights, dt_rank a multiple of 16 up to the kernel's limit, d_state 16, and
    at most FUSED_DT_MAX_ELEMS batch rows x channels; everything else keeps dt_proj as its own GEMM."""
    import mamba_metal_b200.mamba_block as mb
    from mamba_metal_b200 import MambaBlock, ops

    def blk(d_model=256, dt_rank=32, d_state=16, dtype=torch.bfloat16):
        with torch.device("meta"):
            return MambaBlock(d_model, d_state=d_state, dt_rank=dt_rank, dtype=dtype)

    default = mb.FUSED_DT_STEP
    try:
        mb.FUSED_DT_STEP = True
        assert blk()._fused_dt_step(8)
        assert blk(dtype=torch.float16)._fused_dt_step(8)
        assert not blk(dtype=torch.float32)._fused_dt_step(8)             # fp32: separate GEMM
        assert not blk(dt_rank=24)._fused_dt_step(8)                      # not a multiple of 16
        assert not blk(dt_rank=ops.SSM_STEP_FUSED_DT_MAX_RANK + 16)._fused_dt_step(8)
        assert not blk(d_state=8)._fused_dt_step(8)
        b = blk(d_model=2560, dt_rank=160)                                 # 2.8b mixer, 5120 channels
        assert b._fused_dt_step(mb.FUSED_DT_MAX_ELEMS // 5120)
        assert not b._fused_dt_step(mb.FUSED_DT_MAX_ELEMS // 5120 + 1)   # beyond the size limit
        mb.FUSED_DT_STEP = False
        assert not blk()._fused_dt_step(8)
    finally:
        mb.FUSED_DT_STEP = default
