"""MambaBlock / MambaModel / generation on the sm_100a kernels vs the float32 reference restatement."""

import types

import numpy as np
import pytest
import torch

from mamba_metal_b200 import (GraphDecoder, MambaBlock, MambaConfig, MambaModel, generate, generate_fast,
                              generate_ids, init_weights_)
from oracle.model_ref import RefMixer, RefModel, sampling_probs
from tests.helpers import assert_close, assert_close_lowp

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def small_model(seed=0, d_model=64, n_layer=2, vocab=211, dtype=torch.float32):
    cfg = MambaConfig(d_model=d_model, n_layer=n_layer, vocab_size=vocab, dt_rank=8)
    return cfg, init_weights_(MambaModel(cfg, dtype=dtype, device=DEV), seed=seed)


def block_and_ref(d_model=64, seed=0):
    cfg, m = small_model(seed, d_model=d_model, n_layer=1)
    blk = m.layers[0].mixer
    sd = {k.removeprefix("layers.0.mixer."): v.detach().cpu() for k, v in m.state_dict().items()
          if k.startswith("layers.0.mixer.")}
    return blk, RefMixer(sd, "", blk.d_state, blk.dt_rank)


def test_block_forward_prefill_step():
    blk, ref = block_and_ref()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 77, 64, generator=g) * 0.5
    y = blk(x.to(DEV))
    assert_close(y, ref.forward(x), 1e-4, "block forward")
    y, cs, ss = blk.prefill(x.to(DEV))
    yr, csr, ssr = ref.prefill(x)
    assert_close(y, yr, 1e-4, "prefill y")
    assert_close(cs, csr, 1e-5, "conv state")
    assert_close(ss, ssr, 1e-4, "ssm state")
    xt = torch.randn(2, 1, 64, generator=g) * 0.5
    yt, cs2, ss2 = blk.step(xt.to(DEV), cs, ss)
    ytr, csr2, ssr2 = ref.step(xt, csr, ssr)
    assert_close(yt, ytr, 1e-4, "step y")
    assert_close(cs2, csr2, 1e-5, "step conv state")
    assert_close(ss2, ssr2, 1e-4, "step ssm state")
    assert not torch.equal(cs, cs2)  # functional by default: inputs untouched


def test_block_causality():
    """experiments/11-mamba-block/test_block.py:42-61."""
    blk, _ = block_and_ref(seed=42)
    g = torch.Generator().manual_seed(42)
    x1 = torch.randn(1, 64, 64, generator=g) * 0.5
    x2 = x1.clone()
    x2[:, 32:] = torch.randn(1, 32, 64, generator=g) * 0.5
    y1, y2 = blk(x1.to(DEV)).cpu(), blk(x2.to(DEV)).cpu()
    assert (y1[:, :32] - y2[:, :32]).abs().max() < 1e-4
    assert (y1[:, 32:] - y2[:, 32:]).abs().max() > 1e-3


def test_model_matches_reference_and_handoff():
    cfg, m = small_model(1, n_layer=3)
    ref = RefModel({k: v.cpu() for k, v in m.state_dict().items()}, cfg)
    ids = torch.randint(0, cfg.vocab_size, (2, 41), generator=torch.Generator().manual_seed(3))
    lg = m(ids.to(DEV))
    assert lg.shape == (2, 41, cfg.vocab_size)
    assert_close(lg, ref.forward(ids), 1e-4, "logits")
    lp, convs, ssms = m.prefill(ids[:, :40].to(DEV))
    lpr, convr, ssmr = ref.prefill(ids[:, :40])
    assert_close(lp, lpr, 1e-4, "prefill logits")
    for i in range(cfg.n_layer):
        assert_close(convs[i], convr[i], 1e-5, f"conv state {i}")
        assert_close(ssms[i], ssmr[i], 1e-4, f"ssm state {i}")
    st, _, _ = m.step(ids[:, 40:41].to(DEV), convs, ssms)
    assert_close(st[:, 0], lg[:, 40], 1e-4, "step after prefill == full forward")


def test_bf16_model_matches_rounding_reference():
    """A bf16 model (d_model 256, 4 layers) against the oracle run with the reference's bf16 storage
    points (RefModel(act_dtype=bf16)): prefill logits, states and a decode step, compared as bf16-stored
    data (relative L2 within 1e-2 over each tensor and 5e-2 per token / channel)."""
    cfg = MambaConfig(d_model=256, n_layer=4, vocab_size=1000, dt_rank=16)
    m = init_weights_(MambaModel(cfg, dtype=torch.bfloat16, device=DEV), seed=3)
    ref = RefModel({k: v.detach() for k, v in m.state_dict().items()}, cfg, device=DEV, act_dtype=torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (3, 300), generator=torch.Generator().manual_seed(5)).to(DEV)
    lg, convs, ssms = m.prefill(ids)
    lr, convr, ssmr = ref.prefill(ids)
    assert_close_lowp(lg, lr, "bf16 prefill logits", axis=1)
    for i in range(cfg.n_layer):
        assert_close_lowp(convs[i], convr[i], f"bf16 conv state {i}", axis=1)
        assert_close_lowp(ssms[i], ssmr[i], f"bf16 ssm state {i}", axis=1)
    nxt = torch.argmax(lg[:, -1], dim=-1, keepdim=True)
    st, _, _ = m.step(nxt, convs, ssms)
    sr, _, _ = ref.step(nxt, convr, ssmr)
    assert_close_lowp(st, sr, "bf16 step logits")


def test_graph_decoder_matches_eager():
    cfg, m = small_model(2)
    ids = torch.randint(0, cfg.vocab_size, (4, 9), generator=torch.Generator().manual_seed(4)).to(DEV)
    eager = generate_ids(m, ids, 12, use_graph=False)
    graph = generate_ids(m, ids, 12, use_graph=True)
    assert torch.equal(eager, graph)


class ByteTokenizer:
    """Minimal tokenizer for tests: bytes mod vocab, no EOS."""

    eos_token_id = None

    def __init__(self, vocab):
        self.vocab = vocab

    def __call__(self, text, return_tensors="np"):
        return types.SimpleNamespace(input_ids=np.array([[b % self.vocab for b in text.encode()]], dtype=np.int64))

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(33 + (int(i) % 90)) for i in ids)


def test_generate_fast_equals_generate():
    """experiments/17-incremental/test_step.py:31-41: O(L^2) and O(L) greedy outputs identical."""
    cfg, m = small_model(5)
    tok = ByteTokenizer(cfg.vocab_size)
    streamed = []
    for prompt in ("Mamba is a", "Once upon a time", "The capital of Japan is"):
        slow = generate(m, tok, prompt, max_new_tokens=16)
        fast = generate_fast(m, tok, prompt, max_new_tokens=16, on_token=streamed.append)
        assert slow == fast
    assert streamed


def test_temperature_sampling_distribution_and_seeding():
    """generate.py:42-44, :92-93: at temperature T > 0 the next id is a draw from softmax(logits / T).
    The repo's sampler (torch.multinomial on the device) is checked against the oracle's distribution
    over 400,000 draws (total-variation distance; its expected value here is ~0.005) and for
    reproducibility under a fixed torch seed."""
    from mamba_metal_b200.generate import _pick

    logits = (torch.randn(1, 64, generator=torch.Generator().manual_seed(7)) * 2).to(DEV)
    n, T = 400_000, 0.7
    torch.manual_seed(11)
    a = _pick(logits.expand(n, -1), T)
    torch.manual_seed(11)
    b = _pick(logits.expand(n, -1), T)
    assert torch.equal(a, b)
    freq = torch.bincount(a.cpu(), minlength=64).double() / n
    p = sampling_probs(logits.cpu(), T)[0]
    tv = 0.5 * float((freq - p).abs().sum())
    assert tv < 0.012, f"sampled distribution is {tv:.4f} (total variation) from softmax(logits / T)"


def test_sampled_generation_is_seeded():
    """generate_ids / generate_fast with temperature > 0: same torch seed -> same ids; and a sampled
    token is always one the distribution allows (here: all tokens, so only the range is checked)."""
    cfg, m = small_model(6)
    ids = torch.randint(0, cfg.vocab_size, (3, 7), generator=torch.Generator().manual_seed(8)).to(DEV)
    outs = []
    for _ in range(2):
        torch.manual_seed(5)
        outs.append(generate_ids(m, ids, 10, temperature=0.8))
    assert torch.equal(outs[0], outs[1])
    assert int(outs[0].min()) >= 0 and int(outs[0].max()) < cfg.vocab_size
    tok = ByteTokenizer(cfg.vocab_size)
    texts = []
    for _ in range(2):
        torch.manual_seed(9)
        texts.append(generate_fast(m, tok, "Mamba is a", max_new_tokens=12, temperature=0.9))
    assert texts[0] == texts[1]


def test_config2_130m_prefill_and_greedy_decode():
    """Mamba-130m architecture, random init (seed 0), fp32, one 5,601-token prompt,
    parallel prefill, then 50 greedy decode steps; compared with the float32 reference restatement on CPU
    (generate.py:82-108). The oracle decodes free-running (its own argmax feeds its next step), and its
    first 32 greedy tokens must equal the repo's exactly. After step 32 the comparison continues
    teacher-forced, where a differing token is allowed only at an oracle top-2 margin below 1e-3."""
    cfg = MambaConfig(d_model=768, n_layer=24, vocab_size=50280, d_state=16, d_conv=4, expand=2, dt_rank=48)
    m = init_weights_(MambaModel(cfg, device=DEV), seed=0)
    ids = torch.randint(0, cfg.vocab_size, (1, 5601), generator=torch.Generator().manual_seed(0))
    out = generate_ids(m, ids.to(DEV), 50, use_graph=True).cpu()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = RefModel({k: v.cpu() for k, v in m.state_dict().items()}, cfg)
    pre = ref.prefill(ids, last_only=True)
    free, free_logits = ref.greedy(ids, 32, prefilled=pre)
    same = free[0] == out[0, :32]
    assert same.all(), (f"free-running greedy tokens differ from step {int(torch.nonzero(~same)[0])}: "
                        f"repo {out[0, :32].tolist()} oracle {free[0].tolist()}")
    top2 = torch.topk(free_logits[0], 2, dim=-1).values
    print(f"config2: first 32 free-running greedy tokens identical; smallest oracle top-2 margin "
          f"{float((top2[:, 0] - top2[:, 1]).min()):.2e}")
    toks, logits = ref.greedy(ids, 50, forced=out, prefilled=pre)
    top2 = torch.topk(logits[0], 2, dim=-1).values
    decided = (top2[:, 0] - top2[:, 1]) > 1e-3
    mism = (toks[0] != out[0]) & decided
    assert not mism.any(), f"greedy token mismatch at steps {torch.nonzero(mism).flatten().tolist()}"
    print(f"config2: steps 32-49 teacher-forced: {int((toks[0, 32:] != out[0, 32:]).sum())} differing tokens "
          f"(all at margins <= 1e-3)")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_step_fused_dt_matches_dt_gemm(dtype):
    """MambaModel.step with dt_proj computed inside the SSM step kernel (mamba_block.FUSED_DT_STEP) against
    dt_proj as a separate GEMM, from the same prefill state. The GEMM rounds dt to the model dtype and the
    fused step does not, so the two agree to that dtype's accuracy (relative L2 <= 1e-2)."""
    import mamba_metal_b200.mamba_block as mb

    cfg = MambaConfig(d_model=256, n_layer=2, vocab_size=997, dt_rank=32)
    m = init_weights_(MambaModel(cfg, dtype=dtype, device=DEV), seed=5)
    ids = torch.randint(0, cfg.vocab_size, (6, 21), generator=torch.Generator().manual_seed(6)).to(DEV)
    default = mb.FUSED_DT_STEP
    outs = {}
    try:
        with torch.no_grad():
            _, conv, ssm = m.prefill(ids)
            for fused in (False, True):
                mb.FUSED_DT_STEP = fused
                assert m.layers[0].mixer._fused_dt_step(ids.shape[0]) == fused
                logits, _, ssm2 = m.step(ids[:, -1:], [c.clone() for c in conv], [s.clone() for s in ssm])
                outs[fused] = (logits.float(), ssm2[-1].clone())
    finally:
        mb.FUSED_DT_STEP = default
    for a, b in zip(outs[True], outs[False]):
        assert float((a - b).norm() / b.norm()) < 1e-2
