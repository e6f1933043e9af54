"""HF checkpoint loader (mamba_metal/load_hf.py:22-76) on CPU: config aliases, the backbone. prefix, the
tied head, strict key matching. Checkpoints are written here in the HF layout (config.json + safetensors)."""

import json

import pytest
import torch
from safetensors.torch import save_file

from mamba_metal_b200 import MambaConfig, MambaModel, init_weights_
from mamba_metal_b200.load_hf import config_from_hf, load_mamba_hf


def _write_checkpoint(tmp_path, model: MambaModel, cfg_json: dict, head=None):
    sd = {"backbone." + k: v.detach().clone().contiguous() for k, v in model.state_dict().items()}
    if head is not None:
        sd["lm_head.weight"] = head
    save_file(sd, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(cfg_json))


def _small():
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=101, d_state=16, d_conv=4, expand=2, dt_rank=4)
    return cfg, init_weights_(MambaModel(cfg, device="cpu"), seed=3)


def test_round_trip_hf_fields(tmp_path):
    cfg, m = _small()
    # HF transformers field names, plus a stale d_model as some checkpoints carry (load_hf.py:25-28)
    _write_checkpoint(tmp_path, m, {"hidden_size": 64, "d_model": 999, "intermediate_size": 128,
                                    "num_hidden_layers": 2, "vocab_size": 101, "state_size": 16, "conv_kernel": 4,
                                    "time_step_rank": 4, "layer_norm_epsilon": 1e-5},
                      head=m.embeddings.weight.detach().clone())
    loaded, lcfg = load_mamba_hf(tmp_path, device="cpu")
    assert lcfg == cfg
    want = m.state_dict()
    got = loaded.state_dict()
    assert set(got) == set(want)
    for k in want:
        assert torch.equal(got[k], want[k]), k


def test_legacy_aliases():
    c = config_from_hf({"d_model": 768, "n_layer": 24, "vocab_size": 50280, "d_state": 16, "d_conv": 4,
                        "expand": 2})
    assert (c.d_model, c.n_layer, c.d_state, c.d_conv, c.expand, c.dt_rank) == (768, 24, 16, 4, 2, None)


def test_untied_head_and_missing_key_raise(tmp_path):
    cfg, m = _small()
    cj = {"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 2, "vocab_size": 101,
          "state_size": 16, "conv_kernel": 4, "time_step_rank": 4}
    _write_checkpoint(tmp_path, m, cj, head=torch.randn(101, 64))
    with pytest.raises(ValueError):
        load_mamba_hf(tmp_path, device="cpu")
    cj["num_hidden_layers"] = 3  # the checkpoint has two layers: strict loading must refuse
    _write_checkpoint(tmp_path, m, cj)
    with pytest.raises(RuntimeError):
        load_mamba_hf(tmp_path, device="cpu")
