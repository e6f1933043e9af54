"""Loads `state-spaces/mamba-*-hf` checkpoints into a MambaModel (mamba_metal/load_hf.py:1-76).

The parameter names of MambaModel are already the HF ones, and conv1d.weight keeps PyTorch's
(d_inner, 1, d_conv) layout, so the only key transformation is stripping "backbone." (load_hf.py:42-43);
the reference's conv1d transpose (:46-50) exists only because MLX stores (out, k, in/g). A tied
`lm_head.weight` (the head is the embedding, mamba_model.py:67-69) is dropped.

The checkpoint comes from a local directory holding config.json and *.safetensors, or from the Hugging
Face cache through huggingface_hub.snapshot_download (load_hf.py:56-61); this module never needs the
network when the files are local.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from mamba_metal_b200.mamba_model import MambaConfig, MambaModel


def config_from_hf(cfg: dict) -> MambaConfig:
    """MambaConfig from an HF config.json dict (load_hf.py:22-39): HF transformers field names first,
    then the state-spaces aliases; `hidden_size` wins over `d_model`, which some checkpoints carry stale
    (load_hf.py:25-28); expand = intermediate_size // hidden_size when the former is given."""
    d_model = cfg.get("hidden_size") or cfg["d_model"]
    d_inner = cfg.get("intermediate_size") or cfg.get("d_inner")
    expand = d_inner // d_model if d_inner else cfg.get("expand", 2)
    return MambaConfig(
        d_model=d_model,
        n_layer=cfg.get("num_hidden_layers") or cfg["n_layer"],
        vocab_size=cfg["vocab_size"],
        d_state=cfg.get("state_size") or cfg.get("d_state", 16),
        d_conv=cfg.get("conv_kernel") or cfg.get("d_conv", 4),
        expand=expand,
        dt_rank=cfg.get("time_step_rank") or cfg.get("dt_rank"),
        rms_norm_eps=cfg.get("layer_norm_epsilon", 1e-5),
    )


def _local_dir(path_or_repo: str | Path) -> Path:
    p = Path(path_or_repo)
    if p.is_dir():
        return p
    from huggingface_hub import snapshot_download

    return Path(snapshot_download(repo_id=str(path_or_repo),
                                  allow_patterns=["*.json", "*.safetensors", "tokenizer*", "special_tokens*"]))


def load_mamba_hf(path_or_repo: str | Path = "state-spaces/mamba-130m-hf", dtype: torch.dtype = torch.float32,
                  device="cuda") -> tuple[MambaModel, MambaConfig]:
    """Builds a MambaModel (parameters in `dtype`, RMSNorm weights float32) on `device` and loads every
    tensor of the checkpoint's *.safetensors files into it (strict: a missing or unexpected key raises).
    Returns (model, config) like the reference."""
    from safetensors import safe_open

    local = _local_dir(path_or_repo)
    cfg = config_from_hf(json.loads((local / "config.json").read_text()))
    files = sorted(local.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no *.safetensors in {local}")
    sd = {}
    for st in files:
        with safe_open(str(st), framework="pt") as f:
            for key in f.keys():
                sd[key.removeprefix("backbone.")] = f.get_tensor(key)
    head = sd.pop("lm_head.weight", None)
    if head is not None and not torch.equal(head, sd["embeddings.weight"]):
        raise ValueError("checkpoint has an untied lm_head; MambaModel ties the head to the embedding")
    with torch.device("meta"):
        model = MambaModel(cfg, dtype=dtype)
    model = model.to_empty(device=device)
    model.load_state_dict(sd, strict=True)
    return model, cfg
