"""mamba_metal_b200: mamba-metal's hot path (selective scan, causal conv1d, O(1) decode step) as
hand-written sm_100a CUDA behind a C-ABI library, under the reference's Python API.

The package directory is ``mamba_metal_b200`` (the hyphenated name cannot be imported in Python).
Public names mirror mamba_metal/__init__.py:3-20. ``load_mamba_hf`` loads a ``state-spaces/mamba-*-hf``
checkpoint from a local directory or the Hugging Face cache; ``load_kernel`` (the MLX Metal loader) has no
counterpart.
"""

from mamba_metal_b200.generate import GraphDecoder, generate, generate_fast, generate_ids
from mamba_metal_b200.load_hf import load_mamba_hf
from mamba_metal_b200.mamba_block import MambaBlock
from mamba_metal_b200.mamba_model import MambaConfig, MambaModel, MambaResidualBlock, RMSNorm, init_weights_
from mamba_metal_b200.ops import add_rmsnorm, causal_conv1d, causal_conv1d_step, ssm_decode_step
from mamba_metal_b200.selective_scan import selective_scan

__all__ = [
    "GraphDecoder",
    "MambaBlock",
    "MambaConfig",
    "MambaModel",
    "MambaResidualBlock",
    "RMSNorm",
    "add_rmsnorm",
    "causal_conv1d",
    "causal_conv1d_step",
    "generate",
    "generate_fast",
    "generate_ids",
    "load_mamba_hf",
    "init_weights_",
    "selective_scan",
    "ssm_decode_step",
]
