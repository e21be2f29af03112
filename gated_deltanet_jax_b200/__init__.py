"""B200 (sm_100a) gated delta-rule core with the reference package's op API.

Public names follow reference ``src/gated_deltanet_jax/__init__.py``: the config
class, the model classes (PyTorch modules, ``model.py``) and the two ops.
"""

from .configuration import GatedDeltaNetConfig
from .dispatch import delta_rule
from .model import (
    GatedDeltaNet,
    GatedDeltaNetBlock,
    GatedDeltaNetForCausalLM,
    GatedDeltaNetMLP,
    GatedDeltaNetModel,
    ShortConvolution,
)
from .ops import (
    chunk_gated_delta_rule,
    chunk_gated_delta_rule_fwd,
    fused_recurrent_gated_delta_rule,
    fused_recurrent_gated_delta_rule_fwd,
    gated_delta_rule_chunk_layer,
    gated_delta_rule_decode_layer,
    gated_rms_norm,
    short_convolution,
)

__all__ = [
    "GatedDeltaNetConfig",
    "GatedDeltaNet",
    "GatedDeltaNetMLP",
    "GatedDeltaNetBlock",
    "GatedDeltaNetModel",
    "GatedDeltaNetForCausalLM",
    "ShortConvolution",
    "chunk_gated_delta_rule",
    "chunk_gated_delta_rule_fwd",
    "fused_recurrent_gated_delta_rule",
    "fused_recurrent_gated_delta_rule_fwd",
    "delta_rule",
    "gated_delta_rule_chunk_layer",
    "gated_delta_rule_decode_layer",
    "gated_rms_norm",
    "short_convolution",
]
