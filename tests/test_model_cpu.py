"""GatedDeltaNetModel's structure (gated_deltanet_jax_b200/model.py) without a
GPU: the reference's module tree (model.py:58-245) and its parameter shapes at
the default configuration (configuration.py), built on the meta device."""

import torch

from gated_deltanet_jax_b200 import GatedDeltaNetConfig
from gated_deltanet_jax_b200.model import GatedDeltaNetForCausalLM


def test_default_configuration_shapes():
    cfg = GatedDeltaNetConfig(num_hidden_layers=2)
    with torch.device("meta"):
        m = GatedDeltaNetForCausalLM(cfg)
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    D, K, V = 2048, 6 * 256, 6 * 512          # hidden, key_dim, value_dim
    inter = 256 * ((int(D * 4 * 2 / 3) + 255) // 256)
    assert inter == 5632
    want = {
        "model.embed_tokens.weight": (32000, D),
        "model.layers.0.attn_norm.weight": (D,),
        "model.layers.0.attn.q_proj.weight": (K, D),
        "model.layers.0.attn.k_proj.weight": (K, D),
        "model.layers.0.attn.v_proj.weight": (V, D),
        "model.layers.0.attn.a_proj.weight": (6, D),
        "model.layers.0.attn.b_proj.weight": (6, D),
        "model.layers.0.attn.g_proj.weight": (V, D),
        "model.layers.0.attn.o_proj.weight": (D, V),
        "model.layers.0.attn.q_conv.weight": (4, K),
        "model.layers.0.attn.k_conv.weight": (4, K),
        "model.layers.0.attn.v_conv.weight": (4, V),
        "model.layers.0.attn.A_log": (6,),
        "model.layers.0.attn.dt_bias": (6,),
        "model.layers.0.attn.o_norm_weight": (512,),
        "model.layers.0.mlp_norm.weight": (D,),
        "model.layers.0.mlp.gate_proj.weight": (inter, D),
        "model.layers.0.mlp.up_proj.weight": (inter, D),
        "model.layers.0.mlp.down_proj.weight": (D, inter),
        "model.norm.weight": (D,),
        "lm_head.weight": (32000, D),
    }
    for n, s in want.items():
        assert shapes[n] == s, (n, shapes[n], s)
    assert sum(1 for n in shapes if n.startswith("model.layers.1.")) == \
        sum(1 for n in shapes if n.startswith("model.layers.0."))


def test_layer_variants_and_gate_epsilons():
    cfg = GatedDeltaNetConfig(use_gate=False, use_short_conv=False, num_v_heads=12,
                              num_hidden_layers=1)
    with torch.device("meta"):
        m = GatedDeltaNetForCausalLM(cfg)
    at = m.model.layers[0].attn
    assert at.g_proj is None and not hasattr(at, "q_conv")
    assert at.o_norm_eps == 1e-6                     # nnx.RMSNorm without a gate
    assert tuple(at.v_proj.weight.shape) == (12 * 512, 2048)
    assert tuple(at.q_proj.weight.shape) == (6 * 256, 2048)   # q/k keep num_heads heads
    cfg2 = GatedDeltaNetConfig(num_hidden_layers=1)
    with torch.device("meta"):
        m2 = GatedDeltaNetForCausalLM(cfg2)
    assert m2.model.layers[0].attn.o_norm_eps == 1e-5      # FusedRMSNormGated
