"""GatedDeltaNetModel (gated_deltanet_jax_b200/model.py) on the GPU against a
float64 restatement of the reference model (model.py:58-245) assembled from the
oracle's layer pieces (short_conv, layer_gates, chunk_exact, rms_norm_gated),
with the model's own weights.

The reference layer applies no q/k normalisation, so at its default
initialisation the recurrence overflows within a few dozen tokens (in the
reference as well); these tests scale the q/k projections down so that the
exact recurrence stays finite over their sequence lengths."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import GatedDeltaNetConfig
from gated_deltanet_jax_b200.model import GatedDeltaNetForCausalLM, GatedDeltaNetModel
from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().double().cpu().numpy()


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, -1, keepdims=True) + eps) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def restated_forward(model, ids):
    """The reference model's forward in float64 (model.py:113-156, :176-230)."""
    cfg = model.config
    B, T = ids.shape
    lin = lambda m, z: z @ _np(m.weight).T  # noqa: E731
    x = _np(model.embed_tokens.weight)[ids]
    for blk in model.layers:
        at = blk.attn
        h = _rms(x, _np(blk.attn_norm.weight), cfg.norm_eps)
        q, k, v = lin(at.q_proj, h), lin(at.k_proj, h), lin(at.v_proj, h)
        if cfg.use_short_conv:
            q = orc.short_conv(q, _np(at.q_conv.weight))[0]
            k = orc.short_conv(k, _np(at.k_conv.weight))[0]
            v = orc.short_conv(v, _np(at.v_conv.weight))[0]
        else:
            q, k, v = _silu(q), _silu(k), _silu(v)
        q = q.reshape(B, T, at.num_heads, at.head_k_dim)
        k = k.reshape(B, T, at.num_heads, at.head_k_dim)
        v = v.reshape(B, T, at.num_v_heads, at.head_v_dim)
        rep = at.num_v_heads // at.num_heads
        if rep > 1:
            q, k = orc.repeat_heads(q, rep), orc.repeat_heads(k, rep)
        g, beta = orc.layer_gates(lin(at.a_proj, h), lin(at.b_proj, h), _np(at.A_log),
                                  _np(at.dt_bias))
        o, _ = orc.chunk_exact(q, k, v, g, beta)   # both modes compute the recurrence
        gate = None if at.g_proj is None else lin(at.g_proj, h).reshape(o.shape)
        o = orc.rms_norm_gated(o, _np(at.o_norm_weight), gate, at.o_norm_eps)
        x = x + lin(at.o_proj, o.reshape(B, T, -1))
        hm = _rms(x, _np(blk.mlp_norm.weight), cfg.norm_eps)
        m = blk.mlp
        x = x + lin(m.down_proj, _silu(lin(m.gate_proj, hm)) * lin(m.up_proj, hm))
    return _rms(x, _np(model.norm.weight), cfg.norm_eps)


def _model(cfg, dev, seed, dtype=torch.bfloat16, cls=GatedDeltaNetModel):
    torch.manual_seed(seed)
    m = cls(cfg)
    core = m.model if cls is GatedDeltaNetForCausalLM else m
    with torch.no_grad():
        for blk in core.layers:   # keep the unnormalised recurrence finite
            blk.attn.q_proj.weight.mul_(0.5 / blk.attn.head_k_dim ** 0.5)
            blk.attn.k_proj.weight.mul_(0.5 / blk.attn.head_k_dim ** 0.5)
    return m.to(device=dev, dtype=dtype).eval()


def _rel(a, r):
    return float(np.max(np.abs(a - r)) / max(np.max(np.abs(r)), 1e-30))


CASES = [
    # mode, hidden, heads, v_heads, head_dim, expand_v, gate, conv, T
    ("chunk", 256, 2, None, 128, 2.0, True, True, 100),      # the fused layer form
    ("chunk", 128, 2, 4, 64, 1.0, True, True, 70),           # separate ops, grouped heads
    ("fused_recurrent", 256, 2, None, 128, 1.0, True, True, 40),
    ("chunk", 128, 2, None, 32, 2.0, False, False, 50),      # ungated, no convolution
]


@pytest.mark.parametrize("mode,D,H,HV,hd,ev,gate,conv,T", CASES)
def test_model_matches_restated_reference(cuda, mode, D, H, HV, hd, ev, gate, conv, T):
    cfg = GatedDeltaNetConfig(attn_mode=mode, hidden_size=D, num_heads=H, num_v_heads=HV,
                              head_dim=hd, expand_v=ev, use_gate=gate, use_short_conv=conv,
                              num_hidden_layers=2, vocab_size=97)
    model = _model(cfg, cuda, seed=T + hd)
    ids = torch.randint(0, cfg.vocab_size, (2, T), generator=torch.Generator().manual_seed(T))
    with torch.no_grad():
        got = model(ids.to(cuda))
    ref = restated_forward(model, ids.numpy())
    assert np.isfinite(ref).all()
    err = _rel(_np(got), ref)
    # bf16 weights, activations and GEMMs through two blocks
    assert err <= 3e-2, f"rel error {err:.2e}"


def test_model_gradients_route(cuda):
    """With gradients wanted the layer takes the differentiable route (torch
    convolution and norm, the delta rule through gdn_chunk_bwd): its logits and
    the fused inference route's both match the restated reference, and every
    parameter gets a finite gradient."""
    cfg = GatedDeltaNetConfig(hidden_size=256, num_heads=2, head_dim=128, expand_v=2.0,
                              num_hidden_layers=2, vocab_size=97)
    model = _model(cfg, cuda, seed=3, cls=GatedDeltaNetForCausalLM)
    ids = torch.randint(0, 97, (2, 80), generator=torch.Generator().manual_seed(1))
    ref = restated_forward(model.model, ids.numpy()) @ _np(model.lm_head.weight).T
    ids = ids.to(cuda)
    with torch.no_grad():
        fused = model(ids)
    logits = model(ids)
    for got in (fused, logits):
        err = _rel(_np(got), ref)
        assert err <= 3e-2, f"rel error {err:.2e}"
    logits.float().logsumexp(-1).mean().backward()
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    assert len(grads) == len(list(model.parameters()))
    assert all(torch.isfinite(g).all() for g in grads)


def test_model_rejects_unknown_mode(cuda):
    cfg = GatedDeltaNetConfig(attn_mode="linear", hidden_size=128, num_heads=2, head_dim=64,
                              num_hidden_layers=1, vocab_size=11)
    model = _model(cfg, cuda, seed=0)
    with torch.no_grad(), pytest.raises(ValueError, match="Unknown mode"):
        model(torch.zeros(1, 4, dtype=torch.long, device=cuda))
