"""The layer form of the chunked forward (gdn_chunk_fwd_layer): gates from the
raw a_proj / b_proj outputs (model.py:136-139), the chunked forward, and the
gated RMSNorm of every output row (model.py:41-53), in one kernel.  Checked
against the oracle's restatement of each part, composed, and at full size
against the same parts run as separate operations on the GPU."""

import math

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, device_inputs_fast, f64

pytestmark = pytest.mark.gpu


def _layer_extras(B, T, H, dev, seed, with_gate, dtype=torch.bfloat16, steep=False):
    """a, b ~ N(0, 1); A_log, dt_bias as the layer initialises them
    (model.py:103-113), or (steep) dt_bias ~ N(0, 0.5), which gives gates of
    about -5 per token: chunks whose decay spans more than e^40 inside 16
    tokens, the kernel's direct-exponent path."""
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    a = torch.randn(B, T, H, device=dev, generator=gen)
    b = torch.randn(B, T, H, device=dev, generator=gen)
    A_log = torch.log(torch.rand(H, device=dev, generator=gen) * 16 + 1e-4)   # model.py:104-106
    if steep:
        dt_bias = torch.randn(H, device=dev, generator=gen) * 0.5
    else:
        u = torch.rand(H, device=dev, generator=gen)
        dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
        dt_bias = dt + torch.log(-torch.expm1(-dt))                           # model.py:108-113
    gate = torch.randn(B, T, H, 128, device=dev, generator=gen).to(dtype) if with_gate else None
    w = 1.0 + 0.1 * torch.randn(128, device=dev, generator=gen)
    return a, b, A_log, dt_bias, gate, w


@pytest.mark.parametrize("steep", [False, True])
@pytest.mark.parametrize("with_gate,eps", [(True, 1e-5), (False, 1e-6)])
@pytest.mark.parametrize("B,T,H,Hk", [(2, 256, 4, 4), (1, 100, 4, 2), (3, 65, 2, 1),
                                      (1, 1, 2, 2)])
def test_chunk_layer_against_oracle(cuda, steep, with_gate, eps, B, T, H, Hk):
    (q, k, v, _, _, S), _ = device_inputs(B, T, H, 128, 128, seed=B + T + H, dtype="bf16",
                                          dev=cuda, h0_std=0.02)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, cuda, T, with_gate, steep=steep)
    y, hT = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, eps=eps, initial_state=S,
                                             output_final_state=True)
    g, beta = orc.layer_gates(f64(a), f64(b), f64(A_log), f64(dt_bias))
    o, rh = orc.chunk_exact(orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep),
                            f64(v), g, beta, f64(S))
    ry = orc.rms_norm_gated(o, f64(w), None if gate is None else f64(gate), eps)
    assert y.dtype == v.dtype and y.shape == v.shape
    assert_close(f64(y), ry, "bf16", "y")
    assert_close(f64(hT), rh, "bf16", "state")


def test_chunk_layer_full_size_equals_separate_operations(cuda):
    """B=4 T=4096 H=16: the fused kernel against the op followed by the gated
    norm in PyTorch fp32, with the gates computed by PyTorch as the layer does."""
    B, T, H = 4, 4096, 16
    q, k, v, _, _, S = device_inputs_fast(B, T, H, 128, 128, seed=11, dtype="bf16", dev=cuda,
                                          h0_std=0.02)
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, cuda, 11, True)
    y, hT = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, initial_state=S,
                                             output_final_state=True)
    gd = -torch.exp(A_log) * torch.nn.functional.softplus(a + dt_bias)
    bd = torch.sigmoid(b)
    o, h2 = ops.chunk_gated_delta_rule(q, k, v, gd, bd, initial_state=S, output_final_state=True)
    of = o.float()
    ry = of * torch.rsqrt(of.square().mean(-1, keepdim=True) + 1e-5) * w
    ry = ry * torch.nn.functional.silu(gate.float())
    err_y = ((y.float() - ry).abs().max() / ry.abs().max()).item()
    err_h = ((hT - h2).abs().max() / h2.abs().max()).item()
    assert err_y < orc.TOL_BF16_REL, err_y
    assert err_h < orc.TOL_BF16_REL, err_h
    assert torch.isfinite(y).all()


@pytest.mark.parametrize("pair", ["0", "1"])
def test_chunk_layer_forms_agree(cuda, pair):
    """With and without shared preparation (GDN_CHUNK_TC_PAIR forces either
    form; both are clusters of two CTAs exchanging row sums) the outputs are
    bit-identical to the form the dispatcher picks for a small grid (pairs)."""
    B, T, H = 2, 300, 4
    (q, k, v, _, _, S), _ = device_inputs(B, T, H, 128, 128, seed=9, dtype="bf16", dev=cuda,
                                          h0_std=0.02)
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, cuda, 9, True)
    args = (q, k, v, a, b, A_log, dt_bias)
    kw = dict(gate=gate, norm_weight=w, initial_state=S, output_final_state=True)
    y0, h0 = ops.gated_delta_rule_chunk_layer(*args, **kw)
    with _lib.kernel_env("GDN_CHUNK_TC_PAIR", pair):
        y1, h1 = ops.gated_delta_rule_chunk_layer(*args, **kw)
    assert torch.equal(y0, y1) and torch.equal(h0, h1)


def test_chunk_layer_in_place_state_and_empty(cuda):
    B, T, H = 2, 130, 4
    (q, k, v, _, _, S), _ = device_inputs(B, T, H, 128, 128, seed=5, dtype="bf16", dev=cuda,
                                          h0_std=0.02)
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, cuda, 5, True)
    y1, h1 = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                              norm_weight=w, initial_state=S,
                                              output_final_state=True)
    S2 = S.clone()
    y2, _ = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, initial_state=S2,
                                             final_state_out=S2)
    assert torch.equal(y1, y2) and torch.equal(h1, S2)
    # T = 0: nothing to normalise, the state is carried through
    e = [t[:, :0].contiguous() for t in (q, k, v, a, b, gate)]
    y0, h0 = ops.gated_delta_rule_chunk_layer(e[0], e[1], e[2], e[3], e[4], A_log, dt_bias,
                                              gate=e[5], norm_weight=w, initial_state=S,
                                              output_final_state=True)
    assert y0.shape == (B, 0, H, 128) and torch.equal(h0, S)


@pytest.mark.parametrize("lens", [(100, 1, 101), (64, 0, 128, 7)])
def test_chunk_layer_packed_sequences_equal_each_alone(cuda, lens):
    """Packed sequences (cu_seqlens) in one row: every sequence's y and final
    state equal the same layer form run on that sequence alone."""
    T, H = sum(lens), 4
    (q, k, v, _, _, _), _ = device_inputs(1, T, H, 128, 128, seed=T, dtype="bf16", dev=cuda)
    a, b, A_log, dt_bias, gate, w = _layer_extras(1, T, H, cuda, T, True)
    gen = torch.Generator(device=cuda).manual_seed(T + 1)
    S = torch.randn(len(lens), H, 128, 128, device=cuda, generator=gen) * 0.02
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=cuda)
    y, hT = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, initial_state=S,
                                             output_final_state=True, cu_seqlens=cu)
    assert y.shape == v.shape and hT.shape == S.shape
    for s, (t0, t1) in enumerate(zip(cu.tolist(), cu.tolist()[1:])):
        part = [t[:, t0:t1].contiguous() for t in (q, k, v, a, b, gate)]
        ys, hs = ops.gated_delta_rule_chunk_layer(*part[:5], A_log, dt_bias, gate=part[5],
                                                  norm_weight=w, initial_state=S[s:s + 1],
                                                  output_final_state=True)
        assert torch.equal(y[:, t0:t1], ys), s
        assert torch.equal(hT[s:s + 1], hs), s


def test_no_device_error_recorded_chunk_layer(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0
