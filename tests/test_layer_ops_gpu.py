"""The layer's work around the op on the GPU: the short convolution + SiLU
(gdn_short_conv_fwd, model.py:15-40), the gated RMSNorm (gdn_gated_rmsnorm_fwd,
model.py:41-53), and the layer forms at the reference's default head dims
(dk = 256, dv = 512; configuration.py, model.py:70-75) and the general
recurrent shapes.  Checked against the oracle's restatement of each part."""

import math

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, f64

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def _conv_inputs(B, T, C, K, dtype, dev, seed, with_state):
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(B, T, C, device=dev, generator=gen).to(DT[dtype])
    w = torch.randn(K, C, device=dev, generator=gen) * 0.5
    st = torch.randn(B, K - 1, C, device=dev, generator=gen).to(DT[dtype]) if with_state else None
    return x, w, st


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("K", [1, 2, 4])
@pytest.mark.parametrize("T", [1, 7, 64, 65, 300])
@pytest.mark.parametrize("with_state", [False, True])
def test_short_conv_against_oracle(cuda, dtype, K, T, with_state):
    B, C = 3, 96
    x, w, st = _conv_inputs(B, T, C, K, dtype, cuda, seed=T + K, with_state=with_state)
    y, s_out = ops.short_convolution(x, w, conv_state=st, output_final_state=True)
    ry, rs = orc.short_conv(f64(x), f64(w), "silu", None if st is None else f64(st))
    assert y.dtype == x.dtype and y.shape == x.shape
    assert_close(f64(y), ry, dtype, "y")
    np.testing.assert_array_equal(f64(s_out), rs)            # the inputs, moved exactly
    # no activation
    y0, _ = ops.short_convolution(x, w, conv_state=st, activation=None)
    ry0, _ = orc.short_conv(f64(x), f64(w), None, None if st is None else f64(st))
    assert_close(f64(y0), ry0, dtype, "y (no activation)")


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_short_conv_decode_steps_equal_one_call(cuda, dtype):
    """Token by token with the conv state updated in place equals one call over
    the whole sequence, bit for bit (same products in the same order)."""
    B, T, C, K = 4, 37, 2048, 4
    x, w, _ = _conv_inputs(B, T, C, K, dtype, cuda, seed=11, with_state=False)
    y, s_all = ops.short_convolution(x, w, output_final_state=True)
    S = torch.zeros(B, K - 1, C, dtype=x.dtype, device=cuda)
    ys = []
    for t in range(T):
        yt, _ = ops.short_convolution(x[:, t:t + 1], w, conv_state=S, final_state_out=S)
        ys.append(yt)
    assert torch.equal(torch.cat(ys, 1), y)
    assert torch.equal(S, s_all)
    # a long call with the state updated in place (one token tile over all T)
    S2 = torch.zeros_like(S)
    y2, _ = ops.short_convolution(x, w, conv_state=S2, final_state_out=S2)
    assert torch.equal(y2, y) and torch.equal(S2, s_all)


def test_short_conv_flax_kernel_layout_and_empty(cuda):
    x, w, st = _conv_inputs(2, 9, 64, 4, "bf16", cuda, seed=3, with_state=True)
    y1, _ = ops.short_convolution(x, w)
    y2, _ = ops.short_convolution(x, w.reshape(4, 1, 64))       # nnx.Conv kernel (K, 1, C)
    assert torch.equal(y1, y2)
    out = torch.full_like(st, 7)
    y0, s = ops.short_convolution(x[:, :0], w, conv_state=st, final_state_out=out)
    assert y0.shape == (2, 0, 64) and torch.equal(s, st)         # T = 0 carries the state
    assert _lib.load().gdn_device_error(0) == 0


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("dv", [64, 128, 512])
@pytest.mark.parametrize("with_gate", [False, True])
def test_gated_rmsnorm_against_oracle(cuda, dtype, dv, with_gate):
    gen = torch.Generator(device=cuda).manual_seed(dv)
    o = torch.randn(3, 50, 4, dv, device=cuda, generator=gen).to(DT[dtype])
    gate = torch.randn(o.shape, device=cuda, generator=gen).to(DT[dtype]) if with_gate else None
    w = 1.0 + 0.1 * torch.randn(dv, device=cuda, generator=gen)
    y = ops.gated_rms_norm(o, gate, w, eps=1e-5)
    ry = orc.rms_norm_gated(f64(o), f64(w), None if gate is None else f64(gate), 1e-5)
    assert_close(f64(y), ry, dtype, "y")
    y2 = ops.gated_rms_norm(o.clone(), gate, w, eps=1e-5)
    o2 = o.clone()
    ops.gated_rms_norm(o2, gate, w, eps=1e-5, out=o2)             # in place
    assert torch.equal(o2, y) and torch.equal(y2, y)


def _layer_extras(B, T, H, dv, dev, seed, dtype):
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    a = torch.randn(B, T, H, device=dev, generator=gen)
    b = torch.randn(B, T, H, device=dev, generator=gen)
    A_log = torch.log(torch.rand(H, device=dev, generator=gen) * 16 + 1e-4)   # model.py:104-106
    u = torch.rand(H, device=dev, generator=gen)
    dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
    dt_bias = dt + torch.log(-torch.expm1(-dt))                               # model.py:108-113
    gate = torch.randn(B, T, H, dv, device=dev, generator=gen).to(DT[dtype])
    w = 1.0 + 0.1 * torch.randn(dv, device=dev, generator=gen)
    return a, b, A_log, dt_bias, gate, w


def _layer_oracle(q, k, v, a, b, A_log, dt_bias, S, gate, w, rep, eps):
    g, beta = orc.layer_gates(f64(a), f64(b), f64(A_log), f64(dt_bias))
    o, hT = orc.recurrent_ref(orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep),
                              f64(v), g, beta, None if S is None else f64(S))
    return orc.rms_norm_gated(o, f64(w), None if gate is None else f64(gate), eps), hT


@pytest.mark.parametrize("dk,dv,T,H,Hk", [(256, 512, 130, 3, 3), (256, 512, 64, 4, 2),
                                          (128, 256, 100, 2, 2), (256, 128, 65, 2, 1)])
@pytest.mark.parametrize("with_h0", [False, True])
def test_chunk_layer_other_shapes_against_oracle(cuda, dk, dv, T, H, Hk, with_h0):
    """The chunked layer form where it runs as two launches (the chunk kernel
    forming the gates, then the norm in place): the reference's default head
    dims dk = 256, dv = 512 among them."""
    B = 2
    (q, k, v, _, _, S), _ = device_inputs(B, T, H, dk, dv, seed=dk + dv + T, dtype="bf16",
                                          dev=cuda, h0_std=0.02 if with_h0 else None)
    q, k = q[:, :, ::H // Hk].contiguous(), k[:, :, ::H // Hk].contiguous()
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, dv, cuda, seed=T, dtype="bf16")
    y, hT = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, initial_state=S,
                                             output_final_state=True)
    ry, rh = _layer_oracle(q, k, v, a, b, A_log, dt_bias, S, gate, w, H // Hk, 1e-5)
    assert y.shape == v.shape and y.dtype == v.dtype
    assert_close(f64(y), ry, "bf16", "y")
    assert_close(f64(hT), rh, "bf16", "state")
    assert _lib.load().gdn_device_error(0) == 0


def test_chunk_layer_default_dims_equal_separate_operations(cuda):
    """B=8 T=2048 H=6 dk=256 dv=512 (the delta-rule core of the reference's
    default configuration): the layer form against torch gates, the op and
    torch's gated RMSNorm, run as separate operations."""
    B, T, H, dk, dv = 8, 2048, 6, 256, 512
    gen = torch.Generator(device=cuda).manual_seed(5)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=cuda, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, dk, device=cuda, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, dv, device=cuda, generator=gen).bfloat16()
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, dv, cuda, seed=9, dtype="bf16")
    y, hT = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, output_final_state=True)
    g = -torch.exp(A_log) * torch.nn.functional.softplus(a + dt_bias)
    beta = torch.sigmoid(b)
    o, h2 = ops.chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True)
    of = o.float()
    ref = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + 1e-5) * w \
        * torch.nn.functional.silu(gate.float())
    assert_close(f64(y), f64(ref), "bf16", "y")
    assert_close(f64(hT), f64(h2), "bf16", "state")
    assert torch.isfinite(y.float()).all()


@pytest.mark.parametrize("dtype,dk,dv,T", [("bf16", 256, 512, 1), ("fp32", 256, 512, 1),
                                           ("bf16", 64, 64, 5), ("fp32", 128, 96, 3),
                                           ("bf16", 256, 512, 70)])
def test_recurrent_layer_other_shapes_against_oracle(cuda, dtype, dk, dv, T):
    """gdn_recurrent_fwd_layer beyond single-token dk = dv = 128: the general
    recurrent kernel forming the gates per token then the norm, and (T >= 64
    on the tensor-core shapes) the chunked layer form."""
    B, H = 3, 4
    (q, k, v, _, _, S), _ = device_inputs(B, T, H, dk, dv, seed=dk + T, dtype=dtype, dev=cuda,
                                          h0_std=0.02)
    a, b, A_log, dt_bias, gate, w = _layer_extras(B, T, H, dv, cuda, seed=dv, dtype=dtype)
    y, hT = ops.gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                              norm_weight=w, initial_state=S,
                                              output_final_state=True)
    ry, rh = _layer_oracle(q, k, v, a, b, A_log, dt_bias, S, gate, w, 1, 1e-5)
    assert_close(f64(y), ry, dtype, "y")
    assert_close(f64(hT), rh, dtype, "state")
    # in place, no gate
    S2 = S.clone()
    y2, _ = ops.gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, norm_weight=w,
                                              initial_state=S2, final_state_out=S2)
    ry2, _ = _layer_oracle(q, k, v, a, b, A_log, dt_bias, S, None, w, 1, 1e-5)
    assert_close(f64(y2), ry2, dtype, "y (no gate)")
    assert torch.equal(S2, hT)
