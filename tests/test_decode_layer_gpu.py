"""The layer form of the decode step (gdn_recurrent_fwd_layer): gates from the
raw a_proj / b_proj outputs (model.py:136-139), the recurrent step, and the
gated RMSNorm of its output (model.py:41-53), in one kernel.  Checked against
the oracle's restatement of each part, composed."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, f64

pytestmark = pytest.mark.gpu


def _layer_problem(B, H, Hk, dtype, dev, seed, with_gate):
    (q, k, v, _, _, S), _ = device_inputs(B, 1, H, 128, 128, seed=seed, dtype=dtype, dev=dev,
                                          h0_std=0.02)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    a = torch.randn(B, 1, H, device=dev, generator=gen)
    b = torch.randn(B, 1, H, device=dev, generator=gen)
    A_log = torch.log(torch.rand(H, device=dev, generator=gen) * 16 + 1e-4)   # model.py:104-106
    dt_bias = torch.randn(H, device=dev, generator=gen) * 0.5
    gate = torch.randn(B, 1, H, 128, device=dev, generator=gen).to(v.dtype) if with_gate else None
    w = 1.0 + 0.1 * torch.randn(128, device=dev, generator=gen)
    return q, k, v, a, b, A_log, dt_bias, S, gate, w


def _oracle(q, k, v, a, b, A_log, dt_bias, S, gate, w, rep, eps):
    g, beta = orc.layer_gates(f64(a), f64(b), f64(A_log), f64(dt_bias))
    o, hT = orc.recurrent_ref(orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep),
                              f64(v), g, beta, f64(S))
    return orc.rms_norm_gated(o, f64(w), None if gate is None else f64(gate), eps), hT


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("with_gate,eps", [(True, 1e-5), (False, 1e-6)])
@pytest.mark.parametrize("B,H,Hk", [(4, 8, 8), (3, 12, 4), (64, 16, 16)])
def test_decode_layer_against_oracle(cuda, dtype, with_gate, eps, B, H, Hk):
    q, k, v, a, b, A_log, dt_bias, S, gate, w = _layer_problem(B, H, Hk, dtype, cuda,
                                                               seed=B + H, with_gate=with_gate)
    y, hT = ops.gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                              norm_weight=w, eps=eps, initial_state=S,
                                              output_final_state=True)
    ry, rh = _oracle(q, k, v, a, b, A_log, dt_bias, S, gate, w, H // Hk, eps)
    assert y.dtype == v.dtype and y.shape == v.shape
    assert_close(f64(y), ry, dtype, "y")
    assert_close(f64(hT), rh, dtype, "state")


def test_decode_layer_in_place_equals_unfused_step(cuda):
    """The state update is the plain op's, bit for bit; y is its output normalised."""
    B, H = 8, 16
    q, k, v, a, b, A_log, dt_bias, S, gate, w = _layer_problem(B, H, H, "bf16", cuda, seed=3,
                                                               with_gate=True)
    g, beta = orc.layer_gates(f64(a), f64(b), f64(A_log), f64(dt_bias))
    S_ref = S.clone()
    y, _ = ops.gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                             norm_weight=w, initial_state=S, final_state_out=S)
    # the same gates, computed on the device in fp32 the way the kernel does
    gd = -torch.exp(A_log) * torch.nn.functional.softplus(a + dt_bias)
    bd = torch.sigmoid(b)
    o, _ = ops.fused_recurrent_gated_delta_rule(q, k, v, gd, bd, initial_state=S_ref,
                                                final_state_out=S_ref)
    assert_close(f64(S), f64(S_ref), "bf16", "state")
    ry = orc.rms_norm_gated(f64(o), f64(w), f64(gate), 1e-5)
    assert_close(f64(y), ry, "bf16", "y")
    assert np.abs(g - f64(gd)).max() < 1e-4 and np.abs(beta - f64(bd)).max() < 1e-6


def test_no_device_error_recorded_layer(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0
