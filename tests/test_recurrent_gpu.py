"""GPU parity of the fused recurrent kernel (gdn_recurrent_fwd) against the
oracle, the reference's own outputs (golden.npz) and a PyTorch fp32 step."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import ops
from oracle import gdn_oracle as orc
from helpers import (assert_close, device_inputs, device_inputs_fast, f64, to_dev,
                     torch_recurrent_step_fp32)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["c0", "h0", "tail", "layer", "lm", "h1", "d256"])
def test_matches_reference_kernel_outputs(golden, cuda, name):
    """Zero initial state, no final state: the reference call form (ops.py:187)."""
    c = golden[name]
    args = [to_dev(c[x], torch.float32, cuda) for x in ("q", "k", "v", "g", "beta")]
    o, hT = ops.fused_recurrent_gated_delta_rule(*args)
    assert hT is None
    assert o.dtype == torch.float32
    assert_close(f64(o), c["o_recurrent"], "fp32", name)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("dk,dv", [(16, 16), (16, 32), (32, 64), (64, 64), (64, 48),
                                   (128, 128), (128, 256), (256, 512), (256, 16)])
@pytest.mark.parametrize("T", [1, 5, 40])
def test_against_oracle(cuda, dtype, dk, dv, T):
    (q, k, v, g, b, h0), host = device_inputs(2, T, 3, dk, dv, seed=dk + dv + T, dtype=dtype,
                                              dev=cuda, h0_std=0.02)
    o, hT = ops.fused_recurrent_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                                 output_final_state=True)
    ro, rh = orc.recurrent_ref(*host)
    assert o.dtype == q.dtype
    assert_close(f64(o), ro, dtype, "o")
    assert_close(f64(hT), rh, dtype, "state")


def test_in_place_state(cuda):
    (q, k, v, g, b, h0), host = device_inputs(3, 4, 2, 64, 64, seed=1, dtype="bf16",
                                              dev=cuda, h0_std=0.05)
    S = h0.clone()
    o, hT = ops.fused_recurrent_gated_delta_rule(q, k, v, g, b, initial_state=S,
                                                 final_state_out=S)
    assert hT.data_ptr() == S.data_ptr()
    ro, rh = orc.recurrent_ref(*host)
    assert_close(f64(o), ro, "bf16", "o")
    assert_close(f64(S), rh, "bf16", "state")


def test_multi_token_call_equals_single_steps(cuda):
    (q, k, v, g, b, h0), _ = device_inputs(2, 9, 4, 128, 128, seed=2, dtype="bf16",
                                           dev=cuda, h0_std=0.02)
    o_all, h_all = ops.fused_recurrent_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                                        output_final_state=True)
    S = h0.clone()
    outs = []
    for t in range(9):
        sl = slice(t, t + 1)
        o_t, _ = ops.fused_recurrent_gated_delta_rule(q[:, sl], k[:, sl], v[:, sl], g[:, sl],
                                                      b[:, sl], initial_state=S,
                                                      final_state_out=S)
        outs.append(o_t)
    torch.testing.assert_close(torch.cat(outs, 1).float(), o_all.float(), rtol=0, atol=1e-2)
    torch.testing.assert_close(S, h_all, rtol=1e-5, atol=1e-6)


def test_empty_sequence_carries_state(cuda):
    (q, k, v, g, b, h0), _ = device_inputs(1, 0, 2, 32, 32, seed=0, dtype="fp32", dev=cuda,
                                           h0_std=0.1)
    o, hT = ops.fused_recurrent_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                                 output_final_state=True)
    assert o.shape == (1, 0, 2, 32)
    torch.testing.assert_close(hT, h0)


def test_decode_config_full_size(cuda):
    """The decode configuration end to end: B=64, H=16, dk=dv=128, bf16
    q/k/v, fp32 state ~N(0,0.02), all 512 consecutive single-token steps with
    the state updated in place.

    Every head's output against a PyTorch fp32 step at every step, and the
    state after the last step (drift over 512 in-place updates); four sampled
    heads against the float64 oracle over all 512 steps."""
    B, H, dk, dv, steps = 64, 16, 128, 128, 512
    q, k, v, g, b, S = device_inputs_fast(B, steps, H, dk, dv, seed=1, dtype="bf16",
                                          dev=cuda, h0_std=0.02)
    S0 = S.clone()
    S_ref = S.clone()
    outs, err_o = [], []
    for t in range(steps):
        sl = slice(t, t + 1)
        o, _ = ops.fused_recurrent_gated_delta_rule(q[:, sl], k[:, sl], v[:, sl], g[:, sl],
                                                    b[:, sl], initial_state=S, final_state_out=S)
        o_ref, S_ref = torch_recurrent_step_fp32(q[:, t], k[:, t], v[:, t], g[:, t], b[:, t],
                                                 S_ref)
        err_o.append((o[:, 0].float() - o_ref).abs().max() / o_ref.abs().max())
        outs.append(o)
    err_o = torch.stack(err_o).cpu().numpy()
    worst = int(np.argmax(err_o))
    assert err_o.max() <= orc.TOL_BF16_REL, f"step {worst}: o rel error {err_o.max():.3e}"
    assert_close(f64(S), f64(S_ref), "bf16", "state after 512 steps")
    picks = [(0, 0), (5, 3), (31, 15), (63, 7)]
    bi = [p[0] for p in picks]
    hi = [p[1] for p in picks]
    o_all = torch.cat(outs, 1)
    ro, rh = orc.recurrent_ref(f64(q[bi, :, hi][:, :, None]), f64(k[bi, :, hi][:, :, None]),
                               f64(v[bi, :, hi][:, :, None]), f64(g[bi, :, hi][:, :, None]),
                               f64(b[bi, :, hi][:, :, None]), f64(S0[bi, hi][:, None]))
    assert_close(f64(o_all[bi, :, hi]), ro[:, :, 0], "bf16", "sampled o vs oracle (512 steps)")
    assert_close(f64(S[bi, hi]), rh[:, 0], "bf16", "sampled state vs oracle (512 steps)")
    assert np.isfinite(f64(S)).all()


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("with_h0,with_hT", [(True, True), (False, True), (True, False),
                                             (False, False)])
@pytest.mark.parametrize("B,H", [(1, 3), (7, 11), (37, 16)])
def test_decode_step_state_modes(cuda, dtype, with_h0, with_hT, B, H):
    """Single-token steps at dk=dv=128 (the bulk-copy decode kernel): every
    combination of initial / final state, fewer and more heads than SMs."""
    (q, k, v, g, b, h0), host = device_inputs(B, 1, H, 128, 128, seed=B * H, dtype=dtype,
                                              dev=cuda, h0_std=0.05)
    o, hT = ops.fused_recurrent_gated_delta_rule(
        q, k, v, g, b, initial_state=h0 if with_h0 else None, output_final_state=with_hT)
    ro, rh = orc.recurrent_ref(*host[:5], host[5] if with_h0 else None)
    assert_close(f64(o), ro, dtype, "o")
    if with_hT:
        assert_close(f64(hT), rh, dtype, "state")
    else:
        assert hT is None


def test_no_device_error_recorded(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0
