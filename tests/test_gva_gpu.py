"""Grouped value heads on the GPU: q and k with Hk heads, v / g / beta / state
with H = rep * Hk heads.  The reference layer repeats q and k (jnp.repeat,
model.py:132-135) before its ops; the ops here take the unrepeated tensors.
Every kernel must give exactly what it gives on the repeated tensors, and the
oracle's answer on the repeated inputs."""

import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops, sequence_parallel as sp
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, device_inputs_fast, f64

pytestmark = pytest.mark.gpu


def _grouped(q, k, rep):
    """Keep every rep-th head of q and k: the unrepeated tensors whose repeat is
    (q, k) with its heads replaced by copies of the kept ones."""
    qg, kg = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    return qg, kg, qg.repeat_interleave(rep, dim=2), kg.repeat_interleave(rep, dim=2)


@pytest.mark.parametrize("pair", [None, "0", "1"])
@pytest.mark.parametrize("B,T,Hk,rep,dv", [(2, 300, 2, 3, 128), (1, 129, 1, 4, 256),
                                          (3, 64, 4, 2, 64)])
def test_chunk_tensor_core_grouped_equals_repeated(cuda, pair, B, T, Hk, rep, dv):
    """pair None: the two-launch form (the default); "0" / "1": the one-launch
    kernel's unpaired / paired form."""
    H = Hk * rep
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=T + rep, dtype="bf16",
                                           dev=cuda, h0_std=0.02)
    qg, kg, qr, kr = _grouped(q, k, rep)
    with _lib.kernel_env("GDN_CHUNK_KERNEL", None if pair is None else "fused"), \
            _lib.kernel_env("GDN_CHUNK_TC_PAIR", pair):
        o_g, h_g = ops.chunk_gated_delta_rule(qg, kg, v, g, b, initial_state=h0,
                                              output_final_state=True)
        o_r, h_r = ops.chunk_gated_delta_rule(qr, kr, v, g, b, initial_state=h0,
                                              output_final_state=True)
    assert torch.equal(o_g, o_r)
    assert torch.equal(h_g, h_r)


@pytest.mark.parametrize("semantics", ["exact", "reference"])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_chunk_cuda_core_grouped_against_oracle(cuda, semantics, dtype):
    B, T, Hk, rep, dk, dv, C = 1, 100, 2, 3, 32, 48, 32
    H = Hk * rep
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=21, dtype=dtype, dev=cuda,
                                              h0_std=0.02)
    qg, kg, qr, kr = _grouped(q, k, rep)
    o_g, h_g = ops.chunk_gated_delta_rule(qg, kg, v, g, b, initial_state=h0,
                                          output_final_state=True, chunk_size=C,
                                          semantics=semantics)
    o_r, h_r = ops.chunk_gated_delta_rule(qr, kr, v, g, b, initial_state=h0,
                                          output_final_state=True, chunk_size=C,
                                          semantics=semantics)
    assert torch.equal(o_g, o_r) and torch.equal(h_g, h_r)
    hq, hk = f64(qr), f64(kr)
    if semantics == "exact":
        ro, rh = orc.chunk_exact(hq, hk, *host[2:5], host[5], C)
    else:
        ro, rh = orc.chunk_reference_literal(hq, hk, *host[2:5], initial_state=host[5],
                                             output_final_state=True, chunk_size=C)
    assert_close(f64(o_g), ro, dtype, "o")
    assert_close(f64(h_g), rh, dtype, "state")


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("T,dk,dv", [(7, 32, 64), (1, 64, 64), (1, 128, 128), (3, 128, 128)])
def test_recurrent_grouped_against_oracle(cuda, dtype, T, dk, dv):
    """General recurrent kernel, and (T = 1, dk = dv = 128) the bulk-copy decode kernel."""
    B, Hk, rep = 3, 4, 4
    H = Hk * rep
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=T * dk, dtype=dtype,
                                              dev=cuda, h0_std=0.02)
    qg, kg, qr, kr = _grouped(q, k, rep)
    o_g, h_g = ops.fused_recurrent_gated_delta_rule(qg, kg, v, g, b, initial_state=h0,
                                                    output_final_state=True)
    o_r, h_r = ops.fused_recurrent_gated_delta_rule(qr, kr, v, g, b, initial_state=h0,
                                                    output_final_state=True)
    assert torch.equal(o_g, o_r) and torch.equal(h_g, h_r)
    ro, rh = orc.recurrent_ref(f64(qr), f64(kr), *host[2:6])
    assert_close(f64(o_g), ro, dtype, "o")
    assert_close(f64(h_g), rh, dtype, "state")


def test_decode_in_place_grouped(cuda):
    """Decode step with the state updated in place, grouped heads (the layer's GVA)."""
    B, Hk, rep = 8, 2, 6
    H = Hk * rep
    q, k, v, g, b, S = device_inputs_fast(B, 1, H, 128, 128, seed=5, dtype="bf16", dev=cuda,
                                          h0_std=0.02)
    qg, kg, qr, kr = _grouped(q, k, rep)
    S_ref = S.clone()
    o_g, _ = ops.fused_recurrent_gated_delta_rule(qg, kg, v, g, b, initial_state=S,
                                                  final_state_out=S)
    o_r, _ = ops.fused_recurrent_gated_delta_rule(qr, kr, v, g, b, initial_state=S_ref,
                                                  final_state_out=S_ref)
    assert torch.equal(o_g, o_r) and torch.equal(S, S_ref)


def test_sequence_split_grouped(cuda):
    B, T, Hk, rep = 1, 1000, 2, 2
    H = Hk * rep
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, 128, seed=9, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    qg, kg, _, _ = _grouped(q, k, rep)
    o_s, h_s = sp.chunk_gated_delta_rule_split(qg, kg, v, g, b, initial_state=h0,
                                               output_final_state=True, parts=3)
    o_u, h_u = ops.chunk_gated_delta_rule(qg, kg, v, g, b, initial_state=h0,
                                          output_final_state=True)
    assert_close(f64(o_s), f64(o_u), "bf16", "o")
    assert_close(f64(h_s), f64(h_u), "bf16", "state")


def test_rejects_ungrouped_heads(cuda):
    q = torch.zeros(1, 8, 4, 16, device=cuda)
    v = torch.zeros(1, 8, 6, 16, device=cuda)
    g = torch.zeros(1, 8, 6, device=cuda)
    with pytest.raises(ValueError, match="multiple"):
        ops.chunk_gated_delta_rule(q, q, v, g, g)


def test_no_device_error_recorded_gva(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0
