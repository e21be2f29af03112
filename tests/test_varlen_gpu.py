"""Packed variable-length sequences (``cu_seqlens``) on the chunked forward.

Several sequences stored back to back in one row: every sequence must get
what the same kernel gives it on its own, and the oracle's answer.  The rows
of a chunk past a sequence's end hold the next sequence's tokens, so these
tests also check that nothing leaks across a boundary."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, f64

pytestmark = pytest.mark.gpu


def _packed(lengths, H, Hk, dk, dv, dtype, dev, seed):
    T = int(sum(lengths))
    (q, k, v, g, b, _), _ = device_inputs(1, T, H, dk, dv, seed=seed, dtype=dtype, dev=dev)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    h0 = (torch.randn(len(lengths), H, dk, dv, device=dev,
                      generator=torch.Generator(device=dev).manual_seed(seed)) * 0.02)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    return q, k, v, g, b, h0, cu


def _run(pair, fn):
    """fn() on the one-launch tensor-core kernel (the one packed sequences
    take), in its default form (pair None) or forced unpaired / paired."""
    with _lib.kernel_env("GDN_CHUNK_KERNEL", "fused"), _lib.kernel_env("GDN_CHUNK_TC_PAIR", pair):
        return fn()


CASES = [
    # lengths, H, Hk, dk, dv, dtype, chunk  (tensor-core kernel: bf16, dk 128, chunk 64)
    ([200, 1, 63, 64, 65, 0, 130], 2, 2, 128, 128, "bf16", 64),
    ([300, 77], 4, 2, 128, 64, "bf16", 64),
    ([5, 129, 40], 3, 3, 128, 256, "bf16", 64),
    # CUDA-core kernel
    ([33, 0, 70, 16], 2, 1, 32, 48, "fp32", 32),
    ([100, 3], 2, 2, 64, 64, "bf16", 16),
]


@pytest.mark.parametrize("pair", [None, "0", "1"])
@pytest.mark.parametrize("lengths,H,Hk,dk,dv,dtype,C", CASES)
def test_packed_equals_each_sequence_alone(cuda, pair, lengths, H, Hk, dk, dv, dtype, C):
    q, k, v, g, b, h0, cu = _packed(lengths, H, Hk, dk, dv, dtype, cuda, seed=len(lengths) + dk)

    def run():
        o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                           output_final_state=True, chunk_size=C, cu_seqlens=cu)
        parts = []
        for s in range(len(lengths)):
            a0, a1 = int(cu[s]), int(cu[s + 1])
            sl = slice(a0, a1)
            parts.append(ops.chunk_gated_delta_rule(q[:, sl], k[:, sl], v[:, sl], g[:, sl],
                                                    b[:, sl], initial_state=h0[s:s + 1],
                                                    output_final_state=True, chunk_size=C))
        return o, hT, parts

    o, hT, parts = _run(pair, run)
    for s, (o_s, h_s) in enumerate(parts):
        a0, a1 = int(cu[s]), int(cu[s + 1])
        assert torch.equal(o[:, a0:a1], o_s), f"sequence {s}: output"
        assert torch.equal(hT[s:s + 1], h_s), f"sequence {s}: state"


@pytest.mark.parametrize("lengths,H,Hk,dk,dv,dtype,C", CASES)
def test_packed_against_oracle(cuda, lengths, H, Hk, dk, dv, dtype, C):
    q, k, v, g, b, h0, cu = _packed(lengths, H, Hk, dk, dv, dtype, cuda, seed=7 * len(lengths))
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True,
                                       chunk_size=C, cu_seqlens=cu)
    rep = H // Hk
    hq, hk = orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep)
    hv, hg, hb, hh0 = f64(v), f64(g), f64(b), f64(h0)
    for s in range(len(lengths)):
        a0, a1 = int(cu[s]), int(cu[s + 1])
        sl = slice(a0, a1)
        ro, rh = orc.chunk_exact(hq[:, sl], hk[:, sl], hv[:, sl], hg[:, sl], hb[:, sl],
                                 hh0[s:s + 1], C)
        if a1 > a0:
            assert_close(f64(o[:, sl]), ro, dtype, f"sequence {s} o")
        assert_close(f64(hT[s:s + 1]), rh, dtype, f"sequence {s} state")


def test_packed_rejects_bad_offsets(cuda):
    q = torch.zeros(1, 10, 2, 16, device=cuda)
    g = torch.zeros(1, 10, 2, device=cuda)
    for bad in ([0, 4, 3, 10], [1, 10], [0, 9]):
        with pytest.raises(ValueError, match="cu_seqlens"):
            ops.chunk_gated_delta_rule(q, q, q, g, g, cu_seqlens=torch.tensor(bad))
    with pytest.raises(ValueError, match="exact"):
        ops.chunk_gated_delta_rule(q, q, q, g, g, cu_seqlens=torch.tensor([0, 10]),
                                   semantics="reference")


def test_no_device_error_recorded_varlen(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0
