"""Size-independent properties at the full benchmark sizes, where the float64
oracle would take too long: for fixed q, k, g, beta the delta rule is linear
in (v, initial state), so o(v1 + 2 v2, h1 + 2 h2) = o(v1, h1) + 2 o(v2, h2),
and so is the final state.  Checked on the tcgen05 chunk kernel (bf16,
B=4 T=4096 H=16 dk=dv=128), the warp-level chunk path (fp32, same sizes) and
the decode kernel (bf16, B=64 H=16 dk=dv=128, one token).  Also bit-exact
determinism and state carry across a chunk-aligned split of a sequence."""

import pytest
import torch

from gated_deltanet_jax_b200 import ops
from helpers import device_inputs_fast

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


def _linearity(run, v, dev, state_shape, dtype, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    v1 = v.float()
    v2 = torch.randn(v.shape, device=dev, generator=gen)
    h1 = torch.randn(state_shape, device=dev, generator=gen) * 0.02
    h2 = torch.randn(state_shape, device=dev, generator=gen) * 0.02
    cast = lambda x: x.to(dtype).contiguous()  # noqa: E731
    o1, s1 = run(cast(v1), h1)
    o2, s2 = run(cast(v2), h2)
    o3, s3 = run(cast(cast(v1).float() + 2 * cast(v2).float()), h1 + 2 * h2)
    return _rel(o3, o1.float() + 2 * o2.float()), _rel(s3, s1 + 2 * s2)


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-2), ("fp32", 1e-4)])
def test_chunk_linear_in_values_and_state_full_size(cuda, dtype, tol):
    B, T, H, D = 4, 4096, 16, 128
    q, k, v, g, b, _ = device_inputs_fast(B, T, H, D, D, seed=31, dtype=dtype, dev=cuda)

    def run(vv, h0):
        return ops.chunk_gated_delta_rule(q, k, vv, g, b, initial_state=h0,
                                          output_final_state=True)

    eo, es = _linearity(run, v, cuda, (B, H, D, D), q.dtype, 32)
    assert eo < tol, eo
    assert es < tol, es


def test_decode_linear_in_values_and_state_full_size(cuda):
    B, H, D = 64, 16, 128
    q, k, v, g, b, _ = device_inputs_fast(B, 1, H, D, D, seed=41, dtype="bf16", dev=cuda)

    def run(vv, h0):
        return ops.fused_recurrent_gated_delta_rule(q, k, vv, g, b, initial_state=h0,
                                                    output_final_state=True)

    eo, es = _linearity(run, v, cuda, (B, H, D, D), q.dtype, 42)
    assert eo < 2e-2, eo
    assert es < 2e-2, es


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_chunk_forward_deterministic_and_state_carry_exact(cuda, dtype):
    """Repeated calls give the same bits, and a sequence split at a chunk
    boundary, with the fp32 state carried from the first call into the second,
    gives the same bits as one call over the whole sequence."""
    B, T, H, D = 2, 1024, 8, 128
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, D, D, seed=51, dtype=dtype, dev=cuda,
                                           h0_std=0.02)

    def run(sl, h):
        return ops.chunk_gated_delta_rule(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                          v[:, sl].contiguous(), g[:, sl].contiguous(),
                                          b[:, sl].contiguous(), initial_state=h,
                                          output_final_state=True)

    o, hT = run(slice(0, T), h0)
    o2, hT2 = run(slice(0, T), h0)
    assert torch.equal(o, o2) and torch.equal(hT, hT2)
    oa, ha = run(slice(0, 384), h0)
    ob, hb = run(slice(384, T), ha)
    assert torch.equal(torch.cat([oa, ob], 1), o)
    assert torch.equal(hb, hT)
