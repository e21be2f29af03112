"""GPU parity of the backward (gdn_chunk_bwd) against the oracle's reverse-mode
restatement (itself pinned to torch autograd of the recurrence), and of the
ops' autograd against it."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, f64

pytestmark = pytest.mark.gpu

# Gradients are compared relative to their largest entry: fp32 inputs within
# 1e-3, bf16 inputs (fp32 state and accumulation) within the bf16 bar 2e-2.
TOL = {"fp32": 1e-3, "bf16": 2e-2}


def _grads(dtype, B, T, H, dk, dv, seed, dev, with_h0=True, with_dhT=True):
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=seed, dtype=dtype, dev=dev,
                                              h0_std=0.05 if with_h0 else None)
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    do = torch.randn(B, T, H, dv, device=dev, generator=gen).to(q.dtype)
    dhT = torch.randn(B, H, dk, dv, device=dev, generator=gen) if with_dhT else None
    got = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    ref = orc.chunk_exact_backward(*host[:5], host[5], f64(do), None if dhT is None else f64(dhT),
                                   32)
    return got, ref


def _check(got, ref, dtype, with_h0=True):
    names = ["dq", "dk", "dv", "dg", "dbeta", "dh0"]
    for n, a, r in zip(names, got, ref):
        if n == "dh0" and not with_h0:
            continue
        err = orc.rel_err(f64(a), r)
        assert err <= TOL[dtype], f"{n}: rel error {err:.2e}"


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("B,T,H,dk,dv", [(2, 1, 2, 16, 32), (1, 31, 2, 64, 32), (2, 32, 1, 32, 64),
                                         (1, 33, 2, 128, 64), (2, 100, 3, 64, 96),
                                         (1, 200, 2, 128, 128), (1, 128, 2, 128, 256),
                                         (1, 65, 1, 16, 512), (1, 130, 2, 256, 64),
                                         (1, 70, 1, 256, 512)])
def test_backward_against_oracle(cuda, dtype, B, T, H, dk, dv):
    got, ref = _grads(dtype, B, T, H, dk, dv, seed=T + dk, dev=cuda)
    _check(got, ref, dtype)


@pytest.mark.parametrize("with_h0,with_dhT", [(False, False), (False, True), (True, False)])
def test_backward_state_modes(cuda, with_h0, with_dhT):
    got, ref = _grads("fp32", 1, 70, 2, 32, 32, seed=5, dev=cuda, with_h0=with_h0,
                      with_dhT=with_dhT)
    _check(got, ref, "fp32", with_h0=with_h0)


def test_backward_grouped_heads(cuda):
    """q/k with Hk heads: their gradients are the repeated problem's, summed over the group."""
    B, T, Hk, rep, dk, dv = 1, 90, 2, 3, 64, 32
    H = Hk * rep
    (q, k, v, g, b, h0), _ = device_inputs(B, T, H, dk, dv, seed=3, dtype="fp32", dev=cuda,
                                           h0_std=0.05)
    qg, kg = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    qr, kr = qg.repeat_interleave(rep, 2), kg.repeat_interleave(rep, 2)
    do = torch.randn(B, T, H, dv, device=cuda)
    dq_g, dk_g, dv_g, dg_g, db_g, dh_g = ops._chunk_backward(qg, kg, v, g, b, h0, do, None)
    dq_r, dk_r, dv_r, dg_r, db_r, dh_r = ops._chunk_backward(qr, kr, v, g, b, h0, do, None)
    torch.testing.assert_close(dq_g, dq_r.view(B, T, Hk, rep, dk).sum(3), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(dk_g, dk_r.view(B, T, Hk, rep, dk).sum(3), rtol=1e-5, atol=1e-5)
    for a, r in ((dv_g, dv_r), (dg_g, dg_r), (db_g, db_r), (dh_g, dh_r)):
        torch.testing.assert_close(a, r, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("recurrent", [False, True])
def test_autograd_through_ops(cuda, recurrent):
    """loss.backward() through the public ops gives the oracle's gradients."""
    B, T, H, dk, dv = 2, 45, 2, 32, 32
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=11, dtype="fp32", dev=cuda,
                                              h0_std=0.05)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, g, b, h0)]
    fn = ops.fused_recurrent_gated_delta_rule if recurrent else ops.chunk_gated_delta_rule
    o, hT = fn(*leaves[:5], initial_state=leaves[5], output_final_state=True)
    gen = torch.Generator(device=cuda).manual_seed(2)
    do = torch.randn(o.shape, device=cuda, generator=gen)
    dhT = torch.randn(hT.shape, device=cuda, generator=gen)
    ((o * do).sum() + (hT * dhT).sum()).backward()
    ref = orc.chunk_exact_backward(*host[:5], host[5], f64(do), f64(dhT), 32)
    for t, r in zip(leaves, ref):
        assert orc.rel_err(f64(t.grad), r) <= TOL["fp32"]
    # the forward under autograd is the plain forward
    o2, h2 = fn(q, k, v, g, b, initial_state=h0, output_final_state=True)
    torch.testing.assert_close(o.detach(), o2)
    torch.testing.assert_close(hT.detach(), h2)


@pytest.mark.parametrize("Hk", [4, 2])
def test_backward_is_deterministic(cuda, Hk):
    """No atomics anywhere: the same inputs give the same bits on every call."""
    B, T, H, dk, dv = 2, 200, 4, 128, 64
    (q, k, v, g, b, h0), _ = device_inputs(B, T, H, dk, dv, seed=4, dtype="bf16", dev=cuda,
                                           h0_std=0.05)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    gen = torch.Generator(device=cuda).manual_seed(9)
    do = torch.randn(B, T, H, dv, device=cuda, generator=gen).bfloat16()
    dhT = torch.randn(B, H, dk, dv, device=cuda, generator=gen)
    first = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    for _ in range(2):
        again = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
        for a, r in zip(again, first):
            assert torch.equal(a, r)


def test_handoff_workspace_is_compact(cuda):
    """The tensor-core path's workspace (bf16, dk = dv = 128, dense) holds only
    its bf16 hand-off: per (chunk, head) the 32 KB [Z | PT | T] slot, 32 KB of
    bf16 V' and dX rows, the 32 KB h tile and the 36 KB dh tile with the row
    partials; grouped heads add the per value head dq, dk."""
    from gated_deltanet_jax_b200 import _lib
    lib = _lib.load()
    B, T, H = 4, 4096, 16
    items = B * (T // 64) * H
    for_ = lib.gdn_chunk_bwd_workspace_bytes_for
    exact = for_(B, T, H, H, 128, 128, _lib.GDN_DTYPE_BF16)
    assert exact == items * (32768 + 32768 + 32768 + 36864)
    assert exact < 0.45 * lib.gdn_chunk_bwd_workspace_bytes(B, T, H, 128, 128)
    assert for_(B, T, H, 4, 128, 128, _lib.GDN_DTYPE_BF16) == exact + 2 * B * T * H * 128 * 4
    # a call given exactly that workspace (the op allocates this call's size),
    # against the oracle
    got, ref = _grads("bf16", 2, 200, 3, 128, 128, seed=21, dev=cuda)
    _check(got, ref, "bf16")


def test_backward_rejects_unsupported(cuda):
    q = torch.zeros(1, 8, 1, 16, device=cuda, requires_grad=True)
    g = torch.zeros(1, 8, 1, device=cuda)
    with pytest.raises(NotImplementedError):
        ops.chunk_gated_delta_rule(q, q, q, g, g, semantics="reference")


def test_no_device_error_recorded_backward(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0


# ---------------------------------------------------------------------------
# packed sequences (cu_seqlens)
# ---------------------------------------------------------------------------

def _packed_problem(lengths, H, Hk, dk, dv, dtype, dev, seed):
    import numpy as np
    T = int(sum(lengths))
    (q, k, v, g, b, _), _ = device_inputs(1, T, H, dk, dv, seed=seed, dtype=dtype, dev=dev)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    h0 = torch.randn(len(lengths), H, dk, dv, device=dev, generator=gen) * 0.05
    do = torch.randn(1, T, H, dv, device=dev, generator=gen).to(v.dtype)
    dhT = torch.randn(len(lengths), H, dk, dv, device=dev, generator=gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    return q, k, v, g, b, h0, do, dhT, cu


PACKED = [
    ([200, 1, 63, 64, 65, 0, 130], 2, 2, 128, 128, "bf16"),
    ([300, 77], 4, 2, 128, 64, "bf16"),
    ([33, 0, 70, 16], 2, 1, 32, 64, "fp32"),
    ([5, 129, 40], 3, 3, 64, 32, "fp32"),
    ([100, 0, 70], 2, 1, 256, 64, "bf16"),
]


@pytest.mark.parametrize("lengths,H,Hk,dk,dv,dtype", PACKED)
def test_packed_backward_equals_each_sequence_alone(cuda, lengths, H, Hk, dk, dv, dtype):
    """Every packed sequence gets, bit for bit, what the dense backward gives it
    alone on the same kernels.  Dense rows at bf16 dk = dv = 128 run their
    forward pass on the tensor-core scan, packed rows on the warp-level state
    kernel: the dense call is made on the latter too (GDN_BWD_FWDPASS=warp) for
    the bit comparison, and on its default path within the bf16 bar."""
    from gated_deltanet_jax_b200 import _lib
    q, k, v, g, b, h0, do, dhT, cu = _packed_problem(lengths, H, Hk, dk, dv, dtype, cuda,
                                                     seed=len(lengths) + dk)
    got = ops._chunk_backward(q, k, v, g, b, h0, do, dhT, cu)
    for s in range(len(lengths)):
        a0, a1 = int(cu[s]), int(cu[s + 1])
        sl = slice(a0, a1)
        args = (q[:, sl], k[:, sl], v[:, sl], g[:, sl], b[:, sl], h0[s:s + 1], do[:, sl],
                dhT[s:s + 1])
        with _lib.kernel_env("GDN_BWD_FWDPASS", "warp"):
            one = ops._chunk_backward(*args)
        for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta"), got[:5], one[:5]):
            assert torch.equal(a[:, sl], r), f"sequence {s}: {name}"
        assert torch.equal(got[5][s:s + 1], one[5]), f"sequence {s}: dh0"
        if a1 > a0:
            dflt = ops._chunk_backward(*args)
            for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), one, dflt):
                err = orc.rel_err(f64(a), f64(r))
                assert err <= TOL[dtype], f"sequence {s} {name}: rel error {err:.2e}"


@pytest.mark.parametrize("lengths,H,Hk,dk,dv,dtype", PACKED[:2] + PACKED[3:])
def test_packed_backward_against_oracle(cuda, lengths, H, Hk, dk, dv, dtype):
    q, k, v, g, b, h0, do, dhT, cu = _packed_problem(lengths, H, Hk, dk, dv, dtype, cuda,
                                                     seed=3 * len(lengths))
    got = ops._chunk_backward(q, k, v, g, b, h0, do, dhT, cu)
    rep = H // Hk
    hq, hk = orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep)
    hv, hg, hb, hh0, hdo, hdhT = f64(v), f64(g), f64(b), f64(h0), f64(do), f64(dhT)
    for s in range(len(lengths)):
        a0, a1 = int(cu[s]), int(cu[s + 1])
        sl = slice(a0, a1)
        if a1 == a0:
            torch.testing.assert_close(got[5][s], dhT[s])   # no tokens: dh0 = dhT
            continue
        ref = orc.chunk_exact_backward(hq[:, sl], hk[:, sl], hv[:, sl], hg[:, sl], hb[:, sl],
                                       hh0[s:s + 1], hdo[:, sl], hdhT[s:s + 1], 32)
        dq_r = ref[0].reshape(1, a1 - a0, Hk, rep, dk).sum(3)
        dk_r = ref[1].reshape(1, a1 - a0, Hk, rep, dk).sum(3)
        refs = (dq_r, dk_r) + tuple(ref[2:5])
        for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta"), got[:5], refs):
            err = orc.rel_err(f64(a[:, sl]), r)
            assert err <= TOL[dtype], f"sequence {s} {name}: rel error {err:.2e}"
        err = orc.rel_err(f64(got[5][s:s + 1]), ref[5])
        assert err <= TOL[dtype], f"sequence {s} dh0: rel error {err:.2e}"


def test_autograd_through_packed_chunk_op(cuda):
    lengths = [70, 0, 33, 64]
    q, k, v, g, b, h0, do, dhT, cu = _packed_problem(lengths, 2, 2, 32, 32, "fp32", cuda, seed=8)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, g, b, h0)]
    o, hT = ops.chunk_gated_delta_rule(*leaves[:5], initial_state=leaves[5],
                                       output_final_state=True, cu_seqlens=cu)
    ((o * do).sum() + (hT * dhT).sum()).backward()
    want = ops._chunk_backward(q, k, v, g, b, h0, do, dhT, cu)
    for t, r in zip(leaves, want):
        assert torch.equal(t.grad, r)
    o2, h2 = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True,
                                        cu_seqlens=cu)
    assert torch.equal(o.detach(), o2) and torch.equal(hT.detach(), h2)


# The per-chunk preparation at bf16, dk = dv = 128 on dense rows runs on the
# tcgen05 kernel (bf16 operands, fp32 accumulation); GDN_BWD_PREP=warp keeps
# the warp-level one (tf32 operands) for cross-checks.  Both against the
# oracle: partial last chunks, several rows, grouped q/k heads, state in/out.
@pytest.mark.parametrize("prep", ["tcgen05", "tcgen05-warp-fwdpass", "tcgen05-warp-revpass",
                                  "tcgen05-warp-grads", "warp"])
@pytest.mark.parametrize("B,T,H,Hk,with_h0,with_dhT", [(1, 64, 1, 1, False, False),
                                                       (2, 100, 3, 3, True, True),
                                                       (1, 300, 4, 2, True, False),
                                                       (3, 129, 2, 1, False, True)])
def test_backward_preparation_forms_against_oracle(cuda, prep, B, T, H, Hk, with_h0, with_dhT):
    from gated_deltanet_jax_b200 import _lib
    dk = dv = 128
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=T + H, dtype="bf16", dev=cuda,
                                              h0_std=0.05 if with_h0 else None)
    rep = H // Hk
    if rep > 1:   # q/k with Hk heads; the oracle sees them repeated
        q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
        host = list(host)
        host[0] = f64(q.float().repeat_interleave(rep, 2))
        host[1] = f64(k.float().repeat_interleave(rep, 2))
    gen = torch.Generator(device=cuda).manual_seed(T)
    do = torch.randn(B, T, H, dv, device=cuda, generator=gen).bfloat16()
    dhT = torch.randn(B, H, dk, dv, device=cuda, generator=gen) if with_dhT else None
    with _lib.kernel_env("GDN_BWD_PREP", "warp" if prep == "warp" else None), \
            _lib.kernel_env("GDN_BWD_FWDPASS", "warp" if prep.endswith("fwdpass") else None), \
            _lib.kernel_env("GDN_BWD_REVPASS", "warp" if prep.endswith("revpass") else None), \
            _lib.kernel_env("GDN_BWD_GRADS", "warp" if prep.endswith("grads") else None):
        got = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    ref = orc.chunk_exact_backward(*host[:5], host[5], f64(do), None if dhT is None else f64(dhT),
                                   64)
    if rep > 1:   # the gradients of the shared q/k heads sum over each group
        ref = list(ref)
        for idx in (0, 1):
            r = ref[idx]
            ref[idx] = r.reshape(B, T, Hk, rep, dk).sum(3)
    _check(got, ref, "bf16", with_h0=with_h0)
    assert _lib.load().gdn_device_error(1) == 0


def test_backward_preparation_forms_agree_at_size(cuda):
    """B=2 T=2048 H=8 dk=dv=128 bf16: the tcgen05 preparation's gradients
    against the warp-level one's (tf32 operands), within the bf16 bar; and
    repeated calls of the tcgen05 form are bit-identical."""
    from gated_deltanet_jax_b200 import _lib
    B, T, H, dk, dv = 2, 2048, 8, 128, 128
    (q, k, v, g, b, h0), _ = device_inputs(B, T, H, dk, dv, seed=21, dtype="bf16", dev=cuda,
                                           h0_std=0.05)
    gen = torch.Generator(device=cuda).manual_seed(22)
    do = torch.randn(B, T, H, dv, device=cuda, generator=gen).bfloat16()
    dhT = torch.randn(B, H, dk, dv, device=cuda, generator=gen)
    tc = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    tc2 = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    with _lib.kernel_env("GDN_BWD_PREP", "warp"), _lib.kernel_env("GDN_BWD_GRADS", "warp"):
        wp = ops._chunk_backward(q, k, v, g, b, h0, do, dhT)
    for n, a, a2, r in zip(["dq", "dk", "dv", "dg", "dbeta", "dh0"], tc, tc2, wp):
        assert torch.equal(a, a2), n
        err = orc.rel_err(f64(a), f64(r))
        assert err <= TOL["bf16"], f"{n}: rel error {err:.2e}"
