"""CPU tests of the oracle: pinned to the reference's own outputs (golden.npz),
and self-consistent across its chunked, recurrent and two-pass forms."""

import numpy as np
import pytest

from oracle import gdn_oracle as orc


def _f64(case, key):
    return case[key].astype(np.float64)


def test_golden_cases_present(golden):
    assert set(golden) >= {"c0", "h0", "tail", "layer", "lm", "h1"}
    B, T, H, dk, dv, C = golden["c0"]["shape"]
    assert (B, T, H, dk, dv, C) == (1, 256, 2, 64, 64, 64)


@pytest.mark.parametrize("name", ["c0", "h0", "tail", "layer", "lm", "h1", "d256"])
def test_recurrent_matches_reference_kernel(golden, name):
    """recurrent_ref == the reference Pallas kernel (ops.py:162-184), zero state."""
    c = golden[name]
    o, _ = orc.recurrent_ref(*(_f64(c, x) for x in ("q", "k", "v", "g", "beta")))
    assert orc.rel_err(o, c["o_recurrent"]) < 1e-6


@pytest.mark.parametrize("name", ["c0", "h0", "tail", "layer", "lm", "h1", "d256"])
def test_literal_chunk_matches_reference_chunk(golden, name):
    """chunk_reference_literal == the reference chunk path (ops.py:299-346)."""
    c = golden[name]
    C = int(c["shape"][5])
    h0 = _f64(c, "h0") if "h0" in c else None
    o, h = orc.chunk_reference_literal(*(_f64(c, x) for x in ("q", "k", "v", "g", "beta")),
                                       initial_state=h0, output_final_state=True, chunk_size=C)
    assert orc.rel_err(o, c["o_chunk"]) < 1e-6
    assert orc.rel_err(h, c["h_chunk"]) < 1e-6


@pytest.mark.parametrize("name", ["c0", "h0", "tail", "layer", "lm", "h1", "d256"])
def test_exact_chunk_matches_reference_recurrence(golden, name):
    """The exact chunked form reproduces the reference recurrent kernel."""
    c = golden[name]
    C = int(c["shape"][5])
    o, _ = orc.chunk_exact(*(_f64(c, x) for x in ("q", "k", "v", "g", "beta")), chunk_size=C)
    assert orc.rel_err(o, c["o_recurrent"]) < 1e-6


def test_reference_chunk_deviates_from_recurrence(golden):
    """Documented deviation: the reference chunk path is not the recurrence."""
    c = golden["c0"]
    assert orc.rel_err(c["o_chunk"], c["o_recurrent"]) > 0.5


def test_literal_output_permutation(golden):
    """The reference output reshape (ops.py:342) is a pure (token, head)
    permutation of per-position outputs: undoing it on a deviation-free
    input (H=1 identity, else a permuted comparison) is consistent."""
    for name in ("c0", "layer", "tail"):
        c = golden[name]
        B, T, H, dk, dv, C = (int(x) for x in c["shape"])
        src_t, src_h = orc.literal_output_permutation(T, H, C)
        # a bijection onto the valid and padded (token, head) positions
        pairs = set(zip(src_t.ravel().tolist(), src_h.ravel().tolist()))
        assert len(pairs) == T * H
        if H == 1:
            assert np.array_equal(src_t[:, 0], np.arange(T))


@pytest.mark.parametrize("shape", [(2, 130, 3, 16, 32, 32), (1, 64, 2, 32, 16, 16),
                                   (1, 200, 2, 64, 64, 64), (1, 1, 1, 16, 16, 64)])
def test_chunk_exact_equals_recurrent(shape):
    B, T, H, dk, dv, C = shape
    q, k, v, g, beta, h0 = orc.make_inputs(B, T, H, dk, dv, seed=7, h0_std=0.02)
    o1, h1 = orc.recurrent_ref(q, k, v, g, beta, h0)
    o2, h2 = orc.chunk_exact(q, k, v, g, beta, h0, C)
    assert orc.max_abs_err(o1, o2) < 1e-12
    assert orc.max_abs_err(h1, h2) < 1e-12


@pytest.mark.parametrize("parts", [1, 2, 3, 5])
def test_two_pass_split_equals_recurrent(parts):
    q, k, v, g, beta, h0 = orc.make_inputs(1, 300, 2, 16, 32, seed=11, h0_std=0.02)
    o1, h1 = orc.recurrent_ref(q, k, v, g, beta, h0)
    o2, h2 = orc.two_pass_sp(q, k, v, g, beta, h0, parts=parts, chunk_size=32)
    assert orc.max_abs_err(o1, o2) < 1e-12
    assert orc.max_abs_err(h1, h2) < 1e-12


def test_segment_transition_is_affine_map():
    q, k, v, g, beta, h0 = orc.make_inputs(2, 40, 2, 16, 24, seed=3, h0_std=0.1)
    _, S = orc.recurrent_ref(q, k, v, g, beta, None)
    M = orc.segment_transition(k, g, beta)
    _, hT = orc.recurrent_ref(q, k, v, g, beta, h0)
    assert orc.max_abs_err(hT, M @ h0 + S) < 1e-12


def test_split_resume_equals_one_shot():
    q, k, v, g, beta, h0 = orc.make_inputs(1, 150, 2, 32, 32, seed=5, h0_std=0.02)
    o, h = orc.chunk_exact(q, k, v, g, beta, h0, 64)
    oa, ha = orc.chunk_exact(q[:, :77], k[:, :77], v[:, :77], g[:, :77], beta[:, :77], h0, 64)
    ob, hb = orc.chunk_exact(q[:, 77:], k[:, 77:], v[:, 77:], g[:, 77:], beta[:, 77:], ha, 64)
    assert orc.max_abs_err(np.concatenate([oa, ob], 1), o) < 1e-12
    assert orc.max_abs_err(hb, h) < 1e-12


def test_round_bf16():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3e-3, 0.0, 65504.0])
    r = orc.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == 1.015625              # tie rounds up to even mantissa
    assert abs(r[3] - x[3]) / abs(x[3]) < 2 ** -8
    assert r[4] == 0.0


def test_tolerance_rules():
    ref = np.array([1.0, -2.0, 3.0])
    assert orc.within_tolerance(ref + 1e-3, ref, "fp32")[0]
    assert not orc.within_tolerance(ref + 3e-3, ref, "fp32")[0]
    assert orc.within_tolerance(ref + 0.05, ref, "bf16")[0]     # 0.05 / 3 < 2e-2
    assert not orc.within_tolerance(ref + 0.07, ref, "bf16")[0]


def test_work_accounting():
    from gated_deltanet_jax_b200 import roofline as rl
    assert rl.flops_chunk_per_token_head(128, 128, 64) == 180224
    assert rl.flops_chunk_bwd_per_token_head(128, 128, 64) == 507904
    assert rl.bytes_chunk_per_token_head(128, 128) == 1032
    assert rl.bytes_recurrent_per_head_step(128, 128) == 132104


def test_repeat_heads_matches_layer_expansion():
    """repeat_heads is the layer's jnp.repeat(axis=2): value head h uses q/k head h // rep."""
    x = np.arange(2 * 3 * 2 * 4, dtype=np.float64).reshape(2, 3, 2, 4)
    r = orc.repeat_heads(x, 3)
    assert r.shape == (2, 3, 6, 4)
    for h in range(6):
        assert np.array_equal(r[:, :, h], x[:, :, h // 3])


def test_grouped_heads_equal_repeated_recurrence():
    """The grouped-head problem is the plain problem on repeated q, k (oracle level)."""
    q, k, v, g, beta, h0 = orc.make_inputs(1, 40, 6, 16, 24, seed=8, h0_std=0.05)
    qg, kg = q[:, :, ::3].copy(), k[:, :, ::3].copy()   # 2 q/k heads for 6 value heads
    o1, h1 = orc.recurrent_ref(orc.repeat_heads(qg, 3), orc.repeat_heads(kg, 3), v, g, beta, h0)
    o2, h2 = orc.chunk_exact(orc.repeat_heads(qg, 3), orc.repeat_heads(kg, 3), v, g, beta, h0, 16)
    assert orc.max_abs_err(o1, o2) < 1e-12 and orc.max_abs_err(h1, h2) < 1e-12


def _torch_recurrence(q, k, v, g, beta, h0):
    import torch
    h, outs = h0, []
    for t in range(k.shape[1]):
        h = h * torch.exp(g[:, t])[:, :, None, None]
        proj = torch.einsum('bhk,bhkv->bhv', k[:, t], h)
        vn = (v[:, t] - proj) * beta[:, t][:, :, None]
        h = h + k[:, t][:, :, :, None] * vn[:, :, None, :]
        outs.append(torch.einsum('bhkv,bhk->bhv', h, q[:, t]))
    return torch.stack(outs, 1), h


@pytest.mark.parametrize("shape", [(1, 40, 2, 8, 6, 16), (2, 33, 1, 4, 5, 8), (1, 64, 1, 16, 16, 64),
                                   (1, 5, 2, 4, 4, 16)])
def test_backward_matches_autograd_of_recurrence(shape):
    """chunk_exact_backward == torch autograd (float64) through the token recurrence."""
    import torch
    B, T, H, dk, dv, C = shape
    q, k, v, g, beta, h0 = orc.make_inputs(B, T, H, dk, dv, seed=T, h0_std=0.1)
    rng = np.random.default_rng(1)
    do = rng.standard_normal((B, T, H, dv))
    dhT = rng.standard_normal((B, H, dk, dv))
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v, g, beta, h0)]
    o, hT = _torch_recurrence(*ts)
    ((o * torch.tensor(do)).sum() + (hT * torch.tensor(dhT)).sum()).backward()
    got = orc.chunk_exact_backward(q, k, v, g, beta, h0, do, dhT, C)
    for a, t in zip(got, ts):
        ref = t.grad.numpy()
        assert np.abs(a - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max())


def test_layer_gates_and_norm_formulas():
    """model.py:136-139 and :41-53 on hand-checked values."""
    A_log = np.log(np.array([1.0, 2.0]))
    g, beta = orc.layer_gates(np.array([[0.0, 30.0]]), np.array([[0.0, 2.0]]), A_log,
                              np.zeros(2))
    np.testing.assert_allclose(g, [[-np.log(2.0), -2.0 * (30.0 + np.log1p(np.exp(-30.0)))]])
    np.testing.assert_allclose(beta, [[0.5, 1.0 / (1.0 + np.exp(-2.0))]])
    o = np.array([[3.0, -4.0]])
    y = orc.rms_norm_gated(o, np.array([1.0, 2.0]), eps=0.0)
    np.testing.assert_allclose(y, [[3.0 / np.sqrt(12.5), -8.0 / np.sqrt(12.5)]])
    yg = orc.rms_norm_gated(o, np.ones(2), gate=np.array([[0.0, 1.0]]), eps=0.0)
    np.testing.assert_allclose(yg, [[0.0, -4.0 / np.sqrt(12.5) / (1.0 + np.exp(-1.0))]])


@pytest.mark.parametrize("chunked", [False, True])
def test_oracle_linear_in_values_and_state(chunked):
    """For fixed q, k, g, beta the delta rule is linear in (v, initial state):
    the property the full-size GPU tests check the kernels against."""
    rng = np.random.default_rng(11)
    q, k, v1, g, beta, h1 = orc.make_inputs(2, 90, 3, 32, 24, seed=12, h0_std=0.05)
    v2 = rng.standard_normal(v1.shape)
    h2 = rng.standard_normal(h1.shape) * 0.05

    def run(v, h0):
        if chunked:
            return orc.chunk_exact(q, k, v, g, beta, h0, 32)
        return orc.recurrent_ref(q, k, v, g, beta, h0)

    o1, s1 = run(v1, h1)
    o2, s2 = run(v2, h2)
    o3, s3 = run(v1 + 2 * v2, h1 + 2 * h2)
    np.testing.assert_allclose(o3, o1 + 2 * o2, rtol=0, atol=1e-10)
    np.testing.assert_allclose(s3, s1 + 2 * s2, rtol=0, atol=1e-10)


@pytest.mark.parametrize("K", [1, 2, 4])
@pytest.mark.parametrize("activation", ["silu", None])
def test_short_conv_matches_grouped_conv1d(K, activation):
    """The oracle's ShortConvolution (model.py:15-40) against torch's grouped
    conv1d with the same definition: feature_group_count = C (depthwise),
    left padding K - 1, cross-correlation (no kernel flip), no bias."""
    import torch
    rng = np.random.default_rng(K)
    B, T, C = 2, 13, 24
    x = rng.standard_normal((B, T, C))
    w = rng.standard_normal((K, C))
    y, st = orc.short_conv(x, w, activation)
    xt = torch.tensor(x).permute(0, 2, 1)                       # [B, C, T]
    wt = torch.tensor(w).t().reshape(C, 1, K)                   # [C, 1, K]
    ref = torch.nn.functional.conv1d(torch.nn.functional.pad(xt, (K - 1, 0)), wt, groups=C)
    if activation == "silu":
        ref = torch.nn.functional.silu(ref)
    np.testing.assert_allclose(y, ref.permute(0, 2, 1).numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_array_equal(st, x[:, T - (K - 1):T] if K > 1 else x[:, :0])


def test_short_conv_state_carries_across_calls():
    """A sequence convolved in two calls, the first call's final state passed
    to the second, equals one call over the whole sequence (decode
    continuity); short calls (T < K - 1) keep part of the incoming state."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 20, 16))
    w = rng.standard_normal((4, 16))
    y, st = orc.short_conv(x, w)
    for cut in (1, 2, 7, 19):
        y1, s1 = orc.short_conv(x[:, :cut], w)
        y2, s2 = orc.short_conv(x[:, cut:], w, state=s1)
        np.testing.assert_allclose(np.concatenate([y1, y2], 1), y, rtol=1e-12, atol=1e-12)
        np.testing.assert_array_equal(s2, st)
    # one token at a time
    s, ys = None, []
    for t in range(20):
        yt, s = orc.short_conv(x[:, t:t + 1], w, state=s)
        ys.append(yt)
    np.testing.assert_allclose(np.concatenate(ys, 1), y, rtol=1e-12, atol=1e-12)
