"""GPU parity of the chunked forward (gdn_chunk_fwd) against the oracle, the
reference's own outputs (golden.npz) and the recurrent kernel."""

import numpy as np
import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, device_inputs_fast, f64, to_dev

pytestmark = pytest.mark.gpu

GOLDEN_CASES = ["c0", "h0", "tail", "layer", "lm", "h1", "d256"]


def _golden_args(c, dev):
    args = [to_dev(c[x], torch.float32, dev) for x in ("q", "k", "v", "g", "beta")]
    h0 = to_dev(c["h0"], torch.float32, dev) if "h0" in c else None
    return args, h0


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_exact_matches_reference_recurrence(golden, cuda, name):
    """Exact semantics reproduce the reference's recurrent kernel output."""
    c = golden[name]
    args, _ = _golden_args(c, cuda)
    o, hT = ops.chunk_gated_delta_rule(*args, chunk_size=int(c["shape"][5]))
    assert hT is None
    assert_close(f64(o), c["o_recurrent"], "fp32", name)


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_reference_semantics_match_reference_chunk_outputs(golden, cuda, name):
    """semantics='reference' reproduces the reference chunk path as written
    (ops.py:299-346), output permutation and final state included."""
    c = golden[name]
    args, h0 = _golden_args(c, cuda)
    o, hT = ops.chunk_gated_delta_rule(*args, initial_state=h0, output_final_state=True,
                                       chunk_size=int(c["shape"][5]), semantics="reference")
    assert_close(f64(o), c["o_chunk"], "fp32", name + " o")
    assert_close(f64(hT), c["h_chunk"], "fp32", name + " state")


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("dk,dv,C,T", [
    (16, 16, 16, 33), (16, 32, 64, 32), (32, 64, 64, 64), (32, 48, 32, 100),
    (64, 64, 64, 256), (64, 64, 16, 70), (128, 128, 64, 200), (128, 64, 32, 129),
    (256, 512, 64, 130), (256, 32, 16, 40), (128, 128, 64, 1),
])
def test_against_oracle(cuda, dtype, dk, dv, C, T):
    (q, k, v, g, b, h0), host = device_inputs(2, T, 2, dk, dv, seed=dk * 7 + T, dtype=dtype,
                                              dev=cuda, h0_std=0.02)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                       output_final_state=True, chunk_size=C)
    ro, rh = orc.chunk_exact(*host, chunk_size=C)
    assert o.dtype == q.dtype
    assert_close(f64(o), ro, dtype, "o")
    assert_close(f64(hT), rh, dtype, "state")


def test_config0_fp32(cuda):
    """Config 0: B=1 T=256 H=2 dk=dv=64 chunk=64, fp32, zero initial state."""
    (q, k, v, g, b, _), host = device_inputs(1, 256, 2, 64, 64, seed=0, dtype="fp32", dev=cuda)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, output_final_state=True)
    ro, rh = orc.recurrent_ref(*host[:5])
    assert_close(f64(o), ro, "fp32", "o")
    assert_close(f64(hT), rh, "fp32", "state")


def test_split_resume_equals_one_shot(cuda):
    (q, k, v, g, b, h0), _ = device_inputs(2, 300, 3, 64, 64, seed=9, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    o, h = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    s = 137
    oa, ha = ops.chunk_gated_delta_rule(q[:, :s], k[:, :s], v[:, :s], g[:, :s], b[:, :s],
                                        initial_state=h0, output_final_state=True)
    ob, hb = ops.chunk_gated_delta_rule(q[:, s:], k[:, s:], v[:, s:], g[:, s:], b[:, s:],
                                        initial_state=ha, output_final_state=True)
    assert_close(f64(torch.cat([oa, ob], 1)), f64(o), "bf16", "o")
    assert_close(f64(hb), f64(h), "bf16", "state")


def test_chunk_equals_recurrent_kernel(cuda):
    """The tcgen05 chunk kernel against the token-by-token recurrent kernel
    (GDN_RECURRENT_KERNEL=token: whole sequences otherwise go to the chunk
    kernel too)."""
    q, k, v, g, b, h0 = device_inputs_fast(2, 1000, 4, 128, 128, seed=4, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    oc, hc = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    orr, hr = _with_env("GDN_RECURRENT_KERNEL", "token", lambda: ops.fused_recurrent_gated_delta_rule(
        q, k, v, g, b, initial_state=h0, output_final_state=True))
    assert_close(f64(oc), f64(orr), "bf16", "o")
    assert_close(f64(hc), f64(hr), "bf16", "state")
    # and the recurrent op's own whole-sequence path (the one-launch chunk
    # kernel, which needs no workspace), in place
    S = h0.clone()
    o2, _ = ops.fused_recurrent_gated_delta_rule(q, k, v, g, b, initial_state=S,
                                                 final_state_out=S)
    of, hf = _with_kernel("fused", lambda: ops.chunk_gated_delta_rule(
        q, k, v, g, b, initial_state=h0, output_final_state=True))
    assert torch.equal(o2, of) and torch.equal(S, hf)
    assert_close(f64(o2), f64(orr), "bf16", "o (whole-sequence recurrent op)")


def test_prefill_config_full_size(cuda):
    """Config 2: B=4 T=4096 H=16 dk=dv=128 chunk=64, bf16 in, fp32 state.

    Sampled (b, h) sequences against the float64 recurrence over all 4096
    tokens; the whole output for finiteness."""
    B, T, H, dk, dv = 4, 4096, 16, 128, 128
    q, k, v, g, b, _ = device_inputs_fast(B, T, H, dk, dv, seed=2, dtype="bf16", dev=cuda)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, output_final_state=True)
    assert torch.isfinite(o.float()).all() and torch.isfinite(hT).all()
    picks = [(0, 0), (1, 9), (3, 15)]
    bi = [p[0] for p in picks]
    hi = [p[1] for p in picks]
    sel = lambda t: f64(t[bi, :, hi][:, :, None])  # noqa: E731
    ro, rh = orc.recurrent_ref(sel(q), sel(k), sel(v), sel(g), sel(b))
    assert_close(f64(o[bi, :, hi]), ro[:, :, 0], "bf16", "o")
    assert_close(f64(hT[bi, hi]), rh[:, 0], "bf16", "state")
    assert np.isfinite(ro).all()


def _with_env(name, value, fn):
    with _lib.kernel_env(name, value):
        return fn()


def _with_kernel(kind, fn):
    return _with_env("GDN_CHUNK_KERNEL", kind, fn)


@pytest.mark.parametrize("dv", [64, 128, 192, 256])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 300])
@pytest.mark.parametrize("with_h0", [False, True])
def test_tensor_core_path_against_oracle(cuda, dv, T, with_h0):
    """bf16, dk=128, chunk=64: the tcgen05 kernel's shapes, partial chunks included."""
    (q, k, v, g, b, h0), host = device_inputs(2, T, 3, 128, dv, seed=dv + T, dtype="bf16",
                                              dev=cuda, h0_std=0.05)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0 if with_h0 else None,
                                       output_final_state=True)
    ro, rh = orc.chunk_exact(*host[:5], host[5] if with_h0 else None, 64)
    assert_close(f64(o), ro, "bf16", "o")
    assert_close(f64(hT), rh, "bf16", "state")


@pytest.mark.parametrize("B,T,H,dv", [(1, 640, 2, 128), (3, 257, 5, 64), (2, 129, 1, 512)])
def test_tensor_core_matches_cuda_core_kernel(cuda, B, T, H, dv):
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=T, dtype="bf16", dev=cuda,
                                           h0_std=0.02)

    def run():
        return ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                          output_final_state=True)

    o_tc, h_tc = run()
    o_cc, h_cc = _with_kernel("simt", run)
    assert_close(f64(o_tc), f64(o_cc), "bf16", "o")
    assert_close(f64(h_tc), f64(h_cc), "bf16", "state")


@pytest.mark.parametrize("B,T,H,dv", [(2, 700, 3, 128), (1, 193, 2, 256), (1, 64, 1, 128),
                                      (1, 130, 2, 128), (3, 1, 2, 128), (4, 300, 16, 128)])
def test_paired_tiles_match_unpaired(cuda, B, T, H, dv):
    """The one-launch kernel's column-tile pairs that share the per-chunk
    preparation (clusters of two CTAs, each preparing every other chunk for
    both) give bit-identical results to tiles that each prepare every chunk
    themselves."""
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=T + dv, dtype="bf16", dev=cuda,
                                           h0_std=0.02)

    def run():
        return ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                          output_final_state=True)

    with _lib.kernel_env("GDN_CHUNK_KERNEL", "fused"):
        o_p, h_p = _with_env("GDN_CHUNK_TC_PAIR", "1", run)
        o_s, h_s = _with_env("GDN_CHUNK_TC_PAIR", "0", run)
    assert torch.equal(o_p, o_s)
    assert torch.equal(h_p, h_s)


def test_kernels_report_sm100(cuda):
    """The CUDA runtime reports the library's kernels as built for compute
    capability 10.0 (sm_100a), on the device itself."""
    assert _lib.load().gdn_binary_version() == 100


def test_no_device_error_recorded_chunk(cuda):
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_device_error(1) == 0


@pytest.mark.parametrize("gscale,gshift", [(8.0, 0.0), (0.3, 0.25), (0.0, 0.0)])
def test_tensor_core_gate_ranges(cuda, gscale, gshift):
    """Steep decays (spans > 40 inside 16 tokens, the kernel's direct-exponent
    path), gates of both signs, and no decay at all, against the oracle."""
    (q, k, v, g, b, h0), host = device_inputs(2, 200, 2, 128, 128, seed=17, dtype="bf16",
                                              dev=cuda, h0_std=0.05)
    g = (g * gscale + gshift).contiguous()
    host[3] = f64(g)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    ro, rh = orc.chunk_exact(*host[:5], host[5], 64)
    assert np.isfinite(ro).all()
    assert_close(f64(o), ro, "bf16", "o")
    assert_close(f64(hT), rh, "bf16", "state")


@pytest.mark.parametrize("dv", [64, 512])
@pytest.mark.parametrize("T", [1, 65, 300])
@pytest.mark.parametrize("Hk", [2, 1])
def test_tensor_core_dk256_against_oracle(cuda, dv, T, Hk):
    """bf16, dk=256 (the head_dim of the reference's default configuration):
    the tcgen05 kernel with one K/Q stage and two state rows per chain thread,
    partial chunks and grouped q/k heads included."""
    H = 2
    (q, k, v, g, b, h0), host = device_inputs(2, T, H, 256, dv, seed=dv + T + Hk, dtype="bf16",
                                              dev=cuda, h0_std=0.05)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    ro, rh = orc.chunk_exact(orc.repeat_heads(f64(q), rep), orc.repeat_heads(f64(k), rep),
                             *host[2:5], host[5], 64)
    assert_close(f64(o), ro, "bf16", "o")
    assert_close(f64(hT), rh, "bf16", "state")


def test_tensor_core_dk256_matches_cuda_core_kernel(cuda):
    """The reference configuration's head dims (dk=256, dv=512) on both kernels."""
    q, k, v, g, b, h0 = device_inputs_fast(2, 300, 3, 256, 512, seed=5, dtype="bf16", dev=cuda,
                                           h0_std=0.02)

    def run():
        return ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                          output_final_state=True)

    o_tc, h_tc = run()
    o_cc, h_cc = _with_kernel("simt", run)
    assert_close(f64(o_tc), f64(o_cc), "bf16", "o")
    assert_close(f64(h_tc), f64(h_cc), "bf16", "state")


def test_tensor_core_dk256_packed_sequences_equal_each_alone(cuda):
    lens = (100, 0, 129, 7)
    T, H = sum(lens), 2
    q, k, v, g, b, _ = device_inputs_fast(1, T, H, 256, 128, seed=3, dtype="bf16", dev=cuda)
    gen = torch.Generator(device=cuda).manual_seed(4)
    S = torch.randn(len(lens), H, 256, 128, device=cuda, generator=gen) * 0.02
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=cuda)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=S, output_final_state=True,
                                       cu_seqlens=cu)
    for s, (t0, t1) in enumerate(zip(cu.tolist(), cu.tolist()[1:])):
        part = [t[:, t0:t1].contiguous() for t in (q, k, v, g, b)]
        os_, hs = ops.chunk_gated_delta_rule(*part, initial_state=S[s:s + 1],
                                             output_final_state=True)
        assert torch.equal(o[:, t0:t1], os_), s
        assert torch.equal(hT[s:s + 1], hs), s


def test_tensor_core_dk256_steep_gates(cuda):
    (q, k, v, g, b, h0), host = device_inputs(1, 200, 2, 256, 128, seed=23, dtype="bf16",
                                              dev=cuda, h0_std=0.05)
    g = (g * 8.0).contiguous()
    host[3] = f64(g)
    o, hT = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    ro, rh = orc.chunk_exact(*host[:5], host[5], 64)
    assert_close(f64(o), ro, "bf16", "o")
    assert_close(f64(hT), rh, "bf16", "state")


@pytest.mark.parametrize("dtype,B,T,H,dk,dv", [
    ("fp32", 2, 200, 3, 128, 128), ("fp32", 1, 130, 2, 256, 512), ("fp32", 3, 65, 2, 16, 32),
    ("fp32", 1, 1, 2, 64, 96), ("bf16", 2, 150, 2, 64, 64), ("bf16", 1, 100, 3, 128, 96),
])
def test_warp_tensor_core_forward_matches_cuda_core_kernel(cuda, dtype, B, T, H, dk, dv):
    """fp32 inputs (and bf16 shapes outside the tcgen05 kernel) run on the
    warp-level tensor-core kernels with a workspace; the CUDA-core kernel is
    the cross-check, within the fp32 / bf16 bars."""
    (q, k, v, g, b, h0), host = device_inputs(B, T, H, dk, dv, seed=T + dk, dtype=dtype,
                                              dev=cuda, h0_std=0.05)
    from gated_deltanet_jax_b200 import _lib
    assert _lib.load().gdn_chunk_workspace_bytes(B, T, H, dk, dv, 64,
                                                 ops._DTYPES[q.dtype], 0) > 0

    def run():
        return ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                          output_final_state=True)

    o_w, h_w = run()
    o_c, h_c = _with_kernel("simt", run)
    assert_close(f64(o_w), f64(o_c), dtype, "o")
    assert_close(f64(h_w), f64(h_c), dtype, "state")
    ro, rh = orc.chunk_exact(*host, chunk_size=64)
    assert_close(f64(o_w), ro, dtype, "o vs oracle")
    assert_close(f64(h_w), rh, dtype, "state vs oracle")


@pytest.mark.parametrize("B,T,H,Hk,dv", [(2, 700, 3, 3, 128), (1, 193, 2, 1, 256), (3, 1, 2, 2, 64),
                                         (1, 64, 4, 2, 192), (4, 300, 16, 16, 128)])
def test_two_launch_matches_one_launch(cuda, B, T, H, Hk, dv):
    """The two-launch form (preparation over every chunk-head, then the scan)
    against the one-launch kernel: the same recurrence, rounded at different
    points, so within the bf16 bar of each other (and of the oracle)."""
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=T + dv + Hk, dtype="bf16",
                                           dev=cuda, h0_std=0.02)
    q, k = q[:, :, ::H // Hk].contiguous(), k[:, :, ::H // Hk].contiguous()

    def run():
        return ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                          output_final_state=True)

    from gated_deltanet_jax_b200 import _lib as lib_mod
    assert lib_mod.load().gdn_chunk_workspace_bytes(B, T, H, 128, dv, 64, 1, 0) > 0
    o2, h2 = run()
    o1, h1 = _with_kernel("fused", run)
    assert_close(f64(o2), f64(o1), "bf16", "o")
    assert_close(f64(h2), f64(h1), "bf16", "state")
    assert torch.isfinite(o2.float()).all() and torch.isfinite(h2).all()


def test_two_launch_in_place_and_repeatable(cuda):
    """h0 == hT (in-place state) gives what separate buffers give, and a
    repeated call is bit-identical (no atomics, fixed reduction order)."""
    q, k, v, g, b, h0 = device_inputs_fast(2, 333, 4, 128, 128, seed=31, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    o1, h1 = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    o2, h2 = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    S = h0.clone()
    o3, _ = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=S, final_state_out=S)
    assert torch.equal(o1, o2) and torch.equal(h1, h2)
    assert torch.equal(o1, o3) and torch.equal(h1, S)


def test_two_launch_workspace_optional(cuda):
    """gdn_chunk_fwd at the two-launch shapes without a workspace (or with a
    short one) runs the one-launch kernel: bit-identical to forcing it."""
    import ctypes
    from gated_deltanet_jax_b200 import _lib as lib_mod
    lib = lib_mod.load()
    B, T, H, dv = 2, 200, 4, 128
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=5, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    need = lib.gdn_chunk_workspace_bytes(B, T, H, 128, dv, 64, lib_mod.GDN_DTYPE_BF16, 0)
    assert need > 0
    short = torch.empty(need // 2, dtype=torch.uint8, device=cuda)

    def call(ws, ws_bytes):
        o = torch.empty_like(v)
        hT = torch.empty_like(h0)
        rc = lib.gdn_chunk_fwd(ptr(q), ptr(k), ptr(v), ptr(g), ptr(b), ptr(h0), ptr(o), ptr(hT),
                               B, T, H, 128, dv, 64, lib_mod.GDN_DTYPE_BF16, 0, ptr(ws), ws_bytes,
                               ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
        lib_mod.check(rc, "gdn_chunk_fwd")
        torch.cuda.synchronize(cuda)
        return o, hT

    o0, h_0 = call(None, 0)
    o1, h_1 = call(short, short.numel())
    o2, h_2 = _with_kernel("fused", lambda: call(None, 0))
    assert torch.equal(o0, o2) and torch.equal(h_0, h_2)
    assert torch.equal(o1, o2) and torch.equal(h_1, h_2)
    assert lib.gdn_device_error(0) == 0
