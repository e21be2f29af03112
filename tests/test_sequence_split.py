"""Sequence-split forward: host logic on CPU (oracle as the per-segment
function, gloo ranks for the distributed hand-off) and the CUDA path on GPU."""

import datetime
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gated_deltanet_jax_b200 import sequence_parallel as sp
from oracle import gdn_oracle as orc


def oracle_segment_fn(chunk_size=16):
    """Per-segment chunked forward by the float64 oracle on CPU tensors."""
    def fn(q, k, v, g, beta, h0):
        arrs = [x.detach().cpu().numpy().astype(np.float64) for x in (q, k, v, g, beta)]
        h = None if h0 is None else h0.detach().cpu().numpy().astype(np.float64)
        o, hT = orc.chunk_exact(*arrs, h, chunk_size)
        return torch.from_numpy(o), torch.from_numpy(hT)
    return fn


def _t(x):
    return torch.from_numpy(np.asarray(x, np.float64))


@pytest.mark.parametrize("B,T,parts", [(1, 200, 4), (2, 96, 3), (1, 50, 2), (1, 16, 4)])
def test_split_on_one_device_matches_oracle(B, T, parts):
    q, k, v, g, beta, h0 = orc.make_inputs(B, T, 2, 16, 24, seed=T, h0_std=0.05)
    o, hT = sp.chunk_gated_delta_rule_split(*(_t(x) for x in (q, k, v, g, beta)),
                                            initial_state=_t(h0), output_final_state=True,
                                            chunk_size=16, parts=parts,
                                            segment_fn=oracle_segment_fn(16))
    ro, rh = orc.recurrent_ref(q, k, v, g, beta, h0)
    assert orc.max_abs_err(o.numpy(), ro) < 1e-10
    assert orc.max_abs_err(hT.numpy(), rh) < 1e-10


def test_segment_summary_is_affine_map():
    q, k, v, g, beta, h0 = orc.make_inputs(1, 40, 2, 16, 16, seed=1, h0_std=0.1)
    S, M = sp.segment_summary(*(_t(x) for x in (q, k, v, g, beta)), oracle_segment_fn(16))
    _, hT = orc.recurrent_ref(q, k, v, g, beta, h0)
    assert orc.max_abs_err((M @ _t(h0) + S).numpy(), hT) < 1e-10


def _sp_worker(rank, world, port, T, results, local_parts=1, seg=None, auto_by_length=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if auto_by_length:
            # local_parts=None on CPU tensors: a per-rank choice that grows with the
            # rank's own T (as the CUDA choice does), so a shorter last rank would
            # pick fewer parts than the others without the agreement step
            sp.auto_local_parts = lambda B, T_, H, dv, C, dev: max(1, T_ // (2 * C))
        q, k, v, g, beta, h0 = orc.make_inputs(1, T, 2, 16, 16, seed=5, h0_std=0.05)
        seg = seg or T // world
        sl = slice(rank * seg, (rank + 1) * seg if rank < world - 1 else T)
        args = [_t(x[:, sl]) for x in (q, k, v, g, beta)]
        o, hT = sp.chunk_gated_delta_rule_sp(*args, initial_state=_t(h0), output_final_state=True,
                                             chunk_size=16, segment_fn=oracle_segment_fn(16),
                                             local_parts=local_parts)
        ro, rh = orc.recurrent_ref(q, k, v, g, beta, h0)
        results[rank] = (orc.max_abs_err(o.numpy(), ro[:, sl]), orc.max_abs_err(hT.numpy(), rh))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,local_parts", [(2, 1), (3, 1), (2, 3), (3, 2)])
def test_split_across_gloo_ranks_matches_oracle(world, local_parts):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = 29500 + world * 7 + local_parts * 31 + os.getpid() % 500
        procs = [ctx.Process(target=_sp_worker, args=(r, world, port, 160, results, local_parts))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0, f"rank exited with {p.exitcode}"
        for r in range(world):
            eo, eh = results[r]
            assert eo < 1e-10 and eh < 1e-10, (r, eo, eh)


@pytest.mark.gpu
@pytest.mark.parametrize("gscale", [1.0, 0.02])
@pytest.mark.parametrize("B,T,H,parts", [(1, 4096, 4, 4), (2, 1000, 2, 3), (1, 8192, 2, 8)])
def test_split_cuda_matches_unsplit(cuda, B, T, H, parts, gscale):
    """gscale 1: the configurations' gates (about e^-51 per chunk, so little
    state crosses a segment boundary); 0.02: about e^-1 per chunk, so the
    hand-off carries real state over every boundary."""
    from helpers import assert_close, device_inputs_fast, f64
    from gated_deltanet_jax_b200 import ops
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, 128, seed=T, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    g = (g * gscale).contiguous()
    o_ref, h_ref = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                              output_final_state=True)
    o, hT = sp.chunk_gated_delta_rule_split(q, k, v, g, b, initial_state=h0,
                                            output_final_state=True, parts=parts)
    assert_close(f64(o), f64(o_ref), "bf16", "o")
    assert_close(f64(hT), f64(h_ref), "bf16", "state")


@pytest.mark.gpu
def test_long_context_config_against_oracle(cuda):
    """The long-context configuration at full length: B=1 T=65536 H=16
    dk=dv=128, bf16 in, fp32 state.  Two sampled heads over all 65536 tokens
    (1024 chunks) against the float64 oracle, for the one-call kernel and for
    the one-GPU sequence split (4 segments): the drift of the bf16-rounded
    state operand over the whole sequence stays inside the bf16 bar."""
    from helpers import assert_close, device_inputs_fast, f64
    from gated_deltanet_jax_b200 import ops
    B, T, H = 1, 65536, 16
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, 128, seed=4, dtype="bf16", dev=cuda,
                                           h0_std=0.02)
    # half of the heads with the configuration's gates, half with gates 50x
    # milder (about e^-1 per chunk), whose state spans many chunks and every
    # segment boundary of the split
    g = torch.cat([g[:, :, :8], g[:, :, 8:] * 0.02], dim=2).contiguous()
    o1, h1 = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    o2, h2 = sp.chunk_gated_delta_rule_split(q, k, v, g, b, initial_state=h0,
                                             output_final_state=True, parts=4)
    for h in (0, 11):
        host = [f64(t[:, :, h:h + 1]) for t in (q, k, v, g, b)]
        ro, rh = orc.chunk_exact(*host, f64(h0[:, h:h + 1]), 64)
        for name, o, hT in (("one call", o1, h1), ("split", o2, h2)):
            assert_close(f64(o[:, :, h:h + 1]), ro, "bf16", f"{name} head {h} o")
            assert_close(f64(hT[:, h:h + 1]), rh, "bf16", f"{name} head {h} state")
    assert torch.isfinite(o1.float()).all() and torch.isfinite(o2.float()).all()


@pytest.mark.parametrize("P", [1, 2, 3, 5, 8, 9])
def test_scan_fold_equals_sequential_fold(P):
    """The log-depth prefix scan gives the sequential fold's states."""
    gen = torch.Generator().manual_seed(P)
    B, H, dk, dv = 2, 3, 8, 5
    S = torch.randn(P, B, H, dk, dv, generator=gen, dtype=torch.float64)
    M = torch.randn(P, B, H, dk, dk, generator=gen, dtype=torch.float64) / dk ** 0.5
    h0 = torch.randn(B, H, dk, dv, generator=gen, dtype=torch.float64)
    ref = sp.fold_states(h0, [(S[p], M[p]) for p in range(P)])
    got = sp.fold_states_scan(h0, S, M)
    assert got.shape[0] == P + 1
    for p in range(P + 1):
        torch.testing.assert_close(got[p], ref[p], rtol=1e-10, atol=1e-12)


def _nccl_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from helpers import device_inputs_fast, f64
        from gated_deltanet_jax_b200 import ops
        T = 2048 * world
        q, k, v, g, b, h0 = device_inputs_fast(1, T, 4, 128, 128, seed=3, dtype="bf16", dev=dev,
                                               h0_std=0.02)
        g = (g * 0.02).contiguous()   # mild gates: state crosses the rank boundary
        seg = T // world
        sl = slice(rank * seg, (rank + 1) * seg)
        o, hT = sp.chunk_gated_delta_rule_sp(q[:, sl], k[:, sl], v[:, sl], g[:, sl], b[:, sl],
                                             initial_state=h0, output_final_state=True,
                                             local_parts=2)
        o_ref, h_ref = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0,
                                                  output_final_state=True)
        results[rank] = (orc.rel_err(f64(o), f64(o_ref[:, sl])), orc.rel_err(f64(hT), f64(h_ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_split_across_nccl_ranks(cuda):
    """Two GPUs: each rank holds half of the sequence; NCCL all-gather hand-off."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_nccl_worker, args=(r, 2, 29611, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(30)
        for p in procs:
            assert p.exitcode == 0
        for r in range(2):
            eo, eh = results[r]
            assert eo <= orc.TOL_BF16_REL and eh <= orc.TOL_BF16_REL, (r, eo, eh)


def test_split_ranks_agree_on_local_parts_with_a_shorter_last_rank():
    """local_parts=None with a last rank holding fewer tokens: the ranks'
    own choices differ (3 against 1 here); they must agree before the
    all-gather, and the result still matches the oracle."""
    world, T, seg = 3, 250, 96          # ranks hold 96, 96 and 58 tokens
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = 29500 + 401 + os.getpid() % 500
        procs = [ctx.Process(target=_sp_worker,
                             args=(r, world, port, T, results, None, seg, True))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0, f"rank exited with {p.exitcode}"
        for r in range(world):
            eo, eh = results[r]
            assert eo < 1e-10 and eh < 1e-10, (r, eo, eh)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,Hk,dv", [(2, 300, 4, 2, 128), (1, 1000, 2, 2, 64), (3, 64, 2, 1, 192)])
def test_two_phase_scan_transition_is_the_segment_map(cuda, B, T, H, Hk, dv):
    """gdn_chunk_scan's transition columns: [S | M] with hT(h0) = M h0 + S for
    the scan of the same segment from h0 (mild gates, so M is far from zero);
    one preparation serves both scans, and a scan with an output equals the
    one-call forward."""
    from helpers import assert_close, device_inputs_fast, f64
    from gated_deltanet_jax_b200 import ops
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, 128, dv, seed=T + dv, dtype="bf16",
                                           dev=cuda, h0_std=0.05)
    q, k = q[:, :, ::H // Hk].contiguous(), k[:, :, ::H // Hk].contiguous()
    g = (g * 0.02).contiguous()
    ws = ops._chunk_prepare(q, k, g, b)
    none, ext = ops._chunk_scan(q, k, v, g, b, ws, transition=True, output=False)
    assert none is None and ext.shape == (B, H, 128, dv + 128)
    S, M = ext[..., :dv], ext[..., dv:]
    o2, h2 = ops._chunk_scan(q, k, v, g, b, ws, initial_state=h0)
    o1, h1 = ops.chunk_gated_delta_rule(q, k, v, g, b, initial_state=h0, output_final_state=True)
    assert torch.equal(o1, o2) and torch.equal(h1, h2)
    assert_close(f64(M @ h0 + S), f64(h1), "bf16", "M h0 + S")
    # (the map's linear part, which the hand-off carries, against the float64
    # recurrence started from the identity with v = 0, for one head)
    from oracle import gdn_oracle as orc
    eye = np.broadcast_to(np.eye(128), (1, 1, 128, 128)).copy()
    _, rM = orc.recurrent_ref(f64(q[:1, :, :1]), f64(k[:1, :, :1]), np.zeros((1, T, 1, 128)),
                              f64(g[:1, :, :1]), f64(b[:1, :, :1]), eye)
    assert_close(f64(M[:1, :1]), rM, "bf16", "transition vs oracle")


@pytest.mark.gpu
@pytest.mark.parametrize("P,B,H,dv,with_h0", [(1, 1, 2, 32, True), (3, 2, 3, 128, False),
                                               (9, 1, 16, 128, True), (5, 1, 2, 192, True),
                                               (0, 1, 2, 64, True)])
def test_fold_kernel_equals_sequential_fold(cuda, P, B, H, dv, with_h0):
    """gdn_fold_states on the interleaved [S | M] summaries gives the states of
    the float64 sequential fold (fp32 products of 128 terms: 1e-5 relative)."""
    from gated_deltanet_jax_b200 import ops
    gen = torch.Generator(device=cuda).manual_seed(P * 7 + dv)
    dk = 128
    packed = torch.randn(P, B, H, dk, dv + dk, device=cuda, generator=gen)
    packed[..., dv:] /= dk ** 0.5
    h0 = torch.randn(B, H, dk, dv, device=cuda, generator=gen) if with_h0 else None
    got = ops._fold_states(packed, h0, dv)
    pk = packed.double().cpu()
    ref = sp.fold_states(torch.zeros(B, H, dk, dv, dtype=torch.float64) if h0 is None
                         else h0.double().cpu(),
                         [(pk[p, ..., :dv], pk[p, ..., dv:]) for p in range(P)])
    assert got.shape == (P + 1, B, H, dk, dv)
    for p in range(P + 1):
        err = float((got[p].double().cpu() - ref[p]).abs().max() / ref[p].abs().max().clamp_min(1e-30))
        assert err < 1e-5, (p, err)
