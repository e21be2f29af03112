"""Benchmark of the gated delta-rule hot path on B200.

Headline line (one JSON object on rank 0): recurrent decode tokens/s on the
decode workload -- B=64, H=16, dk=dv=128, bf16 q/k/v, fp32 state ~N(0,0.02),
one bench step = 512 consecutive single-token decode steps with the state
updated in place (512 kernel launches, replayed as one CUDA graph).  The
``prefill`` object in the same line reports chunked prefill tokens/s on B=4,
T=4096, H=16, dk=dv=128, chunk=64, bf16 in / fp32 state (two launches per step:
the per-chunk preparation, then the scan, each also timed alone);
``long_context`` B=1 T=65536; ``backward`` the gradients on the prefill workload;
``model_forward`` the full GatedDeltaNetModel forward at the reference's model
configuration (24 layers, B=8 T=2048).

Multi-GPU (torchrun, one rank per GPU): batch x head work is independent, so
every rank runs its own full workload (weak scaling, no collective on the
data path); NCCL is used only for the barrier and the max-over-ranks time.

``--impl reference`` times the CPU restatement of the reference algorithm
(NumPy, all host cores) on a bounded sample of the same decode workload.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

DEC = dict(B=64, H=16, dk=128, dv=128, tokens=512)
NBUF = 4  # decode states used round robin per bench step
PRE = dict(B=4, T=4096, H=16, dk=128, dv=128, chunk=64)
LONG = dict(B=1, T=65536, H=16, dk=128, dv=128, chunk=64, parts=4)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-e2e", action="store_true", help="skip the end-to-end legs")
    p.add_argument("--no-prefill", action="store_true", help="skip the prefill leg")
    p.add_argument("--no-long", action="store_true", help="skip the long-context leg")
    p.add_argument("--no-backward", action="store_true", help="skip the backward leg")
    p.add_argument("--no-layer", action="store_true", help="skip the layer-core legs")
    # A fixed workload for ncu captures (one process, one GPU, no timing):
    #   --profile-workload decode --launches 3        (B=64 H=16 dk=dv=128, state in place)
    #   --profile-workload prefill --launches 2 [--B 4 --T 4096 --H 16 --dk 128 --dv 128]
    #   --profile-workload backward --launches 2 [--B 4 --T 4096]
    #   --profile-workload prefill_layer --launches 2 [--B 4 --T 4096]
    p.add_argument("--profile-workload", choices=["decode", "prefill", "backward",
                                                   "prefill_layer"], default=None)
    p.add_argument("--launches", type=int, default=3)
    p.add_argument("--B", type=int, default=None)
    p.add_argument("--T", type=int, default=None)
    p.add_argument("--H", type=int, default=16)
    p.add_argument("--dk", type=int, default=128)
    p.add_argument("--dv", type=int, default=128)
    return p.parse_args()


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def _profile_traffic(name):
    """Per-launch DRAM bytes recorded from ncu in profiles/<name>.txt, or None."""
    path = os.path.join(REPO, "profiles", name + ".txt")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch\s*=\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"gdn_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or (self.uuid and self.uuid not in parts[0]):
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for _, _, flags in rows for n, f in zip(names, flags)
                          if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU legs (the oracle restatement; never the measured product)
# ---------------------------------------------------------------------------

def _cpu_decode_inputs(seed=0):
    import numpy as np
    from oracle import gdn_oracle as orc
    B, H, dk, dv = DEC["B"], DEC["H"], DEC["dk"], DEC["dv"]
    q, k, v, g, beta, h0 = orc.make_inputs(B, 8, H, dk, dv, seed=seed, h0_std=0.02)
    cast = lambda x: np.ascontiguousarray(x, np.float32)  # noqa: E731
    return [cast(x) for x in (q, k, v, g, beta)], cast(h0)


def _cpu_decode_tokens(inputs, state, ntok, pool, nthreads):
    """Decode `ntok` tokens of the B=64 batch with the float32 NumPy recurrence,
    the batch split over `nthreads` host threads; returns the new state."""
    import numpy as np
    from oracle import gdn_oracle as orc
    q, k, v, g, beta = inputs
    B = q.shape[0]
    parts = np.array_split(np.arange(B), nthreads)

    def run(idx, s):
        sl = slice(idx[0], idx[-1] + 1)
        out = None
        for t in range(ntok):
            tt = t % q.shape[1]
            ts = slice(tt, tt + 1)
            out, s = orc.recurrent_ref(q[sl, ts], k[sl, ts], v[sl, ts], g[sl, ts], beta[sl, ts],
                                       s, dtype=np.float32)
        return s

    futs = [pool.submit(run, idx, state[idx[0]:idx[-1] + 1]) for idx in parts]
    return np.concatenate([f.result() for f in futs], 0)


# Decode tokens of the batch per host dispatch: the CPU baseline and the
# reference arm both step the batch this many tokens per call, so the two time
# one code path at one granularity.
CPU_DECODE_TOKENS = 4


def cpu_decode_timed(steps=None, warmup=1, budget_s=None):
    """Time the host decode recurrence: `warmup` untimed then `steps` timed
    dispatches of CPU_DECODE_TOKENS tokens of the B=64 batch (or as many as fit
    in `budget_s` seconds).  Returns (tokens/s, dispatches, seconds, threads)."""
    import concurrent.futures as cf
    nthreads = os.cpu_count() or 1
    inputs, state = _cpu_decode_inputs()
    with cf.ThreadPoolExecutor(nthreads) as pool:
        for _ in range(warmup):
            state = _cpu_decode_tokens(inputs, state, CPU_DECODE_TOKENS, pool, nthreads)
        n, t0 = 0, time.perf_counter()
        while (n < steps) if steps is not None else (time.perf_counter() - t0 < budget_s or n < 2):
            state = _cpu_decode_tokens(inputs, state, CPU_DECODE_TOKENS, pool, nthreads)
            n += 1
        el = time.perf_counter() - t0
    return DEC["B"] * CPU_DECODE_TOKENS * n / el, n, el, nthreads


def _cpu_decode_sample(n, el, nthreads):
    return (f"{n} dispatches of {CPU_DECODE_TOKENS} decode tokens x B=64 (H=16 dk=dv=128), "
            f"float32 NumPy restatement of the reference recurrence, batch split over "
            f"{nthreads} threads, {el:.1f} s")


def cpu_decode_baseline(budget_s=10.0):
    value, n, el, nthreads = cpu_decode_timed(budget_s=budget_s)
    return {"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
            "sample": _cpu_decode_sample(n, el, nthreads)}


def cpu_prefill_baseline(budget_s=10.0):
    import numpy as np
    from oracle import gdn_oracle as orc
    T, H, dk, dv, C = PRE["T"], PRE["H"], PRE["dk"], PRE["dv"], PRE["chunk"]
    q, k, v, g, beta, _ = orc.make_inputs(1, T, H, dk, dv, seed=0)
    f32 = lambda x: np.ascontiguousarray(x, np.float32)  # noqa: E731
    q, k, v, g, beta = (f32(x) for x in (q, k, v, g, beta))
    ntok, t0, h = 0, time.perf_counter(), None
    seg = 512
    while time.perf_counter() - t0 < budget_s or ntok < seg:
        s = slice(ntok % T, ntok % T + seg)
        _, h = orc.chunk_exact(q[:, s], k[:, s], v[:, s], g[:, s], beta[:, s], h, C, np.float32)
        ntok += seg
    el = time.perf_counter() - t0
    return {"value": ntok / el, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{ntok} tokens of B=1 sequences, H=16 dk=dv=128 chunk=64 (float32 "
                      f"NumPy restatement of the chunked recurrence, BLAS threads), {el:.1f} s"}


def run_reference_arm(a):
    """--impl reference: the CPU restatement, rank 0 only (the same code path
    and dispatch granularity as the GPU arm's cpu_baseline)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    value, n, el, nthreads = cpu_decode_timed(steps=a.steps, warmup=a.warmup)
    ntok_step = CPU_DECODE_TOKENS
    print(json.dumps({
        "impl": "reference", "metric": "recurrent decode tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": el / a.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode B=64 H=16 dk=dv=128, fp32 state ~N(0,0.02); each step a "
                               f"sample of {ntok_step} decode tokens of the batch",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": _cpu_decode_sample(n, el, nthreads) + " (JAX is not "
                                   "installable here, so the reference itself cannot run)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# GPU legs
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self):
        import torch
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=self.dev)

    def barrier(self):
        import torch
        torch.cuda.synchronize(self.dev)
        if self.world > 1:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max(self, x):
        import torch
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def _timed(d, fn, steps, sampler=None):
    """Time exactly `steps` calls of fn on the current stream; max over ranks (ms/step)."""
    import torch
    st = torch.cuda.current_stream(d.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d.barrier()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    torch.cuda.synchronize(d.dev)
    clocks = sampler.stop() if sampler else None
    d.barrier()
    ms = e0.elapsed_time(e1) / steps
    return d.max(ms), clocks


def decode_leg(d, a, lib, uuid):
    import torch
    from gated_deltanet_jax_b200 import _lib, ops
    from gated_deltanet_jax_b200 import roofline as rl
    B, H, dk, dv, TOK = DEC["B"], DEC["H"], DEC["dk"], DEC["dv"], DEC["tokens"]
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(1234 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(TOK, B, 1, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(TOK, B, 1, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(TOK, B, 1, H, dv, device=d.dev, generator=gen).bfloat16()
    g = torch.nn.functional.logsigmoid(torch.randn(TOK, B, 1, H, device=d.dev, generator=gen))
    beta = torch.sigmoid(torch.randn(TOK, B, 1, H, device=d.dev, generator=gen))
    # NBUF independent states used round robin (as the layers of a model would
    # use theirs): 4 x 64 MiB is larger than the 126 MB L2, so every launch
    # reads its state from HBM.  A single 64 MiB state would stay L2-resident.
    S = torch.randn(NBUF, B, H, dk, dv, device=d.dev, generator=gen) * 0.02
    o = torch.empty(TOK, B, 1, H, dv, device=d.dev, dtype=torch.bfloat16)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def one_step(stream, nbuf):
        for t in range(TOK):
            st = S[t % nbuf]
            rc = lib.gdn_recurrent_fwd(ptr(q[t]), ptr(k[t]), ptr(v[t]), ptr(g[t]), ptr(beta[t]),
                                       ptr(st), ptr(o[t]), ptr(st), B, 1, H, dk, dv,
                                       _lib.GDN_DTYPE_BF16, ctypes.c_void_p(stream))
            if rc:
                _lib.check(rc, "gdn_recurrent_fwd")

    def capture(nbuf):
        one_step(torch.cuda.current_stream(d.dev).cuda_stream, nbuf)  # load modules first
        torch.cuda.synchronize(d.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_step(torch.cuda.current_stream(d.dev).cuda_stream, nbuf)
        for _ in range(a.warmup):
            graph.replay()
        return graph

    graph = capture(NBUF)
    sampler = ClockSampler(uuid) if d.rank == 0 else None
    ms, clocks = _timed(d, graph.replay, a.steps, sampler)
    del graph
    value = d.world * B * TOK / (ms / 1e3)
    bytes_launch = B * H * rl.bytes_recurrent_per_head_step(dk, dv, 2)
    launch_s = ms / 1e3 / TOK
    res = {"ms": ms, "value": value, "clocks": clocks, "launch_s": launch_s,
           "bytes_launch": bytes_launch, "launches": a.steps * TOK}
    # The literal single-state form of the workload (its 64 MiB state stays in L2).
    graph = capture(1)
    ms1, _ = _timed(d, graph.replay, a.steps)
    res["launches"] += a.steps * TOK
    del graph
    res["single_state"] = {"value": d.world * B * TOK / (ms1 / 1e3), "unit": "tokens/s",
                           "ms_per_step": ms1,
                           "note": "one 64 MiB state for all 512 steps; it fits the 126 MB L2, "
                                   "so this is not an HBM-bound figure"}

    if not a.no_e2e:
        # Public API with host buffers, driven the way a serving loop drives decode:
        # the per-token op call is captured once, with its copies, into a CUDA graph
        # that is replayed every step.  Per token: one H2D copy of the packed
        # q/k/v/g/beta row from pinned memory (copy stream), the op (compute stream),
        # one D2H copy of o into pinned memory (second copy stream); inputs are
        # double-buffered so token t+1's copy and token t-1's readback overlap token
        # t's kernel.  Every step moves all of its inputs and outputs over PCIe.
        parts = [q[0], k[0], v[0], g[0], beta[0]]
        sizes = [x.nbytes for x in parts]
        offs = [sum(sizes[:i]) for i in range(len(sizes) + 1)]
        tok_bytes = offs[-1]
        hin = torch.empty((TOK, tok_bytes), dtype=torch.uint8).pin_memory()
        for i, src in enumerate((q, k, v, g, beta)):
            hin[:, offs[i]:offs[i + 1]].copy_(src.reshape(TOK, -1).cpu().view(torch.uint8))
        din = torch.empty((2, tok_bytes), dtype=torch.uint8, device=d.dev)
        views = [[din[j, offs[i]:offs[i + 1]].view(parts[i].dtype).view(parts[i].shape)
                  for i in range(len(parts))] for j in range(2)]
        ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
        s_in, s_out = torch.cuda.Stream(d.dev), torch.cuda.Stream(d.dev)

        def e2e_body():
            cur = torch.cuda.current_stream(d.dev)
            s_in.wait_stream(cur)
            s_out.wait_stream(cur)
            ev_k = [None, None]
            outs = []
            for t in range(TOK):
                j = t & 1
                with torch.cuda.stream(s_in):
                    if ev_k[j] is not None:
                        s_in.wait_event(ev_k[j])      # token t-2's kernel is done with din[j]
                    din[j].copy_(hin[t], non_blocking=True)
                    e_in = torch.cuda.Event()
                    e_in.record(s_in)
                cur.wait_event(e_in)
                st = S[t % NBUF]
                ot, _ = ops.fused_recurrent_gated_delta_rule(*views[j], initial_state=st,
                                                             final_state_out=st)
                e_k = torch.cuda.Event()
                e_k.record(cur)
                ev_k[j] = e_k
                with torch.cuda.stream(s_out):
                    s_out.wait_event(e_k)
                    ho[t].copy_(ot, non_blocking=True)
                outs.append(ot)                       # no output buffer is reused in a step
            cur.wait_stream(s_in)
            cur.wait_stream(s_out)

        e2e_body()                                    # eager once (module loads)
        torch.cuda.synchronize(d.dev)
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph):
            e2e_body()
        for _ in range(a.warmup):
            e2e_graph.replay()
        e2e_steps = max(1, min(a.steps, 20))
        ms_e2e, _ = _timed(d, e2e_graph.replay, e2e_steps)
        res["launches"] += e2e_steps * TOK
        torch.cuda.synchronize(d.dev)
        del e2e_graph
        res["e2e"] = {"value": d.world * B * TOK / (ms_e2e / 1e3), "unit": "tokens/s",
                      "h2d_bytes_per_step": int(TOK * tok_bytes),
                      "d2h_bytes_per_step": int(TOK * o[0].nbytes),
                      "steps": e2e_steps,
                      "path": "ops.fused_recurrent_gated_delta_rule per token, captured with its "
                              "copies into a CUDA graph replayed per step: packed q/k/v/g/beta "
                              "H2D from pinned memory and o D2H into pinned memory every token, "
                              "on two copy streams overlapping the kernels; state resident on "
                              "the device"}
    return res


def prefill_leg(d, a, lib, uuid=None):
    import torch
    from gated_deltanet_jax_b200 import _lib, ops
    from gated_deltanet_jax_b200 import roofline as rl
    B, T, H, dk, dv, C = (PRE[x] for x in ("B", "T", "H", "dk", "dv", "chunk"))
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(99 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    o = torch.empty(B, T, H, dv, device=d.dev, dtype=torch.bfloat16)
    hT = torch.empty(B, H, dk, dv, device=d.dev, dtype=torch.float32)
    ws_bytes = lib.gdn_chunk_workspace_bytes(B, T, H, dk, dv, C, _lib.GDN_DTYPE_BF16, 0)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=d.dev)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        rc = lib.gdn_chunk_fwd(ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), None, ptr(o), ptr(hT),
                               B, T, H, dk, dv, C, _lib.GDN_DTYPE_BF16, 0, ptr(ws), ws_bytes,
                               ctypes.c_void_p(torch.cuda.current_stream(d.dev).cuda_stream))
        if rc:
            _lib.check(rc, "gdn_chunk_fwd")

    for _ in range(a.warmup):
        step()
    # ~0.25 ms per launch: time enough launches for the clock sampler to see them.
    steps = max(a.steps, 1000)
    sampler = ClockSampler(uuid) if d.rank == 0 else None
    ms, clocks = _timed(d, step, steps, sampler)
    flops = B * T * H * rl.flops_chunk_per_token_head(dk, dv, C)
    res = {"ms": ms, "value": d.world * B * T / (ms / 1e3), "flops_launch": flops,
           # two launches per call: the per-chunk preparation, then the scan
           "launch_s": ms / 1e3, "launches": 2 * steps, "steps": steps, "clocks": clocks,
           "bytes_launch": B * T * H * rl.bytes_chunk_per_token_head(dk, dv) + B * H * dk * dv * 4}
    if ws_bytes:
        # Each of the two kernels timed on its own over the same workspace: the
        # preparation reads q/k (bf16), g/beta and writes 24 KiB per (chunk,
        # head); the scan reads q/k/v, g/beta and that workspace, writes o and
        # the final state.
        cs = lambda: ctypes.c_void_p(torch.cuda.current_stream(d.dev).cuda_stream)  # noqa: E731

        def prep():
            _lib.check(lib.gdn_chunk_prepare(ptr(q), ptr(k), ptr(g), ptr(beta), B, T, H, H, dk,
                                             _lib.GDN_DTYPE_BF16, ptr(ws), ws_bytes, cs()),
                       "gdn_chunk_prepare")

        def scan():
            _lib.check(lib.gdn_chunk_scan(ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), None, ptr(o),
                                          ptr(hT), B, T, H, H, dk, dv, _lib.GDN_DTYPE_BF16, 0,
                                          ptr(ws), ws_bytes, cs()), "gdn_chunk_scan")

        ksteps = max(a.steps, 200)
        for fn in (prep, scan):
            for _ in range(3):
                fn()
        ms_prep, _ = _timed(d, prep, ksteps)
        ms_scan, _ = _timed(d, scan, ksteps)
        nch = B * H * ((T + C - 1) // C)
        prep_bytes = B * T * H * (2 * dk * 2 + 8) + nch * 24576
        scan_bytes = (B * T * H * ((2 * dk + 2 * dv) * 2 + 8) + nch * 24576
                      + B * H * dk * dv * 4)
        res["launches"] += 2 * (ksteps + 3)
        res["kernels"] = {
            "chunk_prep_kernel": {"ms": ms_prep, "share": ms_prep / (ms_prep + ms_scan),
                                  "bytes_per_launch": prep_bytes,
                                  "gbs": prep_bytes / ms_prep / 1e6},
            "chunk_scan_kernel": {"ms": ms_scan, "share": ms_scan / (ms_prep + ms_scan),
                                  "bytes_per_launch": scan_bytes,
                                  "gbs": scan_bytes / ms_scan / 1e6},
            "note": "each kernel timed alone over the same inputs and workspace "
                    f"({ksteps} launches, CUDA events)"}
    if not a.no_e2e:
        # Through the public op with pinned host buffers, every step: H2D of the
        # step's q/k/v/g/beta, the op, D2H of o and the final state.  Pipelined
        # as a serving loop runs it: inputs upload on one copy stream into one
        # of two device buffer sets while the previous step computes, and
        # results download on a second copy stream (PCIe is full duplex).  The
        # timed region ends after the last step's download.
        hin = [t.cpu().pin_memory() for t in (q, k, v, g, beta)]
        ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
        hh = torch.empty(hT.shape, dtype=hT.dtype).pin_memory()
        dbuf = [[torch.empty_like(t) for t in (q, k, v, g, beta)] for _ in range(2)]
        hbuf = [torch.empty_like(hT) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(d.dev), torch.cuda.Stream(d.dev)
        comp = torch.cuda.current_stream(d.dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        state = {"i": 0, "used": [False, False]}

        def e2e_step():
            i = state["i"]
            j = i % 2
            with torch.cuda.stream(s_in):
                if state["used"][j]:
                    s_in.wait_event(ev_comp[j])       # the op two steps back has read buffer j
                for dst, src in zip(dbuf[j], hin):
                    dst.copy_(src, non_blocking=True)
                ev_in[j].record(s_in)
            comp.wait_event(ev_in[j])
            if state["used"][j]:
                comp.wait_event(ev_out[j])            # buffer j's results have been read out
            ot, _ = ops.chunk_gated_delta_rule(*dbuf[j], final_state_out=hbuf[j])
            ev_comp[j].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[j])
                ho.copy_(ot, non_blocking=True)
                hh.copy_(hbuf[j], non_blocking=True)
                ev_out[j].record(s_out)
            ot.record_stream(s_out)
            state["used"][j] = True
            state["i"] = i + 1

        for _ in range(min(a.warmup, 2)):
            e2e_step()
        torch.cuda.synchronize(d.dev)
        e2e_steps = max(1, min(a.steps, 20))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d.barrier()
        e0.record(comp)
        for _ in range(e2e_steps):
            e2e_step()
        comp.wait_event(ev_out[(state["i"] - 1) % 2])  # the last step's results are on the host
        e1.record(comp)
        torch.cuda.synchronize(d.dev)
        d.barrier()
        ms_e2e = d.max(e0.elapsed_time(e1) / e2e_steps)
        res["launches"] += 2 * e2e_steps
        res["e2e"] = {"value": d.world * B * T / (ms_e2e / 1e3), "unit": "tokens/s",
                      "h2d_bytes_per_step": int(q.nbytes + k.nbytes + v.nbytes + g.nbytes
                                                + beta.nbytes),
                      "d2h_bytes_per_step": int(o.nbytes + hT.nbytes), "steps": e2e_steps,
                      "path": "ops.chunk_gated_delta_rule, pinned host buffers; inputs of the "
                              "next step upload while this step computes and its results "
                              "download (two copy streams)"}
    return res


def _layer_gate_params(H, dev, gen):
    """A_log and dt_bias drawn as the layer initialises them (model.py:103-113):
    A ~ U(1e-4, 16); dt log-uniform in [1e-3, 0.1], dt_bias = softplus^-1(dt)."""
    import math
    import torch
    A_log = torch.log(torch.rand(H, device=dev, generator=gen) * (16 - 1e-4) + 1e-4)
    u = torch.rand(H, device=dev, generator=gen)
    dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
    return A_log, dt + torch.log(-torch.expm1(-dt))


def decode_layer_leg(d, a):
    """One decode token of the layer core (gates from the raw projections, the
    step, the gated RMSNorm) on the decode workload, two ways, each replayed
    from a CUDA graph of 64 tokens: the fused kernel (gdn_recurrent_fwd_layer)
    against the op between the same operations done separately in torch, as
    the reference layer does them (model.py:136-153)."""
    import torch
    from gated_deltanet_jax_b200 import ops
    B, H, dk, dv, TOK = DEC["B"], DEC["H"], DEC["dk"], DEC["dv"], 64
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(4321 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(TOK, B, 1, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(TOK, B, 1, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(TOK, B, 1, H, dv, device=d.dev, generator=gen).bfloat16()
    ra = torch.randn(TOK, B, 1, H, device=d.dev, generator=gen)
    rb = torch.randn(TOK, B, 1, H, device=d.dev, generator=gen)
    gate = torch.randn(TOK, B, 1, H, dv, device=d.dev, generator=gen).bfloat16()
    A_log, dt_bias = _layer_gate_params(H, d.dev, gen)
    w = torch.ones(dv, device=d.dev)
    S = torch.randn(NBUF, B, H, dk, dv, device=d.dev, generator=gen) * 0.02

    def fused():
        for t in range(TOK):
            st = S[t % NBUF]
            ops.gated_delta_rule_decode_layer(q[t], k[t], v[t], ra[t], rb[t], A_log, dt_bias,
                                              gate=gate[t], norm_weight=w, initial_state=st,
                                              final_state_out=st)

    def unfused():
        for t in range(TOK):
            st = S[t % NBUF]
            gd = -torch.exp(A_log) * torch.nn.functional.softplus(ra[t] + dt_bias)
            bd = torch.sigmoid(rb[t])
            o, _ = ops.fused_recurrent_gated_delta_rule(q[t], k[t], v[t], gd, bd,
                                                        initial_state=st, final_state_out=st)
            x = o.float()
            var = x.pow(2).mean(-1, keepdim=True)
            (x * torch.rsqrt(var + 1e-5) * w
             * torch.nn.functional.silu(gate[t].float())).to(o.dtype)

    gd_all = -torch.exp(A_log) * torch.nn.functional.softplus(ra + dt_bias)
    bd_all = torch.sigmoid(rb)

    def op_only():   # the step alone, gates given (what the plain decode leg runs)
        for t in range(TOK):
            st = S[t % NBUF]
            ops.fused_recurrent_gated_delta_rule(q[t], k[t], v[t], gd_all[t], bd_all[t],
                                                 initial_state=st, final_state_out=st)

    res = {}
    for name, fn in (("fused", fused), ("unfused", unfused), ("op_only", op_only)):
        fn()                                   # load modules, allocate
        torch.cuda.synchronize(d.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(a.warmup):
            graph.replay()
        steps = max(1, min(a.steps, 50))
        ms, _ = _timed(d, graph.replay, steps)
        res[name] = ms * 1e3 / TOK
        del graph
    return {"workload": "one decode token of the layer core: B=64 H=16 dk=dv=128 bf16, gates "
                        "from raw a/b projections, gated RMSNorm (eps 1e-5) of the output; "
                        f"states round robin over {NBUF} x 64 MiB; 64 tokens per CUDA graph",
            "fused_us_per_token": res["fused"], "unfused_us_per_token": res["unfused"],
            "op_only_us_per_token": res["op_only"],
            "speedup": res["unfused"] / res["fused"],
            "launches": 3 * TOK * max(1, min(a.steps, 50)),
            "fused_tokens_per_s": d.world * B / (res["fused"] / 1e6),
            "path": "fused: gdn_recurrent_fwd_layer (1 launch per token); unfused: torch gates, "
                    "gdn_recurrent_fwd, torch gated RMSNorm; op_only: gdn_recurrent_fwd with "
                    "precomputed gates and no norm"}


def prefill_layer_leg(d, a):
    """The layer core over the prefill workload (gates from the raw
    projections, the chunked forward, the gated RMSNorm of every output row),
    two ways: the fused kernel (gdn_chunk_fwd_layer) against the op between
    the same operations done separately in torch, as the reference layer does
    them (model.py:136-153); and the op alone with the gates given."""
    import torch
    from gated_deltanet_jax_b200 import ops
    B, T, H, dk, dv = PRE["B"], PRE["T"], PRE["H"], PRE["dk"], PRE["dv"]
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(8765 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    ra = torch.randn(B, T, H, device=d.dev, generator=gen)
    rb = torch.randn(B, T, H, device=d.dev, generator=gen)
    gate = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    A_log, dt_bias = _layer_gate_params(H, d.dev, gen)
    w = torch.ones(dv, device=d.dev)
    hT = torch.empty(B, H, dk, dv, device=d.dev)

    def fused():
        ops.gated_delta_rule_chunk_layer(q, k, v, ra, rb, A_log, dt_bias, gate=gate,
                                         norm_weight=w, final_state_out=hT)

    def unfused():
        gd = -torch.exp(A_log) * torch.nn.functional.softplus(ra + dt_bias)
        bd = torch.sigmoid(rb)
        o, _ = ops.chunk_gated_delta_rule(q, k, v, gd, bd, final_state_out=hT)
        x = o.float()
        var = x.pow(2).mean(-1, keepdim=True)
        (x * torch.rsqrt(var + 1e-5) * w * torch.nn.functional.silu(gate.float())).to(o.dtype)

    gd_all = -torch.exp(A_log) * torch.nn.functional.softplus(ra + dt_bias)
    bd_all = torch.sigmoid(rb)

    def op_only():
        ops.chunk_gated_delta_rule(q, k, v, gd_all, bd_all, final_state_out=hT)

    # Each variant is replayed from a CUDA graph of REP calls, so that the
    # host's per-call Python work (longer than the kernel) is not what is timed.
    REP = 8
    res = {}
    steps = max(1, min(a.steps, 50))
    for name, fn in (("fused", fused), ("unfused", unfused), ("op_only", op_only)):
        fn()                                   # load modules, allocate
        torch.cuda.synchronize(d.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(REP):
                fn()
        for _ in range(a.warmup):
            graph.replay()
        ms, _ = _timed(d, graph.replay, steps)
        res[name] = ms / REP
        del graph
    return {"workload": "the layer core over B=4 T=4096 H=16 dk=dv=128 bf16: gates from raw "
                        "a/b projections, chunked forward, gated RMSNorm (eps 1e-5) of every "
                        "output row; final state out; 8 calls per CUDA graph",
            "fused_ms": res["fused"], "unfused_ms": res["unfused"], "op_only_ms": res["op_only"],
            # fused: one launch per call; unfused and op_only: the op's two each
            "speedup": res["unfused"] / res["fused"], "launches": 5 * REP * steps,
            "fused_tokens_per_s": d.world * B * T / (res["fused"] / 1e3),
            "path": "fused: gdn_chunk_fwd_layer (1 launch; the two column tiles of a row as one "
                    "cluster of two CTAs); unfused: torch gates, "
                    "gdn_chunk_fwd, torch gated RMSNorm; op_only: gdn_chunk_fwd with "
                    "precomputed gates and no norm"}


def prefill_layer_default_leg(d, a):
    """The layer core at the reference's default head dims (head_dim 256,
    expand_v 2: dk=256, dv=512; 6 heads; B=8 T=2048), from the raw q/k/v
    projection outputs: the short convolution + SiLU of q, k and v
    (model.py:15-40, :119-122), the gates from the raw a/b projections
    (:136-139), the chunked forward, the gated RMSNorm of every output row
    (:41-53, :147-153).  Two ways: this library's kernels (gdn_short_conv_fwd
    three times, gdn_chunk_fwd_layer) against the same operations done
    separately in torch around the op, as the reference layer does them."""
    import torch
    import torch.nn.functional as F
    from gated_deltanet_jax_b200 import ops
    B, T, H, dk, dv, KC = 8, 2048, 6, 256, 512, 4
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(5150 + d.rank)
    # raw projection outputs scaled so that the convolved keys and queries have
    # norms of order one (the reference normalises neither)
    xq = (torch.randn(B, T, H * dk, device=d.dev, generator=gen) / dk ** 0.5).bfloat16()
    xk = (torch.randn(B, T, H * dk, device=d.dev, generator=gen) / dk ** 0.5).bfloat16()
    xv = torch.randn(B, T, H * dv, device=d.dev, generator=gen).bfloat16()
    wq, wk, wv = (torch.randn(KC, c, device=d.dev, generator=gen) * 0.5
                  for c in (H * dk, H * dk, H * dv))
    ra = torch.randn(B, T, H, device=d.dev, generator=gen)
    rb = torch.randn(B, T, H, device=d.dev, generator=gen)
    gate = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    A_log, dt_bias = _layer_gate_params(H, d.dev, gen)
    w = torch.ones(dv, device=d.dev)
    hT = torch.empty(B, H, dk, dv, device=d.dev)

    def fused():
        q, _ = ops.short_convolution(xq, wq)
        k, _ = ops.short_convolution(xk, wk)
        v, _ = ops.short_convolution(xv, wv)
        ops.gated_delta_rule_chunk_layer(q.view(B, T, H, dk), k.view(B, T, H, dk),
                                         v.view(B, T, H, dv), ra, rb, A_log, dt_bias,
                                         gate=gate, norm_weight=w, final_state_out=hT)

    def conv_t(x, wt):   # depthwise causal conv1d + SiLU, as separate torch operations
        C = x.shape[-1]
        y = F.conv1d(F.pad(x.transpose(1, 2), (KC - 1, 0)), wt.t().unsqueeze(1).to(x.dtype),
                     groups=C)
        return F.silu(y).transpose(1, 2)

    def unfused():
        q = conv_t(xq, wq).reshape(B, T, H, dk)
        k = conv_t(xk, wk).reshape(B, T, H, dk)
        v = conv_t(xv, wv).reshape(B, T, H, dv)
        gd = -torch.exp(A_log) * F.softplus(ra + dt_bias)
        bd = torch.sigmoid(rb)
        o, _ = ops.chunk_gated_delta_rule(q, k, v, gd, bd, final_state_out=hT)
        x = o.float()
        var = x.pow(2).mean(-1, keepdim=True)
        (x * torch.rsqrt(var + 1e-5) * w * F.silu(gate.float())).to(o.dtype)

    REP = 4
    res = {}
    steps = max(1, min(a.steps, 20))
    for name, fn in (("fused", fused), ("unfused", unfused)):
        fn()                                   # load modules, allocate
        torch.cuda.synchronize(d.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(REP):
                fn()
        for _ in range(a.warmup):
            graph.replay()
        ms, _ = _timed(d, graph.replay, steps)
        res[name] = ms / REP
        del graph
    return {"workload": "the layer core at the reference's default head dims, B=8 T=2048 H=6 "
                        "dk=256 dv=512 bf16: short conv (kernel 4) + SiLU of the raw q/k/v "
                        "projections, gates from raw a/b projections, chunked forward, gated "
                        "RMSNorm (eps 1e-5) of every output row; final state out; 4 calls per "
                        "CUDA graph",
            "fused_ms": res["fused"], "unfused_ms": res["unfused"],
            "speedup": res["unfused"] / res["fused"],
            # fused: three convolutions, the chunk kernel, the in-place norm
            "launches": 5 * REP * steps,
            "fused_tokens_per_s": d.world * B * T / (res["fused"] / 1e3),
            "path": "fused: gdn_short_conv_fwd x3, gdn_chunk_fwd_layer (the dk=256 tcgen05 "
                    "kernel forms the gates; a second launch normalises the output in place); "
                    "unfused: torch conv1d + SiLU, torch gates, gdn_chunk_fwd, torch gated "
                    "RMSNorm"}


def model_core_leg(d, a):
    """The delta-rule core of the reference's default model configuration
    (head_dim 256, expand_v 2: dk=256, dv=512; 6 heads; B=8 T=2048 as the
    full-model configuration quotes): the chunked forward in bf16 and in
    fp32, and the bf16 backward, per layer call (the full model: model_forward_leg)."""
    import torch
    from gated_deltanet_jax_b200 import ops
    from gated_deltanet_jax_b200 import roofline as rl
    B, T, H, dk, dv = 8, 2048, 6, 256, 512
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(97 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1)
    k = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1)
    v = torch.randn(B, T, H, dv, device=d.dev, generator=gen)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    qb, kb, vb = q.bfloat16(), k.bfloat16(), v.bfloat16()
    do = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    steps = max(1, min(a.steps, 10))
    res = {}
    for name, fn in (("fwd_bf16", lambda: ops.chunk_gated_delta_rule(qb, kb, vb, g, beta)),
                     ("fwd_fp32", lambda: ops.chunk_gated_delta_rule(q, k, v, g, beta)),
                     ("bwd_bf16", lambda: ops._chunk_backward(qb, kb, vb, g, beta, None, do,
                                                              None))):
        for _ in range(a.warmup):
            fn()
        ms, _ = _timed(d, fn, steps)
        res[name] = ms
    th = B * T * H
    fl_f = th * rl.flops_chunk_per_token_head(dk, dv, 64)
    fl_b = th * rl.flops_chunk_bwd_per_token_head(dk, dv, 64)
    return {"workload": "delta-rule core of the reference's default configuration: B=8 T=2048 "
                        "H=6 dk=256 dv=512 chunk=64, one layer call",
            "fwd_bf16_ms": res["fwd_bf16"], "fwd_bf16_tflops": fl_f / res["fwd_bf16"] / 1e9,
            "fwd_fp32_ms": res["fwd_fp32"], "fwd_fp32_tflops": fl_f / res["fwd_fp32"] / 1e9,
            "bwd_bf16_ms": res["bwd_bf16"], "bwd_bf16_tflops": fl_b / res["bwd_bf16"] / 1e9,
            "fwd_plus_bwd_bf16_tokens_per_s": d.world * B * T / ((res["fwd_bf16"]
                                                                  + res["bwd_bf16"]) / 1e3),
            "launches": steps * (1 + 3 + 3),
            "path": "bf16 forward: tcgen05 kernel (dk=256 form); fp32 forward: warp-level "
                    "tensor-core kernels (three-term tf32); backward: gdn_chunk_bwd"}


def model_forward_leg(d, a):
    """The full GatedDeltaNetModel forward at the reference's model configuration
    (hidden 2048, 24 layers, 6 heads, head_dim 256, expand_v 2, short convolution
    4, SiLU output gate, RMSNorm, vocab 32000) on B=8 T=2048 token ids: the
    embedding, 24 blocks and the final norm, random init at Flax's default
    scales, bf16.  Projections and MLPs are cuBLAS GEMMs; the short convolutions
    and each layer's gates + chunked delta rule + gated RMSNorm run on this
    library's kernels.  Like the reference (no q/k normalisation in its layer),
    the recurrence overflows at these statistics: a throughput configuration;
    the line reports the fraction of finite outputs."""
    import torch
    from gated_deltanet_jax_b200 import GatedDeltaNetConfig
    from gated_deltanet_jax_b200.model import GatedDeltaNetModel
    B, T = 8, 2048
    cfg = GatedDeltaNetConfig(hidden_size=2048, num_hidden_layers=24, num_heads=6, head_dim=256,
                              expand_v=2.0, conv_size=4, vocab_size=32000, attn_mode="chunk")
    torch.manual_seed(31 + d.rank)
    with torch.device(d.dev):
        model = GatedDeltaNetModel(cfg).to(torch.bfloat16).eval()
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(37 + d.rank)
    ids = torch.randint(0, cfg.vocab_size, (B, T), device=d.dev, generator=gen)
    out = {}

    def step():
        out["x"] = model(ids)

    steps = max(1, min(a.steps, 3))
    with torch.no_grad():
        for _ in range(max(1, min(a.warmup, 2))):
            step()
        ms, _ = _timed(d, step, steps)
    finite = float(torch.isfinite(out["x"]).float().mean())
    nparam = sum(p.numel() for p in model.parameters())
    del model, out
    torch.cuda.empty_cache()
    return {"metric": "full-model forward tokens/s", "value": d.world * B * T / (ms / 1e3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "config": {"workload": "GatedDeltaNetModel forward, hidden 2048, 24 layers, 6 heads, "
                                   "head_dim 256 (dk=256 dv=512), short conv 4, gated RMSNorm, "
                                   "vocab 32000; B=8 T=2048 token ids, bf16, random init",
                       "parameters": nparam},
            "finite_fraction": finite,
            "path": "torch embedding/RMSNorm/GEMMs (cuBLAS); per layer: short convolutions "
                    "(gdn_short_conv_fwd) and gdn_chunk_fwd_layer (gates, tcgen05 dk=256 "
                    "chunk kernel, gated RMSNorm)"}


def backward_leg(d, a, lib):
    """The chunked backward (gdn_chunk_bwd) on the prefill workload: gradients of
    q, k, v, g, beta from dO, every buffer resident, one C-ABI call per step."""
    import torch
    from gated_deltanet_jax_b200 import _lib, roofline as rl
    B, T, H, dk, dv, C = (PRE[x] for x in ("B", "T", "H", "dk", "dv", "chunk"))
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(199 + d.rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))
    do = torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16()
    dq, dk_, dv_ = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg, db = torch.empty_like(g), torch.empty_like(beta)
    ws_bytes = lib.gdn_chunk_bwd_workspace_bytes_for(B, T, H, H, dk, dv, _lib.GDN_DTYPE_BF16)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=d.dev)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        rc = lib.gdn_chunk_bwd(ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), None, ptr(do), None,
                               ptr(dq), ptr(dk_), ptr(dv_), ptr(dg), ptr(db), None,
                               B, T, H, H, dk, dv, _lib.GDN_DTYPE_BF16, ptr(ws), ws_bytes,
                               ctypes.c_void_p(torch.cuda.current_stream(d.dev).cuda_stream))
        if rc:
            _lib.check(rc, "gdn_chunk_bwd")

    for _ in range(a.warmup):
        step()
    steps = max(1, min(a.steps, 30))
    ms, _ = _timed(d, step, steps)
    flops = B * T * H * rl.flops_chunk_bwd_per_token_head(dk, dv, C)
    return {"metric": "chunk backward tokens/s", "value": d.world * B * T / (ms / 1e3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "launches": 4 * steps,
            "config": {"workload": "gradients of q, k, v, g, beta for B=4 T=4096 H=16 "
                                   "dk=dv=128, bf16 in, from a bf16 dO, no initial state",
                       "l2": f"inputs and {ws_bytes / 1e9:.2f} GB of workspace, larger than L2",
                       "path": "gdn_chunk_bwd: per-chunk preparation (with T), forward "
                               "state pass (scan), reverse state pass (reverse scan), per-chunk "
                               "gradients (4 launches, bf16 hand-off in the workspace)"},
            "algorithmic_flops_per_step": flops,
            "achieved_tflops": flops / (ms / 1e3) / 1e12,
            "compute": "tcgen05 tensor cores (bf16 operands staged by TMA, fp32 accumulation "
                       "in TMEM) in all four kernels"}


def long_context_leg(d, a):
    """B=1, T=65536, H=16 over all ranks (strong scaling: the sequence is split
    evenly across ranks, the state handed off by an NCCL all-gather), each rank's
    segment split again into parts on its GPU.  Every rank generates the whole
    sequence from one seed and keeps its segment, so that after the timed region
    each rank can check its outputs and the final state against one unsplit
    launch over the whole sequence on its own GPU (max over ranks reported)."""
    import torch
    from gated_deltanet_jax_b200 import ops, sequence_parallel as sp
    from gated_deltanet_jax_b200 import roofline as rl
    B, T, H, dk, dv, C = (LONG[x] for x in ("B", "T", "H", "dk", "dv", "chunk"))
    seg = T // d.world
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(7)
    nrm = torch.nn.functional.normalize
    full = [nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16(),
            nrm(torch.randn(B, T, H, dk, device=d.dev, generator=gen), dim=-1).bfloat16(),
            torch.randn(B, T, H, dv, device=d.dev, generator=gen).bfloat16(),
            torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=d.dev, generator=gen)),
            torch.sigmoid(torch.randn(B, T, H, device=d.dev, generator=gen))]
    sl = slice(d.rank * seg, (d.rank + 1) * seg)
    q, k, v, g, beta = (x[:, sl].contiguous() for x in full)
    # one GPU: the split is timed against the direct launch below; several GPUs:
    # segments per GPU chosen so that the second pass fills the GPU
    local_parts = (LONG["parts"] if d.world == 1 else
                   sp.auto_local_parts(B, seg, H, dv, C, torch.device(d.dev)))

    def split(marks=None):
        if d.world == 1:
            return sp.chunk_gated_delta_rule_split(q, k, v, g, beta, output_final_state=True,
                                                   parts=local_parts, marks=marks)
        return sp.chunk_gated_delta_rule_sp(q, k, v, g, beta, output_final_state=True,
                                            local_parts=local_parts, marks=marks)

    for _ in range(a.warmup):
        split()
    steps = max(1, min(a.steps, 20))
    ms, _ = _timed(d, split, steps)
    # per-phase times of the split (outside the timed region, max over ranks)
    phase_ms = {}
    for _ in range(3):
        marks = []
        start = torch.cuda.Event(enable_timing=True)
        start.record()
        split(marks)
        torch.cuda.synchronize(d.dev)
        prev = start
        for name, ev in marks:
            phase_ms[name] = phase_ms.get(name, 0.0) + prev.elapsed_time(ev) / 3
            prev = ev
    phase_ms = {n: d.max(t) for n, t in phase_ms.items()}
    path = (f"sequence split over {d.world} GPU(s) x {local_parts} segment(s) per GPU"
            if d.world > 1 or local_parts > 1 else "one launch")
    extra = {"split_phase_ms": phase_ms}
    direct = lambda: ops.chunk_gated_delta_rule(  # noqa: E731
        *full, output_final_state=True)
    if d.world == 1:
        # On one GPU the split is an option, not a necessity: time the direct launch
        # too and report whichever path is faster for this workload.
        for _ in range(a.warmup):
            direct()
        ms_d, _ = _timed(d, direct, steps)
        extra.update({"split_ms_per_step": ms, "unsplit_ms_per_step": ms_d})
        if ms_d < ms:
            ms, path = ms_d, "one launch (no split)"
    # Correctness of the split against one unsplit launch (outside the timed
    # region).  The workload's gates decay the state by about e^-51 per chunk, so
    # almost nothing crosses a segment boundary; the check therefore runs on the
    # same inputs with gates 50x milder (about e^-1 per chunk), whose state spans
    # every boundary.
    full[3] = full[3] * 0.02
    g = full[3][:, sl].contiguous()
    o_s, h_s = split()
    o_ref, h_ref = direct()
    rel = lambda x, r: float((x.float() - r.float()).abs().max() / r.float().abs().max())  # noqa: E731
    extra["max_rel_err"] = {"o": d.max(rel(o_s, o_ref[:, sl])), "state": d.max(rel(h_s, h_ref)),
                            "against": "one unsplit launch over the whole sequence (every rank, "
                                       "its own segment of o; max over ranks), gates x 0.02"}
    flops = T * H * rl.flops_chunk_per_token_head(dk, dv, C)
    res = {"metric": "long-context chunk prefill tokens/s", "value": B * T / (ms / 1e3),
           "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "scaling": "strong",
           "config": {"workload": f"B=1 T={T} H=16 dk=dv=128 chunk=64 bf16, final state out",
                      "path": path, "parallelism": f"sequence split sp{d.world}"},
           "algorithmic_tflops": flops / (ms / 1e3) / 1e12,
           # two launches per chunked call: the split's two passes per step, and (one
           # GPU) the direct call per step
           "launches": 4 * steps + (2 * steps if d.world == 1 else 0)}
    res.update(extra)
    return res


def profile_workload(a):
    """Run one fixed workload ``a.launches`` times on cuda:0 for an ncu capture.

    decode: B=64 H=16 dk=dv=128, bf16 q/k/v, fp32 state ~N(0,0.02) updated in
    place, one token per launch.  prefill: B=4 T=4096 H=16 dk=dv=128, bf16 in,
    fp32 final state out.  backward: gradients of q, k, v, g, beta for the
    prefill workload from a bf16 dO, no initial state.  prefill_layer: the
    prefill workload through gdn_chunk_fwd_layer (gates from raw a/b
    projections initialised as the layer does, a bf16 output gate, norm
    weight 1, eps 1e-5).
    """
    import math
    import torch
    from gated_deltanet_jax_b200 import ops
    dev = torch.device("cuda:0")

    def inputs(B, T, seed):
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        nrm = torch.nn.functional.normalize
        q = nrm(torch.randn(B, T, a.H, a.dk, device=dev, generator=gen), dim=-1).bfloat16()
        k = nrm(torch.randn(B, T, a.H, a.dk, device=dev, generator=gen), dim=-1).bfloat16()
        v = torch.randn(B, T, a.H, a.dv, device=dev, generator=gen).bfloat16()
        g = torch.nn.functional.logsigmoid(torch.randn(B, T, a.H, device=dev, generator=gen))
        beta = torch.sigmoid(torch.randn(B, T, a.H, device=dev, generator=gen))
        return q, k, v, g, beta

    w = a.profile_workload
    if w == "decode":
        B = a.B or 64
        q, k, v, g, beta = inputs(B, 1, 0)
        S = torch.randn(B, a.H, a.dk, a.dv, device=dev) * 0.02
        run = lambda: ops.fused_recurrent_gated_delta_rule(  # noqa: E731
            q, k, v, g, beta, initial_state=S, final_state_out=S)
    elif w == "prefill":
        q, k, v, g, beta = inputs(a.B or 4, a.T or 4096, 0)
        run = lambda: ops.chunk_gated_delta_rule(  # noqa: E731
            q, k, v, g, beta, output_final_state=True)
    elif w == "prefill_layer":
        B, T = a.B or 4, a.T or 4096
        q, k, v, ra, rb = inputs(B, T, 0)
        gen = torch.Generator(device=dev)
        gen.manual_seed(2)
        gate = torch.randn(B, T, a.H, a.dv, device=dev, generator=gen).bfloat16()
        A_log = torch.log(torch.rand(a.H, device=dev, generator=gen) * 16 + 1e-4)
        u = torch.rand(a.H, device=dev, generator=gen)
        dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
        dt_bias = dt + torch.log(-torch.expm1(-dt))
        run = lambda: ops.gated_delta_rule_chunk_layer(  # noqa: E731
            q, k, v, ra, rb, A_log, dt_bias, gate=gate, output_final_state=True)
    else:
        B, T = a.B or 4, a.T or 4096
        q, k, v, g, beta = inputs(B, T, 0)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1)
        do = torch.randn(B, T, a.H, a.dv, device=dev, generator=gen).bfloat16()
        run = lambda: ops._chunk_backward(q, k, v, g, beta, None, do, None)  # noqa: E731
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    print(f"{w}: {a.launches} launches in {time.perf_counter() - t0:.3f} s")


def main():
    a = _args()
    if a.profile_workload:
        profile_workload(a)
        return
    if a.impl == "reference":
        run_reference_arm(a)
        return
    if a.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    import torch
    from gated_deltanet_jax_b200 import _lib
    lib = _lib.load()
    d = Dist()
    peaks, peak_src = _peaks()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(d.dev).uuid)
    except Exception:
        pass

    dec = decode_leg(d, a, lib, uuid)
    pre = None if a.no_prefill else prefill_leg(d, a, lib, uuid)
    lng = None if a.no_long else long_context_leg(d, a)
    bwd = None if a.no_backward else backward_leg(d, a, lib)
    lay = None if a.no_layer else decode_layer_leg(d, a)
    play = None if (a.no_layer or a.no_prefill) else prefill_layer_leg(d, a)
    pdef = None if (a.no_layer or a.no_prefill) else prefill_layer_default_leg(d, a)
    mcore = None if a.no_prefill else model_core_leg(d, a)
    mfwd = None if (a.no_layer or a.no_prefill) else model_forward_leg(d, a)

    cpu = None
    if d.rank == 0 and d.world == 1 and not a.no_cpu:
        cpu = cpu_decode_baseline()
        cpu_pre = None if a.no_prefill else cpu_prefill_baseline()

    if d.rank == 0:
        hbm = float(peaks["hbm_gbs"])
        ach = dec["bytes_launch"] / dec["launch_s"] / 1e9
        traffic = _profile_traffic("recurrent_decode_b64_h16_d128")
        line = {
            "metric": "recurrent decode tokens/s", "value": dec["value"], "unit": "tokens/s",
            "n_gpus": d.world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": dec["ms"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "fused recurrent decode: B=64 H=16 dk=dv=128, bf16 q/k/v, "
                                   "fp32 state ~N(0,0.02) updated in place; one step = 512 "
                                   "consecutive decode tokens (512 launches, one CUDA graph), "
                                   f"round robin over {NBUF} independent 64 MiB states",
                       "global_batch": DEC["B"] * d.world, "seq_len": DEC["tokens"],
                       "parallelism": f"batch x head over {d.world} GPU(s), no collective",
                       "l2": f"inputs larger than L2 ({NBUF} x 64 MiB fp32 states and "
                             "400 MB of q/k/v per step)"},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "peak_source": f"{peak_src} hbm_gbs",
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": dec["bytes_launch"]},
            "gpu_launches": (dec["launches"] + (pre["launches"] if pre else 0)
                             + (bwd["launches"] if bwd else 0) + (lay["launches"] if lay else 0)
                             + (play["launches"] if play else 0)
                             + (pdef["launches"] if pdef else 0)
                             + (mcore["launches"] if mcore else 0)
                             + (lng["launches"] if lng else 0)),
            "clocks": dec["clocks"],
        }
        if "e2e" in dec:
            line["e2e"] = dec["e2e"]
        line["single_state"] = dec["single_state"]
        if cpu:
            line["cpu_baseline"] = cpu
        if pre:
            tf = pre["flops_launch"] / pre["launch_s"] / 1e12
            bf16 = float(peaks["bf16_tflops"])
            pre_line = {
                "metric": "chunk prefill tokens/s", "value": pre["value"], "unit": "tokens/s",
                "ms_per_step": pre["ms"], "steps": pre["steps"], "clocks": pre["clocks"],
                "config": {"workload": "chunked prefill B=4 T=4096 H=16 dk=dv=128 chunk=64, "
                                       "bf16 in, fp32 state, final state out",
                           "l2": "inputs larger than L2 (201 MB q/k/v per GPU)"},
                "roofline": {"bound": "tensor", "achieved": tf, "peak": bf16, "unit": "TFLOP/s",
                             "frac": tf / bf16, "peak_source": f"{peak_src} bf16_tflops (burst)",
                             "traffic": _profile_traffic("chunk_scan_two_launch_b4_t4096_h16_d128"),
                             "traffic_note": "DRAM bytes of one call (both launches) from ncu",
                             "algorithmic_flops_per_launch": pre["flops_launch"],
                             "hbm_achieved_gbs": pre["bytes_launch"] / pre["launch_s"] / 1e9,
                             # min(peak, arithmetic intensity x HBM bandwidth): the attainable
                             # FLOP/s at this kernel's FLOP per algorithmic byte
                             "ai_flop_per_byte": pre["flops_launch"] / pre["bytes_launch"],
                             "frac_of_attainable": tf / min(bf16, pre["flops_launch"]
                                                            / pre["bytes_launch"] * hbm / 1e3)},
            }
            if "kernels" in pre:
                pre_line["kernels"] = pre["kernels"]
            if "e2e" in pre:
                pre_line["e2e"] = pre["e2e"]
            if cpu and cpu_pre:
                pre_line["cpu_baseline"] = cpu_pre
            line["prefill"] = pre_line
        if lng:
            line["long_context"] = lng
        if lay:
            line["decode_layer"] = lay
        if play:
            line["prefill_layer"] = play
        if pdef:
            line["prefill_layer_default_dims"] = pdef
        if mcore:
            line["model_config_core"] = mcore
        if mfwd:
            line["model_forward"] = mfwd
        if bwd:
            if pre:
                bwd["fwd_plus_bwd_tokens_per_s"] = (d.world * PRE["B"] * PRE["T"]
                                                    / ((pre["ms"] + bwd["ms_per_step"]) / 1e3))
            line["backward"] = bwd
        print(json.dumps(line), flush=True)
    d.close()


if __name__ == "__main__":
    main()
