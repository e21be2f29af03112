"""Fixed workloads for profiling the kernels with ncu (one process, one GPU).

    python -m gated_deltanet_jax_b200._profile decode  --launches 3
    python -m gated_deltanet_jax_b200._profile prefill --launches 2 [--B 4 --T 4096]
    python -m gated_deltanet_jax_b200._profile backward --launches 2 [--B 4 --T 4096]
    python -m gated_deltanet_jax_b200._profile prefill_layer --launches 2 [--B 4 --T 4096]

decode:  B=64 H=16 dk=dv=128, bf16 q/k/v, fp32 state ~N(0,0.02) updated in
         place, one token per launch (the decode workload of bench.py).
prefill: B=4 T=4096 H=16 dk=dv=128 chunk=64, bf16 in, fp32 final state out.
backward: gradients of q, k, v, g, beta for the prefill workload from a bf16
         dO, no initial state (one gdn_chunk_bwd call per launch).
prefill_layer: the prefill workload through gdn_chunk_fwd_layer: gates from raw
         a/b projections (A_log, dt_bias as the layer initialises them), a bf16
         output gate, norm weight 1, eps 1e-5, final state out.
"""

from __future__ import annotations

import argparse
import math
import sys
import time

import torch

from . import ops


def _inputs(B, T, H, dk, dv, seed, dev):
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, dk, device=dev, generator=gen), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, dk, device=dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, dv, device=dev, generator=gen).bfloat16()
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=dev, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=gen))
    return q, k, v, g, beta


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("workload", choices=["decode", "prefill", "backward", "prefill_layer"])
    p.add_argument("--launches", type=int, default=3)
    p.add_argument("--B", type=int, default=None)
    p.add_argument("--T", type=int, default=None)
    p.add_argument("--H", type=int, default=16)
    p.add_argument("--dk", type=int, default=128)
    p.add_argument("--dv", type=int, default=128)
    a = p.parse_args(argv)
    dev = torch.device("cuda:0")
    if a.workload == "decode":
        B = a.B or 64
        q, k, v, g, beta = _inputs(B, 1, a.H, a.dk, a.dv, 0, dev)
        S = torch.randn(B, a.H, a.dk, a.dv, device=dev) * 0.02
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.launches):
            ops.fused_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=S,
                                                 final_state_out=S)
    elif a.workload == "prefill":
        B, T = a.B or 4, a.T or 4096
        q, k, v, g, beta = _inputs(B, T, a.H, a.dk, a.dv, 0, dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.launches):
            ops.chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True)
    elif a.workload == "prefill_layer":
        B, T = a.B or 4, a.T or 4096
        q, k, v, ra, rb = _inputs(B, T, a.H, a.dk, a.dv, 0, dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(2)
        gate = torch.randn(B, T, a.H, a.dv, device=dev, generator=gen).bfloat16()
        A_log = torch.log(torch.rand(a.H, device=dev, generator=gen) * 16 + 1e-4)
        u = torch.rand(a.H, device=dev, generator=gen)
        dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
        dt_bias = dt + torch.log(-torch.expm1(-dt))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.launches):
            ops.gated_delta_rule_chunk_layer(q, k, v, ra, rb, A_log, dt_bias, gate=gate,
                                             output_final_state=True)
    else:
        B, T = a.B or 4, a.T or 4096
        q, k, v, g, beta = _inputs(B, T, a.H, a.dk, a.dv, 0, dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1)
        do = torch.randn(B, T, a.H, a.dv, device=dev, generator=gen).bfloat16()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.launches):
            ops._chunk_backward(q, k, v, g, beta, None, do, None)
    torch.cuda.synchronize()
    print(f"{a.workload}: {a.launches} launches in {time.perf_counter() - t0:.3f} s")
    return 0


if __name__ == "__main__":
    sys.exit(main())
