"""Shared helpers for the GPU parity tests: move seeded oracle inputs to the
device in a given dtype, and read device tensors back as float64 for the
oracle (so the oracle sees exactly the values the kernel saw)."""

import numpy as np
import torch

from oracle import gdn_oracle as orc

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def to_dev(x, dtype, dev):
    return torch.as_tensor(np.asarray(x, np.float32)).to(dev).to(dtype).contiguous()


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def device_inputs(B, T, H, dk, dv, seed, dtype, dev, h0_std=None):
    """Seeded inputs on the device; returns (device tensors, float64 copies)."""
    q, k, v, g, beta, h0 = orc.make_inputs(B, T, H, dk, dv, seed=seed, h0_std=h0_std)
    tq, tk, tv = (to_dev(x, DT[dtype], dev) for x in (q, k, v))
    tg, tb = to_dev(g, torch.float32, dev), to_dev(beta, torch.float32, dev)
    th0 = None if h0 is None else to_dev(h0, torch.float32, dev)
    host = [f64(t) for t in (tq, tk, tv, tg, tb)] + [None if th0 is None else f64(th0)]
    return (tq, tk, tv, tg, tb, th0), host


def device_inputs_fast(B, T, H, dk, dv, seed, dtype, dev, h0_std=None):
    """Full-size inputs generated on the device with torch (same distributions)."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    q = torch.randn(B, T, H, dk, device=dev, generator=gen)
    k = torch.randn(B, T, H, dk, device=dev, generator=gen)
    v = torch.randn(B, T, H, dv, device=dev, generator=gen)
    beta = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=gen))
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=dev, generator=gen))
    q = torch.nn.functional.normalize(q, dim=-1).to(DT[dtype]).contiguous()
    k = torch.nn.functional.normalize(k, dim=-1).to(DT[dtype]).contiguous()
    v = v.to(DT[dtype]).contiguous()
    h0 = None
    if h0_std is not None:
        h0 = (torch.randn(B, H, dk, dv, device=dev, generator=gen) * h0_std).contiguous()
    return q, k, v, g.contiguous(), beta.contiguous(), h0


def assert_close(out, ref, dtype, what=""):
    ok, err = orc.within_tolerance(out, ref, dtype)
    kind = "max-abs" if dtype == "fp32" else "rel"
    assert ok, f"{what}: {kind} error {err:.3e} over the {dtype} tolerance"
    return err


def torch_recurrent_step_fp32(q, k, v, g, beta, S):
    """Plain PyTorch fp32 reference of one decode step for every (b, h).

    q,k [B,H,dk], v [B,H,dv], g,beta [B,H], S [B,H,dk,dv] (fp32) -> (o, S')."""
    q, k, v = q.float(), k.float(), v.float()
    S = S * torch.exp(g)[..., None, None]
    proj = torch.einsum("bhk,bhkv->bhv", k, S)
    u = (v - proj) * beta[..., None]
    S = S + k[..., :, None] * u[..., None, :]
    o = torch.einsum("bhkv,bhk->bhv", S, q)
    return o, S
