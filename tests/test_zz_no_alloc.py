"""The allocation-free backward, gdn_chunk_bwd_noalloc, through the C ABI.

It exists for callers that cannot allocate device memory or pass a workspace
(a custom call inside a framework that owns the device memory and gives it no
scratch, a loop that must not stop for cudaMalloc): its scratch is one fixed
array of the library's own device memory that every call on a GPU shares.  So the check is that consecutive
calls each give what gdn_chunk_bwd gives with a workspace of its own on the
same inputs, whatever the previous call left in the array: first the largest
size the array holds, then a smaller call in another dtype (whose
accumulators sit where the first call's were), then the first inputs again.

This file is named to be collected last, so that a run stopping at its first
failure has run every other test before it; it passes on its own too."""

import pytest
import torch

from gated_deltanet_jax_b200 import _lib
from oracle import gdn_oracle as orc
from helpers import device_inputs_fast, f64

pytestmark = pytest.mark.gpu

# Relative to each gradient's largest entry, as the backward's other tests:
# fp32 inputs within 1e-3, bf16 inputs within 2e-2.
TOL = {"fp32": 1e-3, "bf16": 2e-2}
SCRATCH_BYTES = 64 << 20        # GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES


def _p(t):
    return None if t is None else t.data_ptr()


def _problem(B, T, H, Hk, dk, dv, dtype, seed, dev, with_state):
    q, k, v, g, b, h0 = device_inputs_fast(B, T, H, dk, dv, seed=seed, dtype=dtype, dev=dev,
                                           h0_std=0.05 if with_state else None)
    rep = H // Hk
    q, k = q[:, :, ::rep].contiguous(), k[:, :, ::rep].contiguous()
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    do = torch.randn(B, T, H, dv, device=dev, generator=gen).to(v.dtype)
    dhT = torch.randn(B, H, dk, dv, device=dev, generator=gen) if with_state else None
    return dict(ins=(q, k, v, g, b, h0, do, dhT), dims=(B, T, H, Hk, dk, dv),
                dtype=_lib.GDN_DTYPE_BF16 if dtype == "bf16" else _lib.GDN_DTYPE_FP32)


def _outputs(pr):
    q, k, v, g = pr["ins"][:4]
    B, T, H, Hk, dk, dv = pr["dims"]
    f32 = dict(dtype=torch.float32, device=q.device)
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            torch.empty(B, T, H, **f32), torch.empty(B, T, H, **f32),
            torch.empty(B, H, dk, dv, **f32))


def _call(lib, pr, no_alloc):
    outs = _outputs(pr)
    args = [_p(t) for t in pr["ins"]] + [_p(t) for t in outs] + list(pr["dims"]) + [pr["dtype"]]
    stream = torch.cuda.current_stream().cuda_stream
    if no_alloc:
        rc = lib.gdn_chunk_bwd_noalloc(*args, stream)
        _lib.check(rc, "gdn_chunk_bwd_noalloc")
    else:
        B, T, H, Hk, dk, dv = pr["dims"]
        ws_bytes = lib.gdn_chunk_bwd_workspace_bytes(B, T, H, dk, dv)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=pr["ins"][0].device)
        rc = lib.gdn_chunk_bwd(*args, ws.data_ptr(), ws_bytes, stream)
        _lib.check(rc, "gdn_chunk_bwd")
    torch.cuda.synchronize()
    return outs


def _largest_T(lib, B, H, Hk, dk, dv, dtype):
    """Longest sequence whose backward scratch (this call's exact size) fits
    the fixed array (the scratch size grows with T)."""
    need = lambda T: lib.gdn_chunk_bwd_workspace_bytes_for(B, T, H, Hk, dk, dv, dtype)  # noqa: E731
    lo, hi = 1, 1
    while need(hi) <= SCRATCH_BYTES:
        lo, hi = hi, hi * 2
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if need(mid) <= SCRATCH_BYTES:
            lo = mid
        else:
            hi = mid
    return lo


def test_no_alloc_matches_workspace_entry_on_consecutive_calls(cuda):
    lib = _lib.load()
    T_max = _largest_T(lib, 1, 16, 8, 128, 128, _lib.GDN_DTYPE_BF16)
    largest = _problem(1, T_max, 16, 8, 128, 128, "bf16", seed=11, dev=cuda, with_state=True)
    smaller = _problem(2, 100, 3, 3, 64, 64, "fp32", seed=12, dev=cuda, with_state=False)
    names = ("dq", "dk", "dv", "dg", "dbeta", "dh0")
    for step, (pr, dt) in enumerate([(largest, "bf16"), (smaller, "fp32"), (largest, "bf16")]):
        got = _call(lib, pr, no_alloc=True)
        want = _call(lib, pr, no_alloc=False)
        for n, a, r in zip(names, got, want):
            # the backward is deterministic (no atomics, fixed summation order),
            # so the scratch's address must not change a single bit; the bar
            # the other tests use is reported for a mismatch
            assert torch.equal(a, r), (f"call {step}: {n} differs, rel error "
                                       f"{orc.rel_err(f64(a), f64(r)):.2e} (bar {TOL[dt]})")
    assert lib.gdn_device_error(1) == 0


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda):
    """One token more than the largest size above needs more than the fixed
    array: refused before any pointer is read or anything is launched."""
    lib = _lib.load()
    T = _largest_T(lib, 1, 16, 16, 128, 128, _lib.GDN_DTYPE_BF16) + 1
    assert lib.gdn_chunk_bwd_workspace_bytes_for(1, T, 16, 16, 128, 128,
                                                 _lib.GDN_DTYPE_BF16) > SCRATCH_BYTES
    rc = lib.gdn_chunk_bwd_noalloc(*([None] * 14), 1, T, 16, 16, 128, 128,
                                   _lib.GDN_DTYPE_BF16, None)
    assert rc == _lib.GDN_ERR_UNSUPPORTED
    assert b"fixed" in lib.gdn_last_error()
