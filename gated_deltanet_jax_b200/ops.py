"""Gated delta-rule ops with the reference package's names and signatures.

Mirrors ``gated_deltanet_jax.ops`` (reference ``src/gated_deltanet_jax/ops.py``):

* :func:`chunk_gated_delta_rule_fwd` / :func:`chunk_gated_delta_rule`
  -- ops.py:299 and its alias at ops.py:352;
* :func:`fused_recurrent_gated_delta_rule` / :func:`fused_recurrent_gated_delta_rule_fwd`
  -- the Pallas wrapper ops.py:187 and its aliases at ops.py:350-351.

Arrays are CUDA ``torch.Tensor`` s in the reference layout (q, k ``[B,T,H,dk]``,
v ``[B,T,H,dv]``, g, beta ``[B,T,H]``, states ``[B,H,dk,dv]``).  Every call
goes through the C ABI of ``libgdn_b200.so`` on the tensor's current CUDA
stream; there is no CPU path.  Both ops compute the delta-rule recurrence
(the reference's recurrent kernel, ops.py:170-184) with an fp32 state and
return ``o`` in v's dtype.

Differences from the reference, all additive:

* ``fused_recurrent_gated_delta_rule`` also accepts ``initial_state`` and
  ``output_final_state`` (the reference always starts from zeros and returns
  ``(o, None)``, ops.py:168/219); without them it behaves the same.
* ``final_state_out=`` writes the final state into a given fp32 tensor, which
  may be ``initial_state`` itself (in-place decode).
* ``semantics="reference"`` on the chunk op reproduces ops.py:238-346 as
  written, including its deviations from the recurrence.
* Grouped value heads: q and k may carry fewer heads (Hk) than v, g and beta
  (H, a multiple of Hk).  Value head h then uses q/k head ``h * Hk // H``,
  which is what the reference layer obtains by ``jnp.repeat`` of q and k
  before calling its ops (model.py:132-135), without the repeated copies.
* ``cu_seqlens=`` on the chunk op: several sequences packed back to back in
  one row (q ``[1,T,Hk,dk]`` ...), sequence s being tokens
  ``cu_seqlens[s]:cu_seqlens[s+1]``, with one state per sequence.  Each
  sequence gets what a call on it alone gives.  (The reference takes one
  dense batch only.)
* Both ops are differentiable (exact semantics; the chunk op also with
  ``cu_seqlens``): when an input requires grad, the backward runs the
  gdn_chunk_bwd kernels (gdn_chunk_bwd_varlen for packed sequences).  The
  reference has no backward of its own; it differentiates its chunk path with
  JAX.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GDN_DTYPE_FP32, torch.bfloat16: _lib.GDN_DTYPE_BF16}
_SEMANTICS = {"exact": _lib.GDN_SEMANTICS_EXACT, "reference": _lib.GDN_SEMANTICS_REFERENCE}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _prepare(q, k, v, g, beta, initial_state, final_state_out, output_final_state,
             n_states=None):
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if q.dim() != 4 or k.shape != q.shape:
        raise ValueError(f"q and k must both be [B,T,Hk,dk]; got {tuple(q.shape)}, {tuple(k.shape)}")
    B, T, Hk, dk = q.shape
    if v.dim() != 4 or tuple(v.shape[:2]) != (B, T):
        raise ValueError(f"v must be [B,T,H,dv] with B,T={B},{T}; got {tuple(v.shape)}")
    H, dv = v.shape[2], v.shape[3]
    if (Hk == 0) != (H == 0) or (H and H % Hk):
        raise ValueError(f"v's {H} heads must be a multiple of q/k's {Hk} heads")
    for name, t in (("g", g), ("beta", beta)):
        if tuple(t.shape) != (B, T, H):
            raise ValueError(f"{name} must be [B,T,H]=({B},{T},{H}); got {tuple(t.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError(f"q, k, v must share one dtype; got {q.dtype}, {k.dtype}, {v.dtype}")
    if q.dtype not in _DTYPES:
        raise TypeError(f"dtype {q.dtype} not supported (bfloat16 or float32)")
    dev = q.device
    NS = B if n_states is None else n_states   # states: one per batch row or per sequence
    for name, t in (("k", k), ("v", v), ("g", g), ("beta", beta)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, q on {dev}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    g = g.to(torch.float32).contiguous()
    beta = beta.to(torch.float32).contiguous()
    # The kernels read 16-byte aligned rows; a view that starts mid-row (e.g. a
    # token slice of g) is copied into fresh, aligned storage.
    q, k, v, g, beta = (t if t.data_ptr() % 16 == 0 else t.clone()
                        for t in (q, k, v, g, beta))
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (NS, H, dk, dv):
            raise ValueError(f"initial_state must be [{'B' if n_states is None else 'N'},H,dk,dv]"
                             f"=({NS},{H},{dk},{dv}); got {tuple(initial_state.shape)}")
        if initial_state.device != dev:
            raise ValueError(f"initial_state is on {initial_state.device}, q on {dev}")
        h0 = initial_state
        if h0.dtype != torch.float32 or not h0.is_contiguous():
            h0 = h0.to(torch.float32).contiguous()
    hT = None
    if final_state_out is not None:
        if (tuple(final_state_out.shape) != (NS, H, dk, dv) or final_state_out.dtype != torch.float32
                or not final_state_out.is_contiguous() or final_state_out.device != dev):
            raise ValueError("final_state_out must be a contiguous float32 [B,H,dk,dv] tensor "
                             "on the inputs' device")
        hT = final_state_out
    elif output_final_state:
        hT = torch.empty((NS, H, dk, dv), dtype=torch.float32, device=dev)
    o = torch.empty((B, T, H, dv), dtype=v.dtype, device=dev)
    return q, k, v, g, beta, h0, hT, o, (B, T, H, Hk, dk, dv)


def _wants_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad
                                           for t in ts)


class _DeltaRuleFn(torch.autograd.Function):
    """Autograd node of both ops (same function: the recurrence, exact semantics)."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, h0, chunk_size, recurrent, cu_seqlens=None):
        if recurrent:
            o, hT = _recurrent_impl(q, k, v, g, beta, h0, True, None)
        else:
            o, hT = _chunk_impl(q, k, v, g, beta, h0, True, chunk_size, "exact", None,
                                cu_seqlens)
        ctx.set_materialize_grads(False)
        ctx.has_h0 = h0 is not None
        ctx.in_dtypes = (g.dtype, beta.dtype, None if h0 is None else h0.dtype)
        ctx.save_for_backward(q, k, v, g, beta, h0, cu_seqlens)
        return o, hT

    @staticmethod
    def backward(ctx, do, dhT):
        q, k, v, g, beta, h0, cu_seqlens = ctx.saved_tensors
        dq, dk, dv, dg, db, dh0 = _chunk_backward(q, k, v, g, beta, h0, do, dhT, cu_seqlens)
        gd, bd, hd = ctx.in_dtypes
        return (dq, dk, dv, dg.to(gd), db.to(bd), dh0.to(hd) if ctx.has_h0 else None, None,
                None, None)


def _check_cu_seqlens(q, cu_seqlens):
    """Validate packed-sequence offsets (as the forward does); returns N."""
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.dim() != 1 or \
            cu_seqlens.numel() < 1 or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cu_seqlens must be a 1-D int32/int64 tensor of N+1 offsets")
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("with cu_seqlens, q, k, v, g, beta hold one packed row (B == 1)")
    if not cu_seqlens.is_cuda:
        c = cu_seqlens.tolist()
        if c[0] != 0 or c[-1] != q.shape[1] or any(b < a for a, b in zip(c, c[1:])):
            raise ValueError(f"cu_seqlens must rise from 0 to T={q.shape[1]}; got {c}")
    return cu_seqlens.numel() - 1


def _chunk_backward(q, k, v, g, beta, h0, do, dhT, cu_seqlens=None):
    """Gradients of the recurrence through the C ABI: gdn_chunk_bwd, or
    gdn_chunk_bwd_varlen for packed sequences (``cu_seqlens``)."""
    n_seqs = None if cu_seqlens is None else _check_cu_seqlens(q, cu_seqlens)
    q, k, v, g, beta, h0c, _, _, (B, T, H, Hk, dk, dv) = _prepare(
        q, k, v, g, beta, h0, None, False, n_seqs)
    NS = B if n_seqs is None else n_seqs
    dev = q.device
    if do is None:
        do = torch.zeros((B, T, H, dv), dtype=v.dtype, device=dev)
    do = do.to(v.dtype).contiguous()
    if do.data_ptr() % 16:
        do = do.clone()
    dhT_c = None if dhT is None else dhT.to(torch.float32).contiguous()
    dq = torch.empty_like(q)
    dk_ = torch.empty_like(k)
    dv_ = torch.empty_like(v)
    dg = torch.empty((B, T, H), dtype=torch.float32, device=dev)
    db = torch.empty((B, T, H), dtype=torch.float32, device=dev)
    dh0 = torch.empty((NS, H, dk, dv), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        args = (_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0c), _ptr(do),
                _ptr(dhT_c), _ptr(dq), _ptr(dk_), _ptr(dv_), _ptr(dg), _ptr(db), _ptr(dh0))
        if n_seqs is None:
            ws_bytes = lib.gdn_chunk_bwd_workspace_bytes_for(B, T, H, Hk, dk, dv,
                                                             _DTYPES[q.dtype])
            ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
            rc = lib.gdn_chunk_bwd(*args, B, T, H, Hk, dk, dv, _DTYPES[q.dtype], _ptr(ws),
                                   ws_bytes, stream)
            what = "gdn_chunk_bwd"
        else:
            cu = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
            ws_bytes = lib.gdn_chunk_bwd_varlen_workspace_bytes(n_seqs, T, H, dk, dv)
            ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
            rc = lib.gdn_chunk_bwd_varlen(*args, _ptr(cu), n_seqs, T, H, Hk, dk, dv,
                                          _DTYPES[q.dtype], _ptr(ws), ws_bytes, stream)
            what = "gdn_chunk_bwd_varlen"
    _lib.check(rc, what)
    return dq, dk_, dv_, dg, db, dh0


def chunk_gated_delta_rule_fwd(q, k, v, g, beta, initial_state=None, output_final_state=False,
                               chunk_size=64, *, semantics: str = "exact",
                               final_state_out: Optional[torch.Tensor] = None,
                               cu_seqlens: Optional[torch.Tensor] = None
                               ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Chunked gated delta rule (reference ``chunk_gated_delta_rule_fwd``, ops.py:299).

    Returns ``(o, final_state)`` when ``output_final_state`` (or
    ``final_state_out``) is given, else ``(o, None)`` (ops.py:344-346).
    ``chunk_size`` is 16, 32 or 64.  ``semantics="exact"`` (default) equals the
    recurrence; ``"reference"`` reproduces the reference chunk code as written.
    ``cu_seqlens`` (integer ``[N+1]``, non-decreasing from 0 to T) packs N
    sequences into one row: q ``[1,T,Hk,dk]``, states ``[N,H,dk,dv]``.
    Differentiable (exact semantics, dense or packed) when an input requires grad.
    """
    if _wants_grad(q, k, v, g, beta, initial_state):
        if semantics != "exact" or final_state_out is not None:
            raise NotImplementedError("the backward covers exact semantics without "
                                      "final_state_out")
        cu = None
        if cu_seqlens is not None:
            _check_cu_seqlens(q, cu_seqlens)
            cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
        o, hT = _DeltaRuleFn.apply(q, k, v, g, beta, initial_state, int(chunk_size), False, cu)
        return (o, hT) if output_final_state else (o, None)
    return _chunk_impl(q, k, v, g, beta, initial_state, output_final_state, chunk_size,
                       semantics, final_state_out, cu_seqlens)


def _chunk_impl(q, k, v, g, beta, initial_state, output_final_state, chunk_size, semantics,
                final_state_out, cu_seqlens):
    if semantics not in _SEMANTICS:
        raise ValueError(f"semantics must be one of {sorted(_SEMANTICS)}; got {semantics!r}")
    n_seqs = None
    if cu_seqlens is not None:
        n_seqs = _check_cu_seqlens(q, cu_seqlens)
        if semantics != "exact":
            raise ValueError("packed sequences take semantics='exact' only")
    q, k, v, g, beta, h0, hT, o, (B, T, H, Hk, dk, dv) = _prepare(
        q, k, v, g, beta, initial_state, final_state_out, output_final_state, n_seqs)
    lib = _lib.load()
    dtype = _DTYPES[q.dtype]
    sem = _SEMANTICS[semantics]
    with torch.cuda.device(q.device):
        if n_seqs is not None:
            ws_bytes = lib.gdn_chunk_varlen_workspace_bytes(n_seqs, T, H, dk, dv,
                                                            int(chunk_size), dtype, sem)
        else:
            ws_bytes = lib.gdn_chunk_workspace_bytes(B, T, H, dk, dv, int(chunk_size), dtype,
                                                     sem)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if n_seqs is not None:
            cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
            rc = lib.gdn_chunk_fwd_varlen(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                          _ptr(h0), _ptr(o), _ptr(hT), _ptr(cu), n_seqs, T, H, Hk,
                                          dk, dv, int(chunk_size), dtype, sem, _ptr(ws), ws_bytes,
                                          stream)
        elif Hk == H:
            rc = lib.gdn_chunk_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0),
                                   _ptr(o), _ptr(hT), B, T, H, dk, dv, int(chunk_size), dtype,
                                   sem, _ptr(ws), ws_bytes, stream)
        else:
            rc = lib.gdn_chunk_fwd_gva(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0),
                                       _ptr(o), _ptr(hT), B, T, H, Hk, dk, dv, int(chunk_size),
                                       dtype, sem, _ptr(ws), ws_bytes, stream)
    _lib.check(rc, "gdn_chunk_fwd")
    return o, hT


def _two_phase_ok(q, k, v) -> bool:
    """Whether gdn_chunk_prepare / gdn_chunk_scan take these tensors (bf16, dk =
    128, dv a multiple of 64 up to 512, dense rows on a CUDA device)."""
    return (isinstance(q, torch.Tensor) and q.is_cuda and q.dim() == 4
            and q.dtype == torch.bfloat16 and k.dtype == q.dtype and v.dtype == q.dtype
            and q.shape[-1] == 128 and v.shape[-1] % 64 == 0 and 0 < v.shape[-1] <= 512
            and q.shape[0] * v.shape[2] <= 65535 and q.shape[1] > 0 and q.shape[0] > 0)


def _chunk_prepare(q, k, g, beta):
    """gdn_chunk_prepare: the per-chunk operands of (q, k, g, beta) in a new
    workspace (uint8 CUDA tensor) for _chunk_scan."""
    B, T, Hk, dk = q.shape
    H = g.shape[2]
    lib = _lib.load()
    ws_bytes = lib.gdn_chunk_workspace_bytes(B, T, H, dk, 64, 64, _lib.GDN_DTYPE_BF16,
                                             _lib.GDN_SEMANTICS_EXACT)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.gdn_chunk_prepare(_ptr(q), _ptr(k), _ptr(g), _ptr(beta), B, T, H, Hk, dk,
                                   _lib.GDN_DTYPE_BF16, _ptr(ws), ws_bytes,
                                   torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "gdn_chunk_prepare")
    return ws


def _chunk_scan(q, k, v, g, beta, ws, initial_state=None, transition=False, output=True):
    """gdn_chunk_scan over a workspace from _chunk_prepare of the same q, k, g,
    beta.  Returns (o or None, final state); with ``transition`` the final
    state is [B,H,dk,dv+dk]: the end state from a zero start, then the
    transition matrix (initial_state must be None)."""
    B, T, Hk, dk = q.shape
    H, dv = v.shape[2], v.shape[3]
    hT = torch.empty((B, H, dk, dv + (dk if transition else 0)), dtype=torch.float32,
                     device=q.device)
    o = torch.empty((B, T, H, dv), dtype=v.dtype, device=q.device) if output else None
    h0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    lib = _lib.load()
    with torch.cuda.device(q.device):
        rc = lib.gdn_chunk_scan(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0),
                                _ptr(o), _ptr(hT), B, T, H, Hk, dk, dv, _lib.GDN_DTYPE_BF16,
                                int(bool(transition)), _ptr(ws), ws.numel(),
                                torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "gdn_chunk_scan")
    return o, hT


def _fold_states(packed, h0, dv):
    """gdn_fold_states over the gathered summaries ``packed`` [P, B, H, dk,
    dv + dk] fp32 (end state from zero, then transition, per segment) from h0
    [B, H, dk, dv] (None: zero).  Returns [P + 1, B, H, dk, dv]: the state
    entering each segment and, last, the state after the final one."""
    packed = packed.contiguous()
    P, B, H, dk, ld = packed.shape
    out = torch.empty((P + 1, B, H, dk, dv), dtype=torch.float32, device=packed.device)
    h0 = None if h0 is None else h0.to(torch.float32).contiguous()
    lib = _lib.load()
    with torch.cuda.device(packed.device):
        rc = lib.gdn_fold_states(_ptr(packed), packed.data_ptr() + 4 * dv, _ptr(h0), _ptr(out),
                                 P, B * H, dk, dv, ld,
                                 torch.cuda.current_stream(packed.device).cuda_stream)
    _lib.check(rc, "gdn_fold_states")
    return out


def fused_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None,
                                     output_final_state=False, *,
                                     final_state_out: Optional[torch.Tensor] = None
                                     ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Fused recurrent gated delta rule (reference Pallas wrapper, ops.py:187-219).

    With neither ``initial_state`` nor ``output_final_state`` this is the
    reference call: zero initial state, returns ``(o, None)``.  For decode pass
    ``initial_state=S, final_state_out=S`` to update the state in place.
    Differentiable (without ``final_state_out``) when an input requires grad.
    """
    if _wants_grad(q, k, v, g, beta, initial_state):
        if final_state_out is not None:
            raise NotImplementedError("the backward does not cover final_state_out")
        o, hT = _DeltaRuleFn.apply(q, k, v, g, beta, initial_state, 64, True)
        return (o, hT) if output_final_state else (o, None)
    return _recurrent_impl(q, k, v, g, beta, initial_state, output_final_state, final_state_out)


def _recurrent_impl(q, k, v, g, beta, initial_state, output_final_state, final_state_out):
    q, k, v, g, beta, h0, hT, o, (B, T, H, Hk, dk, dv) = _prepare(
        q, k, v, g, beta, initial_state, final_state_out, output_final_state)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if Hk == H:
            rc = lib.gdn_recurrent_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0),
                                       _ptr(o), _ptr(hT), B, T, H, dk, dv, _DTYPES[q.dtype],
                                       stream)
        else:
            rc = lib.gdn_recurrent_fwd_gva(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                           _ptr(h0), _ptr(o), _ptr(hT), B, T, H, Hk, dk, dv,
                                           _DTYPES[q.dtype], stream)
    _lib.check(rc, "gdn_recurrent_fwd")
    return o, hT


def gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, *, gate=None,
                                  norm_weight=None, eps: float = 1e-5, initial_state=None,
                                  output_final_state=False,
                                  final_state_out: Optional[torch.Tensor] = None
                                  ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The GatedDeltaNet layer's core around the recurrent op
    (gdn_recurrent_fwd_layer): the gates from the raw projections, the
    recurrent step, and the gated RMSNorm of its output.  Single-token decode
    at dk = dv = 128 is one kernel; other shapes run the recurrent kernel with
    the gates formed in it, then the norm kernel (whole sequences on the
    tensor-core shapes take the chunked layer form).

    The reference layer (model.py:136-153) runs these as separate operations:
    ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``, the op,
    then ``FusedRMSNormGated`` (model.py:41-53; with ``gate=None`` the plain
    RMSNorm of the ungated layer, whose epsilon is 1e-6).

    q, k ``[B,T,Hk,dk]``; v ``[B,T,H,dv]``; a, b ``[B,T,H]`` (a_proj, b_proj
    outputs); A_log, dt_bias ``[H]``; gate ``[B,T,H,dv]`` in v's dtype or None;
    norm_weight ``[dv]`` (None: ones).  Returns ``(y, final_state)`` like the
    recurrent op (``final_state_out=S`` with ``initial_state=S`` updates S in
    place).  Inference only: there is no backward for this form.
    """
    return _layer_impl("gdn_recurrent_fwd_layer", q, k, v, a, b, A_log, dt_bias, gate,
                       norm_weight, eps, initial_state, output_final_state, final_state_out)


def gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, *, gate=None,
                                 norm_weight=None, eps: float = 1e-5, initial_state=None,
                                 output_final_state=False,
                                 final_state_out: Optional[torch.Tensor] = None,
                                 cu_seqlens: Optional[torch.Tensor] = None
                                 ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The GatedDeltaNet layer's core over a whole sequence (prefill)
    (gdn_chunk_fwd_layer): the gates from the raw projections, the chunked
    forward (exact semantics), and the gated RMSNorm of every output row --
    what model.py:136-153 computes around chunk_gated_delta_rule_fwd as
    separate operations.  One kernel at dk = dv = 128; at the other
    tensor-core shapes (dk = 256, dv a multiple of 64 -- the reference's
    default dk = 256, dv = 512) the chunk kernel forms the gates and a second
    kernel normalises its output in place.

    q, k ``[B,T,Hk,dk]`` and v ``[B,T,H,dv]`` in bfloat16; a, b ``[B,T,H]``;
    A_log, dt_bias ``[H]``; gate ``[B,T,H,dv]`` in v's dtype or None;
    norm_weight ``[dv]`` (None: ones).  Returns ``(y, final_state)`` like
    chunk_gated_delta_rule, packed sequences included (``cu_seqlens``: one row
    of T tokens holding N sequences, states ``[N,H,dk,dv]``).  Inference
    only: there is no backward for this form.
    """
    return _layer_impl("gdn_chunk_fwd_layer", q, k, v, a, b, A_log, dt_bias, gate,
                       norm_weight, eps, initial_state, output_final_state, final_state_out,
                       cu_seqlens)


def _layer_impl(entry, q, k, v, a, b, A_log, dt_bias, gate, norm_weight, eps, initial_state,
                output_final_state, final_state_out, cu_seqlens=None):
    if _wants_grad(q, k, v, a, b, initial_state):
        raise NotImplementedError("the layer forms have no backward")
    n_seqs = None if cu_seqlens is None else _check_cu_seqlens(q, cu_seqlens)
    q, k, v, a, b, h0, hT, y, (B, T, H, Hk, dk, dv) = _prepare(
        q, k, v, a, b, initial_state, final_state_out, output_final_state, n_seqs)
    dev = q.device

    def vec(t, n, name):
        if t is None:
            return None
        t = torch.as_tensor(t, device=dev).to(torch.float32).contiguous()
        if t.shape != (n,):
            raise ValueError(f"{name} must be [{n}]; got {tuple(t.shape)}")
        return t

    A_log, dt_bias = vec(A_log, H, "A_log"), vec(dt_bias, H, "dt_bias")
    w = vec(norm_weight, dv, "norm_weight")
    if w is None:
        w = torch.ones(dv, dtype=torch.float32, device=dev)
    if gate is not None:
        if tuple(gate.shape) != (B, T, H, dv):
            raise ValueError(f"gate must be [B,T,H,dv]=({B},{T},{H},{dv}); got {tuple(gate.shape)}")
        gate = gate.to(device=dev, dtype=v.dtype).contiguous()
        if gate.data_ptr() % 16:
            gate = gate.clone()
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        head = (_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(A_log), _ptr(dt_bias),
                _ptr(h0), _ptr(hT), _ptr(gate), _ptr(w), float(eps), _ptr(y))
        if n_seqs is not None:
            entry += "_varlen"
            cu = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
            rc = getattr(lib, entry)(*head, _ptr(cu), n_seqs, T, H, Hk, dk, dv,
                                     _DTYPES[q.dtype], stream)
        else:
            rc = getattr(lib, entry)(*head, B, T, H, Hk, dk, dv, _DTYPES[q.dtype], stream)
    _lib.check(rc, entry)
    return y, hT


def short_convolution(x, weight, *, activation: Optional[str] = "silu", conv_state=None,
                      output_final_state: bool = False,
                      final_state_out: Optional[torch.Tensor] = None
                      ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """ShortConvolution (model.py:15-40) on the GPU (gdn_short_conv_fwd): a
    causal depthwise convolution over time, kernel K, no bias, then SiLU for
    ``activation`` ``'silu'`` / ``'swish'`` (None: none).

    x ``[B,T,C]`` bfloat16 or float32 on a CUDA device; weight ``[K,C]`` or the
    flax kernel ``[K,1,C]`` (float32).  ``conv_state`` ``[B,K-1,C]`` in x's
    dtype replaces the zero padding before token 0 (the inputs a previous call
    ended with).  Returns ``(y, state)``: state ``[B,K-1,C]`` holds the last
    K - 1 inputs when ``output_final_state`` or ``final_state_out`` (which may
    be ``conv_state``, updated in place) is given, else None.  The reference's
    call is ``short_convolution(x, w)`` (no state).  Inference only.
    """
    if _wants_grad(x, conv_state):
        raise NotImplementedError("the short convolution has no backward here")
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dim() == 3):
        raise ValueError("x must be a [B,T,C] CUDA tensor")
    if x.dtype not in _DTYPES:
        raise TypeError(f"x must be bfloat16 or float32; got {x.dtype}")
    B, T, C = x.shape
    w = torch.as_tensor(weight, device=x.device).to(torch.float32)
    if w.dim() == 3:
        w = w.reshape(w.shape[0], w.shape[-1])
    if w.dim() != 2 or w.shape[1] != C:
        raise ValueError(f"weight must be [K,{C}] or [K,1,{C}]; got {tuple(weight.shape)}")
    K = w.shape[0]
    w = w.contiguous()
    act = {"silu": 1, "swish": 1, None: 0}.get(activation)
    if act is None:
        raise ValueError(f"activation must be 'silu', 'swish' or None; got {activation!r}")
    x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    shape = (B, K - 1, C)

    def state(t, name):
        if t is None:
            return None
        if tuple(t.shape) != shape or t.dtype != x.dtype or t.device != x.device:
            raise ValueError(f"{name} must be {shape} {x.dtype} on {x.device}")
        if not t.is_contiguous() or t.data_ptr() % 16:
            raise ValueError(f"{name} must be contiguous and 16-byte aligned")
        return t

    s_in = state(conv_state, "conv_state")
    s_out = state(final_state_out, "final_state_out")
    if s_out is None and output_final_state:
        s_out = torch.empty(shape, dtype=x.dtype, device=x.device)
    y = torch.empty_like(x)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.gdn_short_conv_fwd(_ptr(x), _ptr(w), _ptr(s_in), _ptr(s_out), _ptr(y), B, T, C,
                                    K, act, _DTYPES[x.dtype],
                                    torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "gdn_short_conv_fwd")
    return y, s_out


def gated_rms_norm(o, gate=None, weight=None, eps: float = 1e-5, *,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FusedRMSNormGated (model.py:41-53) on the GPU (gdn_gated_rmsnorm_fwd):
    ``o * rsqrt(mean(o^2, -1) + eps) * weight``, times ``silu(gate)`` when a
    gate is given.  o ``[..., dv]`` bfloat16 or float32; gate like o or None;
    weight ``[dv]`` (None: ones).  ``out`` may be o (in place)."""
    if not (isinstance(o, torch.Tensor) and o.is_cuda and o.dtype in _DTYPES):
        raise ValueError("o must be a bfloat16 or float32 CUDA tensor")
    dv = o.shape[-1]
    o = o.contiguous()
    if gate is not None:
        if gate.shape != o.shape:
            raise ValueError(f"gate must have o's shape {tuple(o.shape)}")
        gate = gate.to(dtype=o.dtype).contiguous()
        if gate.data_ptr() % 16:
            gate = gate.clone()
    w = torch.ones(dv, dtype=torch.float32, device=o.device) if weight is None else \
        torch.as_tensor(weight, device=o.device).to(torch.float32).contiguous()
    if w.shape != (dv,):
        raise ValueError(f"weight must be [{dv}]")
    y = torch.empty_like(o) if out is None else out
    if y.shape != o.shape or y.dtype != o.dtype or not y.is_contiguous():
        raise ValueError("out must be a contiguous tensor of o's shape and dtype")
    lib = _lib.load()
    with torch.cuda.device(o.device):
        rc = lib.gdn_gated_rmsnorm_fwd(_ptr(o), _ptr(gate), _ptr(w), float(eps), _ptr(y),
                                       o.numel() // max(dv, 1), dv, _DTYPES[o.dtype],
                                       torch.cuda.current_stream(o.device).cuda_stream)
    _lib.check(rc, "gdn_gated_rmsnorm_fwd")
    return y


# Aliases with the reference's public names (ops.py:350-352).
fused_recurrent_gated_delta_rule_fwd = fused_recurrent_gated_delta_rule
fused_recurrent_gated_delta_rule_pallas = fused_recurrent_gated_delta_rule
chunk_gated_delta_rule = chunk_gated_delta_rule_fwd

__all__ = [
    "chunk_gated_delta_rule", "chunk_gated_delta_rule_fwd", "fused_recurrent_gated_delta_rule",
    "fused_recurrent_gated_delta_rule_fwd", "fused_recurrent_gated_delta_rule_pallas",
    "gated_delta_rule_decode_layer",
    "gated_delta_rule_chunk_layer",
    "short_convolution",
    "gated_rms_norm",
]
