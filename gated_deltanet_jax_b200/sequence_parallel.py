"""Sequence-split chunked forward: one long sequence over several segments.

The delta-rule state evolves affinely over a segment of tokens,

    h_end = M h_start + S,     M = prod_t e^{g_t} (I - beta_t k_t k_t^T),

where S is the end state from a zero start and M the end state of the same
recurrence started from the identity with v = 0.  A long sequence is therefore
processed in two passes over contiguous segments:

1. per segment, in parallel: (S_p, M_p) from ONE chunked call on the extended
   value / state  v' = [v | 0],  h0' = [0 | I]  (its final state is [S_p | M_p]);
2. hand-off: S_in(0) = h0,  S_in(p+1) = M_p S_in(p) + S_p;
3. per segment, in parallel: the chunked forward from S_in(p), giving o.

Two placements of the segments:

* :func:`chunk_gated_delta_rule_sp` -- one segment per rank of a
  ``torch.distributed`` group (each rank holds its tokens); the hand-off is one
  all-gather of the (S_p, M_p) pairs, after which every rank folds the prefix
  locally (no sequential chain of sends).
* :func:`chunk_gated_delta_rule_split` -- several segments of one sequence on
  one GPU, laid side by side in the batch dimension so both passes run as single
  wide launches.

Both are exact (same math as the unsplit op, up to rounding).  The per-segment
work runs through ``segment_fn`` -- by default the CUDA chunked op, whose
two-phase form (gdn_chunk_prepare, then gdn_chunk_scan) lets both passes share
one per-chunk preparation and lets pass 1 take the transition columns without
materialising [v | 0] or [0 | I].
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

from . import ops

SegmentFn = Callable[..., Tuple[torch.Tensor, torch.Tensor]]


def _default_segment_fn(chunk_size: int) -> SegmentFn:
    def fn(q, k, v, g, beta, h0):
        return ops.chunk_gated_delta_rule_fwd(q, k, v, g, beta, initial_state=h0,
                                              output_final_state=True, chunk_size=chunk_size)
    return fn


def segment_summary(q, k, v, g, beta, segment_fn: SegmentFn):
    """(S, M) of a segment: end state from zero and the transition matrix.

    One call on v' = [v | 0] with h0' = [0 | I]; the returned state is [S | M]
    with S [B,H,dk,dv] and M [B,H,dk,dk].
    """
    B, T, _, dk = k.shape
    H, dv = v.shape[2], v.shape[-1]   # value heads (q/k may carry fewer, grouped)
    v_ext = torch.cat([v, torch.zeros(B, T, H, dk, dtype=v.dtype, device=v.device)], dim=-1)
    h_ext = torch.zeros(B, H, dk, dv + dk, dtype=torch.float32, device=v.device)
    h_ext[..., dv:] = torch.eye(dk, dtype=torch.float32, device=v.device)
    _, ext = segment_fn(q, k, v_ext.contiguous(), g, beta, h_ext)
    return ext[..., :dv].contiguous(), ext[..., dv:].contiguous()


def fold_states(h0: torch.Tensor, pairs) -> list:
    """States entering each segment: S_in(0) = h0, S_in(p+1) = M_p S_in(p) + S_p.

    ``pairs`` is a sequence of (S_p, M_p); returns [S_in(0), ..., S_in(P)]
    (the last entry is the state after the final segment).
    """
    states = [h0]
    s = h0
    for S_p, M_p in pairs:
        s = torch.matmul(M_p, s) + S_p
        states.append(s)
    return states


def fold_states_scan(h0: torch.Tensor, S: torch.Tensor, M: torch.Tensor) -> torch.Tensor:
    """Same result as :func:`fold_states` in log2(P) rounds of batched products.

    ``S`` [P, ..., dk, dv] and ``M`` [P, ..., dk, dk] are the segments' (S_p, M_p);
    returns [P + 1, ..., dk, dv]: the state entering each segment and, last, the
    state after the final one.  Segment p's map x -> M_p x + S_p composed with
    those before it is built by an inclusive prefix scan (Hillis-Steele): in
    round d, map i absorbs map i - d, (M_i, S_i) <- (M_i M_{i-d}, M_i S_{i-d} + S_i).
    """
    A, C = M, S
    d = 1
    P = S.shape[0]
    while d < P:
        A_new = torch.cat([A[:d], torch.matmul(A[d:], A[:-d])], dim=0)
        C = torch.cat([C[:d], torch.matmul(A[d:], C[:-d]) + C[d:]], dim=0)
        A = A_new
        d *= 2
    after = torch.matmul(A, h0.unsqueeze(0)) + C
    return torch.cat([h0.unsqueeze(0), after], dim=0)


def auto_local_parts(B: int, T: int, H: int, dv: int, chunk_size: int, device) -> int:
    """Segments per GPU so that the second pass fills most SMs: about 0.86 x SMs
    CTAs (one per (segment, head, 64 columns)), at least 4 chunks per segment."""
    if not (isinstance(device, torch.device) and device.type == "cuda"):
        return 1
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    per_part = max(1, B * H * max(1, dv // 64))
    parts = max(1, round(0.86 * sms / per_part))
    return max(1, min(parts, T // (4 * chunk_size)))


def _two_pass(q, k, v, g, beta, initial_state, output_final_state, chunk_size, parts, fn,
              gather, world, rank, marks=None):
    """Both passes over this rank's tokens split into ``parts`` batched segments.

    ``gather`` maps this rank's packed (S, M) pairs [B, parts, H, dk, dv + dk] to
    the list of every rank's, in rank order; segments are ordered rank-major.
    ``marks`` (a list, or None) receives (phase, CUDA event) pairs recorded on
    the current stream after each phase: "pass1", "exchange", "fold", "pass2".
    """
    def mark(name):
        if marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    B, T, _, dk = k.shape
    H, dv = v.shape[2], v.shape[-1]   # value heads (q/k may carry fewer, grouped)
    seg = -(-T // (parts * chunk_size)) * chunk_size          # tokens per segment
    Tp = seg * parts
    pad = Tp - T

    def to_segments(x):
        if pad:
            x = torch.cat([x, torch.zeros((B, pad) + tuple(x.shape[2:]), dtype=x.dtype,
                                          device=x.device)], dim=1)
        return x.reshape((B * parts, seg) + tuple(x.shape[2:])).contiguous()

    qs, ks, vs, gs, bs = (to_segments(x) for x in (q, k, v, g, beta))
    # On the CUDA op (no segment_fn given) with its two-phase form available, the
    # per-chunk preparation runs once for both passes, and pass 1 needs neither
    # [v | 0] nor [0 | I] in memory, nor an output: the scan's transition
    # columns start from the identity with v = 0 by themselves.
    ws = None
    if fn is None:
        qs, ks, vs, gs, bs = (x.contiguous() for x in (qs, ks, vs, gs.float(), bs.float()))
        if ops._two_phase_ok(qs, ks, vs):
            ws = ops._chunk_prepare(qs, ks, gs, bs)
            _, ext = ops._chunk_scan(qs, ks, vs, gs, bs, ws, transition=True, output=False)
            S, M = ext[..., :dv], ext[..., dv:]
        else:
            fn = _default_segment_fn(chunk_size)
    if ws is None:
        S, M = segment_summary(qs, ks, vs, gs, bs, fn)                  # [B*parts, H, ...]
    mark("pass1")
    packed = torch.cat([S, M], dim=-1).view(B, parts, H, dk, dv + dk).contiguous()
    use_kernel = ws is not None and dk == 128 and dv % 32 == 0

    def fold(pairs, h0):
        # [P, B, H, dk, dv + dk] summaries -> [P + 1, B, H, dk, dv]: the state
        # entering each segment, then the state after the last one
        if use_kernel:   # one launch walks every segment: out[p + 1] = M_p out[p] + S_p
            return ops._fold_states(pairs, h0, dv)
        h0 = (torch.zeros(B, H, dk, dv, dtype=S.dtype, device=v.device)
              if h0 is None else h0.to(S.dtype))
        return fold_states_scan(h0, pairs[..., :dv], pairs[..., dv:])

    if world > 1 and parts > 1:
        # This rank's segments composed into one map before the exchange,
        # (M_b, S_b) o (M_a, S_a) = (M_b M_a, M_b S_a + S_b): the all-gather then
        # moves one summary per rank, and the fold over the ranks takes `world`
        # steps instead of world x parts; each rank then walks its own segments
        # from the state entering it.
        loc = packed.transpose(0, 1).contiguous()                       # [parts, B, H, dk, dv+dk]
        acc = loc[0]
        for p in range(1, parts):
            acc = torch.matmul(loc[p, ..., dv:], acc)
            acc[..., :dv] += loc[p, ..., :dv]
        allr = torch.stack(gather(acc.contiguous()), dim=0)             # [world, B, H, dk, dv+dk]
        mark("exchange")
        ranks = fold(allr, initial_state)                               # [world + 1, ...]
        mine = fold(loc, ranks[rank])[:parts]
        final = ranks[world]
    else:
        allp = torch.cat(gather(packed), dim=1).transpose(0, 1)         # [world*parts, B, H, dk, dv+dk]
        mark("exchange")
        states = fold(allp, initial_state)                              # [world*parts + 1, ...]
        mine = states[rank * parts:(rank + 1) * parts]
        final = states[world * parts]
    s_in = mine.transpose(0, 1).reshape(B * parts, H, dk, dv).contiguous()
    mark("fold")
    if ws is not None:
        o, _ = ops._chunk_scan(qs, ks, vs, gs, bs, ws, initial_state=s_in)
    else:
        o, _ = fn(qs, ks, vs, gs, bs, s_in)
    mark("pass2")
    o = o.reshape(B, Tp, H, dv)[:, :T]
    return (o, final) if output_final_state else (o, None)


def chunk_gated_delta_rule_sp(q, k, v, g, beta, initial_state=None, output_final_state=False,
                              chunk_size=64, group=None, segment_fn: Optional[SegmentFn] = None,
                              local_parts: Optional[int] = None, marks: Optional[list] = None):
    """Chunked forward with the sequence split across the ranks of ``group``.

    Every rank passes its own contiguous segment ``[B, T_p, H, D]`` (rank order =
    token order; every rank's T_p is the same, except possibly the last one's).
    Each rank splits its segment again into ``local_parts`` segments that run
    batched on its GPU (None: chosen so the second pass fills the GPU; the ranks
    take the smallest of their choices, so a shorter last segment is fine; an
    explicit value must be the same on every rank); all world x local_parts (S, M)
    pairs are exchanged in one all-gather, after which every rank folds the
    prefix locally with a log-depth scan.
    ``initial_state`` is the state before rank 0's segment and must be the same
    on every rank (or None).  Returns ``(o_segment, final_state or None)``;
    ``final_state`` is the state after the LAST segment, on every rank.
    ``marks``: see ``_two_pass`` (per-phase CUDA events, for timing).
    """
    import torch.distributed as dist

    fn = segment_fn   # None: the CUDA op (its two-phase form where it applies)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)

    def gather(packed):
        out = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(out, packed, group=group)
        return out

    # Every rank must split into the same number of local segments: the
    # all-gather exchanges [B, parts, H, dk, dv + dk] summaries, and the fold
    # indexes them rank-major.  A chosen count depends on this rank's T (the
    # last rank's may be shorter), so the ranks agree on the smallest choice;
    # counts passed in must already agree, or every rank raises.
    auto = local_parts is None
    mine = (auto_local_parts(k.shape[0], k.shape[1], v.shape[2], v.shape[-1], chunk_size,
                             k.device) if auto else max(1, int(local_parts)))
    span = torch.tensor([mine, -mine], dtype=torch.int64, device=k.device)
    dist.all_reduce(span, op=dist.ReduceOp.MIN, group=group)
    lo, hi = int(span[0]), -int(span[1])
    if not auto and lo != hi:
        raise ValueError(f"local_parts differs across ranks ({lo} .. {hi}); pass the same value "
                         "on every rank, or None")
    return _two_pass(q, k, v, g, beta, initial_state, output_final_state, chunk_size, lo, fn,
                     gather, world, rank, marks)


def chunk_gated_delta_rule_split(q, k, v, g, beta, initial_state=None, output_final_state=False,
                                 chunk_size=64, parts: int = 4,
                                 segment_fn: Optional[SegmentFn] = None,
                                 marks: Optional[list] = None):
    """Chunked forward of B long sequences, each split into ``parts`` segments
    that run side by side in the batch dimension of two wide launches.

    The sequence is zero-padded (g = 0, beta = 0, k = v = 0) up to a multiple of
    ``parts * chunk_size``; padded tokens leave the state unchanged.  Returns
    ``(o, final_state or None)`` like the unsplit op.
    """
    fn = segment_fn   # None: the CUDA op (its two-phase form where it applies)
    T = k.shape[1]
    if parts <= 1 or T <= chunk_size:
        o, hT = (fn or _default_segment_fn(chunk_size))(q, k, v, g, beta, initial_state)
        return (o, hT) if output_final_state else (o, None)
    return _two_pass(q, k, v, g, beta, initial_state, output_final_state, chunk_size, parts, fn,
                     lambda packed: [packed], 1, 0, marks)


__all__ = ["chunk_gated_delta_rule_sp", "chunk_gated_delta_rule_split", "segment_summary",
           "fold_states", "fold_states_scan", "auto_local_parts"]
