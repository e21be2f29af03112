"""CPU oracle for the gated delta-rule hot path (test infrastructure only).

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / ``--impl reference`` arms of
``bench.py`` import it.  The CUDA library in ``gated_deltanet_jax_b200`` never
routes through here and fails loudly when its extension is missing.

It restates, in float64 NumPy, the algorithm of the reference package
``gated_deltanet_jax`` (``src/gated_deltanet_jax/ops.py``):

* :func:`recurrent_ref` -- the token-by-token recurrence of the Pallas kernel
  ``fused_recurrent_kernel_simple`` (ops.py:162-184), extended with an optional
  initial state and a returned final state.  This is the exact delta-rule
  semantics the CUDA kernels implement.
* :func:`chunk_exact` -- the chunked (WY / UT transform) form of the same
  recurrence.  Equal to :func:`recurrent_ref` to rounding.
* :func:`chunk_reference_literal` -- a line-by-line restatement of the
  reference's chunk path ``chunk_gated_delta_rule_fwd`` (ops.py:238-346),
  including its four deviations from the recurrence:

  - ``inv(I - A)`` where the recurrence needs ``inv(I + A)`` (ops.py:271-274);
  - the state update ``h <- e^{G_C} h + K^T v_new`` without the intra-chunk
    decay ``e^{G_C - G_j}`` on K (ops.py:329);
  - a partial last chunk pads the *cumulated* G with 0, so the final state is
    decayed by ``e^0`` (ops.py:247, 257, 327);
  - the output reshape ``[B,N,H,C,V] -> [B,N*C,H,V]`` without moving H back
    behind C (ops.py:342), which permutes tokens and heads whenever H > 1.

* :func:`segment_transition` and :func:`two_pass_sp` -- the two-pass sequence
  split used for long sequences: per segment, the affine map
  ``h_end = M h_start + S`` and the hand-off ``S_in(p+1) = M_p S_in(p) + S_p``.

Parity pinning: JAX is not installable in this environment, so the reference
cannot run natively.  ``tests/golden/make_golden.py`` executes the reference's
own ``ops.py`` source under a NumPy stand-in for the ``jax.numpy`` / ``lax.scan``
/ ``pallas_call`` subset it uses, and stores the outputs as fixtures.  The tests
pin :func:`recurrent_ref` and :func:`chunk_reference_literal` against those
fixtures, and :func:`chunk_exact` against :func:`recurrent_ref`.  JAX's own
float32/bfloat16 rounding is not reproduced by the stand-in (it computes in
float64), so the pin covers the algorithm, not JAX's numerics.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

# ---------------------------------------------------------------------------
# Input generation (distributions of the benchmark configurations)
# ---------------------------------------------------------------------------


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _logsigmoid(x):
    # log(sigmoid(x)) = -softplus(-x), computed stably.
    return -np.logaddexp(0.0, -x)


def make_inputs(B: int, T: int, H: int, dk: int, dv: int, seed: int = 0,
                h0_std: Optional[float] = None):
    """Seeded synthetic inputs with the reference benchmark distributions.

    q, k ~ N(0,1) then L2-normalised over the head dimension; v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = logsigmoid(N(0,1)) per (token, head); the
    optional initial state ~ N(0, h0_std) of shape [B,H,dk,dv].
    Returned as float64 arrays in the reference layout [B,T,H,D] / [B,T,H].
    """
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, dk))
    k = rng.standard_normal((B, T, H, dk))
    v = rng.standard_normal((B, T, H, dv))
    beta = _sigmoid(rng.standard_normal((B, T, H)))
    g = _logsigmoid(rng.standard_normal((B, T, H)))
    q = q / np.linalg.norm(q, axis=-1, keepdims=True)
    k = k / np.linalg.norm(k, axis=-1, keepdims=True)
    h0 = None
    if h0_std is not None:
        h0 = rng.standard_normal((B, H, dk, dv)) * h0_std
    return q, k, v, g, beta, h0


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 value (ties to even), returned as float64."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


# ---------------------------------------------------------------------------
# Exact delta-rule recurrence (ops.py:162-184 plus state carry)
# ---------------------------------------------------------------------------


def recurrent_ref(q, k, v, g, beta, h0=None, dtype=np.float64):
    """Token-by-token gated delta rule.

    Follows ``fused_recurrent_kernel_simple`` (ops.py:170-184) for every
    (b, h) at once::

        h = h * exp(g_t)                 # ops.py:178
        proj = k_t . h                   # ops.py:179
        v_new = (v_t - proj) * beta_t    # ops.py:180
        h = h + outer(k_t, v_new)        # ops.py:181
        o_t = h^T q_t                    # ops.py:182

    The reference starts from zeros (ops.py:168) and drops the final state
    (ops.py:219); here ``h0`` (default zeros) seeds the state and the final
    state is returned.  Layouts: q,k [B,T,H,dk], v [B,T,H,dv], g,beta [B,T,H],
    h0 [B,H,dk,dv].  Returns (o [B,T,H,dv], hT [B,H,dk,dv]).
    """
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype)
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    h = np.zeros((B, H, dk, dv), dtype) if h0 is None else np.array(h0, dtype)
    o = np.empty((B, T, H, dv), dtype)
    for t in range(T):
        h = h * np.exp(g[:, t])[:, :, None, None]
        proj = np.einsum('bhk,bhkv->bhv', k[:, t], h)
        v_new = (v[:, t] - proj) * beta[:, t][:, :, None]
        h = h + k[:, t][:, :, :, None] * v_new[:, :, None, :]
        o[:, t] = np.einsum('bhkv,bhk->bhv', h, q[:, t])
    return o, h


# ---------------------------------------------------------------------------
# Chunked form of the exact recurrence
# ---------------------------------------------------------------------------


def _to_chunks(x, C, N):
    """[B,T,H,...] -> [B,H,N,C,...], zero-padding T up to N*C."""
    B, T = x.shape[:2]
    pad = N * C - T
    if pad:
        widths = [(0, 0), (0, pad)] + [(0, 0)] * (x.ndim - 2)
        x = np.pad(x, widths)
    x = x.reshape((B, N, C) + x.shape[2:])
    return np.moveaxis(x, 3, 1)


def chunk_exact(q, k, v, g, beta, h0=None, chunk_size=64, dtype=np.float64):
    """Chunked gated delta rule, algebraically equal to :func:`recurrent_ref`.

    Per chunk of C tokens with in-chunk cumulative gate G (ops.py:238-247):

        A   = tril_{-1}(diag(beta) K K^T * e^{G_i - G_j})
        X   = diag(beta) (V - diag(e^G) K h)
        V'  = (I + A)^{-1} X
        o   = diag(e^G) Q h + tril_0(Q K^T * e^{G_i - G_j}) V'
        h  <- e^{G_C} h + (diag(e^{G_C - G}) K)^T V'

    A partial last chunk is zero-padded (g = 0, beta = 0), which leaves the
    cumulated gate constant, so ``G_C`` is that of the last real token.
    Exponents are formed only on the causal triangle (e^{G_i - G_j}, j <= i),
    never as e^{G_i} * e^{-G_j}.
    """
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype)
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    C = int(chunk_size)
    N = max(1, -(-T // C))
    qc, kc, vc = _to_chunks(q, C, N), _to_chunks(k, C, N), _to_chunks(v, C, N)
    gc, bc = _to_chunks(g, C, N), _to_chunks(beta, C, N)          # [B,H,N,C]
    G = np.cumsum(gc, axis=-1)
    h = np.zeros((B, H, dk, dv), dtype) if h0 is None else np.array(h0, dtype)
    oc = np.empty((B, H, N, C, dv), dtype)
    causal = np.tril(np.ones((C, C), dtype=bool))
    strict = np.tril(np.ones((C, C), dtype=bool), -1)
    eye = np.eye(C, dtype=dtype)
    for n in range(N):
        Kn, Qn, Vn = kc[:, :, n], qc[:, :, n], vc[:, :, n]
        Gn, bn = G[:, :, n], bc[:, :, n]
        diff = Gn[..., :, None] - Gn[..., None, :]
        E = np.exp(np.where(causal, diff, -np.inf))
        A = np.where(strict, bn[..., :, None] * (Kn @ np.swapaxes(Kn, -1, -2)) * E, 0.0)
        P = (Qn @ np.swapaxes(Kn, -1, -2)) * E
        eG = np.exp(Gn)[..., None]
        X = bn[..., None] * (Vn - eG * (Kn @ h))
        Vp = np.linalg.solve(eye + A, X)
        oc[:, :, n] = eG * (Qn @ h) + P @ Vp
        GC = Gn[..., -1]
        Kd = Kn * np.exp(GC[..., None] - Gn)[..., None]
        h = np.exp(GC)[..., None, None] * h + np.swapaxes(Kd, -1, -2) @ Vp
    o = np.moveaxis(oc, 1, 3).reshape(B, N * C, H, dv)[:, :T]
    return o, h


def chunk_exact_backward(q, k, v, g, beta, h0, do, dhT=None, chunk_size=64, dtype=np.float64):
    """Gradients of :func:`chunk_exact` (= of the recurrence) by reverse-mode
    differentiation through its chunked form.  The reference has no backward
    (it relies on JAX autodiff of its chunk path); this is the restatement the
    backward kernel is checked against.

    Given do [B,T,H,dv] (gradient of o) and dhT [B,H,dk,dv] (of the final
    state, None = 0) returns (dq, dk, dv, dg, dbeta, dh0).  Per chunk, with the
    forward's X = diag(beta)(V - diag(e^G) K h), V' = T X, T = (I + A)^{-1}:

        dV'  = P^T dO + Kd dh_out                    (o, h_out)
        dX   = T^T dV',   dT = dV' X^T,   dA = -T^T dT T^T  (strictly lower)
        dh   = e^{G_C} dh_out + Q^T (e^G dO) + K^T dKh,  dKh = -(beta e^G) dX
        gate terms through e^G, e^{G_i - G_j} and e^{G_C - G}; dg is the reverse
        in-chunk cumulative sum of dG.
    """
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype); do = np.asarray(do, dtype)
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    C = int(chunk_size)
    N = max(1, -(-T // C))
    qc, kc, vc, doc = (_to_chunks(x, C, N) for x in (q, k, v, do))
    gc, bc = _to_chunks(g, C, N), _to_chunks(beta, C, N)
    G = np.cumsum(gc, axis=-1)
    causal = np.tril(np.ones((C, C), dtype=bool))
    strict = np.tril(np.ones((C, C), dtype=bool), -1)
    eye = np.eye(C, dtype=dtype)
    sw = lambda x: np.swapaxes(x, -1, -2)  # noqa: E731
    # forward, keeping the state entering every chunk
    h = np.zeros((B, H, dk, dv), dtype) if h0 is None else np.array(h0, dtype)
    hs = []
    for n in range(N):
        hs.append(h)
        Kn, Vn, Gn, bn = kc[:, :, n], vc[:, :, n], G[:, :, n], bc[:, :, n]
        E = np.exp(np.where(causal, Gn[..., :, None] - Gn[..., None, :], -np.inf))
        A = np.where(strict, bn[..., :, None] * (Kn @ sw(Kn)) * E, 0.0)
        X = bn[..., None] * (Vn - np.exp(Gn)[..., None] * (Kn @ h))
        Vp = np.linalg.solve(eye + A, X)
        GC = Gn[..., -1]
        Kd = Kn * np.exp(GC[..., None] - Gn)[..., None]
        h = np.exp(GC)[..., None, None] * h + sw(Kd) @ Vp
    dqc, dkc, dvc = np.zeros_like(qc), np.zeros_like(kc), np.zeros_like(vc)
    dgc, dbc = np.zeros_like(gc), np.zeros_like(bc)
    dh = np.zeros((B, H, dk, dv), dtype) if dhT is None else np.array(dhT, dtype)
    for n in reversed(range(N)):
        h = hs[n]
        Qn, Kn, Vn, dOn = qc[:, :, n], kc[:, :, n], vc[:, :, n], doc[:, :, n]
        Gn, bn = G[:, :, n], bc[:, :, n]
        eG = np.exp(Gn)
        E = np.exp(np.where(causal, Gn[..., :, None] - Gn[..., None, :], -np.inf))
        KK = Kn @ sw(Kn)
        A = np.where(strict, bn[..., :, None] * KK * E, 0.0)
        Tm = np.linalg.inv(eye + A)
        Kh = Kn @ h
        Qh = Qn @ h
        X = bn[..., None] * (Vn - eG[..., None] * Kh)
        Vp = Tm @ X
        P = np.where(causal, (Qn @ sw(Kn)) * E, 0.0)
        GC = Gn[..., -1]
        dec = np.exp(GC[..., None] - Gn)
        Kd = Kn * dec[..., None]
        dG = np.zeros_like(Gn)
        # h_out = e^{G_C} h + Kd^T V'
        dh_out = dh
        dVp = Kd @ dh_out
        dKd = Vp @ sw(dh_out)
        dGC = np.exp(GC) * np.einsum('bhkv,bhkv->bh', h, dh_out) + np.einsum('bhck,bhck->bh', dKd, Kd)
        dG -= np.einsum('bhck,bhck->bhc', dKd, Kd)
        dK = dKd * dec[..., None]
        dh = np.exp(GC)[..., None, None] * dh_out
        # o = e^G (Q h) + P V'
        dVp += sw(P) @ dOn
        dP = np.where(causal, dOn @ sw(Vp), 0.0)
        dQ = eG[..., None] * (dOn @ sw(h))
        dh += sw(Qn) @ (eG[..., None] * dOn)
        dG += eG * np.einsum('bhcv,bhcv->bhc', dOn, Qh)
        dPE = dP * E
        dQ += dPE @ Kn
        dK += sw(dPE) @ Qn
        dPP = dP * P
        dG += dPP.sum(-1) - dPP.sum(-2)
        # V' = T X
        dX = sw(Tm) @ dVp
        dT = dVp @ sw(X)
        dA = np.where(strict, -sw(Tm) @ dT @ sw(Tm), 0.0)
        # X = beta (V - e^G K h)
        dV = bn[..., None] * dX
        dbeta = np.einsum('bhcv,bhcv->bhc', dX, Vn - eG[..., None] * Kh)
        dKh = -(bn * eG)[..., None] * dX
        dG += np.einsum('bhcv,bhcv->bhc', dKh, Kh)
        dK += dKh @ sw(h)
        dh += sw(Kn) @ dKh
        # A = strict(beta_i (K K^T) e^{G_i - G_j})
        dAE = dA * E
        dbeta += (dAE * KK).sum(-1)
        dK += (bn[..., None] * dAE) @ Kn + sw(dAE) @ (bn[..., None] * Kn)
        dAA = dA * A
        dG += dAA.sum(-1) - dAA.sum(-2)
        dG[..., -1] += dGC
        dgc[:, :, n] = np.cumsum(dG[..., ::-1], axis=-1)[..., ::-1]
        dqc[:, :, n], dkc[:, :, n], dvc[:, :, n], dbc[:, :, n] = dQ, dK, dV, dbeta
    unchunk = lambda x: np.moveaxis(x, 1, 3).reshape((B, N * C, H) + x.shape[4:])[:, :T]  # noqa
    dq, dk_, dv_ = unchunk(dqc), unchunk(dkc), unchunk(dvc)
    dg = np.moveaxis(dgc, 1, 3).reshape(B, N * C, H)[:, :T]
    db = np.moveaxis(dbc, 1, 3).reshape(B, N * C, H)[:, :T]
    return dq, dk_, dv_, dg, db, dh


# ---------------------------------------------------------------------------
# Literal restatement of the reference chunk path (ops.py:238-346)
# ---------------------------------------------------------------------------


def chunk_reference_literal(q, k, v, g, beta, initial_state=None,
                            output_final_state=False, chunk_size=64,
                            dtype=np.float64):
    """The reference ``chunk_gated_delta_rule_fwd`` step by step.

    Deliberately keeps the reference's deviations from the recurrence (see the
    module docstring): ``inv(I - A)``, the undecayed K in the state update,
    the zero padding of the cumulated gate, and the output reshape that
    interleaves heads with tokens.  Returns ``(o, final_state or None)``.
    """
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype)
    B, T, H, Kd = k.shape
    Vd = v.shape[-1]
    C = int(chunk_size)
    pad_len = (C - (T % C)) % C

    def pad(x):
        if pad_len > 0:
            return np.pad(x, [(0, 0), (0, pad_len)] + [(0, 0)] * (x.ndim - 2))
        return x

    # chunk_local_cumsum (ops.py:238-247): cumsum per chunk, then cut back to T.
    gp = pad(g)
    Np = gp.shape[1] // C
    G = np.cumsum(gp.reshape(B, Np, C, H), axis=2).reshape(B, Np * C, H)[:, :T]
    # chunk_scaled_dot_kkt (ops.py:249-269): G is re-padded with zeros.
    k_p, G_p, b_p = pad(k), pad(G), pad(beta)
    N = k_p.shape[1] // C
    kch = k_p.reshape(B, N, C, H, Kd).transpose(0, 1, 3, 2, 4)
    gch = G_p.reshape(B, N, C, H).transpose(0, 1, 3, 2)
    bch = b_p.reshape(B, N, C, H).transpose(0, 1, 3, 2)
    A = kch @ np.swapaxes(kch, -1, -2)
    A = A * np.exp(gch[..., :, None] - gch[..., None, :])
    A = np.where(np.tril(np.ones((C, C), dtype=bool), -1), A, 0.0)
    A = A * bch[..., :, None]
    # solve_inv_I_minus_A (ops.py:271-274).
    A_inv = np.linalg.inv(np.eye(C, dtype=dtype) - A)
    # recompute_w_u (ops.py:276-297).
    v_p = pad(v)

    def reshape_chunk(x):
        return np.swapaxes(x.reshape((B, N, C, H) + x.shape[3:]), 2, 3)

    k_c = reshape_chunk(k_p)
    v_c = reshape_chunk(v_p)
    beta_c = reshape_chunk(b_p[..., None])[..., 0]
    g_c = reshape_chunk(G_p[..., None])[..., 0]
    w_c = A_inv @ (k_c * (beta_c * np.exp(g_c))[..., None])
    u_c = A_inv @ (v_c * beta_c[..., None])
    # scan (ops.py:306-341).
    q_c = np.swapaxes(pad(q).reshape(B, N, C, H, Kd), 2, 3)
    h = (np.zeros((B, H, Kd, Vd), dtype) if initial_state is None
         else np.array(initial_state, dtype))
    tril0 = np.tril(np.ones((C, C), dtype=bool))
    outs = []
    for n in range(N):
        k_i, w_i, u_i, g_i, q_i = k_c[:, n], w_c[:, n], u_c[:, n], g_c[:, n], q_c[:, n]
        v_new = u_i - w_i @ h
        g_prob = np.exp(g_i)
        decay = g_prob[..., -1, None, None]
        h_next = h * decay + np.swapaxes(k_i, -1, -2) @ v_new
        o_global = (q_i * g_prob[..., None]) @ h
        S = (q_i @ np.swapaxes(k_i, -1, -2)) * np.exp(g_i[..., :, None] - g_i[..., None, :])
        S = np.where(tril0, S, 0.0)
        outs.append(o_global + S @ v_new)
        h = h_next
    o_scan = np.stack(outs)                                   # [N,B,H,C,V]
    o = np.swapaxes(o_scan, 0, 1).reshape(B, -1, H, Vd)[:, :T]  # ops.py:342-343
    return (o, h) if output_final_state else (o, None)


def literal_output_permutation(T: int, H: int, chunk_size: int):
    """Index map of the reference's output reshape (ops.py:342-343).

    Returns integer arrays (src_t, src_h) of shape [T, H]: the literal output
    at (t, h) holds the per-(token, head) chunk output of (src_t[t,h],
    src_h[t,h]) -- before the final slice to T.
    """
    C = int(chunk_size)
    N = -(-T // C)
    flat = np.arange(N * C * H)          # position in [N,H,C] order
    n, rem = flat // (H * C), flat % (H * C)
    hh, c = rem // C, rem % C
    src_t = (n * C + c).reshape(N * C, H)[:T]
    src_h = hh.reshape(N * C, H)[:T]
    return src_t, src_h


# ---------------------------------------------------------------------------
# Sequence split (two-pass scan over segments)
# ---------------------------------------------------------------------------


def segment_transition(k, g, beta, dtype=np.float64):
    """Linear part M of the affine state map over a segment.

    Over tokens t of one segment the state evolves as
    ``h_t = e^{g_t} (I - beta_t k_t k_t^T) h_{t-1} + beta_t k_t v_t^T``,
    so ``h_end = M h_start + S`` with ``M = prod_t e^{g_t}(I - beta_t k_t k_t^T)``
    (later tokens on the left) and S the end state from a zero start.  M is the
    end state of the same recurrence started from the identity with v = 0.
    Returns M [B,H,dk,dk].
    """
    k = np.asarray(k, dtype)
    B, T, H, dk = k.shape
    ident = np.broadcast_to(np.eye(dk, dtype=dtype), (B, H, dk, dk))
    zeros_v = np.zeros((B, T, H, dk), dtype)
    _, M = recurrent_ref(k, k, zeros_v, g, beta, h0=ident, dtype=dtype)
    return M


def two_pass_sp(q, k, v, g, beta, h0=None, parts=2, chunk_size=64, dtype=np.float64):
    """Two-pass sequence-parallel evaluation over ``parts`` contiguous segments.

    Pass 1 (independent per segment): local end state S_p from a zero start
    and transition M_p.  Hand-off (sequential over segments):
    ``S_in(0) = h0``, ``S_in(p+1) = M_p S_in(p) + S_p``.  Pass 2 (independent
    per segment): the chunked forward from ``S_in(p)``.  Segments are
    chunk-aligned except possibly the last.  Returns (o, hT).
    """
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype)
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    C = int(chunk_size)
    nchunks = -(-T // C)
    per = -(-nchunks // parts) * C
    bounds = [(s, min(T, s + per)) for s in range(0, T, per)]
    S_loc, M_loc = [], []
    for s, e in bounds:
        _, S = chunk_exact(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e],
                           None, C, dtype)
        S_loc.append(S)
        M_loc.append(segment_transition(k[:, s:e], g[:, s:e], beta[:, s:e], dtype))
    s_in = np.zeros((B, H, dk, dv), dtype) if h0 is None else np.array(h0, dtype)
    outs = []
    for (s, e), S, M in zip(bounds, S_loc, M_loc):
        o_p, _ = chunk_exact(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e],
                             s_in, C, dtype)
        outs.append(o_p)
        s_in = M @ s_in + S
    return np.concatenate(outs, axis=1), s_in


# ---------------------------------------------------------------------------
# Tolerances
# ---------------------------------------------------------------------------

#: fp32 inputs: max |out - ref| on o and final state.
TOL_FP32_ABS = 2e-3
#: bf16 inputs with fp32 state: max |out - ref| / max |ref|.
TOL_BF16_REL = 2e-2


def repeat_heads(x: np.ndarray, rep: int) -> np.ndarray:
    """Each head of x [B,T,Hk,...] repeated ``rep`` times in place along axis 2.

    The layer's expansion of q and k for grouped value heads, model.py:132-135
    (``jnp.repeat(x, rep, axis=2)``): value head h uses q/k head h // rep.
    """
    return np.repeat(x, rep, axis=2)


def max_abs_err(out, ref) -> float:
    return float(np.max(np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64))))


def rel_err(out, ref) -> float:
    ref = np.asarray(ref, np.float64)
    scale = float(np.max(np.abs(ref)))
    return max_abs_err(out, ref) / max(scale, 1e-30)


def within_tolerance(out, ref, input_dtype: str) -> Tuple[bool, float]:
    """Apply the parity bar: fp32 -> max-abs <= 2e-3; bf16 -> rel <= 2e-2."""
    if input_dtype in ("fp32", "float32"):
        e = max_abs_err(out, ref)
        return e <= TOL_FP32_ABS, e
    e = rel_err(out, ref)
    return e <= TOL_BF16_REL, e


# ---------------------------------------------------------------------------
# The layer's work on either side of the op (model.py:136-139, :41-53)
# ---------------------------------------------------------------------------


def layer_gates(a, b, A_log, dt_bias, dtype=np.float64):
    """beta and g from the raw a_proj / b_proj outputs, as model.py:136-139:
    ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``, with
    A_log and dt_bias per value head (the last axis of a and b)."""
    a = np.asarray(a, dtype); b = np.asarray(b, dtype)
    A_log = np.asarray(A_log, dtype); dt_bias = np.asarray(dt_bias, dtype)
    beta = 1.0 / (1.0 + np.exp(-b))
    x = a + dt_bias
    softplus = np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))
    return -np.exp(A_log) * softplus, beta


def rms_norm_gated(o, weight, gate=None, eps=1e-5, dtype=np.float64):
    """FusedRMSNormGated (model.py:41-53) over the last axis:
    ``o * rsqrt(mean(o^2) + eps) * weight``, times ``silu(gate)`` if given
    (without a gate, the ungated layer's RMSNorm, model.py:150-151)."""
    o = np.asarray(o, dtype)
    var = np.mean(o * o, axis=-1, keepdims=True)
    y = o / np.sqrt(var + eps) * np.asarray(weight, dtype)
    if gate is not None:
        gt = np.asarray(gate, dtype)
        y = y * gt / (1.0 + np.exp(-gt))
    return y


def short_conv(x, weight, activation="silu", state=None, dtype=np.float64):
    """ShortConvolution (model.py:15-40): ``nnx.Conv`` with
    ``feature_group_count = C`` (depthwise), kernel ``K``, no bias and padding
    ``[(K - 1, 0)]`` (causal), then SiLU for ``'silu'`` / ``'swish'``:

        y[b, t, c] = act(sum_j w[j, c] * x[b, t - (K - 1) + j, c])

    x [B, T, C]; weight [K, C] (the flax kernel (K, 1, C) squeezed).  ``state``
    [B, K - 1, C] stands in for the zero padding (the K - 1 inputs before token
    0).  Returns (y, the last K - 1 inputs, the state a next call continues
    from)."""
    x = np.asarray(x, dtype)
    w = np.asarray(weight, dtype).reshape(-1, x.shape[-1])
    K = w.shape[0]
    B, T, C = x.shape
    pad = np.zeros((B, K - 1, C), dtype) if state is None else np.asarray(state, dtype)
    xe = np.concatenate([pad, x], axis=1)          # token t of x is row t + K - 1
    y = np.zeros((B, T, C), dtype)
    for j in range(K):
        y += w[j] * xe[:, j:j + T]
    if activation in ("silu", "swish"):
        y = y / (1.0 + np.exp(-y))
    return y, xe[:, T:T + K - 1].copy()


__all__ = [
    "make_inputs", "round_bf16", "recurrent_ref", "chunk_exact",
    "chunk_reference_literal", "literal_output_permutation", "segment_transition",
    "two_pass_sp", "TOL_FP32_ABS", "TOL_BF16_REL", "max_abs_err", "rel_err",
    "within_tolerance", "layer_gates", "rms_norm_gated", "short_conv",
]

