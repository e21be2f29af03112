"""Algorithmic work per unit of the delta-rule kernels: the numerators of the
roofline figures that bench.py reports (achieved = work per launch / launch
time).  Units: one token of one value head (chunked forward and backward),
one head for one decode step (recurrent decode)."""


def flops_chunk_per_token_head(dk: int, dv: int, C: int) -> int:
    """FLOP per token-head of the chunked forward.

    K K^T, W and Q K^T over dk; U and P V' over dv (2 C (3 dk + 2 dv)), plus
    W h, Q h and K^T V' (6 dk dv).  The O(C^2) triangular solve is excluded.
    """
    return 2 * C * (3 * dk + 2 * dv) + 6 * dk * dv


def flops_chunk_bwd_per_token_head(dk: int, dv: int, C: int) -> int:
    """FLOP per token-head of the chunked backward (gdn_chunk_bwd).

    Per chunk: Q K^T and K K^T twice (prep and gradients, 4 C^2 dk), W and Z
    (2 C^2 dk), U, P^T dO and Y (3 C^2 dv), dO V'^T and dX V'^T (2 C^2 dv),
    the four dQ / dK products over the chunk (4 C^2 dk); per token the state
    products W h, K^T V' (forward pass), Z dh, Q^T dO, K^T dX (reverse pass)
    and V' dh^T, dO h^T, dX h^T (8 dk dv).  The triangular solve is excluded.
    """
    return 2 * C * (10 * dk + 5 * dv) + 16 * dk * dv


def bytes_recurrent_per_head_step(dk: int, dv: int, in_bytes: int = 2) -> int:
    """HBM bytes per head-step of the decode kernel: fp32 state read + write,
    q/k/v in, o out (input dtype), fp32 g and beta."""
    return 8 * dk * dv + (2 * dk + dv) * in_bytes + dv * in_bytes + 8


def bytes_chunk_per_token_head(dk: int, dv: int, in_bytes: int = 2) -> int:
    """HBM bytes per token-head of the chunked forward (q/k/v in, o out, g/beta)."""
    return (2 * dk + dv) * in_bytes + dv * in_bytes + 8
