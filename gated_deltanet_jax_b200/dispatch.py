"""The layer's mode switch between the two ops.

Mirrors reference ``src/gated_deltanet_jax/model.py:141-146``: ``'chunk'``
calls the chunked op, ``'fused_recurrent'`` the recurrent op, anything else
raises ``ValueError(f"Unknown mode {mode}")``.  Like the reference layer it
passes no initial state and keeps only ``o``.
"""

from __future__ import annotations

from . import ops


def delta_rule(config, q, k, v, g, beta):
    """Return ``o`` of the op ``config.attn_mode`` selects (model.py:141-146)."""
    if config.attn_mode == "chunk":
        o, _ = ops.chunk_gated_delta_rule_fwd(q, k, v, g, beta)
    elif config.attn_mode == "fused_recurrent":
        o, _ = ops.fused_recurrent_gated_delta_rule_fwd(q, k, v, g, beta)
    else:
        raise ValueError(f"Unknown mode {config.attn_mode}")
    return o
