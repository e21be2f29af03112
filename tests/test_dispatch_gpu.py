"""The layer's mode switch (reference model.py:141-146) on the GPU: each mode
reaches its own op, with the reference's call (no initial state, o only)."""

import numpy as np
import pytest

from gated_deltanet_jax_b200 import GatedDeltaNetConfig, delta_rule, ops
from oracle import gdn_oracle as orc
from helpers import assert_close, device_inputs, f64

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,T", [("chunk", 200), ("chunk", 1), ("fused_recurrent", 1),
                                    ("fused_recurrent", 130), ("fused_recurrent", 7)])
def test_mode_switch_calls_its_op(cuda, monkeypatch, mode, T):
    (q, k, v, g, b, _), host = device_inputs(2, T, 3, 128, 128, seed=T, dtype="bf16", dev=cuda)
    calls = []
    for name in ("chunk_gated_delta_rule_fwd", "fused_recurrent_gated_delta_rule_fwd"):
        real = getattr(ops, name)

        def spy(*args, _real=real, _name=name, **kw):
            calls.append((_name, kw))
            return _real(*args, **kw)

        monkeypatch.setattr(ops, name, spy)
    o = delta_rule(GatedDeltaNetConfig(attn_mode=mode), q, k, v, g, b)
    want = {"chunk": "chunk_gated_delta_rule_fwd",
            "fused_recurrent": "fused_recurrent_gated_delta_rule_fwd"}[mode]
    assert [c[0] for c in calls] == [want]
    assert calls[0][1] == {}               # no initial state, no final state (model.py:141-146)
    assert o.shape == (2, T, 3, 128) and o.dtype == v.dtype
    ro, _ = orc.recurrent_ref(*host[:5])
    assert_close(f64(o), ro, "bf16", mode)


def test_unknown_mode_raises_before_any_op(cuda, monkeypatch):
    (q, k, v, g, b, _), _ = device_inputs(1, 4, 1, 16, 16, seed=0, dtype="bf16", dev=cuda)
    monkeypatch.setattr(ops, "chunk_gated_delta_rule_fwd", None)
    monkeypatch.setattr(ops, "fused_recurrent_gated_delta_rule_fwd", None)
    with pytest.raises(ValueError, match="Unknown mode parallel"):
        delta_rule(GatedDeltaNetConfig(attn_mode="parallel"), q, k, v, g, b)
    assert np.isfinite(f64(v)).all()
