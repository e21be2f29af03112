"""Generate the golden fixtures by running the reference's own ``ops.py``.

JAX is not installable in this environment, so the reference package
``gated_deltanet_jax`` cannot be imported normally.  This script installs a
small NumPy stand-in for exactly the JAX surface that
``src/gated_deltanet_jax/ops.py`` touches, loads that file from the read-only
reference checkout, runs its two public ops, and writes the outputs to
``tests/golden/golden.npz``:

* ``jax.numpy``            -> the NumPy namespace (``np.pad``, ``np.cumsum``,
                              ``np.matmul``, ``np.linalg.inv`` ... have the same
                              call forms as used in ops.py)
* ``jax.lax.scan``         -> a Python loop over the leading axis that stacks
                              the per-step outputs
* ``pl.pallas_call``       -> a loop over the grid that hands the kernel NumPy
                              *views* of each block (``BlockSpec.index_map`` x
                              ``block_shape``), so the kernel's block writes land
                              in the output array
* ``pl.program_id``        -> the current grid index
* ``jax.default_backend``  -> ``'cpu'`` (ops.py:197-202 then asks for interpret
                              mode, which the stand-in ignores)

Everything is computed in float64, so the fixtures pin the reference's
algorithm (including its chunk-path deviations), not JAX's float32 or bf16
rounding.  Inputs are stored as float32 values; outputs as float32.

Run once, in a container that has the reference checkout::

    python tests/golden/make_golden.py path/to/reference
    (or GDN_REFERENCE_ROOT=path/to/reference python tests/golden/make_golden.py)

The tests only read the ``.npz``; nothing at test time needs the reference.
"""

from __future__ import annotations

import collections
import importlib.util
import itertools
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.gdn_oracle import make_inputs  # noqa: E402


def _install_jax_standin():
    jax = types.ModuleType("jax")
    jnp = types.ModuleType("jax.numpy")
    for name in dir(np):
        if not name.startswith("_"):
            setattr(jnp, name, getattr(np, name))
    lax = types.ModuleType("jax.lax")

    def scan(f, init, xs):
        carry, ys = init, []
        for i in range(xs[0].shape[0]):
            carry, y = f(carry, tuple(x[i] for x in xs))
            ys.append(y)
        return carry, np.stack(ys)

    lax.scan = scan
    jax.numpy, jax.lax = jnp, lax
    jax.default_backend = lambda: "cpu"
    jax.ShapeDtypeStruct = collections.namedtuple("ShapeDtypeStruct", ["shape", "dtype"])

    experimental = types.ModuleType("jax.experimental")
    pallas = types.ModuleType("jax.experimental.pallas")
    triton = types.ModuleType("jax.experimental.pallas.triton")
    state = {"ids": ()}

    class BlockSpec:
        def __init__(self, index_map=None, block_shape=None):
            self.index_map, self.block_shape = index_map, block_shape

    def program_id(axis):
        return state["ids"][axis]

    def _block(arr, spec, ids):
        blk = spec.index_map(*ids)
        sl = tuple(slice(b * s, (b + 1) * s) for b, s in zip(blk, spec.block_shape))
        return arr[sl]

    def pallas_call(kernel, out_shape, grid, in_specs, out_specs, interpret=False):
        def run(*args):
            out = np.zeros(out_shape.shape, out_shape.dtype)
            for ids in itertools.product(*[range(n) for n in grid]):
                state["ids"] = ids
                refs = [_block(a, s, ids) for a, s in zip(args, in_specs)]
                kernel(*refs, _block(out, out_specs, ids))
            return out
        return run

    pallas.BlockSpec, pallas.program_id, pallas.pallas_call = BlockSpec, program_id, pallas_call
    pallas.triton = triton
    experimental.pallas = pallas
    jax.experimental = experimental
    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.lax": lax, "jax.experimental": experimental,
        "jax.experimental.pallas": pallas, "jax.experimental.pallas.triton": triton,
    })


def _load_reference_ops(ref_root):
    path = os.path.join(ref_root, "src", "gated_deltanet_jax", "ops.py")
    spec = importlib.util.spec_from_file_location("reference_ops", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# name -> (B, T, H, dk, dv, chunk, seed, initial-state std or None)
CASES = {
    # config 0 shapes: B=1 T=256 H=2 dk=dv=64 chunk=64, zero initial state
    "c0": (1, 256, 2, 64, 64, 64, 0, None),
    # initial state, multiple chunks, dk != dv
    "h0": (1, 128, 2, 32, 64, 32, 1, 0.02),
    # partial last chunk (T % chunk != 0)
    "tail": (2, 200, 2, 32, 32, 64, 2, 0.02),
    # reference test shapes: head_dim 32, expand_v 2, 4 heads, T=64
    "layer": (1, 64, 4, 32, 64, 64, 3, None),
    # reference test shapes: head_dim 16, expand_v 2, 4 heads, T=32 (< chunk)
    "lm": (1, 32, 4, 16, 32, 64, 4, None),
    # a single head: the reference output reshape is then the identity
    "h1": (1, 96, 1, 16, 16, 32, 5, 0.02),
    # the head dims of the reference's default configuration (head_dim 256, expand_v 2),
    # with an initial state and a partial last chunk
    "d256": (1, 70, 1, 256, 512, 64, 6, 0.02),
}


def main(ref_root=None):
    ref_root = ref_root or os.environ.get("GDN_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: make_golden.py path/to/reference "
                         "(or set GDN_REFERENCE_ROOT to the reference checkout)")
    _install_jax_standin()
    ops = _load_reference_ops(ref_root)
    out = {}
    for name, (B, T, H, dk, dv, C, seed, h0_std) in CASES.items():
        q, k, v, g, beta, h0 = make_inputs(B, T, H, dk, dv, seed=seed, h0_std=h0_std)
        # The fixtures hold float32 input values; the reference runs on exactly those.
        q, k, v, g, beta = (x.astype(np.float32).astype(np.float64) for x in (q, k, v, g, beta))
        if h0 is not None:
            h0 = h0.astype(np.float32).astype(np.float64)
        o_chunk, h_chunk = ops.chunk_gated_delta_rule(
            q, k, v, g, beta, initial_state=h0, output_final_state=True, chunk_size=C)
        o_rec, none = ops.fused_recurrent_gated_delta_rule(q, k, v, g, beta)
        assert none is None
        out[f"{name}/shape"] = np.array([B, T, H, dk, dv, C])
        for key, arr in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta),
                         ("o_chunk", o_chunk), ("h_chunk", h_chunk), ("o_recurrent", o_rec)):
            out[f"{name}/{key}"] = np.asarray(arr, np.float32)
        if h0 is not None:
            out[f"{name}/h0"] = np.asarray(h0, np.float32)
    dst = os.path.join(HERE, "golden.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst}: {len(CASES)} cases, {os.path.getsize(dst)} bytes")


if __name__ == "__main__":
    main(*sys.argv[1:])
