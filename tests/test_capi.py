"""CPU tests of the C ABI boundary and the host-side argument checks.

No GPU is needed: the library must load, export every symbol include/gdn.h
declares, and reject bad arguments on the host before any CUDA call.
"""

import ctypes
import os
import re
import subprocess

import pytest
import torch

from gated_deltanet_jax_b200 import _lib, ops
from gated_deltanet_jax_b200 import _build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "gdn.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        _build.build()
    return _lib.load()


def test_header_and_binding_agree():
    assert _declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(gdn_\w+)", out))
    assert set(_declared_functions()) <= exported


def test_build_targets_sm100a():
    """Every kernel is compiled for sm_100a only (the GPU test
    test_kernels_report_sm100 asks the CUDA runtime on a device)."""
    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_abi_version(lib):
    assert lib.gdn_abi_version() >> 16 == 1


def _call_recurrent(lib, ptr=16, B=1, T=1, H=1, dk=16, dv=16, dtype=_lib.GDN_DTYPE_BF16):
    p = ctypes.c_void_p(ptr)
    return lib.gdn_recurrent_fwd(p, p, p, p, p, None, p, None, B, T, H, dk, dv, dtype, None)


def _call_chunk(lib, ptr=16, B=1, T=1, H=1, dk=16, dv=16, chunk=64, dtype=_lib.GDN_DTYPE_BF16,
                semantics=_lib.GDN_SEMANTICS_EXACT):
    p = ctypes.c_void_p(ptr)
    return lib.gdn_chunk_fwd(p, p, p, p, p, None, p, None, B, T, H, dk, dv, chunk, dtype,
                             semantics, None, 0, None)


@pytest.mark.parametrize("kw,code", [
    (dict(dk=48), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dk=512), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dv=8), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dv=24), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dv=1024), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dtype=7), _lib.GDN_ERR_INVALID),
    (dict(B=-1), _lib.GDN_ERR_INVALID),
    (dict(ptr=0), _lib.GDN_ERR_INVALID),
    (dict(ptr=18), _lib.GDN_ERR_INVALID),
])
def test_recurrent_rejects_bad_arguments(lib, kw, code):
    assert _call_recurrent(lib, **kw) == code
    assert lib.gdn_last_error()


@pytest.mark.parametrize("kw,code", [
    (dict(chunk=48), _lib.GDN_ERR_UNSUPPORTED),
    (dict(chunk=128), _lib.GDN_ERR_UNSUPPORTED),
    (dict(semantics=5), _lib.GDN_ERR_INVALID),
    (dict(dk=100), _lib.GDN_ERR_UNSUPPORTED),
    (dict(ptr=8), _lib.GDN_ERR_INVALID),
])
def test_chunk_rejects_bad_arguments(lib, kw, code):
    assert _call_chunk(lib, **kw) == code
    msg = lib.gdn_last_error().decode()
    assert msg


@pytest.mark.parametrize("H,Hk", [(6, 4), (4, 0), (4, -1), (3, 6)])
def test_grouped_heads_reject_bad_groups(lib, H, Hk):
    """The _gva entry points need H (value heads) to be a multiple of Hk (q/k heads)."""
    p = ctypes.c_void_p(16)
    rc = lib.gdn_recurrent_fwd_gva(p, p, p, p, p, None, p, None, 1, 4, H, Hk, 16, 16,
                                   _lib.GDN_DTYPE_BF16, None)
    assert rc == _lib.GDN_ERR_INVALID, lib.gdn_last_error()
    assert b"multiple" in lib.gdn_last_error() or b"Hk" in lib.gdn_last_error()
    rc = lib.gdn_chunk_fwd_gva(p, p, p, p, p, None, p, None, 1, 4, H, Hk, 16, 16, 64,
                               _lib.GDN_DTYPE_BF16, _lib.GDN_SEMANTICS_EXACT, None, 0, None)
    assert rc == _lib.GDN_ERR_INVALID, lib.gdn_last_error()


def test_packed_sequences_reject_bad_arguments(lib):
    p = ctypes.c_void_p(16)
    args = lambda cu, n, sem: (p, p, p, p, p, None, p, None, cu, n, 64, 2, 2, 16, 16, 64,
                               _lib.GDN_DTYPE_BF16, sem, None, 0, None)
    assert lib.gdn_chunk_fwd_varlen(*args(None, 2, _lib.GDN_SEMANTICS_EXACT)) == _lib.GDN_ERR_INVALID
    assert lib.gdn_chunk_fwd_varlen(*args(p, -1, _lib.GDN_SEMANTICS_EXACT)) == _lib.GDN_ERR_INVALID
    assert lib.gdn_chunk_fwd_varlen(*args(ctypes.c_void_p(18), 2, _lib.GDN_SEMANTICS_EXACT)) == \
        _lib.GDN_ERR_INVALID
    assert lib.gdn_chunk_fwd_varlen(*args(p, 2, _lib.GDN_SEMANTICS_REFERENCE)) == \
        _lib.GDN_ERR_UNSUPPORTED


def _bwd_args(p, B=1, T=64, H=2, Hk=2, dk=16, dv=32, ws=None, ws_bytes=0, out=None):
    o = p if out is None else out
    return ([p, p, p, p, p, None, p, None, o, o, o, o, o, None]
            + [B, T, H, Hk, dk, dv, _lib.GDN_DTYPE_BF16, ws, ws_bytes, None])


def test_backward_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)
    big = 1 << 30
    assert lib.gdn_chunk_bwd(*_bwd_args(p, dv=48, ws=p, ws_bytes=big)) == _lib.GDN_ERR_UNSUPPORTED
    assert b"dk <= 256" in lib.gdn_last_error()
    assert lib.gdn_chunk_bwd(*_bwd_args(p, dk=512, ws=p, ws_bytes=big)) == _lib.GDN_ERR_UNSUPPORTED
    assert lib.gdn_chunk_bwd(*_bwd_args(p, Hk=3)) == _lib.GDN_ERR_INVALID          # H % Hk
    assert lib.gdn_chunk_bwd(*_bwd_args(p)) == _lib.GDN_ERR_INVALID                # no workspace
    assert b"workspace" in lib.gdn_last_error()
    assert lib.gdn_chunk_bwd(*_bwd_args(p, ws=p, ws_bytes=big,
                                        out=ctypes.c_void_p(24))) == _lib.GDN_ERR_INVALID
    assert b"aligned" in lib.gdn_last_error()
    # packed sequences
    def varlen(cu, n):
        a = _bwd_args(p, ws=p, ws_bytes=big)
        return lib.gdn_chunk_bwd_varlen(*a[:14], cu, n, *a[15:])
    assert varlen(None, 2) == _lib.GDN_ERR_INVALID
    assert varlen(p, -1) == _lib.GDN_ERR_INVALID
    assert varlen(ctypes.c_void_p(18), 2) == _lib.GDN_ERR_INVALID
    assert b"aligned" in lib.gdn_last_error()


def test_backward_workspace_queries(lib):
    dense = lib.gdn_chunk_bwd_workspace_bytes(4, 4096, 16, 128, 128)
    assert dense > 1 << 30
    dense64 = lib.gdn_chunk_bwd_workspace_bytes(4, 4096, 16, 64, 64)
    # packed: an upper bound over any split of the tokens into n_seqs sequences
    assert lib.gdn_chunk_bwd_varlen_workspace_bytes(4, 4 * 4096, 16, 128, 128) >= dense
    assert lib.gdn_chunk_bwd_varlen_workspace_bytes(4, 4 * 4096, 16, 64, 64) >= dense64
    # the exact size of one call: fp32 takes the layout that fits every path, bf16
    # no more (less where the tensor-core hand-off runs: a GPU test checks that)
    for_ = lib.gdn_chunk_bwd_workspace_bytes_for
    assert for_(4, 4096, 16, 16, 128, 128, _lib.GDN_DTYPE_FP32) == dense
    assert for_(4, 4096, 16, 16, 128, 128, _lib.GDN_DTYPE_BF16) <= dense
    assert for_(4, 4096, 16, 16, 64, 64, _lib.GDN_DTYPE_BF16) == dense64
    for bad in ((0, 64, 2, 2, 16, 32, 1), (1, 64, 2, 0, 16, 32, 1), (1, 64, 2, 2, 16, 32, 7)):
        assert for_(*bad) == 0
    assert lib.gdn_chunk_bwd_varlen_workspace_bytes(4, 4 * 4096, 16, 128, 128) > \
        lib.gdn_chunk_bwd_varlen_workspace_bytes(1, 4 * 4096, 16, 128, 128)
    for args in ((0, 64, 2, 16, 32), (1, 0, 2, 16, 32), (1, 64, -1, 16, 32)):
        assert lib.gdn_chunk_bwd_workspace_bytes(*args) == 0
        assert lib.gdn_chunk_bwd_varlen_workspace_bytes(*args) == 0


def test_decode_layer_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)

    def call(T=1, dk=128, dv=128, A=p, gate=None, w=p, eps=1e-5):
        return lib.gdn_recurrent_fwd_layer(p, p, p, p, p, A, p, None, None, gate, w, eps, p,
                                           2, T, 2, 2, dk, dv, _lib.GDN_DTYPE_BF16, None)
    assert call(dk=48) == _lib.GDN_ERR_UNSUPPORTED
    assert call(A=None) == _lib.GDN_ERR_INVALID
    assert call(w=None) == _lib.GDN_ERR_INVALID
    assert call(w=ctypes.c_void_p(20)) == _lib.GDN_ERR_INVALID
    assert call(gate=ctypes.c_void_p(24)) == _lib.GDN_ERR_INVALID
    assert call(eps=-1.0) == _lib.GDN_ERR_INVALID


def test_chunk_layer_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)

    def call(dk=128, dv=128, dtype=_lib.GDN_DTYPE_BF16, A=p, gate=None, w=p, eps=1e-5):
        return lib.gdn_chunk_fwd_layer(p, p, p, p, p, A, p, None, None, gate, w, eps, p,
                                       2, 100, 2, 2, dk, dv, dtype, None)
    assert call(dtype=_lib.GDN_DTYPE_FP32) == _lib.GDN_ERR_UNSUPPORTED
    assert b"bf16" in lib.gdn_last_error()
    assert call(dk=64, dv=64) == _lib.GDN_ERR_UNSUPPORTED
    assert call(dv=96) == _lib.GDN_ERR_UNSUPPORTED
    assert b"multiple of 64" in lib.gdn_last_error()
    assert call(A=None) == _lib.GDN_ERR_INVALID
    assert call(w=None) == _lib.GDN_ERR_INVALID
    assert call(gate=ctypes.c_void_p(24)) == _lib.GDN_ERR_INVALID
    assert call(eps=float("nan")) == _lib.GDN_ERR_INVALID


def test_short_conv_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)
    bf16, fp32 = _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_FP32

    def call(x=p, w=p, si=None, so=None, y=p, B=2, T=10, C=64, K=4, act=1, dtype=bf16):
        return lib.gdn_short_conv_fwd(x, w, si, so, y, B, T, C, K, act, dtype, None)
    assert call(K=0) == _lib.GDN_ERR_UNSUPPORTED
    assert call(K=9) == _lib.GDN_ERR_UNSUPPORTED
    assert call(C=60) == _lib.GDN_ERR_UNSUPPORTED          # bf16: multiple of 8
    assert call(C=62, dtype=fp32) == _lib.GDN_ERR_UNSUPPORTED
    assert call(act=2) == _lib.GDN_ERR_INVALID
    assert call(dtype=7) == _lib.GDN_ERR_INVALID
    assert call(w=None) == _lib.GDN_ERR_INVALID
    assert call(w=ctypes.c_void_p(20)) == _lib.GDN_ERR_INVALID
    assert call(x=ctypes.c_void_p(24)) == _lib.GDN_ERR_INVALID
    assert call(si=ctypes.c_void_p(40)) == _lib.GDN_ERR_INVALID
    assert call(B=-1) == _lib.GDN_ERR_INVALID
    assert call(B=0) == _lib.GDN_OK and call(C=0) == _lib.GDN_OK
    assert call(T=0) == _lib.GDN_OK                          # no state to carry


def test_gated_rmsnorm_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)
    bf16, fp32 = _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_FP32

    def call(o=p, gate=None, w=p, eps=1e-5, y=p, rows=4, dv=128, dtype=bf16):
        return lib.gdn_gated_rmsnorm_fwd(o, gate, w, eps, y, rows, dv, dtype, None)
    assert call(dv=100) == _lib.GDN_ERR_UNSUPPORTED          # bf16: multiple of 8
    assert call(dv=2048) == _lib.GDN_ERR_UNSUPPORTED
    assert call(dv=1024, dtype=fp32) == _lib.GDN_ERR_UNSUPPORTED
    assert call(eps=-1.0) == _lib.GDN_ERR_INVALID
    assert call(w=None) == _lib.GDN_ERR_INVALID
    assert call(gate=ctypes.c_void_p(24)) == _lib.GDN_ERR_INVALID
    assert call(rows=-1) == _lib.GDN_ERR_INVALID
    assert call(rows=0) == _lib.GDN_OK


def test_chunk_layer_varlen_rejects_bad_arguments(lib):
    """Checked on the host before any CUDA call."""
    p = ctypes.c_void_p(16)

    def call(cu=p, n=2, dtype=_lib.GDN_DTYPE_BF16):
        return lib.gdn_chunk_fwd_layer_varlen(p, p, p, p, p, p, p, None, None, None, p, 1e-5, p,
                                              cu, n, 100, 2, 2, 128, 128, dtype, None)
    assert call(n=-1) == _lib.GDN_ERR_INVALID
    assert call(cu=None) == _lib.GDN_ERR_INVALID
    assert call(cu=ctypes.c_void_p(18)) == _lib.GDN_ERR_INVALID
    assert call(dtype=_lib.GDN_DTYPE_FP32) == _lib.GDN_ERR_UNSUPPORTED


def test_empty_problem_is_a_no_op(lib):
    # B*H == 0: nothing to launch, no CUDA call, OK.
    assert _call_recurrent(lib, B=0) == _lib.GDN_OK
    assert _call_chunk(lib, H=0) == _lib.GDN_OK


def test_workspace_query(lib):
    """The two-launch form (bf16, dk 128, dv % 64 == 0, dense): 24 KB per
    chunk-head for the per-chunk operands.  Zero on the other tcgen05 shapes
    (dk 256, packed sequences) and for the reference semantics; non-zero where
    the call runs on the warp-level tensor-core kernels (fp32 inputs, other
    bf16 shapes), growing with the work."""
    bf16, fp32 = _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_FP32
    q = lib.gdn_chunk_workspace_bytes
    assert q(4, 4096, 16, 128, 128, 64, bf16, 0) == 4 * 16 * 64 * 24576
    assert q(1, 65, 2, 128, 192, 64, bf16, 0) == 2 * 2 * 24576    # partial last chunk
    assert q(8, 2048, 6, 256, 512, 64, bf16, 0) == 0
    assert q(2, 100, 2, 128, 128, 64, fp32, _lib.GDN_SEMANTICS_REFERENCE) == 0
    assert q(2, 100, 2, 128, 48, 64, fp32, 0) == 0          # dv % 32 != 0: CUDA cores
    small = q(1, 64, 1, 64, 64, 64, fp32, 0)
    assert small > 0 and q(2, 64, 1, 64, 64, 64, fp32, 0) > small
    assert q(1, 64, 1, 64, 64, 64, bf16, 0) == small        # same fp32 intermediates
    assert q(1, 64, 1, 128, 96, 64, bf16, 0) > 0            # dv % 64 != 0
    assert q(0, 64, 1, 64, 64, 64, fp32, 0) == 0 and q(1, 0, 1, 64, 64, 64, fp32, 0) == 0
    # packed sequences: room for one partial chunk per sequence, and the offsets
    v = lib.gdn_chunk_varlen_workspace_bytes
    assert v(3, 64, 1, 64, 64, 64, fp32, 0) > q(1, 64, 1, 64, 64, 64, fp32, 0)
    assert v(3, 64, 1, 128, 128, 64, bf16, 0) == 0


def test_chunk_rejects_missing_workspace(lib):
    """A call that needs a workspace and gets none is refused on the host."""
    p = ctypes.c_void_p(16)
    rc = lib.gdn_chunk_fwd(p, p, p, p, p, None, p, None, 1, 64, 1, 64, 64, 64,
                           _lib.GDN_DTYPE_FP32, 0, None, 0, None)
    assert rc == _lib.GDN_ERR_INVALID and b"workspace" in lib.gdn_last_error()


def test_error_raises_with_message(lib):
    rc = _call_chunk(lib, chunk=48)
    with pytest.raises(_lib.GDNError, match="chunk=48"):
        _lib.check(rc, "gdn_chunk_fwd")


def _cpu_inputs(B=1, T=4, H=2, dk=16, dv=16, dtype=torch.float32):
    q = torch.zeros(B, T, H, dk, dtype=dtype)
    return q, q.clone(), torch.zeros(B, T, H, dv, dtype=dtype), torch.zeros(B, T, H), \
        torch.zeros(B, T, H)


def test_ops_reject_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        ops.chunk_gated_delta_rule(*_cpu_inputs())
    with pytest.raises(ValueError, match="CUDA"):
        ops.fused_recurrent_gated_delta_rule(*_cpu_inputs())


def test_ops_reject_bad_semantics():
    with pytest.raises(ValueError, match="semantics"):
        ops.chunk_gated_delta_rule(*_cpu_inputs(), semantics="fast")


def test_reference_names_exported():
    import gated_deltanet_jax_b200 as pkg
    for name in ("chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule",
                 "chunk_gated_delta_rule_fwd", "fused_recurrent_gated_delta_rule_fwd",
                 "GatedDeltaNetConfig"):
        assert hasattr(pkg, name)
    assert ops.chunk_gated_delta_rule is ops.chunk_gated_delta_rule_fwd
    assert ops.fused_recurrent_gated_delta_rule_fwd is ops.fused_recurrent_gated_delta_rule


def test_mode_switch_rejects_unknown_mode():
    from gated_deltanet_jax_b200 import GatedDeltaNetConfig, delta_rule
    cfg = GatedDeltaNetConfig(attn_mode="parallel")
    with pytest.raises(ValueError, match="Unknown mode parallel"):
        delta_rule(cfg, *_cpu_inputs())


def test_config_defaults_match_reference():
    from gated_deltanet_jax_b200 import GatedDeltaNetConfig
    c = GatedDeltaNetConfig()
    assert (c.attn_mode, c.hidden_size, c.head_dim, c.num_heads, c.expand_v, c.conv_size,
            c.num_hidden_layers, c.norm_eps, c.vocab_size) == \
        ("chunk", 2048, 256, 6, 2.0, 4, 21, 1e-6, 32000)
    assert c.num_v_heads is None and c.use_gate and c.use_short_conv


def test_two_phase_entry_points_check_arguments_on_the_host(lib):
    """gdn_chunk_prepare / gdn_chunk_scan refuse, before any CUDA call: shapes
    outside bf16 dk=128 dv%64, a missing or short workspace, a transition scan
    with an initial state or without hT, unaligned pointers."""
    p = ctypes.c_void_p(16)
    bf16 = _lib.GDN_DTYPE_BF16
    need = lib.gdn_chunk_workspace_bytes(1, 64, 2, 128, 64, 64, bf16, 0)
    assert need == 2 * 24576
    prep = lambda dk=128, dtype=bf16, ws=p, nb=need: lib.gdn_chunk_prepare(  # noqa: E731
        p, p, p, p, 1, 64, 2, 2, dk, dtype, ws, nb, None)
    assert prep(dk=64) == _lib.GDN_ERR_UNSUPPORTED
    assert prep(dtype=_lib.GDN_DTYPE_FP32) == _lib.GDN_ERR_UNSUPPORTED
    assert prep(ws=None) == _lib.GDN_ERR_INVALID and b"workspace" in lib.gdn_last_error()
    assert prep(nb=need - 1) == _lib.GDN_ERR_INVALID
    assert prep(ws=ctypes.c_void_p(24)) == _lib.GDN_ERR_INVALID

    def scan(h0=None, hT=p, transition=1, dv=64, o=None, q=p):
        return lib.gdn_chunk_scan(q, p, p, p, p, h0, o, hT, 1, 64, 2, 2, 128, dv, bf16,
                                  transition, p, need, None)
    assert scan(h0=p) == _lib.GDN_ERR_INVALID and b"h0 must be NULL" in lib.gdn_last_error()
    assert scan(hT=None) == _lib.GDN_ERR_INVALID
    assert scan(transition=2) == _lib.GDN_ERR_INVALID
    assert scan(dv=96) == _lib.GDN_ERR_UNSUPPORTED
    assert scan(transition=0, o=ctypes.c_void_p(40)) == _lib.GDN_ERR_INVALID
    assert scan(q=None) == _lib.GDN_ERR_INVALID


def test_fold_states_checks_arguments_on_the_host(lib):
    p = ctypes.c_void_p(16)
    fold = lambda dk=128, dv=64, ld=192, P=2, BH=3, out=p: lib.gdn_fold_states(  # noqa: E731
        p, p, None, out, P, BH, dk, dv, ld, None)
    assert fold(dk=64) == _lib.GDN_ERR_UNSUPPORTED
    assert fold(dv=48) == _lib.GDN_ERR_UNSUPPORTED
    assert fold(ld=190) == _lib.GDN_ERR_INVALID and b"ld" in lib.gdn_last_error()
    assert fold(ld=32) == _lib.GDN_ERR_INVALID
    assert fold(P=-1) == _lib.GDN_ERR_INVALID
    assert fold(out=None) == _lib.GDN_ERR_INVALID
    assert fold(out=ctypes.c_void_p(20)) == _lib.GDN_ERR_INVALID
    assert fold(BH=0) == _lib.GDN_OK          # nothing to fold
