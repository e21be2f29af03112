"""ctypes binding of ``libgdn_b200.so`` (the C ABI in ``include/gdn.h``).

Loading fails loudly: there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from typing import Optional

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libgdn_b200.so")

GDN_OK = 0
GDN_ERR_INVALID = 1
GDN_ERR_UNSUPPORTED = 2
GDN_ERR_CUDA = 3

GDN_DTYPE_FP32 = 0
GDN_DTYPE_BF16 = 1

GDN_SEMANTICS_EXACT = 0
GDN_SEMANTICS_REFERENCE = 1

#: Every symbol ``include/gdn.h`` declares.
EXPORTED_SYMBOLS = (
    "gdn_recurrent_fwd",
    "gdn_chunk_fwd",
    "gdn_recurrent_fwd_gva",
    "gdn_recurrent_fwd_layer",
    "gdn_chunk_fwd_layer",
    "gdn_chunk_fwd_layer_varlen",
    "gdn_chunk_fwd_gva",
    "gdn_chunk_fwd_varlen",
    "gdn_chunk_bwd",
    "gdn_chunk_bwd_noalloc",
    "gdn_chunk_bwd_workspace_bytes",
    "gdn_chunk_bwd_workspace_bytes_for",
    "gdn_chunk_bwd_varlen",
    "gdn_chunk_bwd_varlen_workspace_bytes",
    "gdn_chunk_workspace_bytes",
    "gdn_chunk_varlen_workspace_bytes",
    "gdn_chunk_prepare",
    "gdn_chunk_scan",
    "gdn_fold_states",
    "gdn_short_conv_fwd",
    "gdn_gated_rmsnorm_fwd",
    "gdn_last_error",
    "gdn_reload_kernel_overrides",
    "gdn_device_error",
    "gdn_abi_version",
    "gdn_binary_version",
)

_lock = threading.Lock()
_lib = None

_vp, _i, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t


class GDNError(RuntimeError):
    """A non-OK status from the C ABI, with the library's message."""

    def __init__(self, code: int, func: str, message: str):
        self.code = code
        kind = {GDN_ERR_INVALID: "invalid argument", GDN_ERR_UNSUPPORTED: "unsupported",
                GDN_ERR_CUDA: "CUDA error"}.get(code, f"status {code}")
        super().__init__(f"{func}: {kind}: {message}")


def _declare(lib):
    lib.gdn_recurrent_fwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _i, _i, _i, _i, _i, _i, _vp]
    lib.gdn_recurrent_fwd.restype = _i
    lib.gdn_recurrent_fwd_layer.argtypes = ([_vp] * 11 + [ctypes.c_float, _vp] + [_i] * 7
                                            + [_vp])
    lib.gdn_recurrent_fwd_layer.restype = _i
    lib.gdn_chunk_fwd_layer.argtypes = ([_vp] * 11 + [ctypes.c_float, _vp] + [_i] * 7 + [_vp])
    lib.gdn_chunk_fwd_layer.restype = _i
    lib.gdn_chunk_fwd_layer_varlen.argtypes = ([_vp] * 11 + [ctypes.c_float, _vp, _vp]
                                               + [_i] * 7 + [_vp])
    lib.gdn_chunk_fwd_layer_varlen.restype = _i
    lib.gdn_chunk_fwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.gdn_chunk_fwd.restype = _i
    lib.gdn_recurrent_fwd_gva.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                          _i, _i, _i, _i, _i, _i, _i, _vp]
    lib.gdn_recurrent_fwd_gva.restype = _i
    lib.gdn_chunk_fwd_gva.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.gdn_chunk_fwd_gva.restype = _i
    lib.gdn_chunk_fwd_varlen.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                         _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.gdn_chunk_fwd_varlen.restype = _i
    lib.gdn_chunk_bwd.argtypes = [_vp] * 14 + [_i] * 7 + [_vp, _sz, _vp]
    lib.gdn_chunk_bwd.restype = _i
    lib.gdn_chunk_bwd_noalloc.argtypes = [_vp] * 14 + [_i] * 7 + [_vp]
    lib.gdn_chunk_bwd_noalloc.restype = _i
    lib.gdn_chunk_bwd_workspace_bytes.argtypes = [_i] * 5
    lib.gdn_chunk_bwd_workspace_bytes.restype = _sz
    lib.gdn_chunk_bwd_workspace_bytes_for.argtypes = [_i] * 7
    lib.gdn_chunk_bwd_workspace_bytes_for.restype = _sz
    lib.gdn_chunk_bwd_varlen.argtypes = [_vp] * 15 + [_i] * 7 + [_vp, _sz, _vp]
    lib.gdn_chunk_bwd_varlen.restype = _i
    lib.gdn_chunk_bwd_varlen_workspace_bytes.argtypes = [_i] * 5
    lib.gdn_chunk_bwd_varlen_workspace_bytes.restype = _sz
    lib.gdn_chunk_workspace_bytes.argtypes = [_i] * 8
    lib.gdn_chunk_workspace_bytes.restype = _sz
    lib.gdn_chunk_varlen_workspace_bytes.argtypes = [_i] * 8
    lib.gdn_chunk_varlen_workspace_bytes.restype = _sz
    lib.gdn_chunk_prepare.argtypes = [_vp] * 4 + [_i] * 6 + [_vp, _sz, _vp]
    lib.gdn_chunk_prepare.restype = _i
    lib.gdn_chunk_scan.argtypes = [_vp] * 8 + [_i] * 8 + [_vp, _sz, _vp]
    lib.gdn_chunk_scan.restype = _i
    lib.gdn_fold_states.argtypes = [_vp] * 4 + [_i] * 5 + [_vp]
    lib.gdn_fold_states.restype = _i
    lib.gdn_short_conv_fwd.argtypes = [_vp] * 5 + [_i] * 6 + [_vp]
    lib.gdn_short_conv_fwd.restype = _i
    lib.gdn_gated_rmsnorm_fwd.argtypes = [_vp] * 3 + [ctypes.c_float, _vp, ctypes.c_longlong,
                                                      _i, _i, _vp]
    lib.gdn_gated_rmsnorm_fwd.restype = _i
    lib.gdn_last_error.argtypes = []
    lib.gdn_last_error.restype = ctypes.c_char_p
    lib.gdn_reload_kernel_overrides.argtypes = []
    lib.gdn_reload_kernel_overrides.restype = None
    lib.gdn_device_error.argtypes = [_i]
    lib.gdn_device_error.restype = _i
    lib.gdn_abi_version.argtypes = []
    lib.gdn_abi_version.restype = _i
    lib.gdn_binary_version.argtypes = []
    lib.gdn_binary_version.restype = _i


def load(path: str = LIB_PATH):
    """Load (once) and return the library; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m gated_deltanet_jax_b200._build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(path)
            _declare(lib)
            _lib = lib
        return _lib


@contextlib.contextmanager
def kernel_env(name: str, value: Optional[str]):
    """Run the body with environment variable ``name`` set to ``value`` (None:
    unset) as the library's kernel choice, then restore it (cross-checks of one
    kernel against another; the library reads these variables only on
    gdn_reload_kernel_overrides)."""
    old = os.environ.get(name)
    if value is None:
        os.environ.pop(name, None)
    else:
        os.environ[name] = value
    load().gdn_reload_kernel_overrides()
    try:
        yield
    finally:
        if old is None:
            os.environ.pop(name, None)
        else:
            os.environ[name] = old
        load().gdn_reload_kernel_overrides()


def check(rc: int, func: str) -> None:
    if rc != GDN_OK:
        msg = load().gdn_last_error().decode(errors="replace")
        raise GDNError(rc, func, msg)
