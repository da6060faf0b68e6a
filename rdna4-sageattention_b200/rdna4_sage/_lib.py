"""ctypes binding of libsage_b200.so, the sm_100a kernel library (C ABI in include/sage_b200.h).

This takes the place of the reference's HIP launch layer (src/rdna4_sage/_hip.py:31-73: ctypes over
hipModuleLoadData / hipModuleLaunchKernel with packed argument blocks).  The library is built in-tree by
rdna4-sageattention_b200/build_ext.py; when it is missing or fails to load, every kernel call raises
RuntimeError (there is no fallback implementation behind this module).
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libsage_b200.so"
# RDNA4_SAGE_LIB selects another build of the same library (for example one compiled with different
# options); the default is the in-tree build next to this file.
LIB_PATH = os.environ.get("RDNA4_SAGE_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

SAGE_OK = 0
SAGE_ERR_UNSUPPORTED = 1
SAGE_ERR_INVALID = 2
SAGE_ERR_LAUNCH = 3
SAGE_ERR_TIMEOUT = 4
STATUS_NAMES = {0: "ok", 1: "unsupported", 2: "invalid argument", 3: "launch failure", 4: "kernel wait timeout"}

_c_i = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p
_c_f = ctypes.c_float
_c_d = ctypes.c_double
_c_sz = ctypes.c_size_t

# name -> (restype, argtypes); the C-ABI surface of include/sage_b200.h
SIGNATURES = {
    "sage_abi_version": (_c_i, []),
    "sage_last_error": (ctypes.c_char_p, []),
    "sage_qk_row_bytes": (_c_i, [_c_i]),
    "sage_v_amax": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64, _c_p, _c_p]),
    "sage_quant_q": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64, _c_f, _c_p, _c_p, _c_p]),
    "sage_quant_kv": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                             _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "sage_quant_sync_ints": (_c_i, [_c_i, _c_i]),
    "sage_quant_qkv": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64,
                              _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_p, _c_p, _c_p, _c_p, _c_p,
                              _c_p, _c_p, _c_p, _c_p]),
    "sage_quantize": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64,
                             _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_p, _c_p, _c_p, _c_p, _c_p,
                             _c_p, _c_p, _c_p, _c_p]),
    "sage_attn_fwd": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i,
                             _c_i, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p]),
    "sage_attn_fwd_rows": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i,
                                  _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p]),
    "sage_attn_fwd_chunked": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i,
                                     _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p]),
    "sage_workspace_bytes": (_c_sz, [_c_i, _c_i, _c_i, _c_i, _c_i, _c_i]),
    "sage_attention": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64, _c_i64,
                              _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_d, _c_i, _c_p, _c_i64, _c_i64,
                              _c_i64, _c_p, _c_p, _c_sz, _c_p, _c_p]),
    "sage_attention_static": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64,
                                     _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_d, _c_i, _c_p,
                                     _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p]),
    "sage_varlen_workspace_bytes": (_c_sz, [_c_i] * 6),
    "sage_attention_varlen": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_p, _c_p, _c_i, _c_i, _c_i,
                                     _c_i, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_d, _c_i, _c_p, _c_i64,
                                     _c_i64, _c_p, _c_p, _c_sz, _c_p, _c_p]),
    "sage_host_heads_per_chunk": (_c_i, [_c_i] * 7),
    "sage_host_chunk_plan": (_c_i, [_c_i] * 7 + [_c_p, _c_i]),
    "sage_host_workspace_bytes": (_c_sz, [_c_i] * 7),
    "sage_attention_host": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64,
                                   _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_d, _c_i, _c_p,
                                   _c_i64, _c_i64, _c_i64, _c_p, _c_i, _c_p, _c_sz, _c_p, _c_p]),
    "sage_host_multi_workspace_bytes": (_c_sz, [_c_i] * 8),
    "sage_attention_host_multi": (_c_i, [_c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_d, _c_i, _c_p,
                                         _c_i64, _c_i64, _c_i64, _c_p, _c_i, _c_i, _c_p, _c_p, _c_sz, _c_p, _c_p]),
    "sage_selftest_wait_timeout": (_c_i, [_c_p, _c_i, _c_p]),
    "sage_selftest_counter_timeout": (_c_i, [_c_p, _c_p, _c_i, _c_p]),
    "sage_status_sync": (_c_i, [_c_p, _c_p]),
    "sage_debug_record": (_c_i, [_c_i, _c_p]),
    "sage_selftest_debug_store": (_c_i, [_c_p, _c_i, _c_p]),
}
ABI_VERSION = 1

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once); raises RuntimeError if it is missing or incompatible."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"rdna4_sage: {LIB_NAME} is not built (run rdna4-sageattention_b200/build_ext.py)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                if handle.sage_abi_version() != ABI_VERSION:
                    raise RuntimeError(f"rdna4_sage: {LIB_NAME} ABI {handle.sage_abi_version()} != {ABI_VERSION}")
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    """Raise RuntimeError for a nonzero status, with the library's message (as _hip.py:47-49 does)."""
    if rc != SAGE_OK:
        msg = lib().sage_last_error().decode(errors="replace")
        raise RuntimeError(f"rdna4_sage: {what} failed: {STATUS_NAMES.get(rc, rc)}: {msg}")
