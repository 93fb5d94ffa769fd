"""ctypes binding of the in-tree CUDA library ``libgdn_b200.so`` (C ABI in include/gdn_b200.h).

The library is loaded once per process.  There is no fallback: if the shared object is
missing, every operator raises.  Build it with ``python -m`` / ``__graft_entry__.build()``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgdn_b200.so")

GDN_OK = 0
GDN_F32, GDN_BF16 = 0, 1
GDN_CONV_HF, GDN_CONV_ELEM = 0, 1

_i32, _i64, _f32, _vp = C.c_int, C.c_int64, C.c_float, C.c_void_p
_sz = C.c_size_t

# name -> (restype, argtypes); must match include/gdn_b200.h
SIGNATURES = {
    "gdn_last_error": (C.c_char_p, []),
    "gdn_version": (_i32, []),
    "gdn_gated_rmsnorm": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp]),
    "gdn_conv_update": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64,
                               _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "gdn_prefill_conv": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _vp, _vp, _vp, _i64, _vp, _vp, _i32, _i32,
                                _i32, _i32, _vp, _vp]),
    "gdn_recurrent": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp,
                             _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                             _i32, _vp, _vp]),
    "gdn_decode_layer_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "gdn_decode_layer": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _f32,
                                _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _i32, _vp, _vp]),
    "gdn_decode_layer_rows": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp, _i64, _vp, _f32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz,
                                     _i32, _vp, _vp]),
    "gdn_decode_layer_noalloc_max_bytes": (_sz, []),
    "gdn_decode_layer_noalloc_max_ticket_bytes": (_sz, []),
    "gdn_decode_layer_noalloc": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp,
                                        _f32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "gdn_chunk_prefill": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i32, _i64, _vp, _vp,
                                 _vp, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _vp,
                                 _vp]),
    "gdn_chunk_prefill_gates": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _i64,
                                       _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32,
                                       _i32, _vp, _vp]),
    "gdn_rmsnorm": (_i32, [_vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp]),
    "gdn_attn_decode_prep": (_i32, [_vp, _i64, _vp, _vp, _f32, _vp, _vp, _i64, _i32, _vp, _vp, _vp, _vp, _i32,
                                    _i32, _i32, _i32, _i32, _vp]),
    "gdn_attn_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "gdn_attn_decode": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _vp, _vp, _i32, _vp, _f32, _vp, _i32, _i32,
                               _i32, _i32, _vp, _sz, _i32, _vp, _vp]),
    "gdn_ar_buffer_bytes": (_sz, [_i32, _sz, _i32]),
    "gdn_ar_alloc": (_i32, [_sz, C.POINTER(_vp)]),
    "gdn_ar_free": (_i32, [_vp]),
    "gdn_ar_ipc_handle": (_i32, [_vp, _vp]),
    "gdn_ar_ipc_open": (_i32, [_vp, C.POINTER(_vp)]),
    "gdn_ar_ipc_close": (_i32, [_vp]),
    "gdn_allreduce": (_i32, [_vp, _vp, _sz, _i32, _i32, _i32, _vp, _sz, C.c_uint32, _vp, _vp]),
    "gdn_linear": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "gdn_linear_plan": (_i32, [_i32, _i32, _i32, _i32, _i32, _vp]),
    "gdn_linear_ar_buffer_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gdn_linear_allreduce": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _vp,
                                    _i32, _i32, C.c_uint32, _vp, _i32, _vp]),
    "gdn_linear_push": (_i32, [_vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _vp,
                               _i32, _vp]),
    "gdn_ar_norm_buffer_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gdn_allreduce_add_rmsnorm": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _i32, _vp,
                                         _i32, C.c_uint32, _vp, _i32, _vp]),
    "gdn_push_partial": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _i32, _vp]),
    "gdn_pull_add_rmsnorm": (_i32, [_vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _i32, _vp, _i32, _i32,
                                    C.c_uint32, _vp, _i32, _vp]),
    "gdn_add_rmsnorm": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp]),
    "gdn_silu_mul": (_i32, [_vp, _i64, _i32, _vp, _i64, _i64, _i32, _vp]),
}
GDN_IPC_HANDLE_BYTES = 64

_lock = threading.Lock()
_lib = None


def load() -> C.CDLL:
    """Load libgdn_b200.so (raises RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"GDN CUDA library not found at {LIB_PATH}; build it with __graft_entry__.build() "
                    "(there is no CPU fallback)")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Raise RuntimeError with the library's message when a call returned non-zero."""
    if rc != GDN_OK:
        msg = load().gdn_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")
