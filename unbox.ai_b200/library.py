"""ctypes binding of libunbox_b200.so (the C ABI in include/unbox_b200.h).

The library is loaded from ``unbox.ai_b200/lib/``; there is no fallback: if the
file is missing or fails to load, every op raises. Signatures mirror the header
one to one.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libunbox_b200.so")

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
SCHEDULE_AUTO, SCHEDULE_BALANCED, SCHEDULE_SPLIT = 0, 1, 2
FLAG_OVERLAP_PREVIOUS = 1
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = 0, 1, 2, 3, 4
DEVERR = {1: "page id outside the pool", 2: "context longer than its block-table row",
          4: "negative context length", 8: "pipeline wait timed out", 16: "append slot outside the pool",
          32: "rotary position outside the rope table", 64: "cascade work or merge item out of range"}

# exported symbol -> (restype, argtypes); the test suite checks this list against the header
_i32, _i64, _vp, _f32, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "ubx_status_string": (ctypes.c_char_p, [_i32]),
    "ubx_last_error": (ctypes.c_char_p, []),
    "ubx_version": (_i32, []),
    "ubx_kv_append": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _i32, _i32, _i32, _i64,
                             _i32, _vp, _vp]),
    "ubx_slot_mapping": (_i32, [_vp, _i64, _vp, _vp, _i32, _i32, _i32, _vp]),
    "ubx_prefill_kv_write": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i32, _i64, _i64, _i32,
                                    _i32, _i32, _i64, _i32, _vp, _vp, _i32, _vp]),
    "ubx_paged_decode_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_sz)]),
    "ubx_workspace_init": (_i32, [_vp, _sz, _vp]),
    "ubx_paged_decode_attention": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64,
                                          _i64, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32, _i32, _i32,
                                          _vp, _sz, _vp]),
    "ubx_paged_decode_append_attention": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64,
                                                 _vp, _i64, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i64,
                                                 _i32, _f32, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "ubx_qk_norm_rope_append": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _f32, _vp, _i64,
                                       _i32, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp,
                                       _i64, _i32, _i64, _i32, _i32, _i32, _i32, _vp, _vp]),
    "ubx_paged_decode_prep_attention": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _f32, _vp, _i64, _i32,
                                               _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _i32,
                                               _i32, _i32, _i32, _i64, _i32, _f32, _i32, _i32, _i32, _i32, _vp, _sz,
                                               _vp]),
    "ubx_read_device_error": (_i32, [_vp, ctypes.POINTER(ctypes.c_int32), _i32, _vp]),
    "ubx_paged_decode_attention_lse": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp,
                                              _i64, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i64, _i32,
                                              _f32, _i32, _i32, _i32, _i32, _vp, _vp, _sz, _vp]),
    "ubx_cascade_workspace_size": (_i32, [_i32, _i32, _i32, _i32, ctypes.POINTER(_sz)]),
    "ubx_cascade_prefix_attention": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i32,
                                            _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _sz, _vp, _i32, _vp]),
    "ubx_cascade_merge": (_i32, [_vp, _i64, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _i32,
                                 _vp]),
    "ubx_cascade_attention": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64,
                                     _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32,
                                     _i32, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _sz, _vp, _sz,
                                     _vp]),
    "ubx_kv_wire_header_init": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.c_uint64]),
    "ubx_kv_wire_header_check": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, ctypes.c_uint64]),
    "ubx_kv_pages_copy": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i32, _i32,
                                 _i64, _i32, _vp, _vp, _vp]),
    "ubx_enable_peer_access": (_i32, [_i32]),
    "ubx_ipc_get_handle": (_i32, [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)]),
    "ubx_ipc_open_handle": (_i32, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "ubx_ipc_close_handle": (_i32, [_vp]),
    "ubx_paged_decode_attention_noalloc": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp,
                                                  _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32,
                                                  _i32, _i32, _vp, _vp]),
}



class KVWireHeader(ctypes.Structure):
    """ubx_kv_wire_header: the 64-byte header of a KV page message (little-endian)."""
    _fields_ = [("magic", ctypes.c_char * 8), ("version", ctypes.c_uint32), ("header_bytes", ctypes.c_uint32),
                ("dtype", ctypes.c_uint32), ("num_layers", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("block_size", ctypes.c_uint32), ("num_pages", ctypes.c_uint32),
                ("payload_bytes", ctypes.c_uint64), ("checksum", ctypes.c_uint64),
                ("reserved", ctypes.c_uint8 * 8)]


assert ctypes.sizeof(KVWireHeader) == 64

_lib = None
_lock = threading.Lock()


class UbxError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load():
    """Load the shared library (once). Raises if it is absent or unloadable."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} not found: build it with `python __graft_entry__.py build` "
                    "(there is no CPU fallback for this op)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str):
    if status != OK:
        lib = load()
        msg = lib.ubx_last_error().decode() or lib.ubx_status_string(status).decode()
        exc = ValueError if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED) else RuntimeError
        err = exc(f"{what}: {msg}")
        err.status = status
        raise err
