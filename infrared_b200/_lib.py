"""ctypes binding of ``libinfrared_b200.so`` (the C ABI in include/infrared_b200.h).

The library is built in-tree next to this file (``python -m
infrared_b200._build``). Loading fails loudly when it is missing: the
package has no CPU or PyTorch fallback for its kernels.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import (POINTER, c_char_p, c_float, c_int, c_int32, c_int64,
                    c_size_t, c_void_p)
from pathlib import Path

import os

# INFRARED_B200_LIB points at another build of the library (tuning variants).
LIB_PATH = Path(os.environ.get("INFRARED_B200_LIB") or
                Path(__file__).resolve().with_name("libinfrared_b200.so"))

IR_DTYPE_F32, IR_DTYPE_BF16, IR_DTYPE_F16 = 0, 1, 2
IR_OK, IR_ERR_INVALID_ARG, IR_ERR_UNSUPPORTED, IR_ERR_CUDA, IR_ERR_WORKSPACE = range(5)
IR_DECODE_DYNAMIC_TAIL = 1   # ir_decode_shape.flags (the workspace zero-filled)
IR_DECODE_INLINE_MERGE = 2
IR_NOALLOC_WORKSPACE_BYTES = 8 << 20

DEVERR_BITS = {
    0x1: "BLOCK_ID",
    0x2: "CONTEXT_LEN",
    0x4: "SLOT",
    0x8: "NOT_BLOCKED",
    0x10: "MASK",
    0x20: "TIMEOUT",
    0x40: "WRITE_SLOT",
}


class InfraredB200Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"infrared_b200 status {status}: {message}")
        self.status = status


class UnsupportedShape(InfraredB200Error):
    """The shape or dtype is outside what the kernels implement."""


class DecodeShape(ctypes.Structure):
    """Mirror of ``ir_decode_shape``."""

    _fields_ = [
        ("batch", c_int),
        ("num_heads", c_int),
        ("num_kv_heads", c_int),
        ("head_dim", c_int),
        ("block_size", c_int),
        ("max_blocks", c_int),
        ("bt_stride", c_int64),
        ("q_stride", c_int64),
        ("out_stride", c_int64),
        ("num_slots", c_int64),
        ("scale", c_float),
        ("dtype", c_int),
        ("flags", c_int),
    ]


class PrefillShape(ctypes.Structure):
    """Mirror of ``ir_prefill_shape``."""

    _fields_ = [
        ("num_seqs", c_int),
        ("total_q", c_int),
        ("num_heads", c_int),
        ("num_kv_heads", c_int),
        ("head_dim", c_int),
        ("block_size", c_int),
        ("max_blocks", c_int),
        ("bt_stride", c_int64),
        ("q_stride", c_int64),
        ("out_stride", c_int64),
        ("num_slots", c_int64),
        ("scale", c_float),
        ("dtype", c_int),
    ]


# (name, restype, argtypes) of every exported function
_SIGNATURES = {
    "ir_set_prefill_path": (c_int, [c_int]),
    "ir_paged_decode_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_int64, c_void_p, c_void_p,
                                     POINTER(DecodeShape), c_void_p, c_size_t, c_void_p,
                                     c_void_p]),
    "ir_kv_proj_rope_write": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                      c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                      c_int, c_void_p, c_void_p]),
    "ir_peer_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "ir_peer_free": (c_int, [c_void_p]),
    "ir_peer_handle": (c_int, [c_void_p, c_void_p]),
    "ir_peer_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "ir_peer_close": (c_int, [c_void_p]),
    "ir_peer_exchange_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ir_peer_exchange": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, POINTER(c_void_p),
                                 c_size_t, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                 c_void_p]),
    "ir_derive_varlen_metadata": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_int,
                                          c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p]),
    "ir_paged_prefill_plan": (c_int, [POINTER(PrefillShape), POINTER(c_int)]),
    "ir_paged_prefill_workspace_size": (c_size_t, [POINTER(PrefillShape)]),
    "ir_paged_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, POINTER(PrefillShape), c_void_p, c_size_t, c_void_p,
                                 c_void_p]),
    "ir_version": (c_int, []),
    "ir_last_error": (c_char_p, []),
    "ir_deverr_name": (c_char_p, [c_int]),
    "ir_set_decode_path": (c_int, [c_int]),
    "ir_debug_stall_next_decode": (c_int, []),
    "ir_paged_decode_plan": (c_int, [POINTER(DecodeShape), POINTER(c_int), POINTER(c_int)]),
    "ir_paged_decode_workspace_size": (c_size_t, [POINTER(DecodeShape)]),
    "ir_cache_write": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                               c_void_p, c_int64, c_int, c_int, c_int64, c_int,
                               c_void_p, c_void_p]),
    "ir_cache_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                c_int64, c_int, c_void_p, c_void_p]),
    "ir_build_decode_inputs": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int,
                                       c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_int, c_void_p]),
    "ir_derive_block_metadata": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int,
                                         c_int, c_int64, c_int, c_void_p, c_int64,
                                         c_void_p, c_void_p, c_void_p]),
    "ir_paged_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, POINTER(DecodeShape), c_void_p, c_size_t,
                                c_void_p, c_void_p]),
    "ir_paged_decode_write": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                      POINTER(DecodeShape), c_void_p, c_size_t,
                                      c_void_p, c_void_p]),
    "ir_paged_decode_rope_write": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                           c_int64, c_void_p, c_void_p,
                                           POINTER(DecodeShape), c_void_p, c_size_t,
                                           c_void_p, c_void_p]),
    "ir_paged_decode_lse": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, POINTER(DecodeShape), c_void_p,
                                    c_size_t, c_void_p, c_void_p]),
    "ir_lse_merge": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int,
                             c_int, c_int, c_int, c_int, c_void_p]),
    "ir_paged_decode_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, POINTER(DecodeShape), c_void_p,
                                        c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m infrared_b200._build` "
                    "(infrared_b200 has no fallback for its CUDA kernels)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int) -> None:
    """Raise the matching exception for a non-zero status."""
    if status == IR_OK:
        return
    msg = (load().ir_last_error() or b"").decode(errors="replace")
    if status == IR_ERR_UNSUPPORTED:
        raise UnsupportedShape(status, msg)
    raise InfraredB200Error(status, msg)


def exported_names() -> list[str]:
    return list(_SIGNATURES)
