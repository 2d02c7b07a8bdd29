"""The C-ABI library: loads, exports every declared symbol, rejects bad arguments.

Runs without a GPU: only entry points whose argument checks fail before any
CUDA call are invoked.
"""

import ctypes
import re
from pathlib import Path

import pytest

from infrared_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(ir_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_builds_and_loads():
    lib = _lib.load()
    assert lib.ir_version() >= 100


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    decl = declared_functions()
    assert "ir_paged_decode" in decl and "ir_cache_write" in decl
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.exported_names(), f"{name} has no ctypes signature"


def test_deverr_names():
    lib = _lib.load()
    assert lib.ir_deverr_name(0) == b"BLOCK_ID"
    assert lib.ir_deverr_name(6) == b"WRITE_SLOT"
    assert lib.ir_deverr_name(99) == b""


def test_argument_errors_need_no_gpu():
    lib = _lib.load()
    rc = lib.ir_cache_write(None, None, 0, 0, None, None, None, 4, 2, 64, 16, 7, None, None)
    assert rc == _lib.IR_ERR_INVALID_ARG and b"dtype" in lib.ir_last_error()
    rc = lib.ir_cache_write(None, None, 0, 0, None, None, None, 4, 2, 64, 16, 1, None, None)
    assert rc == _lib.IR_ERR_INVALID_ARG
    rc = lib.ir_lse_merge(None, 0, None, 0, None, 0, 0, 1, 1, 64, 1, None)
    assert rc == _lib.IR_ERR_INVALID_ARG
    assert lib.ir_set_decode_path(5) == _lib.IR_ERR_INVALID_ARG
    rc = lib.ir_derive_block_metadata(None, 0, None, 0, 9, 1, 4, 16, None, 0, None, None, None)
    assert rc == _lib.IR_ERR_INVALID_ARG


@pytest.mark.parametrize("field,value,status", [
    ("head_dim", 96, _lib.IR_ERR_UNSUPPORTED),
    ("num_kv_heads", 3, _lib.IR_ERR_INVALID_ARG),      # 28 % 3 != 0
    ("block_size", 0, _lib.IR_ERR_INVALID_ARG),
    ("num_slots", 100, _lib.IR_ERR_INVALID_ARG),       # not a multiple of 16
    ("q_stride", 10, _lib.IR_ERR_INVALID_ARG),
    ("dtype", 9, _lib.IR_ERR_INVALID_ARG),
])
def test_decode_shape_validation(field, value, status):
    lib = _lib.load()
    s = _lib.DecodeShape(batch=2, num_heads=28, num_kv_heads=4, head_dim=128, block_size=16,
                         max_blocks=8, bt_stride=8, q_stride=28 * 128, out_stride=28 * 128,
                         num_slots=1024, scale=0.088, dtype=1)
    setattr(s, field, value)
    rc = lib.ir_paged_decode(None, None, None, None, None, None, ctypes.byref(s), None, 0,
                             None, None)
    assert rc == status, lib.ir_last_error()
    assert lib.ir_paged_decode_workspace_size(ctypes.byref(s)) == 0


def test_group_over_16_unsupported():
    lib = _lib.load()
    s = _lib.DecodeShape(batch=1, num_heads=34, num_kv_heads=2, head_dim=64, block_size=16,
                         max_blocks=1, bt_stride=1, q_stride=34 * 64, out_stride=34 * 64,
                         num_slots=16, scale=0.125, dtype=0)
    assert lib.ir_paged_decode(None, None, None, None, None, None, ctypes.byref(s), None, 0,
                               None, None) == _lib.IR_ERR_UNSUPPORTED
