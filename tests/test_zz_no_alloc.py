"""The allocation-free decode entry point, checked against the regular one.

Some callers may not allocate device memory while they serve: an engine
that hands out all GPU memory from one budget fixed at start-up, a plugin
running inside another runtime's process, or a binding from a language with
no device allocator of its own. They cannot provide the workspace that
``ir_paged_decode`` needs, so ``ir_paged_decode_noalloc`` keeps that scratch
in an array built into the library. These tests call it through the C ABI
(as such a caller would, with no workspace argument) on two calls in a row
with different queries, and check each result against the fp32 oracle at
the bf16 bar of the other parity tests (atol = rtol = 2e-2) and against
``ir_paged_decode``. The C2 shape splits sequences across CTAs, so the merge
kernel reads the pieces the decode kernel left in the shared array, and the
second call reads them over what the first call left there. A shape whose
scratch exceeds the built-in array is refused with a clear error.

This file sorts last so that a run stopping at the first failure has run
every other test before it; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import assert_close_bf16, oracle_decode_device
from infrared_b200 import _lib, ops
from infrared_b200 import workloads as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

TOL = 2e-2


def _shape(w, q, out):
    s = _lib.DecodeShape()
    s.batch = w.batch
    s.num_heads = w.num_heads
    s.num_kv_heads = w.num_kv_heads
    s.head_dim = w.head_dim
    s.block_size = w.block_size
    s.max_blocks = w.max_blocks
    s.bt_stride = w.max_blocks
    s.q_stride = q.stride(0)
    s.out_stride = out.stride(0)
    s.num_slots = w.num_slots
    s.scale = w.scale
    s.dtype = _lib.IR_DTYPE_BF16
    return s


def test_noalloc_matches_regular_decode_on_two_calls_in_a_row():
    lib = _lib.load()
    w = wl.c2(seed=5)
    q1, kp, vp, _, _ = wl.torch_values(w, 11, "cuda")
    q2 = wl.torch_values(w, 12, "cuda")[0]
    bt = torch.from_numpy(w.block_tables).cuda()
    ctx = torch.from_numpy(w.context_lens).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # the built-in scratch serves the static schedule (no dynamic tail units)
    _, ctas, need = ops.decode_plan(q1, kp, bt, w.block_size, w.scale,
                                    inline_merge=False)
    assert 0 < need <= _lib.IR_NOALLOC_WORKSPACE_BYTES
    # more CTAs per kv-head group than sequences: sequences are cut into
    # pieces whose partials go through the scratch array to the merge kernel
    assert ctas > w.batch
    for q in (q1, q2):
        out = torch.empty_like(q)
        rc = lib.ir_paged_decode_noalloc(out.data_ptr(), q.data_ptr(), kp.data_ptr(),
                                         vp.data_ptr(), bt.data_ptr(), ctx.data_ptr(),
                                         ctypes.byref(_shape(w, q, out)), err.data_ptr(),
                                         stream)
        assert rc == _lib.IR_OK, lib.ir_last_error()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert_close_bf16(got, oracle_decode_device(w, q, kp, vp), TOL)
        ref = ops.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got, ref.float().cpu().numpy(), atol=TOL, rtol=TOL)
    assert int(err.item()) == 0


def test_noalloc_refuses_shapes_beyond_its_scratch():
    lib = _lib.load()
    # the partials of 4096 sequences need far more than 8 MiB of scratch
    s = _lib.DecodeShape(batch=4096, num_heads=28, num_kv_heads=4, head_dim=128,
                         block_size=16, max_blocks=256, bt_stride=256, q_stride=28 * 128,
                         out_stride=28 * 128, num_slots=4096 * 256 * 16,
                         scale=128 ** -0.5, dtype=_lib.IR_DTYPE_BF16)
    assert lib.ir_paged_decode_workspace_size(ctypes.byref(s)) > _lib.IR_NOALLOC_WORKSPACE_BYTES
    rc = lib.ir_paged_decode_noalloc(None, None, None, None, None, None, ctypes.byref(s),
                                     None, None)
    assert rc == _lib.IR_ERR_WORKSPACE
    assert b"at most" in lib.ir_last_error()
