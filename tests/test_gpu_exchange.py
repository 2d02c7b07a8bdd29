"""The KV-chunk peer exchange kernel (``ir_peer_exchange``) on one GPU,
through the C ABI.

A world of one rank runs the whole kernel (flags, epochs, merge) with no
peer: its output is the rank's own partial, exactly. A world of two whose
second buffer is a local allocation nobody writes to is the bounded-wait
check: the wait for the missing peer's flags runs out after its limit,
TIMEOUT is reported through the error flag and the context stays usable.
Two real ranks are covered by ``test_gpu_multi.py`` (needs 2 GPUs).
"""

import ctypes
import time

import pytest
import torch

import infrared_b200 as irb
from gpu_helpers import DEV
from infrared_b200 import _lib, ops
from infrared_b200 import workloads as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.error_flag().zero_()
    yield
    ops.error_flag().zero_()


def _alloc(lib, world, rows, d):
    n = lib.ir_peer_exchange_bytes(world, rows, d)
    assert n > 0
    p = ctypes.c_void_p()
    _lib.check(lib.ir_peer_alloc(n, ctypes.byref(p)))
    return p.value


def _exchange(lib, bufs, world, rank, o, lse, out, rows_cap=None):
    b, h, d = out.shape
    nbytes = lib.ir_peer_exchange_bytes(world, rows_cap or b * h, d)
    arr = (ctypes.c_void_p * world)(*bufs)
    stream = ops._stream(torch.cuda.current_device())
    _lib.check(lib.ir_peer_exchange(out.data_ptr(), out.stride(0), o.data_ptr(), lse.data_ptr(),
                                    arr, nbytes, world, rank, b, h, d, ops.dtype_code(out.dtype),
                                    ops.error_flag().data_ptr(), stream))


@pytest.mark.parametrize("d,dtype,b,h,cap", [(128, torch.bfloat16, 5, 7, None),
                                             (64, torch.float16, 5, 7, None),
                                             (128, torch.float32, 5, 7, None),
                                             # a smaller batch than the buffer holds
                                             (128, torch.bfloat16, 5, 7, 64 * 7),
                                             # many rows per warp: 7168 rows on <= 148 CTAs
                                             (128, torch.bfloat16, 256, 28, None)])
def test_world_of_one_returns_own_partial(d, dtype, b, h, cap):
    lib = _lib.load()
    g = torch.Generator(device=DEV)
    g.manual_seed(d)
    o = torch.randn(b, h, d, generator=g, device=DEV)
    lse = torch.randn(b, h, generator=g, device=DEV)
    lse[1, 3] = -float("inf")  # an empty range: zeros, like ir_lse_merge
    want = o.clone()
    want[1, 3] = 0
    want = want.to(dtype)
    buf = _alloc(lib, 1, cap or b * h, d)
    try:
        outs = []
        for _ in range(3):  # the epoch advances; every call gives the same rows
            out = torch.empty(b, h, d, dtype=dtype, device=DEV)
            _exchange(lib, [buf], 1, 0, o, lse, out, cap)
            outs.append(out)
        torch.cuda.synchronize()
        for out in outs:
            assert torch.equal(out, want)
        # captured in a CUDA graph and replayed
        s = torch.cuda.Stream(DEV)
        s.wait_stream(torch.cuda.current_stream())
        cap_out = torch.empty(b, h, d, dtype=dtype, device=DEV)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                _exchange(lib, [buf], 1, 0, o, lse, cap_out, cap)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            cap_out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(cap_out, want)
        del graph
        ops.check_device_errors()
    finally:
        torch.cuda.synchronize()
        _lib.check(lib.ir_peer_free(buf))


def test_missing_peer_times_out_and_context_survives():
    """Several rows per warp (1792 rows on at most one CTA per SM): a warp
    whose wait for the silent peer ran out leaves that peer out of its later
    rows, so the call takes about one wait limit (2 s), not one per row."""
    lib = _lib.load()
    b, h, d = 64, 28, 128
    o = torch.ones(b, h, d, device=DEV)
    lse = torch.zeros(b, h, device=DEV)
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device=DEV)
    own = _alloc(lib, 2, b * h, d)
    silent = _alloc(lib, 2, b * h, d)  # stands for a peer that never stores
    try:
        t0 = time.perf_counter()
        _exchange(lib, [own, silent], 2, 0, o, lse, out)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 8
        with pytest.raises(irb.DeviceError, match="TIMEOUT"):
            ops.check_device_errors()
        # the missing partial is left out: the rank's own rows come back
        assert torch.equal(out, o.to(torch.bfloat16))
    finally:
        torch.cuda.synchronize()
        _lib.check(lib.ir_peer_free(own))
        _lib.check(lib.ir_peer_free(silent))
    # the context still computes correctly
    w = wl.custom(47, 3, 28, 4, 128, 16, 50, 300, "bfloat16")
    q, kp, vp, _, _ = wl.torch_values(w, 5, DEV)
    bt = torch.from_numpy(w.block_tables).to(DEV)
    ctx = torch.from_numpy(w.context_lens).to(DEV)
    a = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    c = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    torch.cuda.synchronize()
    assert torch.equal(a, c) and torch.isfinite(a.float()).all()
    ops.check_device_errors()


def test_exchange_rejects_bad_arguments():
    lib = _lib.load()
    o = torch.zeros(1, 1, 128, device=DEV)
    lse = torch.zeros(1, 1, device=DEV)
    out = torch.empty(1, 1, 128, dtype=torch.bfloat16, device=DEV)
    buf = _alloc(lib, 1, 1, 128)
    try:
        arr = (ctypes.c_void_p * 1)(buf)
        err = ops.error_flag().data_ptr()
        st = ops._stream(torch.cuda.current_device())
        nbytes = lib.ir_peer_exchange_bytes(1, 1, 128)
        for world, rank, d in [(1, 1, 128), (9, 0, 128), (1, 0, 130), (1, 0, 256)]:
            rc = lib.ir_peer_exchange(out.data_ptr(), 128, o.data_ptr(), lse.data_ptr(), arr,
                                      nbytes, world, rank, 1, 1, d, ops.dtype_code(out.dtype),
                                      err, st)
            assert rc != 0
        # more rows than the buffer was laid out for; a batch * heads past 2^31
        for batch, heads in [(2, 1), (1 << 20, 1 << 12)]:
            rc = lib.ir_peer_exchange(out.data_ptr(), 128, o.data_ptr(), lse.data_ptr(), arr,
                                      nbytes, 1, 0, batch, heads, 128,
                                      ops.dtype_code(out.dtype), err, st)
            assert rc == _lib.IR_ERR_INVALID_ARG
            assert b"rows exceed" in lib.ir_last_error()
    finally:
        _lib.check(lib.ir_peer_free(buf))
