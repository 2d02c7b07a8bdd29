"""The in-kernel merge of short rows (``IR_DECODE_INLINE_MERGE``).

With a zero-filled workspace the TMA decode kernel counts the pieces of every
row split into at most 4 pieces; the warp that writes the last piece merges
the row right away and the merge kernel skips it. Checked here:

* C2 (rows of 2-3 pieces: all merged in the kernel), C3 with the fused cache
  write, and C4 (rows of ~37 pieces: left to the merge kernel) against the
  fp32 oracle at the bf16 bar (atol = rtol = 2e-2), and against the same
  call without the feature; LSE mode;
* deterministic results over repeated calls;
* the counters are zero after every call: eager, in CUDA-graph replays, and
  after a call whose wait ran out (the stall test hook);
* an output whose rows are not 16-byte aligned makes the library use the
  CUDA-core kernel, whose scalar stores need no alignment.
"""

import time

import numpy as np
import pytest
import torch

import infrared_b200 as irb
from gpu_helpers import DEV, assert_close_bf16, dev_meta, host_f32, oracle_decode_device
from infrared_b200 import _lib, ops
from infrared_b200 import workloads as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.set_decode_path(0)
    ops.error_flag().zero_()
    yield
    ops.set_decode_path(0)
    ops.check_device_errors()


def _ws(w, q, kp, bt, inline=True):
    _, _, need = ops.decode_plan(q, kp, bt, w.block_size, w.scale, inline_merge=inline)
    return ops.decode_workspace(need, DEV, dynamic=False, inline_merge=inline)


def _counters_zero(ws, w):
    torch.cuda.synchronize()
    n = 256 + 4 * w.num_kv_heads * w.batch
    return int(ws[:n].count_nonzero()) == 0


@pytest.mark.parametrize("name", ["c2", "c4"])
def test_inline_merge_matches_oracle_and_merge_kernel(name):
    w = {"c2": lambda: wl.c2(seed=11), "c4": lambda: wl.c4(seed=11)}[name]()
    q, kp, vp, _, _ = wl.torch_values(w, 12, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_in = _ws(w, q, kp, bt, True)
    ws_off = _ws(w, q, kp, bt, False)
    out_in = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_in)
    out_off = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_off)
    assert _counters_zero(ws_in, w)
    want = oracle_decode_device(w, q, kp, vp)
    assert_close_bf16(host_f32(out_in), want)
    # the same fold in the same order as the merge kernel: same rows
    np.testing.assert_allclose(host_f32(out_in), host_f32(out_off), atol=1e-2, rtol=1e-2)
    for _ in range(3):
        again = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_in)
        assert torch.equal(again, out_in)
    assert _counters_zero(ws_in, w)


def test_inline_merge_fused_write_c3():
    w = wl.c3(seed=12)
    q, kp, vp, kn, vn = wl.torch_values(w, 13, DEV)
    bt, ctx, sm = dev_meta(w)
    ws = _ws(w, q, kp, bt)
    out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size, ws=ws)
    assert _counters_zero(ws, w)
    assert torch.equal(kp[sm], kn) and torch.equal(vp[sm], vn)
    assert_close_bf16(host_f32(out), oracle_decode_device(w, q, kp, vp))


def test_inline_merge_lse_mode():
    w = wl.c2(seed=13)
    q, kp, vp, _, _ = wl.torch_values(w, 14, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_in, ws_off = _ws(w, q, kp, bt, True), _ws(w, q, kp, bt, False)
    o_i, l_i = ops.paged_decode_lse(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_in)
    o_o, l_o = ops.paged_decode_lse(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_off)
    assert _counters_zero(ws_in, w)
    assert_close_bf16(host_f32(o_i), oracle_decode_device(w, q, kp, vp))
    np.testing.assert_allclose(host_f32(o_i), host_f32(o_o), atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(host_f32(l_i), host_f32(l_o), atol=1e-5, rtol=1e-5)


def test_inline_merge_in_cuda_graph_replays():
    w = wl.c2(seed=14)
    q, kp, vp, _, _ = wl.torch_values(w, 15, DEV)
    bt, ctx, _ = dev_meta(w)
    ws = _ws(w, q, kp, bt)
    want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws)
    out = torch.empty_like(q)
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(3):
                irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, out=out, ws=ws)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(4):
        out.zero_()
        g.replay()
        assert _counters_zero(ws, w)
        assert torch.equal(out, want)
    del g


def test_inline_merge_timeout_leaves_counters_at_zero():
    w = wl.c2(seed=15)
    q, kp, vp, _, _ = wl.torch_values(w, 16, DEV)
    bt, ctx, _ = dev_meta(w)
    ws = _ws(w, q, kp, bt)
    want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws)
    torch.cuda.synchronize()
    assert _lib.load().ir_debug_stall_next_decode() == 0
    t0 = time.perf_counter()
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30
    with pytest.raises(irb.DeviceError, match="TIMEOUT"):
        ops.check_device_errors()
    assert _counters_zero(ws, w)
    again = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws)
    assert torch.equal(again, want)


def test_output_rows_not_16_byte_aligned_use_the_cuda_core_kernel():
    w = wl.custom(17, 5, 28, 4, 128, 16, 100, 700, "bfloat16", std=0.5)
    q, kp, vp, _, _ = wl.torch_values(w, 17, DEV)
    bt, ctx, _ = dev_meta(w)
    h, d = w.num_heads, w.head_dim
    # rows 4 elements (8 bytes) apart from a 16-byte boundary
    store = torch.zeros(w.batch, h * d + 4, dtype=torch.bfloat16, device=DEV)
    out = store[:, :h * d].view(w.batch, h, d)
    assert out.stride(0) == h * d + 4
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, out=out)
    torch.cuda.synchronize()
    assert_close_bf16(host_f32(out), oracle_decode_device(w, q, kp, vp))
    assert not host_f32(store[:, h * d:]).any()   # nothing written past the rows


def test_one_workspace_serves_calls_of_any_shape_and_kernel():
    """One zeroed workspace used in turn by an fp32 call (CUDA-core kernel, no
    counters), bf16 calls of different batches (in-kernel merge) and a call
    without the flag: the counter header sits at the same place in every
    layout, so no call's data lands on another call's counters."""
    cases = [wl.custom(21, 8, 14, 2, 64, 16, 1, 512, "float32"),
             wl.c2(seed=21),
             wl.custom(22, 7, 28, 4, 128, 16, 300, 3000, "bfloat16", std=0.5),
             wl.custom(23, 8, 14, 2, 64, 16, 1, 512, "bfloat16"),
             wl.c2(seed=22)]
    need = 0
    inputs = []
    for w in cases:
        q, kp, vp, _, _ = wl.torch_values(w, 31, DEV)
        bt, ctx, _ = dev_meta(w)
        need = max(need, ops.decode_plan(q, kp, bt, w.block_size, w.scale,
                                         inline_merge=True)[2])
        inputs.append((w, q, kp, vp, bt, ctx))
    ws = ops.decode_workspace(need, DEV, inline_merge=True)
    unmarked = ws.view(torch.uint8)[:]           # same memory, no flags: static layout
    for rep in range(2):
        for i, (w, q, kp, vp, bt, ctx) in enumerate(inputs):
            use = unmarked if (rep == 1 and i == 2) else ws
            out = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=use)
            want = oracle_decode_device(w, q, kp, vp)
            if w.dtype == "float32":
                np.testing.assert_allclose(host_f32(out), want, atol=1e-5, rtol=1e-5)
            else:
                assert_close_bf16(host_f32(out), want)
            assert _counters_zero(ws, w)
