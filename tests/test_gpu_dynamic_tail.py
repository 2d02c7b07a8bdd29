"""The decode kernel's dynamic tail (``IR_DECODE_DYNAMIC_TAIL``).

With a workspace whose header is zero, the TMA decode kernel streams a static
share per CTA and then hands out the last part of the tiles as small units
that CTAs claim from counters in that header. Checked here:

* the dynamic schedule matches the fp32 oracle at the bf16 bar (atol = rtol
  = 2e-2) and the static schedule on the same inputs, for C2, C3 (fused cache
  write, shared prefixes), C4 (4 x 32k), a batch larger than one CTA's
  threads with many short contexts, and contexts of 0 among the last
  sequences; in LSE mode too;
* it is deterministic: which CTA takes which unit does not change a bit;
* the counters are back at zero after every call — eager, replayed in a
  CUDA graph, and after a call whose wait ran out (the stall test hook);
* unknown flag bits are refused by the C ABI.
"""

import ctypes
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

HEADER = 256


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.set_decode_path(0)
    ops.error_flag().zero_()
    yield
    ops.set_decode_path(0)
    ops.check_device_errors()


def _workspaces(w, q, kp, bt):
    _, _, need_dyn = ops.decode_plan(q, kp, bt, w.block_size, w.scale, dynamic=True)
    _, _, need_static = ops.decode_plan(q, kp, bt, w.block_size, w.scale, dynamic=False)
    assert need_dyn > need_static   # the dynamic units' partial slots
    dyn = ops.decode_workspace(need_dyn, DEV, dynamic=True)
    static = torch.zeros(need_dyn, dtype=torch.uint8, device=DEV)  # unmarked: static
    return dyn, static


def _header_is_zero(ws):
    torch.cuda.synchronize()
    return int(ws[:HEADER].count_nonzero()) == 0


def _many_short(seed=0):
    """520 sequences (more than one CTA's threads) of 16-80 tokens, the last
    ones partly empty: the dynamic units lie in the last 32 sequences."""
    w = wl.custom(seed, 520, 28, 4, 128, 16, 16, 80, "bfloat16", std=0.5)
    w.context_lens[-6:-3] = 0
    w.slot_mapping[:] = wl.tail_slots(w.block_tables, w.context_lens, w.block_size)
    return w


@pytest.mark.parametrize("name", ["c2", "c4", "many_short"])
def test_dynamic_matches_oracle_and_static(name):
    w = {"c2": lambda: wl.c2(seed=3), "c4": lambda: wl.c4(seed=3),
         "many_short": _many_short}[name]()
    q, kp, vp, _, _ = wl.torch_values(w, 4, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_dyn, ws_static = _workspaces(w, q, kp, bt)
    out_d = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    assert _header_is_zero(ws_dyn)
    out_s = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_static)
    torch.cuda.synchronize()
    want = oracle_decode_device(w, q, kp, vp)
    assert_close_bf16(host_f32(out_d), want)
    assert_close_bf16(host_f32(out_s), want)
    # the same rows whichever schedule: only the fp32 split points differ
    np.testing.assert_allclose(host_f32(out_d), host_f32(out_s), atol=1e-2, rtol=1e-2)
    # deterministic: units land in fixed slots whatever CTA takes them
    for _ in range(3):
        again = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
        assert torch.equal(again, out_d)
    assert _header_is_zero(ws_dyn)
    if name == "many_short":
        assert not host_f32(out_d)[-6:-3].any()   # empty contexts give zero rows


def test_dynamic_fused_write_c3():
    w = wl.c3(seed=4)
    q, kp, vp, kn, vn = wl.torch_values(w, 5, DEV)
    bt, ctx, sm = dev_meta(w)
    ws_dyn, _ = _workspaces(w, q, kp, bt)
    out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size,
                                 ws=ws_dyn)
    assert _header_is_zero(ws_dyn)
    assert torch.equal(kp[sm], kn) and torch.equal(vp[sm], vn)
    assert_close_bf16(host_f32(out), oracle_decode_device(w, q, kp, vp))


def test_dynamic_lse_mode_matches_static():
    w = wl.c2(seed=5)
    q, kp, vp, _, _ = wl.torch_values(w, 6, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_dyn, ws_static = _workspaces(w, q, kp, bt)
    o_d, l_d = ops.paged_decode_lse(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    o_s, l_s = ops.paged_decode_lse(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_static)
    assert _header_is_zero(ws_dyn)
    assert_close_bf16(host_f32(o_d), oracle_decode_device(w, q, kp, vp))
    # P enters the P.V product rounded to bf16, so the two schedules' fp32
    # outputs differ by that rounding (about 5e-5 here), not by fp32 ulps
    np.testing.assert_allclose(host_f32(o_d), host_f32(o_s), atol=1e-3, rtol=1e-2)
    np.testing.assert_allclose(host_f32(l_d), host_f32(l_s), atol=1e-4, rtol=1e-5)


def test_dynamic_in_cuda_graph_replays():
    w = wl.c2(seed=6)
    q, kp, vp, _, _ = wl.torch_values(w, 7, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_dyn, _ = _workspaces(w, q, kp, bt)
    want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    out = torch.empty_like(q)
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(3):
                irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, out=out,
                                 ws=ws_dyn)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(5):
        out.zero_()
        g.replay()
        assert _header_is_zero(ws_dyn)
        assert torch.equal(out, want)
    del g


def test_dynamic_timeout_leaves_counters_at_zero():
    """The stall hook makes one CTA's wait run out: TIMEOUT is reported, every
    CTA still counts itself done, so the header is zero again and the next
    dynamic call is right."""
    w = wl.c2(seed=7)
    q, kp, vp, _, _ = wl.torch_values(w, 8, DEV)
    bt, ctx, _ = dev_meta(w)
    ws_dyn, _ = _workspaces(w, q, kp, bt)
    want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    torch.cuda.synchronize()
    assert _lib.load().ir_debug_stall_next_decode() == 0
    t0 = time.perf_counter()
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30
    with pytest.raises(irb.DeviceError, match="TIMEOUT"):
        ops.check_device_errors()
    assert _header_is_zero(ws_dyn)
    again = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, ws=ws_dyn)
    assert torch.equal(again, want)


def test_unknown_flag_bits_are_refused():
    lib = _lib.load()
    s = _lib.DecodeShape(batch=1, num_heads=28, num_kv_heads=4, head_dim=128, block_size=16,
                         max_blocks=4, bt_stride=4, q_stride=28 * 128, out_stride=28 * 128,
                         num_slots=64, scale=128 ** -0.5, dtype=_lib.IR_DTYPE_BF16, flags=6)
    assert lib.ir_paged_decode_workspace_size(ctypes.byref(s)) == 0
    assert lib.ir_paged_decode_plan(ctypes.byref(s), None, None) == _lib.IR_ERR_INVALID_ARG
    assert b"flags" in lib.ir_last_error()
