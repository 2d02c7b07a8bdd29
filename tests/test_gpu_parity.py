"""Parity of the CUDA path with the reference's naive attention (via the pinned oracle).

Bars (written in each test): cache write / gather / metadata bit-exact;
fp32 outputs within 1e-5 max-abs of the reference; bf16 / fp16 outputs
within atol = rtol = 2e-2 of the fp32 reference computed on the same
(rounded) inputs.
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import (DEV, assert_close_bf16, dev_meta, dev_values, host_f32,
                         oracle_decode, oracle_decode_device)
import infrared_b200 as irb
from infrared_b200 import ops
from infrared_b200 import workloads as wl
from oracle import paged_attention_np as orc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

FP32_TOL = 1e-5


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.set_decode_path(0)
    ops.error_flag().zero_()
    yield
    ops.set_decode_path(0)
    ops.check_device_errors()


# ----------------------------------------------------------- golden fixtures


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("name", sorted(cases.ATTENTION_CASES))
def test_golden_fp32(golden, name, fused):
    """fp32 through the C ABI vs the reference's own outputs (max-abs <= 1e-5)."""
    assert str(golden[f"{name}/input_digest"]) == cases.input_digest(name)
    w, *vals = cases.attention_inputs(name)
    q, kp, vp, kn, vn = dev_values(vals, torch.float32)
    bt, ctx, sm = dev_meta(w)
    if fused:
        out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size)
    else:
        irb.cache_write(kn, vn, kp, vp, sm)
        out = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    got = host_f32(out)
    assert np.abs(got - golden[f"{name}/out"]).max() <= FP32_TOL
    # pool after the write, bit-exact with the reference's pool
    assert cases.digest(host_f32(kp)[None], host_f32(vp)[None]) == \
        str(golden[f"{name}/pool_digest"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", sorted(cases.ATTENTION_CASES))
def test_golden_cases_half(name, dtype):
    w, *vals = cases.attention_inputs(name)
    q, kp, vp, kn, vn = dev_values(vals, dtype)
    bt, ctx, sm = dev_meta(w)
    want = oracle_decode(w, *[host_f32(t) for t in (q, kp, vp, kn, vn)])
    out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size)
    assert_close_bf16(host_f32(out), want)


@pytest.mark.parametrize("name", ["g2_d64_bs16", "g7_d128_bs16", "g1_d64_bs8",
                                  "g8_d128_bs16", "g7_d64_bs16_shared"])
def test_tma_and_cuda_core_paths_agree(name):
    w, *vals = cases.attention_inputs(name)
    q, kp, vp, kn, vn = dev_values(vals, torch.bfloat16)
    bt, ctx, sm = dev_meta(w)
    irb.cache_write(kn, vn, kp, vp, sm)
    assert ops.decode_plan(q, kp, bt, w.block_size)[0] == 2
    want = oracle_decode(w, *[host_f32(t) for t in (q, kp, vp)])
    outs = {}
    for path in (1, 2, 3):   # CUDA cores, TMA one copy per tile, TMA per (head, half)
        ops.set_decode_path(path)
        outs[path] = host_f32(irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size))
        assert_close_bf16(outs[path], want)
    assert np.abs(outs[1] - outs[2]).max() < 2e-2
    assert np.array_equal(outs[2], outs[3])


# ----------------------------------------------------------- sweeps


SWEEP = [
    # (B, H, Hkv, D, bs, ctx_lo, ctx_hi)
    (7, 28, 4, 128, 16, 1, 600),
    (9, 14, 2, 64, 16, 1, 333),
    (5, 32, 4, 128, 32, 17, 700),
    (5, 8, 1, 128, 64, 1, 400),
    (4, 12, 4, 64, 8, 1, 300),
    (3, 40, 8, 128, 16, 200, 260),   # group 5
    (2, 48, 4, 64, 16, 1, 500),      # group 12 -> CUDA-core path
    (3, 64, 4, 128, 16, 1, 200),     # group 16 -> CUDA-core path
    (6, 6, 6, 64, 16, 1, 90),        # MHA
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("cfg", SWEEP)
def test_sweep(cfg, dtype):
    b, h, hkv, d, bs, lo, hi = cfg
    w = wl.custom(100 + b * h, b, h, hkv, d, bs, lo, hi,
                  "float32" if dtype == torch.float32 else "bfloat16", shared_frac=0.3)
    vals = wl.numpy_values(w, 5)
    q, kp, vp, kn, vn = dev_values(vals, dtype)
    bt, ctx, sm = dev_meta(w)
    want = oracle_decode(w, *[host_f32(t) for t in (q, kp, vp, kn, vn)])
    out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, bs)
    if dtype == torch.float32:
        assert np.abs(host_f32(out) - want).max() <= FP32_TOL
    else:
        assert_close_bf16(host_f32(out), want)


@pytest.mark.parametrize("b", [3, 12, 40])
def test_split_merge_warp_tiers(b):
    """The split-sequence merge folds a row's pieces with 16, 8 or 4 warps
    by the shares per sequence (148 shares at this geometry: B = 3, 12, 40
    take 16, 8 and 4 warps); every tier matches the oracle."""
    w = wl.custom(300 + b, b, 28, 4, 128, 16, 1000, 3000, "bfloat16")
    vals = wl.numpy_values(w, 6)
    q, kp, vp, _, _ = dev_values(vals, torch.bfloat16)
    bt, ctx, _ = dev_meta(w)
    want = oracle_decode(w, *[host_f32(t) for t in (q, kp, vp)])
    out = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    assert_close_bf16(host_f32(out), want)


# ----------------------------------------------------------- full-size configs


def test_c2_full_size():
    w = wl.c2(seed=0)
    q, kp, vp, _, _ = wl.torch_values(w, 1, DEV)
    bt, ctx, _ = dev_meta(w)
    out = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    want = oracle_decode_device(w, q, kp, vp)
    assert_close_bf16(host_f32(out), want)
    # deterministic: same inputs, same bits
    out2 = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    assert torch.equal(out, out2)


def test_c3_full_size_fused_write_and_shared_prefixes():
    w = wl.c3(seed=0)
    q, kp, vp, kn, vn = wl.torch_values(w, 2, DEV)
    bt, ctx, sm = dev_meta(w)
    out = irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size)
    # the write is bit-exact at every tail slot and the rest of the pool is untouched
    assert torch.equal(kp[sm], kn) and torch.equal(vp[sm], vn)
    want = oracle_decode_device(w, q, kp, vp)
    assert_close_bf16(host_f32(out), want)


def test_c4_long_context_and_kv_chunk_merge():
    """One GPU: full 32k-context decode, then the same KV cut into 2/4/8 chunks
    decoded separately (paged_decode_lse) and merged (lse_merge)."""
    w = wl.c4(seed=0)
    q, kp, vp, _, _ = wl.torch_values(w, 3, DEV)
    bt, ctx, _ = dev_meta(w)
    full = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    want = oracle_decode_device(w, q, kp, vp)
    assert_close_bf16(host_f32(full), want)
    nblk = w.block_tables.shape[1]
    for parts in (2, 4, 8):
        per = nblk // parts
        os_, ls_ = [], []
        for p in range(parts):
            btp = bt[:, p * per:(p + 1) * per].contiguous()
            ctxp = torch.full_like(ctx, per * w.block_size)
            o, lse = irb.paged_decode_lse(q, kp, vp, btp, ctxp, w.scale, w.block_size)
            os_.append(o)
            ls_.append(lse)
        merged = irb.lse_merge(torch.stack(os_), torch.stack(ls_), torch.bfloat16)
        assert_close_bf16(host_f32(merged), want)
        assert np.abs(host_f32(merged) - host_f32(full)).max() < 2e-2
        # the packed layout of an all-gather ([P, B*H*D + B*H]) merges in place
        n_o = os_[0].numel()
        packed = torch.cat([torch.cat([o.reshape(-1), l.reshape(-1)])[None]
                            for o, l in zip(os_, ls_)])
        o_view = packed[:, :n_o].unflatten(1, os_[0].shape)
        l_view = packed[:, n_o:].unflatten(1, ls_[0].shape)
        assert torch.equal(irb.lse_merge(o_view, l_view, torch.bfloat16), merged)


def test_lse_outputs_match_oracle_partials():
    w = wl.custom(31, 6, 28, 4, 128, 16, 1, 900, "bfloat16")
    vals = wl.numpy_values(w, 9)
    q, kp, vp, _, _ = dev_values(vals, torch.bfloat16)
    bt, ctx, _ = dev_meta(w)
    o, lse = irb.paged_decode_lse(q, kp, vp, bt, ctx, w.scale, w.block_size)
    ref_o, ref_lse = orc.partial_attention(host_f32(q), host_f32(kp)[None], host_f32(vp)[None],
                                           0, w.block_tables, w.context_lens, 16, w.scale,
                                           w.n_rep, 0, 1 << 30)
    np.testing.assert_allclose(host_f32(o), ref_o, atol=2e-2, rtol=2e-2)
    np.testing.assert_allclose(host_f32(lse), ref_lse, atol=1e-3, rtol=1e-4)


# ----------------------------------------------------------- cache write / gather


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_cache_write_bit_exact(dtype):
    g = torch.Generator(device=DEV).manual_seed(0)
    n_slots, hkv, d, n = 4096, 4, 128, 300
    kp = torch.randn(n_slots, hkv, d, device=DEV, generator=g).to(dtype)
    vp = torch.randn(n_slots, hkv, d, device=DEV, generator=g).to(dtype)
    slots = torch.randperm(n_slots, device=DEV, generator=g)[:n]
    slots[::17] = -1                                  # padding rows are skipped
    big = torch.randn(n, hkv + 2, d, device=DEV, generator=g).to(dtype)
    k = big[:, :hkv]                                  # token stride (hkv+2)*d
    v = torch.randn(n, hkv, d, device=DEV, generator=g).to(dtype)
    want_k, want_v = kp.clone(), vp.clone()
    keep = slots >= 0
    want_k[slots[keep]] = k[keep]
    want_v[slots[keep]] = v[keep]
    irb.cache_write(k, v, kp, vp, slots)
    assert torch.equal(kp, want_k) and torch.equal(vp, want_v)


def test_cache_write_duplicate_identical_rows():
    """CUDA-graph pad rows repeat row 0: same slot, same data -> well defined."""
    kp = torch.zeros(64, 2, 64, device=DEV, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    k = torch.randn(1, 2, 64, device=DEV).to(torch.bfloat16).repeat(4, 1, 1)
    slots = torch.tensor([5, 5, 5, 5], device=DEV)
    irb.cache_write(k, k, kp, vp, slots)
    assert torch.equal(kp[5], k[0]) and torch.equal(vp[5], k[0])


def test_cache_write_out_of_range_slot_flags():
    kp = torch.zeros(64, 2, 64, device=DEV)
    k = torch.ones(2, 2, 64, device=DEV)
    irb.cache_write(k, k, kp, kp.clone(), torch.tensor([3, 64], device=DEV))
    with pytest.raises(irb.DeviceError, match="SLOT"):
        ops.check_device_errors()
    assert kp[3].eq(1).all() and kp.sum() == 128


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gather_bit_exact(dtype):
    pool = torch.randn(512, 2, 64, device=DEV).to(dtype)
    gs = torch.randint(0, 512, (3, 40), device=DEV)
    assert torch.equal(irb.cache_gather(pool, gs), pool[gs])


def test_mirror_pool_write_gather():
    pool = irb.PagedKVPool(2, 16, 16, 2, 64, torch.bfloat16, DEV)
    k = torch.randn(5, 2, 64, device=DEV).to(torch.bfloat16)
    slots = torch.tensor([0, 17, 33, 200, 255], device=DEV)
    pool.write(1, k, -k, slots)
    kk, vv = pool.gather(1, slots[None])
    assert torch.equal(kk[0], k) and torch.equal(vv[0], -k)
    assert pool.k[0].abs().sum() == 0


# ----------------------------------------------------------- metadata derivation


@pytest.mark.parametrize("name", sorted(cases.GRAPH_CASES))
@pytest.mark.parametrize("mask_dtype", [torch.float32, torch.bfloat16])
def test_derive_block_metadata_bit_exact(golden, name, mask_dtype):
    tables, num_cached, last, bucket, t_max, bs = cases.graph_case_args(name)
    gs_np, mask_np = golden[f"{name}/gather_slots"], golden[f"{name}/mask"]
    want_bt, want_ctx, ok = orc.derive_block_metadata(gs_np, mask_np, bs)
    assert ok
    gs = torch.from_numpy(gs_np).to(DEV)
    mask = torch.from_numpy(mask_np).to(DEV).to(mask_dtype)
    bt, ctx = irb.derive_block_metadata(gs, mask, bs)
    np.testing.assert_array_equal(bt.cpu().numpy(), want_bt)
    np.testing.assert_array_equal(ctx.cpu().numpy(), want_ctx)


def test_derive_block_metadata_flags():
    gs = torch.tensor([[32, 33, 34, 7]], device=DEV)
    mask = torch.zeros(1, 1, 1, 4, device=DEV)
    irb.derive_block_metadata(gs, mask, 16)
    with pytest.raises(irb.DeviceError, match="NOT_BLOCKED"):
        ops.check_device_errors()
    mask[..., 1] = torch.finfo(torch.float32).min
    irb.derive_block_metadata(torch.tensor([[32, 33, 34, 35]], device=DEV), mask, 16)
    with pytest.raises(irb.DeviceError, match="MASK"):
        ops.check_device_errors()


# ----------------------------------------------------------- edge cases


def test_edge_context_lengths():
    """ctx 0 (zero row), 1, exact multiples of 16, the full table width."""
    b = 6
    w = wl.custom(41, b, 28, 4, 128, 16, 1, 256, "bfloat16", num_blocks=256, max_blocks=16)
    w.context_lens[:] = np.array([0, 1, 16, 32, 255, 256], np.int32)
    w.block_tables[:] = np.random.default_rng(0).permutation(w.num_blocks)[: b * 16] \
        .reshape(b, 16).astype(np.int32)
    vals = wl.numpy_values(w, 1)
    for dtype in (torch.bfloat16, torch.float32):
        q, kp, vp, _, _ = dev_values(vals, dtype)
        bt, ctx, _ = dev_meta(w)
        out = host_f32(irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16))
        want = oracle_decode(w, *[host_f32(t) for t in (q, kp, vp)])
        assert (out[0] == 0).all()
        if dtype == torch.bfloat16:
            assert_close_bf16(out, want)
        else:
            np.testing.assert_allclose(out, want, atol=FP32_TOL, rtol=0)


def test_empty_batch_is_noop():
    q = torch.empty(0, 28, 128, device=DEV, dtype=torch.bfloat16)
    kp = torch.zeros(64, 4, 128, device=DEV, dtype=torch.bfloat16)
    out = irb.paged_decode(q, kp, kp, torch.zeros(0, 4, dtype=torch.int32, device=DEV),
                           torch.zeros(0, dtype=torch.int32, device=DEV), 0.1, 16)
    assert out.shape == (0, 28, 128)


def test_bad_block_id_and_context_are_flagged_not_faulted():
    w = wl.custom(42, 3, 28, 4, 128, 16, 40, 100, "bfloat16")
    q, kp, vp, _, _ = dev_values(wl.numpy_values(w, 2), torch.bfloat16)
    bt, ctx, _ = dev_meta(w)
    bt[1, 0] = w.num_blocks + 5
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    with pytest.raises(irb.DeviceError, match="BLOCK_ID"):
        ops.check_device_errors()
    bt, ctx, _ = dev_meta(w)
    ctx[2] = w.max_blocks * 16 + 1
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    with pytest.raises(irb.DeviceError, match="CONTEXT_LEN"):
        ops.check_device_errors()


def test_fused_write_requires_tail_slot():
    w = wl.custom(43, 3, 28, 4, 128, 16, 40, 100, "bfloat16")
    q, kp, vp, kn, vn = dev_values(wl.numpy_values(w, 2), torch.bfloat16)
    bt, ctx, sm = dev_meta(w)
    sm[0] += 1 if int(w.context_lens[0]) % 16 else -1
    irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, 16)
    with pytest.raises(irb.DeviceError, match="WRITE_SLOT"):
        ops.check_device_errors()


# ----------------------------------------------------------- the reference seam mirror


def _seam(w, vals, dtype):
    q, kp, vp, kn, vn = dev_values(vals, dtype)
    pool = irb.PagedKVPool(1, w.num_blocks, w.block_size, w.num_kv_heads, w.head_dim, dtype,
                           DEV)
    pool.k[0].copy_(kp)
    pool.v[0].copy_(vp)
    t = int(w.context_lens.max())
    gs = torch.from_numpy(orc.gather_slots_from_tables(w.block_tables, w.context_lens,
                                                       w.block_size, t)).to(DEV)
    mask = torch.from_numpy(orc.decode_mask(w.context_lens, t)).to(DEV).to(dtype)
    ws = torch.from_numpy(w.slot_mapping).to(DEV)
    return q[:, None], kn[:, None], vn[:, None], pool, ws, gs, mask


@pytest.mark.parametrize("use_fused", [True, False])
def test_mirror_paged_attention_matches_golden(golden, use_fused):
    name = "c1"
    w, *vals = cases.attention_inputs(name)
    q, k, v, pool, ws, gs, mask = _seam(w, vals, torch.float32)
    ctx = irb.PagedContext(pool, ws, gs, use_triton=use_fused)
    out = irb.paged_attention(q, k, v, ctx, mask, 0, w.scale, w.n_rep)
    assert out.shape == q.shape
    assert np.abs(host_f32(out)[:, 0] - golden[f"{name}/out"]).max() <= FP32_TOL
    assert cases.digest(host_f32(pool.k), host_f32(pool.v)) == str(golden[f"{name}/pool_digest"])


def test_reference_cuda_kernel_test_ported():
    """infrared tests/test_triton_attention.py:155-187 at the decode shape:
    b=2, h_kv=2, n_rep=2, d=64 fp32, vs the naive path at atol=rtol=1e-2."""
    torch.manual_seed(0)
    b, h_kv, n_rep, d = 2, 2, 2, 64
    q = torch.randn(b, 1, h_kv * n_rep, d, device=DEV)
    k = torch.randn(b, 1, h_kv, d, device=DEV)
    v = torch.randn(b, 1, h_kv, d, device=DEV)
    mask = torch.zeros(b, 1, 1, 1, device=DEV)
    # each row's history is its own new token, in a one-slot block of its own
    pool = irb.PagedKVPool(1, b, 1, h_kv, d, torch.float32, DEV)
    ws = torch.arange(b, device=DEV)
    gs = ws[:, None].clone()
    got = irb.paged_attention(q, k, v, irb.PagedContext(pool, ws, gs), mask, 0, d ** -0.5,
                              n_rep)
    qn, kn, vn = (host_f32(x) for x in (q, k, v))
    want = orc.masked_attention(qn, orc.repeat_kv(kn, n_rep), orc.repeat_kv(vn, n_rep),
                                host_f32(mask), d ** -0.5)
    np.testing.assert_allclose(host_f32(got), want, atol=1e-2, rtol=1e-2)
    np.testing.assert_allclose(host_f32(got), want, atol=FP32_TOL, rtol=0)


def test_mirror_rejects_batched_prefill_and_cpu():
    w, *vals = cases.attention_inputs("g2_d64_bs16")
    q, k, v, pool, ws, gs, mask = _seam(w, vals, torch.float32)
    ctx = irb.PagedContext(pool, ws, gs)
    with pytest.raises(NotImplementedError):
        irb.paged_attention(q.expand(-1, 2, -1, -1), k, v, ctx, mask, 0, w.scale, w.n_rep)
    with pytest.raises(ValueError):
        irb.paged_decode(q[:, 0].cpu(), pool.k[0], pool.v[0],
                         torch.zeros(w.batch, 1, dtype=torch.int32), torch.zeros(
                             w.batch, dtype=torch.int32), 0.1, 16)


def test_cuda_graph_capture_and_replay():
    """The fused path captured once and replayed over new inputs == eager."""
    w = wl.custom(44, 8, 28, 4, 128, 16, 20, 300, "bfloat16")
    vals = wl.numpy_values(w, 3)
    q, k, v, pool, ws, gs, mask = _seam(w, vals, torch.bfloat16)
    pool_ref_k, pool_ref_v = pool.k.clone(), pool.v.clone()
    static = [t.clone() for t in (q, k, v, ws, gs, mask)]

    def step(qq, kk, vv, wws, ggs, mm):
        return irb.paged_attention(qq, kk, vv, irb.PagedContext(pool, wws, ggs), mm, 0,
                                   w.scale, w.n_rep)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step(*static)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out_static = step(*static)
    for seed in (10, 11):
        g = torch.Generator(device=DEV).manual_seed(seed)
        newq = torch.randn(q.shape, device=DEV, generator=g).to(q.dtype)
        static[0].copy_(newq)
        graph.replay()
        pool.k.copy_(pool_ref_k)
        pool.v.copy_(pool_ref_v)
        eager = step(newq, k, v, ws, gs, mask)
        assert torch.equal(out_static, eager)


def test_workspace_reuse_across_shapes():
    """Split sequences are merged from pieces in the workspace; the workspace
    needs no initialisation and one buffer serves calls of any shape."""
    w = wl.custom(45, 16, 28, 4, 128, 16, 100, 3000, "bfloat16")
    q, kp, vp, _, _ = dev_values(wl.numpy_values(w, 4), torch.bfloat16)
    bt, ctx, _ = dev_meta(w)
    _, ctas, nbytes = ops.decode_plan(q, kp, bt, 16, w.scale)
    assert ctas > w.batch   # sequences really are split across CTAs
    ws = torch.full((nbytes,), 0x7f, dtype=torch.uint8, device=DEV)   # garbage on purpose
    outs = [irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16, ws=ws) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    assert_close_bf16(host_f32(outs[0]), oracle_decode(w, *[host_f32(t) for t in (q, kp, vp)]))
    # a smaller batch after a larger one reuses the workspace (its tiles are
    # shared out differently, so it agrees within tolerance)
    small = irb.paged_decode(q[:3], kp, vp, bt[:3], ctx[:3], w.scale, 16, ws=ws)
    assert_close_bf16(host_f32(small), host_f32(outs[0][:3]))
    with pytest.raises(ValueError, match="workspace"):
        irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16, ws=ws[:256])



# ----------------------------------------------------------- graph-input builder


@pytest.mark.parametrize("name", sorted(cases.GRAPH_CASES))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_graph_inputs_match_reference_bit_exact(golden, name, dtype):
    """ir_build_decode_inputs == infrared's build_decode_static_inputs (golden outputs)."""
    from infrared_b200.graph_inputs import build_decode_static_inputs

    tables, num_cached, last, bucket, t_max, bs = cases.graph_case_args(name)
    got = build_decode_static_inputs(tables, num_cached, last, bucket, t_max, bs, DEV, dtype)
    for key in ("ids", "positions", "write_slots", "gather_slots"):
        np.testing.assert_array_equal(got.__getattribute__(key).cpu().numpy(),
                                      golden[f"{name}/{key}"])
    want_mask = torch.from_numpy(golden[f"{name}/mask"]).to(dtype)
    want_mask[want_mask != 0] = torch.finfo(dtype).min
    assert torch.equal(got.mask.cpu(), want_mask)


def test_graph_inputs_errors_and_known_answers():
    from infrared_b200.graph_inputs import build_decode_static_inputs

    inp = build_decode_static_inputs([[0, 1], [2]], [5, 2], [7, 9], 4, 16, 4, DEV,
                                     torch.float32)
    assert inp.write_slots[:2].tolist() == [5, 10]
    assert torch.equal(inp.gather_slots[2], inp.gather_slots[0])
    with pytest.raises(ValueError, match="exceeds t_max"):
        build_decode_static_inputs([[0]], [10], [1], 1, 8, 8, DEV, torch.float32)
    with pytest.raises(ValueError, match="bucket_b"):
        build_decode_static_inputs([[0]], [1], [1], 0, 8, 8, DEV, torch.float32)



# ----------------------------------------------------------- failure path


def test_bounded_wait_runs_out_and_context_survives():
    """A decode whose pipeline barrier never completes (the test hook expects
    bytes no copy delivers) gives up after its wait limit, reports TIMEOUT
    through the error flag, and the next decode on the same context is right."""
    import time

    from infrared_b200 import _lib

    w = wl.custom(46, 4, 28, 4, 128, 16, 100, 400, "bfloat16")
    q, kp, vp, _, _ = dev_values(wl.numpy_values(w, 3), torch.bfloat16)
    bt, ctx, _ = dev_meta(w)
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    torch.cuda.synchronize()
    assert _lib.load().ir_debug_stall_next_decode() == 0
    t0 = time.perf_counter()
    irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30
    with pytest.raises(irb.DeviceError, match="TIMEOUT"):
        ops.check_device_errors()
    out = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, 16)
    assert_close_bf16(host_f32(out), oracle_decode(w, *[host_f32(t) for t in (q, kp, vp)]))
