"""Paged prefill / mixed varlen attention (ir_paged_prefill) against the oracle.

Bars: fp32 within 1e-5 max-abs of the reference's own golden outputs; bf16 /
fp16 within atol = rtol = 2e-2 of the fp32 oracle on the same rounded
inputs, on every kernel form: tcgen05 tensor cores (path 2), the CTA-pair
tensor-core form (path 3, cta_group::2, head_dim 128) and rows-as-decode
(path 1).
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import DEV, assert_close_bf16, host_f32
import infrared_b200 as irb
from infrared_b200 import ops
from oracle import paged_attention_np as orc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.set_prefill_path(0)
    ops.error_flag().zero_()
    yield
    ops.set_prefill_path(0)
    ops.check_device_errors()


def _device_case(c, dtype):
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    kp, vp = t(c["pool_k"]).to(dtype), t(c["pool_v"]).to(dtype)
    ws = t(c["frame"]["write_slots"])
    irb.cache_write(t(c["k"]).to(dtype), t(c["v"]).to(dtype), kp, vp, ws)
    return (t(c["q"]).to(dtype), kp, vp, t(c["block_tables"]), t(c["context_lens"]),
            t(c["q_start"]))


@pytest.mark.parametrize("name", sorted(cases.PREFILL_CASES))
def test_prefill_golden_fp32(golden, name):
    c = cases.prefill_inputs(name)
    q, kp, vp, bt, ctx, qs = _device_case(c, torch.float32)
    assert ops.prefill_plan(q, kp, bt, qs, c["bs"])[0] == 1
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, c["scale"], c["bs"])
    assert np.abs(host_f32(out) - golden[f"prefill/{name}/out"]).max() <= 1e-5


@pytest.mark.parametrize("path", [2, 3, 1])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", sorted(cases.PREFILL_CASES))
def test_prefill_golden_half(name, dtype, path):
    c = cases.prefill_inputs(name)
    if path == 3 and c["q"].shape[-1] != 128:
        pytest.skip("the CTA-pair form takes head_dim 128")
    q, kp, vp, bt, ctx, qs = _device_case(c, dtype)
    ops.set_prefill_path(path)
    assert ops.prefill_plan(q, kp, bt, qs, c["bs"])[0] == path
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, c["scale"], c["bs"])
    want = orc.prefill_from_tables(host_f32(q), host_f32(kp)[None], host_f32(vp)[None], 0,
                                   c["block_tables"], c["context_lens"], c["q_start"], c["bs"],
                                   c["scale"], c["n_rep"])
    assert_close_bf16(host_f32(out), want)


def _random_frame(seed, h, hkv, d, bs, chunks, dtype):
    rng = np.random.default_rng(seed)
    ctx = np.array([st + ql for st, ql in chunks], np.int32)
    nblk = [-(-int(x) // bs) for x in ctx]
    num_blocks = sum(nblk) + 3
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(chunks), max(nblk)), np.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    q_start = np.concatenate([[0], np.cumsum([ql for _, ql in chunks])]).astype(np.int32)
    nq = int(q_start[-1])
    q = torch.from_numpy(rng.standard_normal((nq, h, d), dtype=np.float32)).to(DEV).to(dtype)
    kp = torch.from_numpy(rng.standard_normal((num_blocks * bs, hkv, d),
                                              dtype=np.float32)).to(DEV).to(dtype)
    vp = torch.from_numpy(rng.standard_normal((num_blocks * bs, hkv, d),
                                              dtype=np.float32)).to(DEV).to(dtype)
    return (q, kp, vp, torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV),
            torch.from_numpy(q_start).to(DEV), bt, ctx, q_start)


SWEEP = [
    # (H, Hkv, D, bs, [(cached, forwarded), ...])
    (28, 4, 128, 16, [(0, 300), (17, 1), (500, 129), (0, 1), (64, 64)]),
    (14, 2, 64, 16, [(0, 257), (3, 5), (128, 128)]),
    (8, 8, 128, 32, [(10, 200), (0, 33)]),
    (16, 2, 128, 8, [(100, 150), (1, 1), (0, 7)]),
    (12, 4, 64, 64, [(0, 129), (250, 20)]),
    (8, 1, 128, 128, [(130, 140), (0, 3)]),
    (4, 4, 64, 256, [(300, 70)]),
]


@pytest.mark.parametrize("path", [2, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cfg", SWEEP)
def test_prefill_sweep_tensor_cores(cfg, dtype, path):
    h, hkv, d, bs, chunks = cfg
    if path == 3 and d != 128:
        pytest.skip("the CTA-pair form takes head_dim 128")
    q, kp, vp, bt, ctx, qs, bt_np, ctx_np, qs_np = _random_frame(7 + h + d + bs, h, hkv, d, bs,
                                                                 chunks, dtype)
    ops.set_prefill_path(path)
    assert ops.prefill_plan(q, kp, bt, qs, bs)[0] == path
    scale = d ** -0.5
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, scale, bs)
    want = orc.prefill_from_tables(host_f32(q), host_f32(kp)[None], host_f32(vp)[None], 0,
                                   bt_np, ctx_np, qs_np, bs, scale, h // hkv)
    assert_close_bf16(host_f32(out), want)


def test_prefill_long_prompt_rows_against_oracle():
    """One 2048-token prompt at the Qwen2.5-7B geometry; rows spread over the
    q tiles (incl. the diagonal tiles' first and last rows) vs the oracle."""
    h, hkv, d, bs = 28, 4, 128, 16
    q, kp, vp, bt, ctx, qs, bt_np, ctx_np, qs_np = _random_frame(5, h, hkv, d, bs, [(0, 2048)],
                                                                 torch.bfloat16)
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, d ** -0.5, bs)
    rows = [0, 1, 127, 128, 129, 1000, 1023, 1024, 2046, 2047]
    qh = host_f32(q)
    kh, vh = host_f32(kp)[None], host_f32(vp)[None]
    for r in rows:
        sub_q = qh[r:r + 1]
        want = orc.prefill_from_tables(sub_q, kh, vh, 0, bt_np, np.array([r + 1], np.int32),
                                       np.array([0, 1], np.int32), bs, d ** -0.5, h // hkv)
        assert_close_bf16(host_f32(out[r:r + 1]), want)


def test_prefill_paths_agree_and_are_deterministic():
    h, hkv, d, bs = 28, 4, 128, 16
    q, kp, vp, bt, ctx, qs, *_ = _random_frame(9, h, hkv, d, bs, [(40, 200), (0, 1), (3, 77)],
                                               torch.bfloat16)
    a = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.088, bs)
    b = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.088, bs)
    assert torch.equal(a, b)
    ops.set_prefill_path(1)
    c = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.088, bs)
    assert (a.float() - c.float()).abs().max().item() < 2e-2
    ops.set_prefill_path(3)
    e = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.088, bs)
    f = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.088, bs)
    assert torch.equal(e, f)
    assert (a.float() - e.float()).abs().max().item() < 2e-2


# (H, Hkv, bs, [(cached, forwarded), ...]) at head_dim 128: long prompts whose
# 256-row pair items end ragged (both halves, one half, a lone row)
PAIR_FRAMES = [
    (28, 4, 16, [(0, 700), (37, 300), (0, 1), (5, 257), (0, 256)]),
    (28, 4, 64, [(0, 1024), (900, 129)]),
    (16, 2, 128, [(70, 513), (0, 255)]),
    (8, 8, 8, [(3, 300)]),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cfg", PAIR_FRAMES)
def test_prefill_cta_pairs_long_prompts(cfg, dtype):
    """The CTA-pair form on long prompts (on request; auto keeps the
    single-CTA form): rows of both halves of every pair item against the
    oracle (a sample of rows per sequence for the long ones), and close to
    the single-CTA form."""
    h, hkv, bs, chunks = cfg
    d = 128
    q, kp, vp, bt, ctx, qs, bt_np, ctx_np, qs_np = _random_frame(11 + h + bs, h, hkv, d, bs,
                                                                 chunks, dtype)
    assert ops.prefill_plan(q, kp, bt, qs, bs)[0] == 2
    ops.set_prefill_path(3)
    assert ops.prefill_plan(q, kp, bt, qs, bs)[0] == 3
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, d ** -0.5, bs)
    qh, kh, vh = host_f32(q), host_f32(kp)[None], host_f32(vp)[None]
    got = host_f32(out)
    for s_i, (cached, ql) in enumerate(chunks):
        r0 = int(qs_np[s_i])
        rows = sorted({0, 1, 127, 128, 129, 255, 256, ql // 2, ql - 2, ql - 1} & set(range(ql)))
        for r in rows:
            want = orc.prefill_from_tables(qh[r0 + r:r0 + r + 1], kh, vh, 0, bt_np[s_i:s_i + 1],
                                           np.array([cached + r + 1], np.int32),
                                           np.array([0, 1], np.int32), bs, d ** -0.5, h // hkv)
            assert_close_bf16(got[r0 + r:r0 + r + 1], want)
    ops.set_prefill_path(2)
    single = irb.paged_prefill(q, kp, vp, bt, ctx, qs, d ** -0.5, bs)
    assert (out.float() - single.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("path", [2, 3])
def test_prefill_stale_pool_rows_past_context_stay_out(path):
    """Pool slots past a sequence's context inside its last block hold NaN:
    no output row may see them (the kernels zero those V rows in shared
    memory and mask those keys)."""
    h, hkv, d, bs = 28, 4, 128, 16
    chunks = [(0, 300), (13, 250), (0, 37)]
    q, kp, vp, bt, ctx, qs, bt_np, ctx_np, qs_np = _random_frame(21, h, hkv, d, bs, chunks,
                                                                 torch.bfloat16)
    for s_i, n in enumerate(ctx_np):
        last = int(bt_np[s_i, (int(n) - 1) // bs])
        for pos in range(int(n), -(-int(n) // bs) * bs):
            slot = last * bs + pos % bs
            kp[slot] = float("nan")
            vp[slot] = float("nan")
    ops.set_prefill_path(path)
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, d ** -0.5, bs)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    want = orc.prefill_from_tables(host_f32(q), host_f32(kp)[None], host_f32(vp)[None], 0,
                                   bt_np, ctx_np, qs_np, bs, d ** -0.5, h // hkv)
    assert_close_bf16(host_f32(out), want)


def test_prefill_bad_context_is_flagged_not_faulted():
    h, hkv, d, bs = 8, 2, 64, 16
    q, kp, vp, bt, ctx, qs, *_ = _random_frame(3, h, hkv, d, bs, [(0, 40), (5, 10)],
                                               torch.bfloat16)
    bad = ctx.clone()
    bad[0] = 20                       # shorter than its 40 query rows
    irb.paged_prefill(q, kp, vp, bt, bad, qs, 0.125, bs)
    with pytest.raises(ops.DeviceError, match="CONTEXT_LEN"):
        ops.check_device_errors()
    # the next call on the same context is fine
    out = irb.paged_prefill(q, kp, vp, bt, ctx, qs, 0.125, bs)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


def test_prefill_empty_frame():
    q = torch.empty(0, 8, 64, device=DEV, dtype=torch.bfloat16)
    kp = torch.zeros(64, 2, 64, device=DEV, dtype=torch.bfloat16)
    bt = torch.zeros(0, 4, dtype=torch.int32, device=DEV)
    ctx = torch.zeros(0, dtype=torch.int32, device=DEV)
    qs = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = irb.paged_prefill(q, kp, kp, bt, ctx, qs, 0.125, 16)
    assert out.shape == (0, 8, 64)


# ----------------------------------------------------------- infrared's frame form


def _frame_tensors(c, dtype):
    fr = c["frame"]
    mask = torch.from_numpy(orc.varlen_mask(fr["q_seq_ids"], fr["q_pos"], fr["k_seq_ids"],
                                            fr["k_pos"])).to(DEV)
    if dtype != torch.float32:
        mask = mask.to(dtype)   # finfo(fp32).min -> -inf in 16 bits: still "blocked"
    return torch.from_numpy(fr["gather_slots"]).to(DEV), mask


@pytest.mark.parametrize("mask_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", sorted(cases.PREFILL_CASES))
def test_derive_varlen_metadata_bit_exact(name, mask_dtype):
    c = cases.prefill_inputs(name)
    gs, mask = _frame_tensors(c, mask_dtype)
    bt, ctx, qs = ops.derive_varlen_metadata(gs, mask, c["bs"])
    want_bt, want_ctx, want_qs, ok = orc.varlen_metadata(c["frame"]["gather_slots"],
                                                         host_f32(mask), c["bs"])
    assert ok
    np.testing.assert_array_equal(ctx.cpu().numpy(), want_ctx)
    np.testing.assert_array_equal(qs.cpu().numpy(), want_qs)
    np.testing.assert_array_equal(bt.cpu().numpy()[:, :want_bt.shape[1]], want_bt)


def test_derive_varlen_metadata_flags_broken_frames():
    c = cases.prefill_inputs("varlen_mix")
    gs, mask = _frame_tensors(c, torch.float32)
    bad = mask.clone()
    bad[0, 0, 3, 1] = torch.finfo(torch.float32).min   # a hole inside row 3's range
    ops.derive_varlen_metadata(gs, bad, c["bs"])
    with pytest.raises(ops.DeviceError, match="MASK"):
        ops.check_device_errors()
    gs2 = gs.clone()
    gs2[0, 5] += 1                                       # not block structured
    ops.derive_varlen_metadata(gs2, mask, c["bs"])
    with pytest.raises(ops.DeviceError, match="NOT_BLOCKED"):
        ops.check_device_errors()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", sorted(cases.PREFILL_CASES))
def test_mirror_paged_attention_prefill_frames(golden, name, dtype):
    """infrared's seam signature with a packed frame: write, then prefill."""
    from infrared_b200.attention import clear_metadata_cache

    c = cases.prefill_inputs(name)
    fr = c["frame"]
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    pool = irb.PagedKVPool(1, c["num_blocks"], c["bs"], c["hkv"], c["d"], dtype, DEV)
    pool.k[0].copy_(t(c["pool_k"]).to(dtype))
    pool.v[0].copy_(t(c["pool_v"]).to(dtype))
    gs, mask = _frame_tensors(c, dtype)
    paged = irb.PagedContext(pool, t(fr["write_slots"]), gs, use_triton=True)
    q, k, v = (t(c[n]).to(dtype)[None] for n in ("q", "k", "v"))
    clear_metadata_cache()
    out = irb.paged_attention(q, k, v, paged, mask, 0, c["scale"], c["n_rep"])
    assert out.shape == q.shape
    if dtype == torch.float32:
        assert np.abs(host_f32(out[0]) - golden[f"prefill/{name}/out"]).max() <= 1e-5
    else:
        want = orc.prefill_from_tables(host_f32(q[0]), host_f32(pool.k[0])[None],
                                       host_f32(pool.v[0])[None], 0, c["block_tables"],
                                       c["context_lens"], c["q_start"], c["bs"], c["scale"],
                                       c["n_rep"])
        assert_close_bf16(host_f32(out[0]), want)
