"""The CPU oracle, pinned against outputs of the reference engine itself.

The fixtures in tests/golden/golden.npz were produced by running infrared's
own naive path, graph-input builder and blockwise twin
(tests/golden/make_golden.py). These tests check the numpy restatement in
oracle/ against every one of them, plus the reference tests' own known
answers (infrared tests/test_cuda_graph.py:60-112,
tests/test_triton_attention.py:58-82).
"""

import numpy as np
import pytest

import cases
from infrared_b200 import workloads as wl
from oracle import paged_attention_np as orc


@pytest.mark.parametrize("name", sorted(cases.ATTENTION_CASES))
def test_oracle_matches_reference_naive_path(golden, name):
    assert str(golden[f"{name}/input_digest"]) == cases.input_digest(name), \
        "seeded inputs drifted from the ones the fixture was made with"
    w, q, kp, vp, kn, vn = cases.attention_inputs(name)
    s = cases.seam_tensors(w, q, kp, vp, kn, vn)
    out = orc.paged_attention_naive(s["q"], s["k"], s["v"], s["pool_k"], s["pool_v"],
                                    s["write_slots"], s["gather_slots"], s["mask"], 0,
                                    w.scale, w.n_rep)
    np.testing.assert_allclose(out[:, 0], golden[f"{name}/out"], atol=1e-5, rtol=0)
    # the pool after the scatter is bit-identical to the reference's
    assert cases.digest(s["pool_k"], s["pool_v"]) == str(golden[f"{name}/pool_digest"])


@pytest.mark.parametrize("name", sorted(cases.ATTENTION_CASES))
def test_block_table_oracle_equals_seam_oracle(golden, name):
    """decode_from_tables (block tables + context lens) == the seam's naive path."""
    w, q, kp, vp, kn, vn = cases.attention_inputs(name)
    kp2, vp2 = kp[None].copy(), vp[None].copy()
    orc.pool_write(kp2, vp2, 0, kn, vn, w.slot_mapping)
    out = orc.decode_from_tables(q, kp2, vp2, 0, w.block_tables, w.context_lens,
                                 w.block_size, w.scale, w.n_rep)
    np.testing.assert_allclose(out, golden[f"{name}/out"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("block_n", cases.BLOCKWISE_BLOCKS)
def test_blockwise_oracle_matches_reference_twin(golden, block_n):
    w, q, kp, vp, kn, vn = cases.attention_inputs("g7_d64_bs16_shared")
    s = cases.seam_tensors(w, q, kp, vp, kn, vn)
    orc.pool_write(s["pool_k"], s["pool_v"], 0, kn, vn, s["write_slots"])
    k_all = orc.repeat_kv(orc.pool_gather(s["pool_k"], 0, s["gather_slots"]), w.n_rep)
    v_all = orc.repeat_kv(orc.pool_gather(s["pool_v"], 0, s["gather_slots"]), w.n_rep)
    out = orc.blockwise_attention(s["q"], k_all, v_all, s["mask"], w.scale, block_n)
    np.testing.assert_allclose(out[:, 0], golden[f"blockwise/{block_n}"], atol=1e-5, rtol=0)
    one_shot = orc.masked_attention(s["q"], k_all, v_all, s["mask"], w.scale)
    np.testing.assert_allclose(out, one_shot, atol=1e-5, rtol=0)


@pytest.mark.parametrize("name", sorted(cases.GRAPH_CASES))
def test_graph_inputs_match_reference(golden, name):
    tables, num_cached, last, bucket, t_max, bs = cases.graph_case_args(name)
    inp = orc.build_decode_inputs(tables, num_cached, last, bucket, t_max, bs)
    for key in ("ids", "positions", "write_slots", "gather_slots"):
        np.testing.assert_array_equal(inp[key], golden[f"{name}/{key}"])
    np.testing.assert_array_equal(inp["mask"], golden[f"{name}/mask"])


def test_graph_inputs_known_answers():
    """Reference tests/test_cuda_graph.py:60-92: block_size 4, tables [[0,1],[2]],
    num_cached [5, 2] -> write slots 5 and 10, mask boundaries 6 and 3."""
    inp = orc.build_decode_inputs([[0, 1], [2]], [5, 2], [7, 9], 4, 16, 4)
    assert inp["write_slots"][0] == 5 and inp["write_slots"][1] == 10
    assert inp["positions"][0, 0] == 5 and inp["ids"][0, 0] == 7
    neg = np.finfo(np.float32).min
    assert (inp["mask"][0, 0, 0, :6] == 0).all() and (inp["mask"][0, 0, 0, 6:] == neg).all()
    assert (inp["mask"][1, 0, 0, :3] == 0).all() and (inp["mask"][1, 0, 0, 3:] == neg).all()
    # pad rows replicate row 0 (reference :95-112)
    for pad in (2, 3):
        for key in ("ids", "positions", "write_slots", "gather_slots", "mask"):
            np.testing.assert_array_equal(inp[key][pad], inp[key][0])
    with pytest.raises(ValueError, match="exceeds t_max"):
        orc.build_decode_inputs([[0]], [10], [1], 1, 8, 8)


@pytest.mark.parametrize("name", sorted(cases.GRAPH_CASES))
def test_metadata_derivation_round_trip(golden, name):
    """(gather_slots, mask) -> (block_tables, context_lens) inverts the engine's build."""
    tables, num_cached, last, bucket, t_max, bs = cases.graph_case_args(name)
    gs, mask = golden[f"{name}/gather_slots"], golden[f"{name}/mask"]
    bt, ctx, ok = orc.derive_block_metadata(gs, mask, bs)
    assert ok
    for i in range(bucket):
        j = i if i < len(tables) else 0
        assert ctx[i] == num_cached[j] + 1
        nblk = -(-int(ctx[i]) // bs)
        np.testing.assert_array_equal(bt[i, :nblk], tables[j][:nblk])
    rebuilt = orc.gather_slots_from_tables(bt, ctx, bs, gs.shape[1])
    np.testing.assert_array_equal(rebuilt, gs)


def test_metadata_derivation_flags_bad_rows():
    gs = np.array([[32, 33, 34, 7]], np.int64)       # position 3 not in block 2
    mask = orc.decode_mask([4], 4)
    assert not orc.derive_block_metadata(gs, mask, 16)[2]
    gs2 = np.array([[32, 33, 34, 35]], np.int64)
    bad_mask = mask.copy()
    bad_mask[0, 0, 0, 1] = np.finfo(np.float32).min  # hole inside the prefix
    assert not orc.derive_block_metadata(gs2, bad_mask, 16)[2]
    assert orc.derive_block_metadata(gs2, mask, 16)[2]


@pytest.mark.parametrize("splits", [(0, 17, 64, 1000), (0, 1, 2, 3, 1000), (0, 1000)])
def test_lse_merge_of_partials_equals_one_shot(splits):
    w, q, kp, vp, kn, vn = cases.attention_inputs("g7_d64_bs16_shared")
    full = orc.decode_from_tables(q, kp[None], vp[None], 0, w.block_tables, w.context_lens,
                                  w.block_size, w.scale, w.n_rep)
    parts = [orc.partial_attention(q, kp[None], vp[None], 0, w.block_tables, w.context_lens,
                                   w.block_size, w.scale, w.n_rep, lo, hi)
             for lo, hi in zip(splits[:-1], splits[1:])]
    o = np.stack([p[0] for p in parts])
    lse = np.stack([p[1] for p in parts])
    np.testing.assert_allclose(orc.lse_merge(o, lse), full, atol=1e-5, rtol=0)


def test_lse_merge_empty_rows_are_zero():
    o = np.ones((2, 1, 1, 4), np.float32)
    lse = np.full((2, 1, 1), -np.inf, np.float32)
    assert (orc.lse_merge(o, lse) == 0).all()


def test_zero_context_row_is_zero():
    w = wl.custom(3, 3, 4, 2, 64, 16, 5, 20, "float32")
    w.context_lens[1] = 0
    q, kp, vp, _, _ = wl.numpy_values(w, 0)
    out = orc.decode_from_tables(q, kp[None], vp[None], 0, w.block_tables, w.context_lens,
                                 16, w.scale, w.n_rep)
    assert (out[1] == 0).all() and np.abs(out[0]).sum() > 0


def test_workload_properties():
    w = wl.c3(seed=0)
    assert w.batch == 256 and w.n_rep == 7
    assert (w.context_lens >= 128).all() and (w.context_lens <= 2048).all()
    members = w.shared["prefix_of"]
    assert 0.15 * w.batch <= len(members) + len(w.shared["groups"]) <= 0.45 * w.batch
    used = set()
    for i in range(w.batch):
        nblk = -(-int(w.context_lens[i]) // w.block_size)
        own = w.block_tables[i, :nblk]
        k = members.get(i, (None, 0))[1]
        if k:
            donor = members[i][0]
            np.testing.assert_array_equal(own[:k], w.block_tables[donor, :k])
        # the write slot is the tail position, in a block no other row holds
        p = int(w.context_lens[i]) - 1
        assert w.slot_mapping[i] == own[p // 16] * 16 + p % 16
        used.update(int(x) for x in own[k:])
    assert len(used) == sum(-(-int(c) // 16) for c in w.context_lens) - \
        sum(k for _, k in members.values())
    tails = [w.block_tables[i, (int(w.context_lens[i]) - 1) // 16] for i in range(w.batch)]
    assert len(set(int(t) for t in tails)) == w.batch


def test_c2_bytes_in_expected_range_and_match_oracle_count():
    w = wl.c2(seed=0)
    assert w.batch == 64 and (w.context_lens >= 512).all() and (w.context_lens <= 4096).all()
    assert 200e6 < w.algorithmic_bytes() < 400e6
    assert w.algorithmic_bytes() == orc.decode_bytes(w.context_lens, 28, 4, 128, 2,
                                                     w.max_blocks)


@pytest.mark.parametrize("name", sorted(cases.ROPE_CASES))
def test_rope_oracle_matches_reference(golden, name):
    """apply_rope == infrared's apply_rotary_pos_emb bit for bit (fp32, same
    tables); rope_tables == RotaryEmbedding up to the last-bit differences of
    fp32 pow/cos between numpy and torch, amplified by the position (up to
    300 rad here); attention on the rotated q/k == the reference's output."""
    w, q, kp, vp, kn, vn = cases.attention_inputs(name)
    cos, sin = golden[f"rope/{name}/cos"], golden[f"rope/{name}/sin"]
    q_rot = orc.apply_rope(q, cos, sin)
    k_rot = orc.apply_rope(kn, cos, sin)
    np.testing.assert_array_equal(q_rot, golden[f"rope/{name}/q_rot"])
    np.testing.assert_array_equal(k_rot, golden[f"rope/{name}/k_rot"])
    c2, s2 = orc.rope_tables(w.context_lens - 1, w.head_dim, cases.ROPE_CASES[name])
    np.testing.assert_allclose(c2, cos, atol=1e-4, rtol=0)
    np.testing.assert_allclose(s2, sin, atol=1e-4, rtol=0)
    kp2, vp2 = kp[None].copy(), vp[None].copy()
    orc.pool_write(kp2, vp2, 0, k_rot, vn, w.slot_mapping)
    out = orc.decode_from_tables(q_rot, kp2, vp2, 0, w.block_tables, w.context_lens,
                                 w.block_size, w.scale, w.n_rep)
    np.testing.assert_allclose(out, golden[f"rope/{name}/out"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("name", sorted(cases.PREFILL_CASES))
def test_prefill_oracle_matches_reference(golden, name):
    """Prefill with a cached prefix and packed mixed steps: the oracle's mask is
    infrared's mask bit for bit, the pool after the write is infrared's, and
    the block-table prefill equals infrared's naive path (fp32, 1e-5)."""
    c = cases.prefill_inputs(name)
    fr = c["frame"]
    mask = orc.varlen_mask(fr["q_seq_ids"], fr["q_pos"], fr["k_seq_ids"], fr["k_pos"])
    assert cases.digest(mask) == str(golden[f"prefill/{name}/mask_digest"])
    kp, vp = c["pool_k"][None].copy(), c["pool_v"][None].copy()
    orc.pool_write(kp, vp, 0, c["k"], c["v"], fr["write_slots"])
    assert cases.digest(kp, vp) == str(golden[f"prefill/{name}/pool_digest"])
    out = orc.prefill_from_tables(c["q"], kp, vp, 0, c["block_tables"], c["context_lens"],
                                  c["q_start"], c["bs"], c["scale"], c["n_rep"])
    np.testing.assert_allclose(out, golden[f"prefill/{name}/out"], atol=1e-5, rtol=0)
    # the frame's (gather_slots, mask) give back the block-table form
    bt, ctx, q_start, ok = orc.varlen_metadata(fr["gather_slots"], mask, c["bs"])
    assert ok
    np.testing.assert_array_equal(ctx, c["context_lens"])
    np.testing.assert_array_equal(q_start, c["q_start"])
    for s in range(len(ctx)):
        nb = -(-int(ctx[s]) // c["bs"])
        np.testing.assert_array_equal(bt[s, :nb], c["block_tables"][s, :nb])


def test_varlen_metadata_rejects_non_contiguous_rows():
    mask = orc.varlen_mask([0, 0], [1, 2], [0, 0, 0], [0, 1, 2])
    mask[0, 0, 1, 1] = orc.F32_MIN          # a hole inside row 1's range
    _, _, _, ok = orc.varlen_metadata(np.arange(3)[None], mask, 1)
    assert not ok
