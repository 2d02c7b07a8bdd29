"""CPU oracle for the paged-decode attention path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference engine's naive paged-attention
path so that the CUDA kernels in ``infrared_b200`` can be checked against it.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline. The product path never calls into it.

Every function names the reference ``file:line`` it follows (paths are inside
the infrared project). The restatement is pinned against outputs of the
reference itself: ``tests/golden/make_golden.py`` imports infrared, runs its
naive path on seeded inputs and stores the outputs as fixtures, and
``tests/test_oracle.py`` checks this module against every fixture.

Numerics follow the reference's fp32 path: scores are computed as float32
dot products, scaled, the additive mask added, a float32 softmax taken and the
probabilities multiplied with V in float32. bf16 / fp16 inputs are upcast to
float32 first (numpy has no bf16); that fp32 result is the tolerance target
for half-precision kernels.
"""

from __future__ import annotations

import math

import numpy as np

F32_MIN = float(np.finfo(np.float32).min)


# --- PagedKVPool (infrared/cache/paged_kv_cache.py) --------------------------


def pool_write(pool_k: np.ndarray, pool_v: np.ndarray, layer_idx: int,
               k: np.ndarray, v: np.ndarray, slots: np.ndarray) -> None:
    """Scatter ``k, v [N, Hkv, D]`` into ``pool[layer_idx, slots]`` in place.

    Follows ``PagedKVPool.write`` (infrared/cache/paged_kv_cache.py:48-57):
    ``self.k[layer_idx, slots] = k``. With duplicate slots numpy, like torch's
    ``index_put`` on CPU, keeps the last row written.
    """
    pool_k[layer_idx, slots] = k
    pool_v[layer_idx, slots] = v


def pool_gather(pool: np.ndarray, layer_idx: int,
                gather_slots: np.ndarray) -> np.ndarray:
    """``gather_slots [B, T]`` -> ``[B, T, Hkv, D]`` rows of ``pool[layer_idx]``.

    Follows ``PagedKVPool.gather`` (infrared/cache/paged_kv_cache.py:59-72).
    """
    b, t = gather_slots.shape
    rows = pool[layer_idx, gather_slots.reshape(-1)]
    return rows.reshape(b, t, *pool.shape[2:])


# --- attention math (infrared/model/layers.py) -------------------------------


def repeat_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """``[B, S, Hkv, D]`` -> ``[B, S, Hkv*n_rep, D]``; head j reads kv head j // n_rep.

    Follows ``repeat_kv`` (infrared/model/layers.py:92-99).
    """
    if n_rep == 1:
        return x
    return np.repeat(x, n_rep, axis=2)


def softmax_f32(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Numerically stable float32 softmax (the ``torch.softmax`` step)."""
    x = x.astype(np.float32, copy=False)
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def masked_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                     mask: np.ndarray, scale: float) -> np.ndarray:
    """Scaled dot-product attention with an additive mask, in float32.

    Follows ``masked_attention`` (infrared/model/layers.py:102-118):
    ``scores = einsum("bqhd,bkhd->bhqk", q, k) * scale + mask``, float32
    softmax over keys, then ``einsum("bhqk,bkhd->bqhd", attn, v)``.
    Shapes: q ``[B, Sq, H, D]``, k/v ``[B, T, H, D]``, mask broadcastable to
    ``[B, H, Sq, T]``. Returns ``[B, Sq, H, D]`` float32.
    """
    q = q.astype(np.float32, copy=False)
    k = k.astype(np.float32, copy=False)
    v = v.astype(np.float32, copy=False)
    qh = np.transpose(q, (0, 2, 1, 3))            # [B, H, Sq, D]
    kh = np.transpose(k, (0, 2, 3, 1))            # [B, H, D, T]
    vh = np.transpose(v, (0, 2, 1, 3))            # [B, H, T, D]
    scores = np.matmul(qh, kh) * np.float32(scale) + mask.astype(np.float32)
    attn = softmax_f32(scores, axis=-1)
    out = np.matmul(attn, vh)                     # [B, H, Sq, D]
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))


# --- the dispatcher's naive path (infrared/model/triton_attention.py) --------


def paged_attention_naive(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                          pool_k: np.ndarray, pool_v: np.ndarray,
                          write_slots: np.ndarray, gather_slots: np.ndarray,
                          mask: np.ndarray, layer_idx: int, scale: float,
                          n_rep: int) -> np.ndarray:
    """Write this step's K/V into the pool, then gather + attend.

    Follows ``paged_attention`` with ``use_triton=False``
    (infrared/model/triton_attention.py:81-107) and ``_paged_attention_naive``
    (:110-129): scatter first, gather ``[B, T, Hkv, D]``, ``repeat_kv``, then
    ``masked_attention``. ``pool_k``/``pool_v`` are updated in place.
    """
    hkv, d = k.shape[-2], k.shape[-1]
    pool_write(pool_k, pool_v, layer_idx, k.reshape(-1, hkv, d),
               v.reshape(-1, hkv, d), write_slots)
    k_all = repeat_kv(pool_gather(pool_k, layer_idx, gather_slots), n_rep)
    v_all = repeat_kv(pool_gather(pool_v, layer_idx, gather_slots), n_rep)
    return masked_attention(q, k_all, v_all, mask, scale)


def blockwise_attention(q: np.ndarray, k_all: np.ndarray, v_all: np.ndarray,
                        mask: np.ndarray, scale: float,
                        block_n: int | None = None) -> np.ndarray:
    """Online-softmax twin of ``masked_attention`` walking keys in blocks.

    Follows ``paged_attention_blockwise_reference``
    (infrared/model/triton_attention.py:135-177): running max ``m``, running
    sum ``l`` and a rescaled accumulator, natural ``exp``, final ``acc / l``.
    """
    q = q.astype(np.float32)
    b, sq, h, d = q.shape
    t = k_all.shape[1]
    block_n = block_n or t
    qh = np.transpose(q, (0, 2, 1, 3))
    kh = np.transpose(k_all.astype(np.float32), (0, 2, 1, 3))
    vh = np.transpose(v_all.astype(np.float32), (0, 2, 1, 3))
    m_i = np.full((b, h, sq, 1), -np.inf, np.float32)
    l_i = np.zeros((b, h, sq, 1), np.float32)
    acc = np.zeros((b, h, sq, d), np.float32)
    for j in range(0, t, block_n):
        k_blk = kh[:, :, j:j + block_n]
        v_blk = vh[:, :, j:j + block_n]
        m_blk = mask[:, :, :, j:j + block_n].astype(np.float32)
        qk = np.matmul(qh, np.swapaxes(k_blk, -1, -2)) * np.float32(scale) + m_blk
        m_ij = np.maximum(m_i, qk.max(axis=-1, keepdims=True))
        p = np.exp(qk - m_ij)
        alpha = np.exp(m_i - m_ij)
        l_i = l_i * alpha + p.sum(axis=-1, keepdims=True)
        acc = acc * alpha + np.matmul(p, v_blk)
        m_i = m_ij
    out = acc / l_i
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))


# --- decode-step metadata (infrared/engine/paged_engine.py, cuda_graph.py) ---


def rope_tables(positions, head_dim: int, theta: float):
    """fp32 ``(cos, sin)`` of shape ``positions.shape + (head_dim,)``:
    ``inv_freq = 1 / theta ** (arange(0, D, 2) / D)``, ``emb = cat(f, f)``
    with ``f = position * inv_freq`` (infrared/model/layers.py:121-136).
    numpy's cos/sin may differ from torch's in the last bit; parity tests
    take the tables from the golden fixtures."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                          / np.float32(head_dim)))).astype(np.float32)
    f = np.asarray(positions, dtype=np.float32)[..., None] * inv
    emb = np.concatenate([f, f], axis=-1).astype(np.float32)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """``(x1, x2) -> (-x2, x1)`` over the last dim (infrared/model/layers.py:72-76)."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` in fp32, one op at a time
    (infrared/model/layers.py:79-89); ``x [B, heads, D]``, ``cos/sin [B, D]``
    broadcast over the heads."""
    x = x.astype(np.float32)
    c = cos.astype(np.float32)[:, None, :]
    s = sin.astype(np.float32)[:, None, :]
    a = (x * c).astype(np.float32)
    b = (rotate_half(x) * s).astype(np.float32)
    return (a + b).astype(np.float32)


def slot_of(block_table, pos: int, block_size: int) -> int:
    """Flat slot of logical position ``pos``.

    Follows ``PagedBatchEngine._slot`` (infrared/engine/paged_engine.py:621-625).
    """
    return int(block_table[pos // block_size]) * block_size + pos % block_size


def decode_mask(context_lens, max_len: int,
                min_value: float = F32_MIN) -> np.ndarray:
    """Additive decode mask ``[B, 1, 1, max_len]``: 0 before ``ctx``, min after.

    Follows ``PagedBatchEngine._decode_mask`` (infrared/engine/paged_engine.py:630-638).
    """
    lens = np.asarray(context_lens, dtype=np.int64)[:, None]
    invalid = np.arange(max_len)[None, :] >= lens
    mask = np.where(invalid, np.float32(min_value), np.float32(0.0))
    return mask[:, None, None, :].astype(np.float32)


def build_decode_inputs(block_tables, num_cached, last_tokens, bucket_b: int,
                        t_max: int, block_size: int,
                        min_value: float = F32_MIN) -> dict:
    """Fixed-shape decode inputs for a batch bucket and a ``t_max`` key axis.

    Follows ``build_decode_static_inputs`` (infrared/engine/cuda_graph.py:105-155):
    row i holds sequence i (rows past the real batch repeat row 0); the new
    token sits at position ``num_cached`` and is written to
    ``slot(block_table, num_cached)``; ``gather_slots`` lists the slots of
    positions ``[0, num_cached]`` and is zero-padded to ``t_max``; the mask
    blocks columns ``>= num_cached + 1``. Raises ``ValueError`` as the
    reference does for an empty/oversized batch or a context past ``t_max``.
    """
    b = len(last_tokens)
    if not 0 < b <= bucket_b:
        raise ValueError(f"need 0 < b ({b}) <= bucket_b ({bucket_b})")
    ids = np.zeros((bucket_b, 1), np.int64)
    positions = np.zeros((bucket_b, 1), np.int64)
    write_slots = np.zeros((bucket_b,), np.int64)
    gather_slots = np.zeros((bucket_b, t_max), np.int64)
    ctx_lens = []
    for i in range(bucket_b):
        j = i if i < b else 0
        bt, nc = block_tables[j], num_cached[j]
        ctx = nc + 1
        if ctx > t_max:
            raise ValueError(f"context_len {ctx} exceeds t_max {t_max}")
        ids[i, 0] = last_tokens[j]
        positions[i, 0] = nc
        write_slots[i] = slot_of(bt, nc, block_size)
        pos = np.arange(ctx)
        bt_arr = np.asarray(bt, np.int64)
        gather_slots[i, :ctx] = bt_arr[pos // block_size] * block_size + pos % block_size
        ctx_lens.append(ctx)
    mask = decode_mask(ctx_lens, t_max, min_value)
    return {"ids": ids, "positions": positions, "write_slots": write_slots,
            "gather_slots": gather_slots, "mask": mask,
            "context_lens": np.asarray(ctx_lens, np.int64)}


def derive_block_metadata(gather_slots: np.ndarray, mask: np.ndarray,
                          block_size: int):
    """Recover ``(block_tables, context_lens)`` from ``(gather_slots, mask)``.

    Inverse of the metadata build in ``_decode_logits_eager``
    (infrared/engine/paged_engine.py:309-315) and ``build_decode_static_inputs``
    (infrared/engine/cuda_graph.py:146-155): ``context_len`` is the number of
    zero (allowed) mask columns of the row, and block j of the row is
    ``gather_slots[b, j*bs] // bs`` for every block that holds a valid
    position (0 past the context). Returns ``(bt int32 [B, ceil(T/bs)],
    ctx int32 [B], ok bool)``; ``ok`` is False when a row is not
    block-structured (a valid position whose slot is not
    ``bt[p//bs]*bs + p%bs``) or its mask is not a prefix of zeros.
    """
    b, t = gather_slots.shape
    m = mask.reshape(b, t)
    allowed = m == 0
    ctx = allowed.sum(axis=1).astype(np.int32)
    nb = -(-t // block_size)
    bt = np.zeros((b, nb), np.int32)
    ok = True
    for i in range(b):
        c = int(ctx[i])
        if not allowed[i, :c].all():
            ok = False
        if c == 0:
            continue
        first = gather_slots[i, 0:c:block_size]
        bt[i, :len(first)] = first // block_size
        pos = np.arange(c)
        want = bt[i, pos // block_size].astype(np.int64) * block_size + pos % block_size
        if not np.array_equal(want, gather_slots[i, :c]):
            ok = False
    return bt, ctx, ok


# --- the block-table form used by the kernels ---------------------------------


def gather_slots_from_tables(block_tables: np.ndarray, context_lens: np.ndarray,
                             block_size: int, t: int | None = None) -> np.ndarray:
    """``[B, T]`` slot list of each row's history, zero past the context.

    The per-row build of ``_decode_logits_eager`` (infrared/engine/paged_engine.py:309-314).
    """
    ctx = np.asarray(context_lens, np.int64)
    t = int(ctx.max()) if t is None else t
    b = len(ctx)
    out = np.zeros((b, max(t, 1)), np.int64)
    for i in range(b):
        pos = np.arange(int(ctx[i]))
        out[i, :len(pos)] = (block_tables[i, pos // block_size].astype(np.int64)
                             * block_size + pos % block_size)
    return out


def decode_from_tables(q: np.ndarray, pool_k: np.ndarray, pool_v: np.ndarray,
                       layer_idx: int, block_tables: np.ndarray,
                       context_lens: np.ndarray, block_size: int, scale: float,
                       n_rep: int) -> np.ndarray:
    """Decode attention for ``q [B, H, D]`` over block-table histories.

    The naive read path (gather -> repeat_kv -> masked_attention,
    infrared/model/triton_attention.py:110-129) with ``gather_slots`` and the
    decode mask rebuilt from ``(block_tables, context_lens)``. A row with a
    zero context returns zeros, the convention of the reference's fused
    kernel (``l_safe`` guard, infrared/model/triton_attention.py:293-297).
    Sequences are processed one at a time so memory stays bounded.
    Returns ``[B, H, D]`` float32.
    """
    b, h, d = q.shape
    out = np.zeros((b, h, d), np.float32)
    for i in range(b):
        c = int(context_lens[i])
        if c == 0:
            continue
        gs = gather_slots_from_tables(block_tables[i:i + 1], context_lens[i:i + 1],
                                      block_size, c)
        k_all = repeat_kv(pool_gather(pool_k, layer_idx, gs), n_rep)
        v_all = repeat_kv(pool_gather(pool_v, layer_idx, gs), n_rep)
        mask = np.zeros((1, 1, 1, c), np.float32)
        out[i] = masked_attention(q[i:i + 1, None], k_all, v_all, mask, scale)[0, 0]
    return out


# --- prefill / mixed varlen (Sq > 1) -----------------------------------------


def varlen_mask(q_seq_ids, q_pos, k_seq_ids, k_pos) -> np.ndarray:
    """Additive ``[1, 1, Q, K]`` mask of a packed multi-sequence frame: a query
    token attends a key of the same sequence at or before its position
    (infrared/model/inputs.py:64-94, ``build_varlen_mask``)."""
    q_seq_ids, q_pos = np.asarray(q_seq_ids), np.asarray(q_pos)
    k_seq_ids, k_pos = np.asarray(k_seq_ids), np.asarray(k_pos)
    allowed = (q_seq_ids[:, None] == k_seq_ids[None, :]) & (k_pos[None, :] <= q_pos[:, None])
    return np.where(allowed, np.float32(0), np.float32(F32_MIN))[None, None].astype(np.float32)


def varlen_frame(block_tables, starts, q_lens, block_size: int):
    """The packed frame of infrared's mixed step for sequences whose first
    ``starts[s]`` tokens are cached and ``q_lens[s]`` new tokens are forwarded
    (infrared/engine/paged_engine.py:478-496): per query token its write slot,
    sequence id and position; per gathered key its slot, sequence id and
    position. Returns a dict of numpy arrays."""
    ws, gs, qs, qp, ks, kp = [], [], [], [], [], []
    for i, (st, ql) in enumerate(zip(starts, q_lens)):
        for p in range(st, st + ql):
            ws.append(slot_of(block_tables[i], p, block_size))
            qs.append(i)
            qp.append(p)
        for p in range(st + ql):
            gs.append(slot_of(block_tables[i], p, block_size))
            ks.append(i)
            kp.append(p)
    return {"write_slots": np.array(ws, np.int64), "gather_slots": np.array(gs, np.int64)[None],
            "q_seq_ids": np.array(qs), "q_pos": np.array(qp), "k_seq_ids": np.array(ks),
            "k_pos": np.array(kp)}


def varlen_metadata(gather_slots: np.ndarray, mask: np.ndarray, block_size: int):
    """Inverse of :func:`varlen_frame` + :func:`varlen_mask` for one packed
    frame (``gather_slots [1, K]``, ``mask [1, 1, Q, K]``): every query row must
    allow one contiguous key range ``[lo, lo + n)``; consecutive rows with the
    same ``lo`` form a sequence whose history is its key range of the last
    row, block-structured from ``lo``. Returns ``(block_tables, context_lens,
    q_start, ok)``; ``ok`` is False when the frame does not have that form."""
    m = mask.reshape(mask.shape[-2], mask.shape[-1])
    gsl = gather_slots.reshape(-1)
    q, k = m.shape
    allowed = m == 0
    ok = True
    lo = np.zeros(q, np.int64)
    cnt = allowed.sum(axis=1).astype(np.int64)
    for i in range(q):
        nz = np.flatnonzero(allowed[i])
        if len(nz) == 0 or nz[-1] - nz[0] + 1 != len(nz):
            ok = False
            lo[i] = nz[0] if len(nz) else 0
            continue
        lo[i] = nz[0]
    starts = [0] + [i for i in range(1, q) if lo[i] != lo[i - 1]]
    q_start = np.array(starts + [q], np.int32)
    nseq = len(starts)
    ctx = np.zeros(nseq, np.int32)
    max_blocks = max(1, -(-int(cnt.max()) // block_size)) if q else 1
    bt = np.zeros((nseq, max_blocks), np.int32)
    for s in range(nseq):
        r0, r1 = q_start[s], q_start[s + 1]
        c = int(cnt[r1 - 1])
        ctx[s] = c
        if np.any(np.diff(cnt[r0:r1]) != 1):
            ok = False
        base = int(lo[r0])
        hist = gsl[base:base + c]
        first = hist[0:c:block_size]
        bt[s, :len(first)] = first // block_size
        pos = np.arange(c)
        want = bt[s, pos // block_size].astype(np.int64) * block_size + pos % block_size
        if not np.array_equal(want, hist):
            ok = False
    return bt, ctx, q_start, ok


def prefill_from_tables(q: np.ndarray, pool_k: np.ndarray, pool_v: np.ndarray,
                        layer_idx: int, block_tables: np.ndarray, context_lens,
                        q_start, block_size: int, scale: float, n_rep: int) -> np.ndarray:
    """Causal attention of packed query rows ``q [Q, H, D]`` over block-table
    histories: sequence ``s`` owns rows ``[q_start[s], q_start[s+1])``, its
    last ``q_len`` positions ``ctx - q_len .. ctx - 1``; a row at position
    ``p`` attends positions ``0..p`` (the naive path with the causal /
    varlen masks of infrared/model/inputs.py:38-94). Returns float32."""
    out = np.zeros(q.shape, np.float32)
    for s in range(len(context_lens)):
        r0, r1 = int(q_start[s]), int(q_start[s + 1])
        c, ql = int(context_lens[s]), r1 - r0
        if ql == 0:
            continue
        gs = gather_slots_from_tables(block_tables[s:s + 1], context_lens[s:s + 1],
                                      block_size, c)
        k_all = repeat_kv(pool_gather(pool_k, layer_idx, gs), n_rep)
        v_all = repeat_kv(pool_gather(pool_v, layer_idx, gs), n_rep)
        pos = np.arange(c - ql, c)
        allowed = np.arange(c)[None, :] <= pos[:, None]
        mask = np.where(allowed, np.float32(0), np.float32(F32_MIN))[None, None]
        out[r0:r1] = masked_attention(q[r0:r1][None], k_all, v_all, mask, scale)[0]
    return out


# --- split-KV partials and their merge (no reference counterpart) ------------


def partial_attention(q: np.ndarray, pool_k: np.ndarray, pool_v: np.ndarray,
                      layer_idx: int, block_tables: np.ndarray,
                      context_lens: np.ndarray, block_size: int, scale: float,
                      n_rep: int, tok_begin: int, tok_end: int):
    """Attention of ``q [B, H, D]`` over positions ``[tok_begin, tok_end)`` only.

    Returns ``(o [B, H, D] normalised over that range, lse [B, H])`` with
    ``lse = log(sum(exp(score)))`` in natural-log units; a row with no key in
    the range gives ``o = 0`` and ``lse = -inf``. The reference defers
    split-KV (infrared ``docs/research/t4-triton-cudagraph-api.md:130``); this
    is the standard log-sum-exp decomposition of its softmax, restated from
    the mathematics: softmax over a union of key sets equals the
    ``exp(lse_p - LSE)``-weighted sum of the per-set softmax outputs.
    """
    b, h, d = q.shape
    o = np.zeros((b, h, d), np.float32)
    lse = np.full((b, h), -np.inf, np.float32)
    for i in range(b):
        c = int(context_lens[i])
        lo, hi = max(0, tok_begin), min(c, tok_end)
        if hi <= lo:
            continue
        pos = np.arange(lo, hi)
        slots = (block_tables[i, pos // block_size].astype(np.int64) * block_size
                 + pos % block_size)
        kk = repeat_kv(pool_k[layer_idx, slots][None], n_rep)[0].astype(np.float32)
        vv = repeat_kv(pool_v[layer_idx, slots][None], n_rep)[0].astype(np.float32)
        s = np.einsum("hd,thd->ht", q[i].astype(np.float32), kk) * np.float32(scale)
        m = s.max(axis=1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(axis=1, keepdims=True)
        o[i] = np.einsum("ht,thd->hd", e / l, vv)
        lse[i] = (m + np.log(l))[:, 0]
    return o, lse


def lse_merge(o_parts: np.ndarray, lse_parts: np.ndarray) -> np.ndarray:
    """Combine ``P`` partials ``o [P, B, H, D]``, ``lse [P, B, H]`` into ``[B, H, D]``.

    ``out = sum_p exp(lse_p - LSE) * o_p`` with ``LSE = log sum_p exp(lse_p)``;
    partials with ``lse = -inf`` get zero weight and a row whose partials are
    all empty gives zeros.
    """
    lse = lse_parts.astype(np.float64)
    mx = np.max(lse, axis=0)
    mx_safe = np.where(np.isfinite(mx), mx, 0.0)
    w = np.exp(lse - mx_safe[None])
    w = np.where(np.isfinite(lse), w, 0.0)
    tot = w.sum(axis=0)
    tot_safe = np.where(tot > 0, tot, 1.0)
    out = (w[..., None] * o_parts.astype(np.float64)).sum(axis=0) / tot_safe[..., None]
    return out.astype(np.float32)


# --- algorithmic byte count (the roofline numerator) -------------------------


def decode_bytes(context_lens, num_heads: int, num_kv_heads: int, head_dim: int,
                 elem_bytes: int, max_blocks: int, with_write: bool = False) -> int:
    """Useful HBM bytes of one decode call over ``context_lens``.

    K and V of every cached token of every kv head, plus q read, out written,
    the block table and the context lengths; with ``with_write`` the new
    token's K/V read and written once more.
    """
    ctx = np.asarray(context_lens, np.int64)
    b = len(ctx)
    e = 2 * num_kv_heads * head_dim * elem_bytes
    total = int(ctx.sum()) * e
    total += 2 * b * num_heads * head_dim * elem_bytes
    total += b * max_blocks * 4 + 4 * b
    if with_write:
        total += 2 * 2 * b * num_kv_heads * head_dim * elem_bytes
    return total


def log2e() -> float:
    return 1.0 / math.log(2.0)
