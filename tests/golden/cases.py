"""Seeded cases behind the golden fixtures (shared by make_golden.py and the tests).

Each case is a workload from ``infrared_b200.workloads`` plus a value seed;
inputs are regenerated from the seeds with numpy's PCG64 (identical on every
machine) and checked against the stored input digest before use.
"""

from __future__ import annotations

import hashlib

import numpy as np

from infrared_b200 import workloads as wl

# name -> (workload factory, value seed)
ATTENTION_CASES = {
    "c1": (lambda: wl.c1(seed=0), 1),
    "g2_d64_bs16": (lambda: wl.custom(11, 3, 4, 2, 64, 16, 1, 70, "float32"), 2),
    "g7_d128_bs16": (lambda: wl.custom(12, 5, 21, 3, 128, 16, 1, 300, "float32"), 3),
    "g1_d64_bs8": (lambda: wl.custom(13, 4, 8, 8, 64, 8, 1, 100, "float32"), 4),
    "g12_d128_bs32": (lambda: wl.custom(14, 2, 24, 2, 128, 32, 30, 200, "float32"), 5),
    "g8_d128_bs16": (lambda: wl.custom(15, 6, 16, 2, 128, 16, 1, 40, "float32"), 6),
    "g3_d64_bs4": (lambda: wl.custom(16, 3, 12, 4, 64, 4, 1, 50, "float32"), 7),
    "g7_d64_bs16_shared": (lambda: wl.custom(17, 12, 14, 2, 64, 16, 40, 160, "float32",
                                             shared_frac=0.5), 8),
}


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def attention_inputs(name: str):
    """``(workload, q, k_pool, v_pool, k_new, v_new)`` of a case (fp32 numpy)."""
    factory, vseed = ATTENTION_CASES[name]
    w = factory()
    q, kp, vp, kn, vn = wl.numpy_values(w, vseed)
    return w, q, kp, vp, kn, vn


def input_digest(name: str) -> str:
    w, q, kp, vp, kn, vn = attention_inputs(name)
    return digest(w.context_lens, w.block_tables, w.slot_mapping, q, kp, vp, kn, vn)


def seam_tensors(w, q, kp, vp, kn, vn):
    """The reference seam's arguments for a decode step of workload ``w``:
    ``q [B,1,H,D]``, ``k/v [B,1,Hkv,D]``, pools ``[1, slots, Hkv, D]``,
    ``write_slots [B]``, ``gather_slots [B, T]`` and mask ``[B,1,1,T]``."""
    from oracle import paged_attention_np as orc

    t = int(w.context_lens.max())
    gs = orc.gather_slots_from_tables(w.block_tables, w.context_lens, w.block_size, t)
    mask = orc.decode_mask(w.context_lens, t)
    return {
        "q": q[:, None], "k": kn[:, None], "v": vn[:, None],
        "pool_k": kp[None].copy(), "pool_v": vp[None].copy(),
        "write_slots": w.slot_mapping.copy(), "gather_slots": gs, "mask": mask,
    }


# fixed-shape graph inputs (reference: build_decode_static_inputs)
GRAPH_CASES = {
    "graph_a": dict(seed=21, b=5, bucket_b=8, t_max=96, block_size=8, num_blocks=64),
    "graph_b": dict(seed=22, b=3, bucket_b=4, t_max=64, block_size=16, num_blocks=32),
}


def graph_case_args(name: str):
    p = GRAPH_CASES[name]
    rng = np.random.default_rng(p["seed"])
    bs = p["block_size"]
    perm = list(rng.permutation(p["num_blocks"]))
    tables, num_cached, last = [], [], []
    for _ in range(p["b"]):
        nc = int(rng.integers(0, p["t_max"]))
        nblk = nc // bs + 1
        tables.append([int(perm.pop()) for _ in range(nblk)])
        num_cached.append(nc)
        last.append(int(rng.integers(0, 1000)))
    return tables, num_cached, last, p["bucket_b"], p["t_max"], bs


BLOCKWISE_BLOCKS = (1, 3, 16, 100)

# rotary embedding at the new token's position (position = context_len - 1):
# case -> theta of infrared's RotaryEmbedding
ROPE_CASES = {"c1": 1e6, "g7_d128_bs16": 1e4, "g8_d128_bs16": 1e6, "g2_d64_bs16": 1e6}


# prefill / mixed varlen frames (reference: paged_engine.py:170-221 prefill with a
# cached prefix, :461-516 packed mixed step): name -> (seed, H, Hkv, D, block size,
# [(cached tokens, forwarded tokens) per sequence])
PREFILL_CASES = {
    "prefill_one": (31, 14, 2, 64, 16, [(37, 63)]),
    "varlen_mix": (32, 8, 2, 128, 16, [(0, 20), (50, 1), (30, 17), (0, 5)]),
    "varlen_bs8": (33, 12, 4, 64, 8, [(9, 33), (64, 2), (1, 40)]),
    "varlen_g7": (34, 7, 1, 128, 16, [(0, 130), (200, 1), (3, 40)]),
}


def prefill_inputs(name: str) -> dict:
    """Seeded fp32 inputs of a prefill case: block tables, the packed frame, q and
    this step's K/V for every forwarded token, and the initial pools."""
    from oracle import paged_attention_np as orc

    seed, h, hkv, d, bs, chunks = PREFILL_CASES[name]
    rng = np.random.default_rng(seed)
    starts = [c[0] for c in chunks]
    qls = [c[1] for c in chunks]
    ctx = np.array([st + ql for st, ql in chunks], np.int32)
    nblk = [-(-int(c) // bs) for c in ctx]
    num_blocks = sum(nblk) + 4
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(chunks), max(nblk)), np.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    q_start = np.concatenate([[0], np.cumsum(qls)]).astype(np.int32)
    nq = int(q_start[-1])
    return {
        "h": h, "hkv": hkv, "d": d, "bs": bs, "scale": d ** -0.5, "n_rep": h // hkv,
        "starts": starts, "q_lens": qls, "block_tables": bt, "context_lens": ctx,
        "q_start": q_start, "num_blocks": num_blocks,
        "q": rng.standard_normal((nq, h, d), dtype=np.float32),
        "k": rng.standard_normal((nq, hkv, d), dtype=np.float32),
        "v": rng.standard_normal((nq, hkv, d), dtype=np.float32),
        "pool_k": rng.standard_normal((num_blocks * bs, hkv, d), dtype=np.float32),
        "pool_v": rng.standard_normal((num_blocks * bs, hkv, d), dtype=np.float32),
        "frame": orc.varlen_frame(bt, starts, qls, bs),
    }
