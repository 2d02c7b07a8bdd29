"""Seeded synthetic decode workloads at the benchmark geometries.

Metadata (context lengths, block tables, write slots) comes from numpy's
PCG64 generator so it is identical on every machine; K/V/q values are drawn
either with numpy (small cases whose golden outputs are committed) or with a
seeded ``torch.Generator`` on the device (benchmark sizes).

Configurations (Qwen2.5 geometries; there is no public dataset for this
path, inputs are synthetic by design):

* ``c1`` fp32, 14 q / 2 kv heads, D=64, scale 1/8, B=8, ctx ~ U[1, 512],
  block 16, pool of 512 blocks, block tables = slices of a random permutation.
* ``c2`` bf16, 28 q / 4 kv heads, D=128, B=64, ctx ~ U[512, 4096],
  pool of 32768 blocks, values N(0, 1) * 0.5.
* ``c3`` as c2 with B=256, ctx ~ U[128, 2048], new-token slots in randomly
  allocated tail blocks, ~30 % of sequences sharing 1-8 leading blocks.
* ``c4`` bf16 7B geometry, B=4, ctx = 32768 each (split-KV / multi-GPU).
* ``p1`` prefill (Sq > 1): bf16 7B attention geometry, 8 prompts of 4096
  tokens each forwarded at once (causal), block 16.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Workload:
    name: str
    batch: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    dtype: str                 # "float32" | "bfloat16" | "float16"
    scale: float
    std: float
    context_lens: np.ndarray   # int32 [B]
    block_tables: np.ndarray   # int32 [B, max_blocks]
    slot_mapping: np.ndarray   # int64 [B], slot of position ctx-1
    shared: dict = field(default_factory=dict)

    @property
    def n_rep(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def max_blocks(self) -> int:
        return self.block_tables.shape[1]

    @property
    def num_slots(self) -> int:
        return self.num_blocks * self.block_size

    @property
    def elem_bytes(self) -> int:
        return 4 if self.dtype == "float32" else 2

    def kv_bytes(self) -> int:
        """K and V bytes the decode must read (per referencing sequence)."""
        return int(self.context_lens.astype(np.int64).sum()) * 2 * self.num_kv_heads * \
            self.head_dim * self.elem_bytes

    def algorithmic_bytes(self, with_write: bool = False) -> int:
        """Useful HBM bytes of one decode call (K/V + q + out + tables)."""
        b, h, d, e = self.batch, self.num_heads, self.head_dim, self.elem_bytes
        total = self.kv_bytes() + 2 * b * h * d * e + b * self.max_blocks * 4 + 4 * b
        if with_write:
            total += 2 * 2 * b * self.num_kv_heads * d * e
        return total


def tail_slots(block_tables: np.ndarray, context_lens: np.ndarray, bs: int) -> np.ndarray:
    """Slot of position ``ctx - 1`` of every row (where the new token goes)."""
    out = np.zeros(len(context_lens), np.int64)
    for i, c in enumerate(context_lens):
        if c > 0:
            p = int(c) - 1
            out[i] = int(block_tables[i, p // bs]) * bs + p % bs
    return out


def assign_blocks(rng: np.random.Generator, context_lens: np.ndarray, bs: int,
                  num_blocks: int, max_blocks: int | None = None,
                  shared_frac: float = 0.0, max_prefix: int = 8) -> tuple[np.ndarray, dict]:
    """Block tables drawn from one random permutation of the pool's block ids.

    With ``shared_frac > 0`` about that fraction of sequences are put in
    small groups that reuse the first 1..``max_prefix`` full blocks of the
    group's first member (ref-counted prefix sharing, as the reference's
    ``BlockManager.match_prefix`` produces); shared blocks never hold a
    position at or after ``ctx - 1`` of any member, so every write lands in
    a private tail block.
    """
    b = len(context_lens)
    nblk = (context_lens.astype(np.int64) + bs - 1) // bs
    mb = int(nblk.max()) if max_blocks is None else max_blocks
    bt = np.zeros((b, max(mb, 1)), np.int32)
    free = list(rng.permutation(num_blocks))
    groups: list[list[int]] = []
    if shared_frac > 0:
        chosen = rng.permutation(b)[: int(round(shared_frac * b))]
        i = 0
        while i < len(chosen):
            size = int(rng.integers(2, 5))
            groups.append([int(x) for x in chosen[i:i + size]])
            i += size
        groups = [g for g in groups if len(g) >= 2]
    prefix_of: dict[int, tuple[int, int]] = {}   # member -> (donor, n_shared)
    for g in groups:
        donor = g[0]
        limit = min((int(context_lens[m]) - 1) // bs for m in g)
        n_shared = min(int(rng.integers(1, max_prefix + 1)), limit)
        if n_shared < 1:
            continue
        for m in g[1:]:
            prefix_of[m] = (donor, n_shared)
    # donors first so their blocks exist when members copy them
    order = sorted(range(b), key=lambda i: i in prefix_of)
    shared_blocks = 0
    for i in order:
        n = int(nblk[i])
        start = 0
        if i in prefix_of:
            donor, k = prefix_of[i]
            bt[i, :k] = bt[donor, :k]
            start = k
            shared_blocks += k
        for j in range(start, n):
            bt[i, j] = free.pop()
    info = {"groups": groups, "prefix_of": prefix_of, "shared_block_refs": shared_blocks}
    return bt, info


def c1(seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    b, bs, nb = 8, 16, 512
    ctx = rng.integers(1, 513, size=b).astype(np.int32)
    bt, info = assign_blocks(rng, ctx, bs, nb, max_blocks=32)
    return Workload("c1", b, 14, 2, 64, bs, nb, "float32", 1.0 / 8.0, 1.0, ctx, bt,
                    tail_slots(bt, ctx, bs), info)


def c2(seed: int = 0, batch: int = 64) -> Workload:
    rng = np.random.default_rng(seed)
    bs, nb = 16, max(32768, batch * 256)
    ctx = rng.integers(512, 4097, size=batch).astype(np.int32)
    bt, info = assign_blocks(rng, ctx, bs, nb, max_blocks=4096 // bs)
    return Workload("c2", batch, 28, 4, 128, bs, nb, "bfloat16", 128 ** -0.5, 0.5, ctx, bt,
                    tail_slots(bt, ctx, bs), info)


def c3(seed: int = 0, batch: int = 256) -> Workload:
    rng = np.random.default_rng(seed)
    bs, nb = 16, max(32768, batch * 128)
    ctx = rng.integers(128, 2049, size=batch).astype(np.int32)
    bt, info = assign_blocks(rng, ctx, bs, nb, max_blocks=2048 // bs, shared_frac=0.3)
    return Workload("c3", batch, 28, 4, 128, bs, nb, "bfloat16", 128 ** -0.5, 0.5, ctx, bt,
                    tail_slots(bt, ctx, bs), info)


def c4(seed: int = 0, batch: int = 4, ctx_len: int = 32768) -> Workload:
    rng = np.random.default_rng(seed)
    bs = 16
    nb = batch * ctx_len // bs
    ctx = np.full(batch, ctx_len, np.int32)
    bt, info = assign_blocks(rng, ctx, bs, nb, max_blocks=ctx_len // bs)
    return Workload("c4", batch, 28, 4, 128, bs, nb, "bfloat16", 128 ** -0.5, 0.5, ctx, bt,
                    tail_slots(bt, ctx, bs), info)


def custom(seed: int, batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
           block_size: int, ctx_lo: int, ctx_hi: int, dtype: str = "bfloat16",
           num_blocks: int | None = None, shared_frac: float = 0.0,
           std: float = 1.0, max_blocks: int | None = None) -> Workload:
    """A seeded workload of any geometry (parity sweeps)."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int32)
    need = int(((ctx.astype(np.int64) + block_size - 1) // block_size).sum())
    nb = num_blocks or max(need + 8, 16)
    mb = max_blocks or max(1, (ctx_hi + block_size - 1) // block_size)
    bt, info = assign_blocks(rng, ctx, block_size, nb, max_blocks=mb, shared_frac=shared_frac)
    return Workload(f"custom{seed}", batch, num_heads, num_kv_heads, head_dim, block_size, nb,
                    dtype, head_dim ** -0.5, std, ctx, bt, tail_slots(bt, ctx, block_size), info)


CONFIGS = {"c1": c1, "c2": c2, "c3": c3, "c4": c4}


def numpy_values(w: Workload, seed: int):
    """q [B, H, D], k/v pools [num_slots, Hkv, D], k_new/v_new [B, Hkv, D] as float32
    numpy arrays drawn from N(0, 1) * std (small cases; exact on every machine)."""
    rng = np.random.default_rng(seed)
    f = np.float32
    q = (rng.standard_normal((w.batch, w.num_heads, w.head_dim)) * w.std).astype(f)
    kp = (rng.standard_normal((w.num_slots, w.num_kv_heads, w.head_dim)) * w.std).astype(f)
    vp = (rng.standard_normal((w.num_slots, w.num_kv_heads, w.head_dim)) * w.std).astype(f)
    kn = (rng.standard_normal((w.batch, w.num_kv_heads, w.head_dim)) * w.std).astype(f)
    vn = (rng.standard_normal((w.batch, w.num_kv_heads, w.head_dim)) * w.std).astype(f)
    return q, kp, vp, kn, vn


def torch_values(w: Workload, seed: int, device):
    """The same tensors drawn on ``device`` with a seeded torch generator, in the
    workload's dtype (benchmark sizes)."""
    import torch

    dt = getattr(torch, w.dtype)
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def randn(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
                * w.std).to(dt)

    q = randn(w.batch, w.num_heads, w.head_dim)
    kp = randn(w.num_slots, w.num_kv_heads, w.head_dim)
    vp = randn(w.num_slots, w.num_kv_heads, w.head_dim)
    kn = randn(w.batch, w.num_kv_heads, w.head_dim)
    vn = randn(w.batch, w.num_kv_heads, w.head_dim)
    return q, kp, vp, kn, vn


# --- prefill frames -----------------------------------------------------------


@dataclass
class PrefillWorkload:
    """Packed prefill frame: sequence s has ``starts[s]`` cached tokens and
    forwards ``q_lens[s]`` new ones (rows ``q_start[s] .. q_start[s+1]-1``)."""

    name: str
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    starts: np.ndarray
    q_lens: np.ndarray
    block_tables: np.ndarray
    num_blocks: int
    dtype: str = "bfloat16"

    @property
    def context_lens(self) -> np.ndarray:
        return (self.starts + self.q_lens).astype(np.int32)

    @property
    def q_start(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.q_lens)]).astype(np.int32)

    @property
    def total_q(self) -> int:
        return int(self.q_lens.sum())

    @property
    def scale(self) -> float:
        return self.head_dim ** -0.5

    def flops(self) -> int:
        """Useful FLOPs: every query row at position p scores p + 1 keys
        (QK^T and P.V, 2 * D each, per query head)."""
        tot = 0
        for st, ql in zip(self.starts.tolist(), self.q_lens.tolist()):
            # sum over p in [st, st + ql) of (p + 1)
            tot += ql * (2 * st + ql + 1) // 2
        return 4 * self.head_dim * self.num_heads * tot


def prefill_frame(name: str, seed: int, starts, q_lens, num_heads: int = 28,
                  num_kv_heads: int = 4, head_dim: int = 128, block_size: int = 16,
                  dtype: str = "bfloat16") -> PrefillWorkload:
    rng = np.random.default_rng(seed)
    starts = np.asarray(starts, np.int64)
    q_lens = np.asarray(q_lens, np.int64)
    ctx = starts + q_lens
    nblk = -(-ctx // block_size)
    num_blocks = int(nblk.sum())
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(ctx), int(nblk.max())), np.int32)
    off = 0
    for i, n in enumerate(nblk.tolist()):
        bt[i, :n] = perm[off:off + n]
        off += n
    return PrefillWorkload(name, num_heads, num_kv_heads, head_dim, block_size, starts, q_lens,
                           bt, num_blocks, dtype)


def p1(seed: int = 0, batch: int = 8, prompt: int = 4096) -> PrefillWorkload:
    return prefill_frame("p1", seed, [0] * batch, [prompt] * batch)


PREFILL_CONFIGS = {"p1": p1}
