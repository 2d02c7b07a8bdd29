"""Paged decode over the GPUs of one node (one process per GPU, torch.distributed).

Two partitionings, neither of which exists in infrared (it is single-GPU):

* **by sequence** — each GPU owns disjoint sequences, their blocks and its
  own pool; nothing is exchanged (``shard_sequences`` balances the ranges
  by tokens).
* **by KV chunk** (one long context over several GPUs) — GPU g keeps blocks
  ``[g*n//G, (g+1)*n//G)`` of every sequence's n blocks
  (``kv_chunk_tables``), computes the softmax-normalised partial output and
  its log-sum-exp over that range (``ir_paged_decode_lse``), and one
  all-gather of the fp32 partials (o and lse packed in one buffer:
  ``B*H*(D+1)*4`` bytes per GPU) lets every rank combine them with
  ``ir_lse_merge``. Data only moves through the collective into each rank's
  own memory — no kernel reads another GPU's memory.

The compute steps are parameters of ``chunked_decode`` so the exchange can
be exercised on CPU ranks (gloo) with the oracle in tests; ``partial_fn``
writes into the packed send buffer, so the partials are not copied again.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard_sequences(context_lens, world: int) -> list[tuple[int, int]]:
    """Contiguous sequence ranges ``[(lo, hi), ...]``, one per rank, cut where
    the running token count crosses ``r * total / world``; while there are at
    least ``world`` sequences every range holds at least one."""
    ctx = np.asarray(context_lens, dtype=np.int64)
    n = len(ctx)
    if world <= 0:
        raise ValueError("world must be positive")
    pref = np.concatenate([[0], np.cumsum(ctx)])
    cuts = [0]
    for r in range(1, world):
        c = int(np.searchsorted(pref, pref[-1] * r / world, side="left"))
        if n >= world:
            c = min(max(c, cuts[-1] + 1), n - (world - r))
        cuts.append(min(max(c, cuts[-1]), n))
    cuts.append(n)
    return [(cuts[i], cuts[i + 1]) for i in range(world)]


def kv_chunk_tables(block_tables: np.ndarray, context_lens, block_size: int, world: int,
                    rank: int):
    """This rank's block-table columns and context lengths for a KV-chunk split.

    Rank g takes blocks ``[g*n//world, (g+1)*n//world)`` of a sequence with
    ``n = ceil(ctx / block_size)`` blocks; its local context is the number of
    positions of the sequence that fall in those blocks (0 if none).
    Returns ``(tables int32 [B, max_local], ctx int32 [B], first_block [B])``.
    """
    ctx = np.asarray(context_lens, dtype=np.int64)
    b = len(ctx)
    nblk = (ctx + block_size - 1) // block_size
    lo = (rank * nblk) // world
    hi = ((rank + 1) * nblk) // world
    width = int((hi - lo).max()) if b else 0
    tables = np.zeros((b, max(width, 1)), np.int32)
    local = np.zeros(b, np.int32)
    for i in range(b):
        cols = block_tables[i, lo[i]:hi[i]]
        tables[i, :len(cols)] = cols
        local[i] = max(0, min(int(ctx[i]), int(hi[i]) * block_size) - int(lo[i]) * block_size)
    return tables, local, lo.astype(np.int64)


def _cuda_partial(q, k_pool, v_pool, tables, ctx, scale, block_size, o, lse):
    from . import ops

    ops.paged_decode_lse(q, k_pool, v_pool, tables, ctx, scale, block_size, o=o, lse=lse)


def _cuda_merge(o_parts, lse_parts, dtype):
    from . import ops

    return ops.lse_merge(o_parts, lse_parts, dtype)


def chunked_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                   tables: torch.Tensor, ctx: torch.Tensor, scale: float, block_size: int,
                   out_dtype: torch.dtype | None = None, group=None,
                   partial_fn=_cuda_partial, merge_fn=_cuda_merge) -> torch.Tensor:
    """Decode attention of ``q [B, H, D]`` over a KV range held on this rank,
    combined across all ranks of ``group``; every rank returns the full
    ``[B, H, D]`` result. Each rank passes its own ``tables``/``ctx``
    (``kv_chunk_tables``) and pool; ``q`` is the same on every rank."""
    b, h, d = q.shape
    world = dist.get_world_size(group)
    packed = torch.empty(b * h * (d + 1), dtype=torch.float32, device=q.device)
    o = packed[: b * h * d].view(b, h, d)
    lse = packed[b * h * d:].view(b, h)
    partial_fn(q, k_pool, v_pool, tables, ctx, scale, block_size, o, lse)
    gathered = torch.empty(world * packed.numel(), dtype=torch.float32, device=q.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    gathered = gathered.view(world, packed.numel())
    o_parts = gathered[:, : b * h * d].unflatten(1, (b, h, d))   # views, no copy
    lse_parts = gathered[:, b * h * d:].unflatten(1, (b, h))
    return merge_fn(o_parts, lse_parts, out_dtype or q.dtype)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest ``value`` over all ranks (per-rank timings -> job time)."""
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
