"""``paged_attention`` with the reference engine's signature, on the B200 kernels.

Mirrors ``paged_attention(q, k, v, paged, mask, layer_idx, scale, n_rep)``
of infrared (``infrared/model/triton_attention.py:81-107``): it writes this
step's K/V into the pool, then attends over each row's history and returns
``[B, Sq, H, D]``. Decode steps (``Sq == 1``) run the decode kernels; packed
prefill / mixed frames (``B == 1``, ``Sq > 1``: one prompt with a cached
prefix, or infrared's mixed prefill + decode step) run the tensor-core
prefill kernel.

The reference hands the kernel a per-row slot list ``gather_slots [B, T]``
and an additive mask ``[B, 1, 1, T]``; the B200 kernels read whole blocks
through ``block_tables`` and ``context_lens``. ``ir_derive_block_metadata``
converts one into the other on the device once per forward: the same
``(PagedContext, mask)`` pair is passed to every layer, so the result is
cached on that pair (a strong reference keeps the objects, and so their
ids, alive).
"""

from __future__ import annotations

import threading

import torch

from . import ops

_cache_lock = threading.Lock()
_cache: dict = {}


def block_metadata(paged, mask: torch.Tensor):
    """``(block_tables int32, context_lens int32)`` for this forward's context."""
    with _cache_lock:
        hit = _cache.get("key")
        if hit is not None and hit[0] is paged and hit[1] is mask:
            return _cache["value"]
    bt, ctx = ops.derive_block_metadata(paged.gather_slots, mask, paged.pool.block_size)
    with _cache_lock:
        _cache["key"] = (paged, mask)
        _cache["value"] = (bt, ctx)
    return bt, ctx


def varlen_metadata(paged, mask: torch.Tensor):
    """``(block_tables, context_lens, q_start)`` of a packed Sq > 1 frame,
    derived on the device once per forward (cached like :func:`block_metadata`)."""
    with _cache_lock:
        hit = _cache.get("vkey")
        if hit is not None and hit[0] is paged and hit[1] is mask:
            return _cache["vvalue"]
    value = ops.derive_varlen_metadata(paged.gather_slots, mask, paged.pool.block_size)
    with _cache_lock:
        _cache["vkey"] = (paged, mask)
        _cache["vvalue"] = value
    return value


def prefill_frame(q: torch.Tensor, paged, mask: torch.Tensor, layer_idx: int,
                  scale: float) -> torch.Tensor:
    """Read path of a packed frame ``q [1, Q, H, D]`` whose K/V are in the pool."""
    _, nq, h, d = q.shape
    pool = paged.pool
    bt, ctx, q_start = varlen_metadata(paged, mask)
    out = torch.empty((1, nq, h, d), dtype=q.dtype, device=q.device)
    ops.paged_prefill(q.reshape(nq, h, d), pool.k[layer_idx], pool.v[layer_idx], bt, ctx,
                      q_start, scale, pool.block_size, out=out.view(nq, h, d))
    return out


def clear_metadata_cache() -> None:
    with _cache_lock:
        _cache.clear()


def paged_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, paged,
                    mask: torch.Tensor, layer_idx: int, scale: float,
                    n_rep: int) -> torch.Tensor:
    """Write this step's K/V into the paged pool, then decode-attend over history.

    Shapes: ``q [B, 1, H, D]`` (RoPE applied), ``k, v [B, 1, Hkv, D]``,
    ``mask [B, 1, 1, T]`` additive (0 where allowed). ``paged.use_triton``
    True runs the fused write + decode kernel (``ir_paged_decode_write``;
    the write slot of each row must be the slot of its last history
    position, which the engine's decode step guarantees), False runs the
    cache write and the decode as two launches.
    """
    b, sq, h, d = q.shape
    hkv = k.shape[-2]
    if h != hkv * n_rep:
        raise ValueError(f"num_heads {h} != num_kv_heads {hkv} * n_rep {n_rep}")
    pool = paged.pool
    if sq != 1:
        if b != 1:
            raise NotImplementedError(
                "Sq > 1 is served for packed frames (B == 1), the form infrared's paged "
                "engine uses for prefill and mixed steps")
        pool.write(layer_idx, k.reshape(-1, hkv, d), v.reshape(-1, hkv, d),
                   paged.write_slots)
        return prefill_frame(q, paged, mask, layer_idx, scale)
    bt, ctx = block_metadata(paged, mask)
    q3 = q.reshape(b, h, d)
    out = torch.empty((b, 1, h, d), dtype=q.dtype, device=q.device)
    if paged.use_triton:
        ops.paged_decode_write(q3, k.reshape(b, hkv, d), v.reshape(b, hkv, d),
                               pool.k[layer_idx], pool.v[layer_idx], paged.write_slots,
                               bt, ctx, scale, pool.block_size, out=out.view(b, h, d))
    else:
        pool.write(layer_idx, k.reshape(-1, hkv, d), v.reshape(-1, hkv, d),
                   paged.write_slots)
        ops.paged_decode(q3, pool.k[layer_idx], pool.v[layer_idx], bt, ctx, scale,
                         pool.block_size, out=out.view(b, h, d))
    return out
