"""``PagedKVPool`` / ``PagedContext`` with the reference engine's interface.

Same names, fields, shapes and call semantics as infrared's
``infrared/cache/paged_kv_cache.py``: the pool is
``[num_layers, num_blocks * block_size, num_kv_heads, head_dim]`` for K and
for V, a token at physical slot ``s`` is row ``s``, ``write`` scatters a
step's K/V by slot (reference :48-57) and ``gather`` reads histories back
(:59-72). Here both go through the B200 kernels (``ir_cache_write`` /
``ir_cache_gather``); the pool lives on a CUDA device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


class PagedKVPool:
    """Shared flat K/V slot pool on one GPU, addressed by ``block * block_size + offset``."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int,
                 num_kv_heads: int, head_dim: int, dtype: torch.dtype,
                 device: torch.device | str = "cuda") -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("infrared_b200.PagedKVPool lives on a CUDA device (no CPU path)")
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_slots = num_blocks * block_size
        shape = (num_layers, self.num_slots, num_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)

    def write(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor,
              slots: torch.Tensor) -> None:
        """Scatter ``k, v [N, Hkv, D]`` into ``slots [N]`` of layer ``layer_idx``.

        A negative slot skips its row (padding).
        """
        ops.cache_write(k, v, self.k[layer_idx], self.v[layer_idx], slots)

    def gather(self, layer_idx: int, gather_slots: torch.Tensor):
        """``gather_slots [B, T]`` -> ``(k, v)`` each ``[B, T, Hkv, D]``."""
        return (ops.cache_gather(self.k[layer_idx], gather_slots),
                ops.cache_gather(self.v[layer_idx], gather_slots))


@dataclass(slots=True)
class PagedContext:
    """Per-forward paged metadata, as in the reference (paged_kv_cache.py:75-91).

    ``write_slots [N]`` int64 — slots of this step's new K/V; ``gather_slots
    [B, T]`` int64 — each query row's history slots (right-padded);
    ``use_triton`` — the reference's request for its fused kernel; here it
    selects the fused B200 path (write + decode in one launch) when True and
    a separate cache write + decode when False.
    """

    pool: PagedKVPool
    write_slots: torch.Tensor
    gather_slots: torch.Tensor
    use_triton: bool = True
