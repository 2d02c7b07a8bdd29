"""Fixed-shape CUDA-graph decode inputs built on the device.

Same signature, outputs and errors as infrared's ``build_decode_static_inputs``
(infrared/engine/cuda_graph.py:105-155): row i of a batch bucket holds
sequence i (rows past the batch repeat row 0); the new token sits at position
``num_cached`` and goes to ``slot(block_table, num_cached)``; ``gather_slots``
lists the slots of positions ``[0, num_cached]`` zero-padded to ``t_max``; the
additive mask blocks columns past the context with ``finfo(dtype).min``.
infrared fills ``gather_slots`` one element at a time from Python (≈262 k
scalar tensor writes for a bucket of 128 over t_max 2048); here the host only
packs the block tables into one int32 array and ``ir_build_decode_inputs``
writes every output in one launch.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .ops import _dev_index, _stream, dtype_code
from ._lib import check


@dataclass(slots=True)
class DecodeInputs:
    """``ids [B,1]``, ``positions [B,1]``, ``write_slots [B]``, ``gather_slots [B,t_max]``,
    ``mask [B,1,1,t_max]`` — the fields of infrared's DecodeInputs (cuda_graph.py:84-102)."""

    ids: torch.Tensor
    positions: torch.Tensor
    write_slots: torch.Tensor
    gather_slots: torch.Tensor
    mask: torch.Tensor


def build_decode_static_inputs(block_tables: list[list[int]], num_cached: list[int],
                               last_tokens: list[int], bucket_b: int, t_max: int,
                               block_size: int, device, dtype: torch.dtype,
                               decode_inputs_cls=DecodeInputs):
    """Device-built equivalent of infrared's ``build_decode_static_inputs``."""
    b = len(last_tokens)
    if not 0 < b <= bucket_b:
        raise ValueError(f"need 0 < b ({b}) <= bucket_b ({bucket_b})")
    for i in range(bucket_b):
        ctx = num_cached[i if i < b else 0] + 1
        if ctx > t_max:
            raise ValueError(f"context_len {ctx} exceeds t_max {t_max}")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("infrared_b200 builds graph inputs on a CUDA device")
    width = -(-t_max // block_size)
    tables = np.zeros((b, width), np.int32)
    for i in range(b):
        need = min(len(block_tables[i]), width)
        tables[i, :need] = block_tables[i][:need]
    host = torch.from_numpy(tables)
    bt = host.to(device, non_blocking=False)
    nc = torch.tensor(num_cached[:b], dtype=torch.int32).to(device)
    last = torch.tensor(last_tokens[:b], dtype=torch.int64).to(device)
    ids = torch.empty((bucket_b, 1), dtype=torch.long, device=device)
    positions = torch.empty((bucket_b, 1), dtype=torch.long, device=device)
    write_slots = torch.empty((bucket_b,), dtype=torch.long, device=device)
    gather_slots = torch.empty((bucket_b, t_max), dtype=torch.long, device=device)
    mask = torch.empty((bucket_b, 1, 1, t_max), dtype=dtype, device=device)
    dev = _dev_index(ids)
    with torch.cuda.device(dev):   # the launch goes to this device's stream
        check(_lib.load().ir_build_decode_inputs(
            bt.data_ptr(), width, nc.data_ptr(), last.data_ptr(), b, bucket_b, t_max,
            block_size, ids.data_ptr(), positions.data_ptr(), write_slots.data_ptr(),
            gather_slots.data_ptr(), mask.data_ptr(), dtype_code(dtype), _stream(dev)))
    return decode_inputs_cls(ids, positions, write_slots, gather_slots, mask)
