"""Shared helpers of the GPU parity tests (device tensors + oracle references)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import paged_attention_np as orc

DEV = "cuda"


def dev_meta(w):
    bt = torch.from_numpy(w.block_tables).to(DEV)
    ctx = torch.from_numpy(w.context_lens).to(DEV)
    sm = torch.from_numpy(w.slot_mapping).to(DEV)
    return bt, ctx, sm


def dev_values(vals, dtype):
    return [torch.from_numpy(x).to(DEV).to(dtype) for x in vals]


def host_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def oracle_decode(w, q, kp, vp, kn=None, vn=None):
    """fp32 oracle of decode (after writing kn/vn at the tail slots if given) for
    host arrays that are already rounded to the kernel's input dtype."""
    kp2, vp2 = kp[None].copy(), vp[None].copy()
    if kn is not None:
        orc.pool_write(kp2, vp2, 0, kn, vn, w.slot_mapping)
    return orc.decode_from_tables(q, kp2, vp2, 0, w.block_tables, w.context_lens,
                                  w.block_size, w.scale, w.n_rep)


def oracle_decode_device(w, q, kp, vp, rows=None):
    """fp32 oracle for large device-resident inputs: gathers each sequence's
    history on the device with torch indexing, one sequence at a time."""
    out = np.zeros((w.batch, w.num_heads, w.head_dim), np.float32)
    rows = range(w.batch) if rows is None else rows
    for i in rows:
        c = int(w.context_lens[i])
        if c == 0:
            continue
        pos = np.arange(c)
        slots = (w.block_tables[i, pos // w.block_size].astype(np.int64) * w.block_size
                 + pos % w.block_size)
        st = torch.from_numpy(slots).to(kp.device)
        kh = orc.repeat_kv(host_f32(kp[st])[None], w.n_rep)
        vh = orc.repeat_kv(host_f32(vp[st])[None], w.n_rep)
        qi = host_f32(q[i])[None, None]
        out[i] = orc.masked_attention(qi, kh, vh, np.zeros((1, 1, 1, c), np.float32),
                                      w.scale)[0, 0]
    return out


def assert_close_bf16(got: np.ndarray, want: np.ndarray, tol: float = 2e-2):
    """The bf16 bar: atol = rtol = 2e-2 against the fp32 reference."""
    np.testing.assert_allclose(got, want, atol=tol, rtol=tol)
