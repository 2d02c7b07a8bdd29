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
  ``ir_lse_merge``; or (``PeerExchange``) each rank stores its partial
  straight into every rank's exchange buffer over NVLink and merges the
  world's partials as each 16-byte chunk's flag shows it arrived, in one
  kernel.
  Kernels only STORE to peer memory; every read is of the rank's own
  memory.

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


class PeerExchange:
    """Exchange of KV-chunk partials by peer stores (``ir_peer_exchange``)
    instead of an all-gather: each rank allocates one zeroed exchange
    buffer, the buffers are mapped into every process with CUDA IPC (handles
    traded once with ``all_gather_object``), and every call stores this
    rank's ``(o, lse)`` into all peers' buffers over NVLink and merges the
    world's partials as their flags arrive, in one kernel. The buffers hold
    ``batch`` sequences; a call may pass fewer (the same number on every
    rank). All ranks must call :meth:`merge` the same number of times with
    the same shapes; :meth:`close` unmaps and frees (collective)."""

    def __init__(self, batch: int, num_heads: int, head_dim: int, device, group=None):
        import ctypes

        from . import _lib
        from ._lib import check

        self._lib, self._check = _lib.load(), check
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.batch, self.num_heads, self.head_dim = batch, num_heads, head_dim
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device(self.device.type, torch.cuda.current_device())
        rows = batch * num_heads
        nbytes = self._lib.ir_peer_exchange_bytes(self.world, rows, head_dim)
        if nbytes == 0:
            raise ValueError("unsupported world size or shape for the peer exchange")
        self._ptrs = None
        own = ctypes.c_void_p()
        opened = []
        failure = None
        with torch.cuda.device(self.device):  # the buffer lives on the exchange's GPU
            check(self._lib.ir_peer_alloc(nbytes, ctypes.byref(own)))
            ptrs = []
            try:
                handle = (ctypes.c_char * 64)()
                check(self._lib.ir_peer_handle(own, handle))
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
                for r, hd in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(own.value)
                    else:
                        pp = ctypes.c_void_p()
                        check(self._lib.ir_peer_open(ctypes.c_char_p(hd), ctypes.byref(pp)))
                        opened.append(pp.value)
                        ptrs.append(pp.value)
            except Exception as exc:  # noqa: BLE001 - every rank learns of it below
                failure = exc
            # every rank takes part in this vote, so a rank that could not map a
            # peer's buffer makes all ranks give up together instead of waiting
            ok = torch.tensor([0 if failure else 1], dtype=torch.int32, device=self.device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if failure is not None or int(ok.item()) == 0:
                for ptr in opened:
                    self._lib.ir_peer_close(ptr)
                self._lib.ir_peer_free(own)
                raise RuntimeError("peer exchange setup failed on "
                                   + ("this rank: " + repr(failure) if failure else
                                      "another rank")) from failure
        self._own = own.value
        self._nbytes = nbytes
        self._ptrs = ptrs
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def merge(self, o: torch.Tensor, lse: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Push ``o [B, H, D]`` / ``lse [B, H]`` (fp32, contiguous; ``B`` at most
        the exchange's batch) of this rank and write the combined result of
        all ranks into ``out [B, H, D]``."""
        from .ops import _dev_index, _stream, dtype_code, error_flag

        b, h, d = o.shape[0] if o.dim() == 3 else -1, self.num_heads, self.head_dim
        if not 0 <= b <= self.batch:
            raise ValueError(f"o must be [B <= {self.batch}, {h}, {d}], got {tuple(o.shape)}")
        for name, t, shape in (("o", o, (b, h, d)), ("lse", lse, (b, h)), ("out", out, (b, h, d))):
            if tuple(t.shape) != shape:
                raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
            if t.device != self.device:
                raise ValueError(f"{name} is on {t.device}, the exchange on {self.device}")
        if o.dtype != torch.float32 or lse.dtype != torch.float32:
            raise TypeError("o and lse must be float32")
        if not (o.is_contiguous() and lse.is_contiguous()) or out.stride(2) != 1 or \
                out.stride(1) != d:
            raise ValueError("o / lse must be contiguous and out's rows [H, D] dense")
        if self._ptrs is None:
            raise RuntimeError("the exchange has been closed")
        dev = _dev_index(o)
        err = error_flag(dev).data_ptr()
        stream = _stream(dev)
        with torch.cuda.device(dev):   # the launch goes to this device's stream
            self._check(self._lib.ir_peer_exchange(out.data_ptr(), out.stride(0), o.data_ptr(),
                                                   lse.data_ptr(), self._bufs, self._nbytes,
                                                   self.world, self.rank, b, self.num_heads,
                                                   self.head_dim, dtype_code(out.dtype), err,
                                                   stream))
        return out

    def close(self) -> None:
        if self._ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for r, ptr in enumerate(self._ptrs):
                if r != self.rank:
                    self._check(self._lib.ir_peer_close(ptr))
            dist.barrier(group=self.group)
            self._check(self._lib.ir_peer_free(self._own))
        self._ptrs = None


def chunked_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                   tables: torch.Tensor, ctx: torch.Tensor, scale: float, block_size: int,
                   out_dtype: torch.dtype | None = None, group=None,
                   partial_fn=_cuda_partial, merge_fn=_cuda_merge,
                   exchange: PeerExchange | None = None) -> torch.Tensor:
    """Decode attention of ``q [B, H, D]`` over a KV range held on this rank,
    combined across all ranks of ``group``; every rank returns the full
    ``[B, H, D]`` result. Each rank passes its own ``tables``/``ctx``
    (``kv_chunk_tables``) and pool; ``q`` is the same on every rank. With an
    ``exchange`` the partials move by peer stores (:class:`PeerExchange`),
    otherwise by one NCCL all-gather."""
    b, h, d = q.shape
    world = dist.get_world_size(group)
    packed = torch.empty(b * h * (d + 1), dtype=torch.float32, device=q.device)
    o = packed[: b * h * d].view(b, h, d)
    lse = packed[b * h * d:].view(b, h)
    partial_fn(q, k_pool, v_pool, tables, ctx, scale, block_size, o, lse)
    if exchange is not None:
        out = torch.empty((b, h, d), dtype=out_dtype or q.dtype, device=q.device)
        return exchange.merge(o, lse, out)
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
