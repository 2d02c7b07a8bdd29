"""Multi-GPU host logic on CPU ranks (gloo, world size 2 and 3).

The exchange of ``chunked_decode`` (pack, all-gather, unpack, merge) runs
with the oracle as the compute steps and must equal the single-process
oracle; the partition helpers are checked directly.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from infrared_b200 import dist as irdist
from infrared_b200 import workloads as wl
from oracle import paged_attention_np as orc


def test_shard_sequences_balances_tokens():
    ctx = np.random.default_rng(0).integers(100, 4000, size=64)
    for world in (1, 2, 4, 8):
        ranges = irdist.shard_sequences(ctx, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == 64
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert all(hi > lo for lo, hi in ranges)
        tokens = [ctx[lo:hi].sum() for lo, hi in ranges]
        assert max(tokens) - min(tokens) <= 2 * ctx.max()
    few = irdist.shard_sequences([5, 5], 4)   # fewer sequences than ranks
    assert len(few) == 4 and sum(hi - lo for lo, hi in few) == 2


def test_kv_chunk_tables_cover_every_block_once():
    w = wl.custom(2, 5, 8, 2, 64, 16, 1, 500, "float32")
    for world in (2, 3, 8):
        seen = [[] for _ in range(w.batch)]
        total = np.zeros(w.batch, np.int64)
        for r in range(world):
            t, c, first = irdist.kv_chunk_tables(w.block_tables, w.context_lens, 16, world, r)
            total += c
            for i in range(w.batch):
                nb = -(-int(c[i]) // 16)
                seen[i].extend(t[i, :nb].tolist())
                assert first[i] == (r * (-(-int(w.context_lens[i]) // 16))) // world
        np.testing.assert_array_equal(total, w.context_lens)
        for i in range(w.batch):
            nb = -(-int(w.context_lens[i]) // 16)
            assert seen[i] == w.block_tables[i, :nb].tolist()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        w = wl.custom(21, 4, 14, 2, 64, 16, 1, 700, "float32")
        qv, kp, vp, _, _ = wl.numpy_values(w, 3)
        tables, ctx, first = irdist.kv_chunk_tables(w.block_tables, w.context_lens, 16, world,
                                                    rank)

        def partial(qq, kpool, vpool, tbl, cx, scale, bs, o, lse):
            po, pl = orc.partial_attention(qq.numpy(), kpool.numpy()[None], vpool.numpy()[None],
                                           0, tbl.numpy(), cx.numpy(), bs, scale, w.n_rep,
                                           0, 1 << 30)
            o.copy_(torch.from_numpy(po))
            lse.copy_(torch.from_numpy(pl))

        def merge(o_parts, lse_parts, dtype):
            return torch.from_numpy(orc.lse_merge(o_parts.numpy(), lse_parts.numpy()))

        out = irdist.chunked_decode(torch.from_numpy(qv), torch.from_numpy(kp),
                                    torch.from_numpy(vp), torch.from_numpy(tables),
                                    torch.from_numpy(ctx), w.scale, 16,
                                    partial_fn=partial, merge_fn=merge)
        want = orc.decode_from_tables(qv, kp[None], vp[None], 0, w.block_tables, w.context_lens,
                                      16, w.scale, w.n_rep)
        err = float(np.abs(out.numpy() - want).max())
        t = irdist.max_over_ranks(float(rank) + 0.5)
        q.put((rank, err, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_chunked_decode_exchange_on_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, t in results:
        assert err < 1e-5, (rank, err)
        assert t == world - 0.5   # max over ranks
