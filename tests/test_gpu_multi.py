"""KV-chunk decode over 2-8 GPUs (as many as the box has): the peer-store
exchange against the NCCL all-gather path and the single-GPU decode (needs
2 GPUs; skipped otherwise).

Each rank is a spawned process on its own GPU. Bars: the peer exchange equals
the NCCL path within fp32 merge rounding (1e-3) and the single-GPU decode
within the bf16 bar (2e-2); repeated calls (the exchange's epoch counters
advancing) and CUDA-graph replays give the same result every time. A wide
batch (256 sequences x 28 heads = 7168 rows, many rows per exchange warp)
checks the exchange's bounded grid: no timeout, and the same bits as the
NCCL path, whose merge kernel does the same arithmetic in the same order.
"""

import datetime
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    import infrared_b200 as irb
    from infrared_b200 import dist as irdist
    from infrared_b200 import ops
    from infrared_b200 import workloads as wl

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=world,
                            rank=rank, device_id=dev, timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        w = wl.c4(seed=0, batch=3, ctx_len=4608)
        q, kp, vp, _, _ = wl.torch_values(w, 7, dev)
        tables_np, ctx_np, _ = irdist.kv_chunk_tables(w.block_tables, w.context_lens,
                                                      w.block_size, world, rank)
        tables = torch.from_numpy(tables_np).to(dev)
        ctx = torch.from_numpy(ctx_np).to(dev)
        full = irb.paged_decode(q, kp, vp, torch.from_numpy(w.block_tables).to(dev),
                                torch.from_numpy(w.context_lens).to(dev), w.scale, w.block_size)
        ref = irdist.chunked_decode(q, kp, vp, tables, ctx, w.scale, w.block_size)
        ex = irdist.PeerExchange(w.batch, w.num_heads, w.head_dim, dev)
        outs = [irdist.chunked_decode(q, kp, vp, tables, ctx, w.scale, w.block_size,
                                      exchange=ex) for _ in range(6)]
        torch.cuda.synchronize()
        res["p2p_vs_nccl"] = (outs[0].float() - ref.float()).abs().max().item()
        res["p2p_vs_full"] = (outs[0].float() - full.float()).abs().max().item()
        res["repeat_equal"] = all(torch.equal(outs[0], o) for o in outs[1:])
        # captured in a CUDA graph and replayed: epochs advance on the device
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                cap = irdist.chunked_decode(q, kp, vp, tables, ctx, w.scale, w.block_size,
                                            exchange=ex)
        torch.cuda.current_stream(dev).wait_stream(s)
        eq = True
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            eq = eq and torch.equal(cap, outs[0])
        res["graph_equal"] = eq
        del g
        ops.check_device_errors()
        ex.close()
        # a wide batch: far more rows than one wave of exchange CTAs
        w2 = wl.c4(seed=1, batch=256, ctx_len=1104)
        q2, kp2, vp2, _, _ = wl.torch_values(w2, 9, dev)
        t2_np, c2_np, _ = irdist.kv_chunk_tables(w2.block_tables, w2.context_lens,
                                                 w2.block_size, world, rank)
        t2 = torch.from_numpy(t2_np).to(dev)
        c2 = torch.from_numpy(c2_np).to(dev)
        ref2 = irdist.chunked_decode(q2, kp2, vp2, t2, c2, w2.scale, w2.block_size)
        ex2 = irdist.PeerExchange(w2.batch, w2.num_heads, w2.head_dim, dev)
        got2 = [irdist.chunked_decode(q2, kp2, vp2, t2, c2, w2.scale, w2.block_size,
                                      exchange=ex2) for _ in range(3)]
        torch.cuda.synchronize()
        res["wide_max_diff"] = max((g2.float() - ref2.float()).abs().max().item()
                                   for g2 in got2)
        res["wide_equal"] = all(torch.equal(g2, ref2) for g2 in got2)
        ops.check_device_errors()
        ex2.close()
        res["errors"] = 0
    except Exception as e:  # noqa: BLE001 - reported to the parent test
        res["exception"] = repr(e)
    finally:
        dist.destroy_process_group()
    results.put((rank, res))


def test_peer_exchange_gpus():
    world = min(torch.cuda.device_count(), 8)
    ctx = torch.multiprocessing.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, res = results.get(timeout=300)
        got[rank] = res
    for p in procs:
        p.join(timeout=60)
    for rank, res in sorted(got.items()):
        assert "exception" not in res, f"rank {rank}: {res}"
        assert res["p2p_vs_nccl"] < 1e-3, res
        assert res["p2p_vs_full"] < 2e-2, res
        assert res["repeat_equal"] and res["graph_equal"], res
        assert res["wide_equal"], res


def test_kernels_follow_the_tensors_device():
    """A call whose tensors live on another GPU than the calling thread's
    current device (infrared's engine loop runs in a worker thread whose
    current device is 0) runs on the tensors' GPU and gives the same result."""
    import infrared_b200 as irb
    from infrared_b200 import ops
    from infrared_b200 import workloads as wl

    dev = torch.device("cuda", 1)
    w = wl.custom(3, 5, 28, 4, 128, 16, 100, 900, "bfloat16")
    q, kp, vp, kn, vn = wl.torch_values(w, 3, dev)
    bt = torch.from_numpy(w.block_tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    sm = torch.from_numpy(w.slot_mapping).to(dev)
    with torch.cuda.device(1):
        want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
        torch.cuda.synchronize()
    with torch.cuda.device(0):
        got = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
        ops.cache_write(kn, vn, kp, vp, sm)
        torch.cuda.synchronize(dev)
    assert torch.equal(got, want)
    assert torch.equal(kp[sm], kn) and torch.equal(vp[sm], vn)
    ops.check_device_errors(1)
