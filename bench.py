#!/usr/bin/env python
"""Paged-decode attention throughput on B200 — one JSON line per run.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c4|c5|p1]

A step is one decode-attention call (one layer) over one batch of the
workload: ``c2`` (default) is the Qwen2.5-7B geometry batch of 64 sequences
with contexts U[512, 4096]; ``c3`` adds the fused K/V cache write over 256
sequences with shared prefixes; ``c4`` is 4 x 32k contexts; ``c5`` is a
whole greedy decode step of a random-init Qwen2.5-7B (tok/s); ``p1`` is a
causal prefill of 8 x 4096-token prompts (TFLOP/s, tcgen05). At N GPUs (one
process per GPU, launched by torchrun) every rank decodes its own batch of
the workload — the sequences are sharded, there is no collective on the data
path — so the scaling is weak and ``value`` is the bytes all ranks moved
divided by the slowest rank's time.

* ``value``: HBM GB/s of useful bytes (K/V of every cached token of every
  sequence, q, out, block tables) with inputs resident on the device; the K
  steps are captured in one CUDA graph and timed with CUDA events; inputs
  rotate over 3 pool sets and each step touches > L2 (126 MB) of K/V.
* ``e2e``: the same metric through the public Python API
  (``infrared_b200.paged_decode``) with host buffers: every step copies q,
  block tables and context lengths from pinned host memory and reads the
  output back (inputs packed in one pinned buffer; double-buffered: the next
  step's copy in and the previous step's copy out overlap this step's kernel
  on two copy streams; kernels run in order).
* ``roofline``: the decode call's bytes / its measured duration against the
  measured HBM copy bandwidth in MEASURED_PEAKS.json.
* ``prefill_p1`` (default config): P1 (8 causal 4096-token prompts) on the
  tcgen05 prefill kernel, TFLOP/s against the measured bf16 peak, per GPU.
* ``c5_engine`` (default config): config C5 decoded through infrared's own
  ``PagedBatchEngine`` (CUDA graphs, the shim installed), the 128 requests
  sharded over the job's GPUs; tok/s from the engine's own loop.
* ``kv_chunk`` (default config, every N): config C4 (4 x 32k contexts)
  with each sequence's KV split across the same N GPUs, partials exchanged
  by peer stores over NVLink in one kernel (``p2p``) and by an NCCL
  all-gather + merge (``nccl``); strong scaling of one fixed batch.
* ``cpu_baseline`` / ``--impl reference``: infrared's own naive CPU path,
  ``paged_attention(..., PagedContext(use_triton=False))``
  (infrared/model/triton_attention.py:81-129), over the whole batch of the
  workload per call, on all host cores (infrared from the git-ignored
  ``baseline/_ref`` install); where that install is absent, the numpy
  restatement in oracle/ on one sequence per call (``kind: "port"``).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-decode attn HBM GB/s (% of ~8 TB/s) + decode tok/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=["c2", "c3", "c4", "c5", "p1", "kernels"],
                   default="c2")
    p.add_argument("--sets", type=int, default=3)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--only", default="",
                   help="--config kernels: run one case (cache_write_c3, cache_write_bulk, "
                        "lse_merge_c4, lse_merge_b256, kv_proj_c5, kv_proj_c5_torch, "
                        "peer_exchange_world1_b256)")
    p.add_argument("--inline-merge", action="store_true",
                   help="merge rows of <= 4 pieces in the decode kernel (zeroed workspace)")
    p.add_argument("--dynamic-tail", action="store_true",
                   help="decode with static shares + dynamic tail units")
    p.add_argument("--engine", action="store_true",
                   help="c5 through infrared's own PagedBatchEngine (CUDA graphs, shim)")
    p.add_argument("--no-prefill", action="store_true",
                   help="leave out the P1 prefill leg of the default config")
    p.add_argument("--no-engine", action="store_true",
                   help="leave out the C5 leg through infrared's engine (default config)")
    p.add_argument("--no-kv-chunk", action="store_true",
                   help="leave out the C4 KV-chunk leg of the default config")
    p.add_argument("--soak", type=float, default=1.5,
                   help="seconds of untimed replays before timing (clock sampling)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                   help="c4 over several GPUs: partials by peer stores or an NCCL all-gather")
    p.add_argument("--batch", type=int, default=0,
                   help="override the workload's per-GPU batch (c2/c3/c4)")
    p.add_argument("--prefill-path", type=int, default=0, choices=[0, 1, 2, 3],
                   help="p1: prefill kernel override (ir_set_prefill_path): 0 auto, 1 rows "
                        "as decode rows, 2 tcgen05, 3 tcgen05 CTA pairs")
    p.add_argument("--decode-path", type=int, default=0,
                   help="kernel override (ir_set_decode_path): 0 auto, 1 CUDA-core, "
                        "2 TMA, 3 TMA with one copy per head and half")
    return p.parse_args()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ CPU side


def cpu_sample_workload(w, seqs, seed=0):
    """Compact host copy of a few sequences of ``w`` (their blocks renumbered)."""
    from infrared_b200 import workloads as wl

    rng = np.random.default_rng(seed)
    bs = w.block_size
    ctx = w.context_lens[seqs].astype(np.int32)
    nblk = (ctx.astype(np.int64) + bs - 1) // bs
    bt = np.zeros((len(seqs), int(nblk.max())), np.int32)
    perm = rng.permutation(int(nblk.sum()))
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    sub = wl.Workload(w.name + "-sample", len(seqs), w.num_heads, w.num_kv_heads, w.head_dim,
                      bs, int(nblk.sum()), "float32", w.scale, w.std, ctx, bt,
                      wl.tail_slots(bt, ctx, bs))
    q, kp, vp, _, _ = wl.numpy_values(sub, seed)
    return sub, q, kp[None], vp[None]


def infrared_importable() -> bool:
    """infrared (the reference) from the repository's git-ignored install."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "infrared" / "__init__.py").exists():
        return False
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    try:
        import infrared.model.triton_attention  # noqa: F401
    except Exception:  # noqa: BLE001
        return False
    return True


def time_infrared_decode(w, steps, warmup, budget_s, with_write=False):
    """infrared's own naive paged decode (pool write, gather, repeat_kv, masked
    attention; infrared/model/triton_attention.py:81-129) over the whole batch
    of ``w`` per call, on every host core; stops after ``steps`` calls or
    ``budget_s`` seconds of timed calls (at least one). Returns (GB/s of the
    workload's useful bytes, seconds, calls, threads)."""
    import torch
    from infrared.cache.paged_kv_cache import PagedContext, PagedKVPool
    from infrared.model.triton_attention import paged_attention

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    dt = getattr(torch, w.dtype)
    g = torch.Generator().manual_seed(0)

    def randn(*shape):
        return (torch.randn(*shape, generator=g) * w.std).to(dt)

    pool = PagedKVPool(num_layers=1, num_blocks=w.num_blocks, block_size=w.block_size,
                       num_kv_heads=w.num_kv_heads, head_dim=w.head_dim, dtype=dt)
    pool.k[0].copy_(randn(w.num_slots, w.num_kv_heads, w.head_dim))
    pool.v[0].copy_(randn(w.num_slots, w.num_kv_heads, w.head_dim))
    q = randn(w.batch, 1, w.num_heads, w.head_dim)
    k_new = randn(w.batch, 1, w.num_kv_heads, w.head_dim)
    v_new = randn(w.batch, 1, w.num_kv_heads, w.head_dim)
    # the engine's decode inputs (infrared/engine/paged_engine.py:300-314, 630-638)
    ctx = torch.from_numpy(w.context_lens.astype(np.int64))
    t = int(ctx.max())
    pos = torch.arange(t)
    bt = torch.from_numpy(w.block_tables.astype(np.int64))
    gather = bt[:, pos // w.block_size] * w.block_size + pos % w.block_size
    valid = pos[None, :] < ctx[:, None]
    gather = torch.where(valid, gather, torch.zeros_like(gather))
    mask = torch.zeros(w.batch, 1, 1, t, dtype=dt)
    mask = mask.masked_fill(~valid[:, None, None, :], torch.finfo(dt).min)
    paged = PagedContext(pool, torch.from_numpy(w.slot_mapping.astype(np.int64)), gather,
                         use_triton=False)

    def call():
        paged_attention(q, k_new, v_new, paged, mask, 0, w.scale, w.n_rep)

    for _ in range(max(0, warmup)):
        call()
    n, t0 = 0, time.perf_counter()
    while n < max(steps, 1):
        call()
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    secs = time.perf_counter() - t0
    nbytes = w.algorithmic_bytes(with_write=with_write)
    return nbytes * n / secs / 1e9, secs, n, torch.get_num_threads()


def cpu_baseline_leg(w, config, steps, warmup, budget_s):
    """``cpu_baseline`` object: infrared's own path where it is installed,
    else the numpy restatement on one sequence per call."""
    if infrared_importable():
        gbs, secs, n, threads = time_infrared_decode(w, steps, warmup, budget_s,
                                                     with_write=config == "c3")
        return {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                "kind": "reference",
                "sample": f"infrared's paged_attention(use_triton=False) (pool write, gather, "
                          f"repeat_kv, masked attention; torch CPU, {w.dtype}) over the full "
                          f"{config} batch of {w.batch} sequences per call: {n} call(s), "
                          f"{secs:.1f} s, torch threads {threads}",
                "host_cpus": os.cpu_count(), "same_config": True}
    gbs, secs, n = time_cpu_oracle(w, steps=10 ** 6, warmup=1, budget_s=budget_s)
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"oracle naive path (gather+repeat_kv+softmax, numpy fp32) on {n} "
                      f"single-sequence samples of {config} ({secs:.1f} s), bytes counted at "
                      f"the workload's bf16 size (infrared not installed)",
            "host_cpus": os.cpu_count(), "same_config": False}


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:  # noqa: BLE001
        return 1


def time_cpu_oracle(w, steps, warmup, budget_s=None):
    """Time the oracle's naive path over one sequence per step (rotating)."""
    from oracle import paged_attention_np as orc

    order = list(range(w.batch))
    samples = [cpu_sample_workload(w, [i], seed=i) for i in order[:8]]
    times, nbytes = [], []
    t_start = time.perf_counter()
    for it in range(warmup + steps):
        sub, q, kp, vp = samples[it % len(samples)]
        t0 = time.perf_counter()
        orc.decode_from_tables(q, kp, vp, 0, sub.block_tables, sub.context_lens,
                               sub.block_size, sub.scale, sub.n_rep)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
            nbytes.append(sub.algorithmic_bytes() * w.elem_bytes // 4)
        if budget_s is not None and it >= warmup and time.perf_counter() - t_start > budget_s:
            break
    total_t = sum(times)
    gbs = sum(nbytes) / total_t / 1e9
    return gbs, total_t, len(times)


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        import torch

        self.proc = None
        try:
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", bus, "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------ GPU side


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_workload(name, rank, batch=0):
    from infrared_b200 import workloads as wl

    if batch:
        return wl.CONFIGS[name](seed=rank, batch=batch)
    return wl.CONFIGS[name](seed=rank)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import infrared_b200 as irb
    from infrared_b200 import ops
    from infrared_b200 import workloads as wl

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
    ops.set_decode_path(args.decode_path)
    # every rank decodes a batch of the same shape (workload seed 0: the same
    # context lengths and bytes), its own values (seeded by rank)
    w = make_workload(args.config, 0, args.batch)
    fused = args.config == "c3"
    bt = torch.from_numpy(w.block_tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    sm = torch.from_numpy(w.slot_mapping).to(dev)
    sets = [wl.torch_values(w, 1000 * rank + s, dev) for s in range(args.sets)]
    out = torch.empty_like(sets[0][0])
    dynamic = args.dynamic_tail
    inline = args.inline_merge
    _, _, ws_bytes = ops.decode_plan(sets[0][0], sets[0][1], bt, w.block_size, w.scale,
                                     dynamic=dynamic, inline_merge=inline)
    # a zeroed, marked workspace: short rows merged in the decode kernel and,
    # if asked for, the tail handed out dynamically
    ws = ops.decode_workspace(ws_bytes, dev, dynamic=dynamic, inline_merge=inline)
    nbytes = w.algorithmic_bytes(with_write=fused)

    def step(i):
        q, kp, vp, kn, vn = sets[i % len(sets)]
        if fused:
            irb.paged_decode_write(q, kn, vn, kp, vp, sm, bt, ctx, w.scale, w.block_size,
                                   out=out, ws=ws)
        else:
            irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, out=out, ws=ws)

    def measure_e2e():
        """Public API with pinned host buffers; every step copies its inputs in
        and its result out. The step's inputs sit in one pinned buffer (one
        copy in); double-buffered: step i+1's inputs copy in on one copy stream
        and step i's result copies out on another while kernels run in order."""
        parts = [sets[0][0], bt, ctx] + ([sets[0][3], sets[0][4], sm] if fused else [])
        offs, total = [], 0
        for t in parts:
            offs.append(total)
            total += -(-t.numel() * t.element_size() // 256) * 256
        host_in = torch.empty(total, dtype=torch.uint8).pin_memory()
        for t, o in zip(parts, offs):
            nb = t.numel() * t.element_size()
            host_in[o:o + nb].copy_(t.cpu().reshape(-1).view(torch.uint8))

        def views(buf):
            return [buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                    for t, o in zip(parts, offs)]

        _, kp0, vp0, _, _ = sets[0]
        bufs = []
        for _ in range(2):
            din = torch.empty(total, dtype=torch.uint8, device=dev)
            bufs.append({"din": din, "in": views(din), "out": torch.empty_like(out),
                         "host_out": torch.empty(out.shape, dtype=out.dtype).pin_memory(),
                         "in_ready": torch.cuda.Event(), "done": torch.cuda.Event()})
        compute = torch.cuda.current_stream(dev)
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_step(i):
            bf = bufs[i % 2]
            h2d_s.wait_event(bf["done"])          # step i-2 finished with this buffer
            with torch.cuda.stream(h2d_s):
                bf["din"].copy_(host_in, non_blocking=True)
                bf["in_ready"].record(h2d_s)
            compute.wait_event(bf["in_ready"])
            x = bf["in"]
            if fused:
                irb.paged_decode_write(x[0], x[3], x[4], kp0, vp0, x[5], x[1], x[2], w.scale,
                                       w.block_size, out=bf["out"], ws=ws)
            else:
                irb.paged_decode(x[0], kp0, vp0, x[1], x[2], w.scale, w.block_size,
                                 out=bf["out"], ws=ws)
            bf["done"].record(compute)
            d2h_s.wait_event(bf["done"])
            with torch.cuda.stream(d2h_s):
                bf["host_out"].copy_(bf["out"], non_blocking=True)

        for i in range(max(args.warmup, 3)):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        ev[0].record(compute)
        h2d_s.wait_event(ev[0])
        for i in range(args.steps):
            e2e_step(i)
        compute.wait_stream(d2h_s)
        ev[1].record(compute)
        ev[1].synchronize()
        e2e_ms = ev[0].elapsed_time(ev[1])
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        h2d = sum(t.numel() * t.element_size() for t in parts)
        d2h = out.numel() * out.element_size()
        return e2e_ms, h2d, d2h

    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize(dev)
        ops.check_device_errors(dev)
        # K steps in one graph: the timed region is a single replay
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                step(i)
        # per-call duration of the decode path (eager, events on the stream)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        clocks = ClockSampler(local)
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < args.soak:   # clocks settle under load
            graph.replay()
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
        clk = clocks.stop()
        ms = ev[0].elapsed_time(ev[1])
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        ops.check_device_errors(dev)

        e2e_ms = h2d = d2h = None
        if not args.no_e2e:
            e2e_ms, h2d, d2h = measure_e2e()

    path, ctas, _ = ops.decode_plan(sets[0][0], sets[0][1], bt, w.block_size, w.scale)
    peak, peak_kind = measured_peaks()
    per_step_ms = ms / args.steps
    job_bytes = nbytes
    if world > 1:   # the bytes every rank moved, summed
        t = torch.tensor([nbytes], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        job_bytes = int(t.item())
    value = job_bytes * args.steps / (ms / 1e3) / 1e9
    per_gpu = nbytes / (per_step_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)*0.5 q/K/V, uniform context lengths, random block "
                "tables (no dataset: the reference benchmarks none)",
        "config": {
            "workload": {"c2": "C2: Qwen2.5-7B attention (28 q / 4 kv heads, head_dim 128), "
                               "B=64/GPU, ctx U[512,4096], block 16, 32768-block pool",
                         "c3": "C3: fused K/V write + decode, B=256/GPU, ctx U[128,2048], "
                               "~30% shared prefixes",
                         "c4": "C4: B=4 x ctx 32768 per GPU"}[args.config],
            "global_batch": w.batch * world,
            "batch_per_gpu": w.batch,
            "tokens_per_gpu": int(w.context_lens.sum()),
            "bytes_per_step_per_gpu": nbytes,
            "bytes_per_step_job": job_bytes,
            "shards": "every rank: the same context lengths (equal bytes), its own values",
            "parallelism": f"sequence-sharded x{world}, no collective",
            "l2": "inputs larger than L2: >=200 MB of K/V per step, 3 rotating pool sets",
            "timing": "K steps in one CUDA graph, CUDA events, max over ranks",
            "kernel_path": {1: "cuda-core", 2: "tma+mma.sync"}[path] +
                           (" (copy per head)" if args.decode_path == 3 else ""),
            "schedule": ("static shares + dynamic tail units" if dynamic and path == 2
                         else "static shares") +
                        (", rows of <= 4 pieces merged in the decode kernel"
                         if inline and path == 2 else ", split rows merged by the merge kernel"),
            "ctas_per_kv_head": ctas,
        },
        "decode_tok_s_per_layer": round(world * w.batch / (per_step_ms / 1e3), 1),
        "hbm_frac_per_gpu": round(per_gpu / peak, 4),
        "roofline": {
            "bound": "hbm",
            "achieved": round(per_gpu, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(per_gpu / peak, 4),
            "peak_kind": peak_kind,
            "traffic": traffic_from_profiles(args.config),
            "scope": "one decode call (decode kernel + merge kernel), per GPU",
        },
        "e2e": None if e2e_ms is None else {
            "value": round(job_bytes * args.steps / (e2e_ms / 1e3) / 1e9, 1),
            "unit": "GB/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": round(e2e_ms / args.steps, 5),
        },
        "clocks": clk,
        "gpu_launches": 2 * args.steps,
    }
    del graph
    if args.config == "c2" and not args.no_kv_chunk:
        line["kv_chunk"] = kv_chunk_leg(args, dev, world, rank)
    if args.config == "c2" and not args.no_prefill:
        line["prefill_p1"] = p1_summary(dev, world, rank)
    if args.config == "c2" and not args.no_engine:
        line["c5_engine"] = c5_engine_summary(dev, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_leg(w, args.config, 10 ** 6, 1, args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def traffic_from_profiles(config):
    """DRAM bytes per decode call from the committed ncu summary, if present."""
    f = ROOT / "profiles" / f"decode_{config}_traffic.json"
    if f.exists():
        try:
            return json.loads(f.read_text()).get("dram_bytes_per_call")
        except Exception:  # noqa: BLE001
            return None
    return None


def run_reference(args):
    world, rank, _ = dist_info()
    if rank != 0:
        return
    if args.config == "c5":
        print(json.dumps({"impl": "reference", "unavailable": "c5 is a whole Qwen2.5-7B decode "
                          "step; the reference's CPU path restated here is the attention path "
                          "(configs c2/c3/c4)"}), flush=True)
        return
    if args.config == "p1":
        run_reference_prefill(args)
        return
    if args.config == "kernels":
        print(json.dumps({"impl": "reference", "unavailable": "the standalone-kernel leg has "
                          "no reference counterpart (infrared has no kernels of its own)"}),
              flush=True)
        return
    w = make_workload(args.config, 0, args.batch)
    if infrared_importable():
        # each step: one call of infrared's own naive path over the whole batch;
        # warm-up capped at one call and the timed calls at about a minute so
        # the run ends within minutes whatever --steps says
        gbs, secs, n, threads = time_infrared_decode(w, args.steps, min(args.warmup, 1), 60.0,
                                                     with_write=args.config == "c3")
        kind = "reference"
        sample = (f"infrared's paged_attention(use_triton=False) (pool write, gather, "
                  f"repeat_kv, masked attention; torch CPU, {w.dtype}) over the full "
                  f"{args.config} batch of {w.batch} sequences per step; {n} step(s) timed")
        workload = f"{args.config} at full size (the GPU arm's config), infrared's own code"
        dtype = {"bfloat16": "bf16", "float16": "f16"}.get(w.dtype, "f32")
        same = True
    else:
        gbs, secs, n = time_cpu_oracle(w, steps=args.steps, warmup=args.warmup)
        threads, kind, dtype, same = 1, "port", "f32", False
        sample = ("reference naive CPU path restated in oracle/ (numpy): one sequence of "
                  "the workload per step (infrared not installed)")
        workload = f"{args.config} geometry, one sequence per step (bounded sample)"
    per_step = secs / max(n, 1)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": n,
        "warmup": min(args.warmup, 1) if kind == "reference" else args.warmup,
        "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic (same generator and geometry as the GPU arm)",
        "config": {"workload": workload, "global_batch": w.batch, "same_config": same},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                         "kind": kind, "sample": sample, "host_cpus": os.cpu_count()},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_prefill(args):
    """The reference's naive CPU path for a prefill (gather, repeat_kv, causal
    masked attention; restated in oracle/) on one 512-token prompt of the P1
    geometry per step, timed on the host cores."""
    import torch

    from infrared_b200 import workloads as wl
    from oracle import paged_attention_np as orc

    w = wl.prefill_frame("p1-sample", 0, [0], [512])
    rng = np.random.default_rng(0)
    slots = w.num_blocks * w.block_size
    kp = (rng.standard_normal((1, slots, w.num_kv_heads, w.head_dim), np.float32) * 0.5)
    vp = (rng.standard_normal((1, slots, w.num_kv_heads, w.head_dim), np.float32) * 0.5)
    q = rng.standard_normal((w.total_q, w.num_heads, w.head_dim), np.float32) * 0.5
    torch.set_num_threads(cpu_threads())

    def one():
        orc.prefill_from_tables(q, kp, vp, 0, w.block_tables, w.context_lens, w.q_start,
                                w.block_size, w.scale, w.num_heads // w.num_kv_heads)

    for _ in range(max(1, min(args.warmup, 2))):
        one()
    n, t0 = 0, time.perf_counter()
    while n < max(args.steps, 1) and time.perf_counter() - t0 < 20.0:
        one()
        n += 1
    secs = time.perf_counter() - t0
    tflops = w.flops() * n / secs / 1e12
    line = {
        "impl": "reference", "metric": "paged prefill attention TFLOP/s (causal, useful FLOPs)",
        "value": round(tflops, 5), "unit": "TFLOP/s", "n_gpus": 1, "steps": n,
        "warmup": args.warmup, "ms_per_step": round(secs / n * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (P1 geometry)",
        "config": {"workload": "P1 geometry, one 512-token prompt per step (bounded sample)"},
        "cpu_baseline": {"value": round(tflops, 5), "unit": "TFLOP/s", "cores": cpu_threads(),
                         "kind": "port",
                         "sample": "reference naive CPU prefill restated in oracle/ (numpy): "
                                   "one 512-token prompt, 28 heads, per step"},
        "e2e": {"value": round(tflops, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _graph_ms(step, steps, dev, world, soak_s=0.3):
    """Per-replay time (ms) of ``steps`` calls of ``step`` captured in one CUDA
    graph, max over ranks; every rank replays the same number of times."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist

    for i in range(3):
        step(i)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with torch.cuda.stream(stream):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                step(i)
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
        est = ev[0].elapsed_time(ev[1])
        if world > 1:
            est = irdist.max_over_ranks(est, device=dev)
        for _ in range(int(min(500, soak_s * 1e3 / max(est, 1e-3)))):
            graph.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
    ms = ev[0].elapsed_time(ev[1])
    if world > 1:
        ms = irdist.max_over_ranks(ms, device=dev)
    del graph
    return ms


def kv_chunk_leg(args, dev, world, rank, steps=100):
    """C4 (4 sequences x 32768 tokens) with every sequence's KV split across
    the job's N GPUs: per step each rank decodes its chunk (partial out +
    log-sum-exp), the partials cross NVLink and every rank merges them; at
    N = 1 the plain decode of the whole KV. Strong scaling of one fixed batch;
    GB/s = the batch's useful bytes / step time (max over ranks)."""
    import torch

    import infrared_b200 as irb
    from infrared_b200 import dist as irdist
    from infrared_b200 import workloads as wl

    w = wl.c4(seed=0)
    total = w.algorithmic_bytes()
    res = {"workload": "C4: B=4 x ctx 32768 (Qwen2.5-7B attention), each sequence's KV "
                       "split over the N GPUs", "n_gpus": world, "scaling": "strong",
           "bytes_per_step_total": total, "steps": steps,
           "timing": "K steps in one CUDA graph, CUDA events, max over ranks"}
    if world == 1:
        bt = torch.from_numpy(w.block_tables).to(dev)
        ctx = torch.from_numpy(w.context_lens).to(dev)
        sets = [wl.torch_values(w, 7 + s, dev) for s in range(3)]
        out = torch.empty_like(sets[0][0])

        def one(i):
            q, kp, vp, _, _ = sets[i % 3]
            irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size, out=out)

        ms = _graph_ms(one, steps, dev, world) / steps
        res["single_gpu"] = {"ms_per_step": round(ms, 5),
                             "value": round(total / (ms / 1e3) / 1e9, 1), "unit": "GB/s"}
        del sets
        return res
    tables_np, ctx_np, _ = irdist.kv_chunk_tables(w.block_tables, w.context_lens,
                                                  w.block_size, world, rank)
    tables = torch.from_numpy(tables_np).to(dev)
    ctx = torch.from_numpy(ctx_np).to(dev)
    local_bytes = int(ctx_np.astype(np.int64).sum()) * 2 * w.num_kv_heads * w.head_dim * 2
    nsets = max(3, -(-3 * 126 * 2 ** 20 // max(local_bytes, 1)))
    sets = [wl.torch_values(w, 7 + s, dev) for s in range(nsets)]   # same q on every rank
    res["bytes_per_step_per_gpu"] = local_bytes
    for kind in ("p2p", "nccl"):
        ex = None
        if kind == "p2p":
            try:
                ex = irdist.PeerExchange(w.batch, w.num_heads, w.head_dim, dev)
            except RuntimeError as exc:   # every rank raises together
                res[kind] = {"error": str(exc)[:200]}
                continue

        def one(i, ex=ex):
            q, kp, vp, _, _ = sets[i % nsets]
            irdist.chunked_decode(q, kp, vp, tables, ctx, w.scale, w.block_size, exchange=ex)

        ms = _graph_ms(one, steps, dev, world) / steps
        res[kind] = {"ms_per_step": round(ms, 5),
                     "value": round(total / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
                     "exchange": "peer stores over NVLink + merge, one kernel" if ex else
                                 "NCCL all-gather + ir_lse_merge"}
        if ex is not None:
            ex.close()
    del sets
    return res


def run_chunked(args):
    """C4 over N GPUs: every sequence's KV split into N chunks, one per GPU;
    partials exchanged by peer stores over NVLink (``--exchange p2p``, one
    kernel that also merges) or all-gathered over NCCL and merged
    (``--exchange nccl``); strong scaling."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist
    from infrared_b200 import workloads as wl

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    w = make_workload("c4", 0, args.batch)
    tables_np, ctx_np, _ = irdist.kv_chunk_tables(w.block_tables, w.context_lens,
                                                  w.block_size, world, rank)
    tables = torch.from_numpy(tables_np).to(dev)
    ctx = torch.from_numpy(ctx_np).to(dev)
    local_bytes = int(ctx_np.astype(np.int64).sum()) * 2 * w.num_kv_heads * w.head_dim * 2
    nsets = max(args.sets, -(-3 * 126 * 2 ** 20 // max(local_bytes, 1)))
    sets = [wl.torch_values(w, 7 + s, dev) for s in range(nsets)]   # same q on every rank
    total_bytes = w.algorithmic_bytes()
    ex = irdist.PeerExchange(w.batch, w.num_heads, w.head_dim, dev) \
        if args.exchange == "p2p" else None

    def step(i):
        q, kp, vp, _, _ = sets[i % nsets]
        return irdist.chunked_decode(q, kp, vp, tables, ctx, w.scale, w.block_size, exchange=ex)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    # K steps (decode + exchange + merge each) in one CUDA graph
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with torch.cuda.stream(stream):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                step(i)
        # soak for a replay count every rank agrees on (replays hold collectives)
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
        est_ms = irdist.max_over_ranks(ev[0].elapsed_time(ev[1]), device=dev)
        n_soak = int(min(2000, args.soak * 1e3 / max(est_ms, 1e-3)))
        clocks = ClockSampler(local)
        for _ in range(n_soak):
            graph.replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
        clk = clocks.stop()
    ms = irdist.max_over_ranks(ev[0].elapsed_time(ev[1]), device=dev)
    del graph
    # e2e: q from pinned host memory in, result out, every step
    q_host = sets[0][0].cpu().pin_memory()
    out_host = torch.empty(q_host.shape, dtype=q_host.dtype).pin_memory()
    q_dev = torch.empty_like(sets[0][0])
    _, kp0, vp0, _, _ = sets[0]

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        o = irdist.chunked_decode(q_dev, kp0, vp0, tables, ctx, w.scale, w.block_size,
                                  exchange=ex)
        out_host.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    ev[0].record()
    for _ in range(args.steps):
        e2e_step()
    ev[1].record()
    ev[1].synchronize()
    e2e_ms = irdist.max_over_ranks(ev[0].elapsed_time(ev[1]), device=dev)
    peak, peak_kind = measured_peaks()
    per_step = ms / args.steps
    per_gpu = (local_bytes + total_bytes - w.kv_bytes()) / (per_step / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(total_bytes * args.steps / (ms / 1e3) / 1e9, 1),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per_step, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)*0.5 q/K/V, random block tables",
        "config": {"workload": "C4: B=4 x ctx 32768, KV chunked over the GPUs",
                   "global_batch": w.batch, "bytes_per_step_total": total_bytes,
                   "parallelism": f"KV-chunk split x{world}: partials " + (
                       "stored into every rank's buffer over NVLink (peer stores, "
                       "epoch-counted arrival)" if ex is not None else
                       "all-gathered (NCCL)") + ", log-sum-exp merged on every rank",
                   "l2": f"{nsets} rotating pool sets (> 3x L2 between reuses)",
                   "timing": "K steps in one CUDA graph (NCCL captured), CUDA events, "
                             "max over ranks"},
        "decode_tok_s_per_layer": round(w.batch / (per_step / 1e3), 1),
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind,
                     "traffic": None,
                     "scope": "one rank: its KV chunk + q/out per step, incl. the exchange"},
        "e2e": {"value": round(total_bytes * args.steps / (e2e_ms / 1e3) / 1e9, 1),
                "unit": "GB/s", "h2d_bytes_per_step": q_host.numel() * 2,
                "d2h_bytes_per_step": out_host.numel() * 2,
                "ms_per_step": round(e2e_ms / args.steps, 5)},
        "clocks": clk,
        "gpu_launches": 3 * args.steps,   # decode, split merge, exchange or lse merge
    }
    if ex is not None:
        ex.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_model(args):
    """C5: one greedy decode token of a random-init Qwen2.5-7B for a batch of
    128 sequences (contexts U[1024, 2048]), attention on the fused cache-write
    + decode kernel, the rest of the step on library GEMMs; the step is one
    CUDA graph replayed token after token. At N GPUs every rank holds the
    weights and decodes its share of the 128 sequences (strong scaling, no
    collective on the data path)."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist
    from infrared_b200 import model_step as ms

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    global_batch = args.batch or 128
    ctx_all = ms.random_context_lens(global_batch, 1024, 2048, seed=0)
    lo, hi = irdist.shard_sequences(ctx_all, world)[rank]
    warm = max(args.warmup, 3)
    max_new = 2 * warm + args.steps + min(args.steps, 100) + 8
    model = ms.Qwen2DecodeStep(ms.QWEN25_7B, ctx_all[lo:hi], max_new=max_new, device=dev,
                               seed=rank)
    w_bytes = model.weight_bytes()
    for _ in range(warm):                      # eager steps (plans, workspaces, cuBLAS)
        model.step()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            logits = model.step()
        for _ in range(warm):
            graph.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        kv_first = model.kv_bytes_per_step()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        clocks = ClockSampler(local)
        ev[0].record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev[1].record(stream)
        ev[1].synchronize()
        clk = clocks.stop()
    ms_dev = ev[0].elapsed_time(ev[1])
    kv_bytes = (kv_first + model.kv_bytes_per_step()) // 2   # contexts grow by one a step
    ms_job = irdist.max_over_ranks(ms_dev, device=dev) if world > 1 else ms_dev
    # e2e: the engine's loop -- every step copies ids, positions and block
    # tables in from pinned host memory, replays and reads the sampled ids back
    b = model.batch
    h_ids = torch.empty(b, dtype=torch.int64).pin_memory()
    h_pos = torch.empty(b, dtype=torch.int64).pin_memory()
    h_bt = model.block_tables.cpu().pin_memory()
    h_ids.copy_(model.ids.cpu())
    h_pos.copy_(model.positions.cpu())
    e2e_steps = min(args.steps, 100)
    if model.positions.max().item() + e2e_steps + 1 > model.max_blocks * model.bs:
        e2e_steps = 0
    with torch.cuda.stream(stream):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            model.ids.copy_(h_ids, non_blocking=True)
            model.positions.copy_(h_pos, non_blocking=True)
            model.block_tables.copy_(h_bt, non_blocking=True)
            graph.replay()
            h_ids.copy_(model.ids, non_blocking=True)
            stream.synchronize()
            h_pos += 1
        e2e_s = time.perf_counter() - t0
    e2e_s = irdist.max_over_ranks(e2e_s, device=dev) if world > 1 else e2e_s
    del graph, logits
    peak, peak_kind = measured_peaks()
    per_step = ms_job / args.steps
    step_bytes = w_bytes + kv_bytes
    gbs = step_bytes / (ms_dev / args.steps / 1e3) / 1e9
    tok_s = global_batch * args.steps / (ms_job / 1e3)
    line = {
        "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": warm, "ms_per_step": round(per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init weights N(0,0.02), KV history N(0,0.5), random "
                "token ids, random block tables (no checkpoint or dataset)",
        "config": {"workload": "C5: Qwen2.5-7B decode step (28 layers, hidden 3584, 28/4 "
                               "heads, inter 18944, vocab 152064), ctx U[1024,2048], block "
                               "16, greedy, one CUDA graph per token",
                   "global_batch": global_batch, "batch_per_gpu": b,
                   "parallelism": f"sequence-sharded x{world}, weights replicated",
                   "l2": "inputs larger than L2: ~14 GB of weights + KV read per step",
                   "timing": "K graph replays, CUDA events, max over ranks"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": peak_kind, "traffic": None,
                     "scope": "whole decode step on one GPU: weights + KV history read "
                              "(rank 0)", "weight_bytes": w_bytes, "kv_bytes": kv_bytes},
        "e2e": {"value": round(global_batch * e2e_steps / e2e_s, 1) if e2e_steps else None,
                "unit": "tok/s", "h2d_bytes_per_step": 2 * b * 8 + h_bt.numel() * 4,
                "d2h_bytes_per_step": b * 8, "steps": e2e_steps},
        "clocks": clk,
        "gpu_launches": 2 * ms.QWEN25_7B.layers * args.steps,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def build_infrared_qwen7b(dev, dtype, seed=0, std=0.02):
    """infrared's own ``Qwen2ForCausalLM`` (infrared/model/qwen2.py:71-118) at
    the Qwen2.5-7B geometry with random weights N(0, std) (norm weights 1),
    built on the meta device and materialised on ``dev`` in ``dtype`` (no
    host copy of 15 GB). The RoPE frequencies are recomputed after
    materialising and cast to the model dtype, as ``from_pretrained``'s
    ``.to(dtype)`` leaves them."""
    import torch
    from infrared.model.config import Qwen2Config
    from infrared.model.qwen2 import Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944,
                      num_hidden_layers=28, num_attention_heads=28, num_key_value_heads=4,
                      head_dim=128, rms_norm_eps=1e-6, rope_theta=1_000_000.0,
                      max_position_embeddings=32768, tie_word_embeddings=False,
                      bos_token_id=151643, eos_token_ids=())
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device("meta"):
            model = Qwen2ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    model = model.to_empty(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith("norm.weight"):
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, std, generator=g)
        d = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=dev,
                                                     dtype=torch.float32) / d))
        model.rotary.inv_freq = inv.to(dtype)
    return model.eval(), cfg


def engine_leg(steps, warmup, dev, world, rank, local, global_batch=128,
               timeout_s=600.0):
    """Decode through infrared's own ``PagedBatchEngine`` (see
    :func:`run_model_engine`) on this rank's share of ``global_batch``
    requests; every rank takes part in the final reductions whatever happened
    in its own run (a failure is reported, never left to hang the others).
    Returns the job's figures (max time, summed tokens over ranks)."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist
    from infrared_b200 import model_step as ms
    from infrared_b200 import shim

    res = {"error": None, "ok": False, "secs": float("nan"), "tokens": 0, "graph_ms": [],
           "prefill_s": float("nan"), "total_s": float("nan"), "steps_logged": 0,
           "clocks": None, "b": 0, "t_max": 0, "w_bytes": 0, "kv_bytes": 0}
    warm = max(warmup, 3)
    model = engine = handle = None
    try:
        from infrared.engine.paged_engine import PagedBatchEngine
        from infrared.engine.static_batch import BatchRequest

        ctx_all = ms.random_context_lens(global_batch, 1024, 2048, seed=0)
        lo, hi = irdist.shard_sequences(ctx_all, world)[rank]
        ctx = [int(c) for c in ctx_all[lo:hi]]
        b = len(ctx)
        max_new = warm + steps + 1          # the first token comes from the prefill
        model, cfg = build_infrared_qwen7b(dev, torch.bfloat16, seed=rank)
        handle = shim.install(graph_inputs=True, fuse_rope=True, prefill=True)
        t_max = -(-(max(ctx) + max_new + 1) // 16) * 16
        engine = PagedBatchEngine(model, max_num_seqs=b, block_size=16,
                                  num_blocks=b * (t_max // 16) + 16,
                                  enable_prefix_caching=False, enable_cuda_graph=True,
                                  graph_max_seq_len=t_max)
        steps_log = []
        orig_step = engine._decode_step

        def timed_decode_step():
            n = len(engine.scheduler.running)
            t0 = time.perf_counter()
            orig_step()
            steps_log.append((t0, time.perf_counter(), n))

        engine._decode_step = timed_decode_step
        orig_run = engine._run

        def run_on_device():          # the engine's worker thread on this rank's GPU
            torch.cuda.set_device(dev)
            orig_run()

        engine._run = run_on_device
        # device time of each graph decode (input build + replay), CUDA events
        graph_events = []
        orig_decoder = engine._cuda_graph_decoder

        def timed_decoder():
            dec = orig_decoder()
            if not getattr(dec, "_irb_timed", False):
                orig_decode = dec.decode

                def decode(*a, **k):
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    out = orig_decode(*a, **k)
                    e1.record()
                    graph_events.append((e0, e1))
                    return out

                dec.decode = decode
                dec._irb_timed = True
            return dec

        engine._cuda_graph_decoder = timed_decoder
        rng = np.random.default_rng(100 + rank)
        pends = [engine.submit(BatchRequest(
            [int(x) for x in rng.integers(0, cfg.vocab_size, c)], max_new_tokens=max_new,
            eos_token_ids=())) for c in ctx]
        clocks = ClockSampler(local)
        t_start = time.perf_counter()
        engine.start()
        error = None
        try:
            for pd in pends:
                pd.result(timeout=timeout_s)
        except Exception as exc:  # noqa: BLE001 - reported in the line
            error = repr(exc)[:300]
        finally:
            engine.stop()
            handle.uninstall()
        t_total = time.perf_counter() - t_start
        clk = clocks.stop()
        torch.cuda.synchronize(dev)
        graph_ms = [e0.elapsed_time(e1) for e0, e1 in graph_events[warm:warm + steps]]
        timed = steps_log[warm:warm + steps]
        ok = error is None and len(timed) == steps and all(n == b for _, _, n in timed)
        secs = (timed[-1][1] - timed[0][0]) if ok else float("nan")
        tokens = sum(n for _, _, n in timed)
        prefill_s = (steps_log[0][0] - t_start) if steps_log else float("nan")
        kv_tokens = sum(ctx) + b * (warm + steps // 2)
        res.update(ok=ok, secs=secs, tokens=tokens, graph_ms=graph_ms, prefill_s=prefill_s,
                   total_s=t_total, steps_logged=len(steps_log), clocks=clk, b=b,
                   t_max=t_max, error=error,
                   w_bytes=sum(p.numel() * p.element_size() for p in model.parameters()),
                   kv_bytes=kv_tokens * 2 * cfg.num_key_value_heads * cfg.head_dim * 2 *
                   cfg.num_hidden_layers)
    except Exception as exc:  # noqa: BLE001 - reported, and the reductions still run
        res["error"] = repr(exc)[:300]
        res["ok"] = False
    finally:
        if handle is not None:
            handle.uninstall()   # idempotent: restores infrared's functions
        del engine, model
        torch.cuda.empty_cache()
    if world > 1:
        t = torch.tensor([res["secs"] if res["ok"] else -1.0, float(res["tokens"]),
                          float(res["ok"])], dtype=torch.float64, device=dev)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        mn = t.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        sm = t.clone()
        dist.all_reduce(sm)
        res["ok"] = bool(mn[2].item())
        res["secs"], res["tokens"] = float(mx[0].item()), int(sm[1].item())
    res["warm"] = warm
    return res


def c5_engine_summary(dev, world, rank, local, steps=20, warmup=3):
    """The ``c5_engine`` object of the default line: C5 decoded through
    infrared's own PagedBatchEngine at this job's N GPUs (128 requests
    sharded over the ranks; see :func:`run_model_engine`)."""
    if not infrared_importable():
        return {"unavailable": "infrared is not installed in baseline/_ref "
                               "(python -m oracle.reference_install)"}
    r = engine_leg(steps, warmup, dev, world, rank, local, global_batch=128, timeout_s=300.0)
    ok = r["ok"]
    return {
        "workload": "C5: random-init Qwen2.5-7B in infrared's Qwen2ForCausalLM served by "
                    "infrared's PagedBatchEngine (CUDA-graph decode, shim installed), 128 "
                    "requests with prompts U[1024,2048], sharded over the GPUs",
        "metric": "decode tok/s", "n_gpus": world, "global_batch": 128, "steps": steps,
        "scaling": "strong (fixed 128 sequences; every GPU reads the full weights)",
        "value": round(r["tokens"] / r["secs"], 1) if ok else None, "unit": "tok/s",
        "ms_per_step": round(r["secs"] / steps * 1e3, 4) if ok else None,
        "graph_decode_device_ms_per_step": round(statistics.mean(r["graph_ms"]), 4)
        if r["graph_ms"] else None,
        "prefill_s": round(r["prefill_s"], 2), "error": r["error"],
        "timing": "wall time of the engine's own decode loop, max over ranks; the device "
                  "part timed with CUDA events around each graph decode",
    }


def run_model_engine(args):
    """C5 through infrared's own engine: a random-init Qwen2.5-7B in infrared's
    ``Qwen2ForCausalLM``, served by infrared's ``PagedBatchEngine`` with
    CUDA-graph decode (infrared/engine/paged_engine.py:248-288,
    infrared/engine/cuda_graph.py:202-287), the B200 kernels installed behind
    its seam (``shim.install``: RoPE + cache write + decode in one kernel,
    prefill on the tensor-core kernel, graph inputs built on the device).
    128 requests (prompts of U[1024, 2048] random tokens) are submitted; the
    engine prefills each, then decodes them as one batch. tok/s = decoded
    tokens / wall time of the engine's decode steps (its own loop: graph
    replay, per-sequence greedy sampling on the host, scheduling), after
    warm-up steps that include the graph capture. At N GPUs every rank runs
    its own engine over its share of the 128 requests (no collective)."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist
    from infrared_b200 import model_step as ms
    from infrared_b200 import shim

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)
    if not infrared_importable():
        if rank == 0:
            print(json.dumps({"metric": METRIC, "unavailable": "infrared is not installed in "
                              "baseline/_ref (python -m oracle.reference_install)"}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    r = engine_leg(args.steps, args.warmup, dev, world, rank, local,
                   global_batch=args.batch or 128, timeout_s=1800.0)
    ok, secs, tokens, warm, b = r["ok"], r["secs"], r["tokens"], r["warm"], r["b"]
    global_batch = args.batch or 128
    error, prefill_s, t_total, clk = r["error"], r["prefill_s"], r["total_s"], r["clocks"]
    graph_ms, t_max = r["graph_ms"], r["t_max"]
    steps_log = [None] * r["steps_logged"]
    per_step_ms = secs / args.steps * 1e3 if ok else None
    tok_s = tokens / secs if ok else None
    w_bytes, kv_bytes = r["w_bytes"], r["kv_bytes"]
    peak, peak_kind = measured_peaks()
    step_gbs = (w_bytes + kv_bytes) / (per_step_ms / 1e3) / 1e9 if ok else None
    line = {
        "metric": METRIC, "value": round(tok_s, 1) if ok else None, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": warm,
        "ms_per_step": round(per_step_ms, 4) if ok else None, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init weights N(0,0.02), random prompt token ids (no "
                "checkpoint or dataset)",
        "config": {"workload": "C5 through infrared's PagedBatchEngine: Qwen2.5-7B (28 layers, "
                               "hidden 3584, 28/4 heads, inter 18944, vocab 152064) in "
                               "infrared's Qwen2ForCausalLM, prompts U[1024,2048], block 16, "
                               "greedy, CUDA-graph decode",
                   "global_batch": global_batch, "batch_per_gpu": b,
                   "parallelism": f"sequence-sharded x{world}: one engine per GPU, weights "
                                  "replicated",
                   "shim": "install(graph_inputs=True, fuse_rope=True, prefill=True)",
                   "l2": "inputs larger than L2: ~15 GB of weights + KV read per step",
                   "timing": "wall time of the engine's decode steps (its own loop), max "
                             "over ranks"},
        "engine": {"prefill_s": round(prefill_s, 2), "total_s": round(t_total, 2),
                   "decode_steps_logged": len(steps_log), "error": error,
                   "graph_decode_device_ms_per_step": round(statistics.mean(graph_ms), 4)
                   if graph_ms else None,
                   "note": "a decode step's wall time = the graph decode on the device "
                           "(inputs built by ir_build_decode_inputs, then the replay of the "
                           "28-layer forward) + infrared's host loop (per-sequence greedy "
                           "sampling, each a device sync; block bookkeeping)"},
        "roofline": {"bound": "hbm", "achieved": round(step_gbs, 1) if ok else None,
                     "peak": peak, "unit": "GB/s",
                     "frac": round(step_gbs / peak, 4) if ok else None, "peak_kind": peak_kind,
                     "traffic": None, "weight_bytes": w_bytes, "kv_bytes": kv_bytes,
                     "scope": "whole engine decode step on one GPU (weights + KV history "
                              "read per wall-clock step, host work included)"},
        "e2e": {"value": round(tok_s, 1) if ok else None, "unit": "tok/s",
                "h2d_bytes_per_step": b * (t_max // 16) * 4 + b * 12,
                "d2h_bytes_per_step": b * 8,
                "note": "the engine loop is end to end: host block tables in, sampled ids "
                        "out, every step"},
        "clocks": clk,
        "gpu_launches": (2 * 28 + 2) * args.steps,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_kernels(args):
    """The path's smaller kernels alone, each timed over K launches captured in
    one CUDA graph (CUDA events): the standalone K/V cache write
    (``ir_cache_write``) at the C3 batch (256 new tokens) and at a bulk size
    (65536 tokens, larger than L2), the log-sum-exp merge (``ir_lse_merge``)
    of 8 KV-chunk partials at C4 (4 x 28 rows) and at 256 x 28 rows, and the
    peer-exchange kernel (``ir_peer_exchange``) in a world of one GPU (the
    flag protocol, the merge and the row writes without NVLink; a capture of
    its multi-GPU form would hold one GPU's kernel while the other's waits on
    it). GB/s = algorithmic bytes (reads + writes) / launch time."""
    import ctypes

    import torch

    from infrared_b200 import _lib, ops
    from infrared_b200 import workloads as wl

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    res = {}

    def timed(name, fn, nbytes, steps):
        if args.only and name != args.only:
            return
        ms = _graph_ms(lambda i: fn(i), steps, dev, 1) / steps
        res[name] = {"us_per_launch": round(ms * 1e3, 3), "bytes": nbytes,
                     "GB_s": round(nbytes / (ms / 1e3) / 1e9, 1)}

    # cache write: C3's 256 tokens, and a bulk write larger than L2
    w3 = wl.c3(seed=0)
    pool_k = torch.randn(w3.num_slots, 4, 128, generator=g, device=dev).to(torch.bfloat16)
    pool_v = torch.randn(w3.num_slots, 4, 128, generator=g, device=dev).to(torch.bfloat16)
    for name, n in (("cache_write_c3", 256), ("cache_write_bulk", 65536)):
        sets = []
        for i in range(3):
            slots = torch.randperm(w3.num_slots, generator=g, device=dev)[:n]
            if n == 256 and i == 0:
                slots = torch.from_numpy(w3.slot_mapping).to(dev)
            k = torch.randn(n, 4, 128, generator=g, device=dev).to(torch.bfloat16)
            v = torch.randn(n, 4, 128, generator=g, device=dev).to(torch.bfloat16)
            sets.append((k, v, slots.contiguous()))
        timed(name, lambda i, sets=sets: ops.cache_write(sets[i % 3][0], sets[i % 3][1],
                                                         pool_k, pool_v, sets[i % 3][2]),
              2 * 2 * n * 4 * 128 * 2 + n * 8, args.steps)
    # log-sum-exp merge of 8 partials
    for name, b in (("lse_merge_c4", 4), ("lse_merge_b256", 256)):
        o = torch.randn(8, b, 28, 128, generator=g, device=dev)
        lse = torch.randn(8, b, 28, generator=g, device=dev)
        out = torch.empty(b, 28, 128, dtype=torch.bfloat16, device=dev)
        timed(name, lambda i, o=o, lse=lse, out=out: ops.lse_merge(o, lse, torch.bfloat16,
                                                                    out=out),
              o.numel() * 4 + lse.numel() * 4 + out.numel() * 2, args.steps)
    # K/V projection + bias + RoPE + cache write at the C5 layer shape (128 new
    # tokens, hidden 3584, 4 kv heads x 128), and the same work in PyTorch
    if not args.only or args.only.startswith("kv_proj"):
        hid, hkv, d, n = 3584, 4, 128, 128
        x = torch.randn(n, hid, generator=g, device=dev).to(torch.bfloat16)
        wk = (torch.randn(hkv * d, hid, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wv = (torch.randn(hkv * d, hid, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        bk = (torch.randn(hkv * d, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        bv = (torch.randn(hkv * d, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=dev, dtype=torch.float32) / d))
        f = torch.randint(0, 2048, (n,), generator=g, device=dev).float()[:, None] * inv
        cos, sin = torch.cat((f, f), -1).cos(), torch.cat((f, f), -1).sin()
        slots = torch.randperm(pool_k.shape[0], generator=g, device=dev)[:n].contiguous()
        kvp = torch.zeros(pool_k.shape[0], hkv, d, dtype=torch.bfloat16, device=dev)
        vvp = torch.zeros_like(kvp)
        nb = 2 * hkv * d * hid * 2 + n * hid * 2 + 2 * n * hkv * d * 2

        def torch_path(i):
            k = torch.nn.functional.linear(x, wk, bk).view(n, hkv, d)
            v = torch.nn.functional.linear(x, wv, bv).view(n, hkv, d)
            c, s_ = cos[:, None].to(k.dtype), sin[:, None].to(k.dtype)
            k = k * c + torch.cat((-k[..., d // 2:], k[..., :d // 2]), -1) * s_
            kvp[slots] = k
            vvp[slots] = v

        timed("kv_proj_c5", lambda i: ops.kv_proj_rope_write(x, wk, wv, bk, bv, cos, sin,
                                                             slots, kvp, vvp), nb, args.steps)
        timed("kv_proj_c5_torch", torch_path, nb, args.steps)
    # peer exchange, world of one (7168 rows of 128)
    b, h, d = 256, 28, 128
    o = torch.randn(b, h, d, generator=g, device=dev)
    lse = torch.randn(b, h, generator=g, device=dev)
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device=dev)
    nbytes = lib.ir_peer_exchange_bytes(1, b * h, d)
    buf = ctypes.c_void_p()
    _lib.check(lib.ir_peer_alloc(nbytes, ctypes.byref(buf)))
    arr = (ctypes.c_void_p * 1)(buf.value)

    def exchange(i):
        _lib.check(lib.ir_peer_exchange(out.data_ptr(), out.stride(0), o.data_ptr(),
                                        lse.data_ptr(), arr, nbytes, 1, 0, b, h, d,
                                        ops.dtype_code(out.dtype),
                                        ops.error_flag(local).data_ptr(), ops._stream(local)))

    timed("peer_exchange_world1_b256", exchange, o.numel() * 4 + lse.numel() * 4 +
          out.numel() * 2, args.steps)
    torch.cuda.synchronize(dev)
    ops.check_device_errors(dev)
    _lib.check(lib.ir_peer_free(buf))
    peak, peak_kind = measured_peaks()
    first = res.get("cache_write_bulk") or next(iter(res.values()))
    line = {"metric": "standalone kernel GB/s (algorithmic bytes / launch time)",
            "value": first["GB_s"], "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": 3, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic", "kernels": res, "peak": peak, "peak_kind": peak_kind,
            "config": {"workload": "cache write (C3 256 tokens; 65536 tokens), lse merge "
                                   "(8 parts x 4/256 x 28 rows), peer exchange world of one",
                       "timing": "K launches in one CUDA graph, CUDA events"}}
    print(json.dumps(line), flush=True)


PREFILL_PATHS = {1: "rows as decode rows", 2: "tcgen05",
                 3: "tcgen05 CTA pairs (cta_group::2, 256-row tiles)"}


def p1_summary(dev, world, rank, steps=10, warmup=3):
    """The ``prefill_p1`` object of the default line: P1 (8 causal 4096-token
    prompts, Qwen2.5-7B attention geometry) on the tcgen05 prefill kernel,
    launches timed back to back with CUDA events; TFLOP/s of useful (causal)
    FLOPs against the measured bf16 peak; every rank runs its own prompts."""
    import torch

    from infrared_b200 import dist as irdist
    from infrared_b200 import ops
    from infrared_b200 import workloads as wl

    w = wl.p1(seed=rank)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    slots = w.num_blocks * w.block_size

    def randn(*shape):
        return (torch.randn(*shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)

    kp = randn(slots, w.num_kv_heads, w.head_dim)
    vp = randn(slots, w.num_kv_heads, w.head_dim)
    q = randn(w.total_q, w.num_heads, w.head_dim)
    bt = torch.from_numpy(w.block_tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    qs = torch.from_numpy(w.q_start).to(dev)
    out = torch.empty_like(q)
    path, _ = ops.prefill_plan(q, kp, bt, qs, w.block_size, w.scale)
    for _ in range(warmup):
        ops.paged_prefill(q, kp, vp, bt, ctx, qs, w.scale, w.block_size, out=out)
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(steps):
        ops.paged_prefill(q, kp, vp, bt, ctx, qs, w.scale, w.block_size, out=out)
    ev[1].record()
    ev[1].synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    ms_job = irdist.max_over_ranks(ms, device=dev) if world > 1 else ms
    ops.check_device_errors(dev)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tflops = w.flops() / (ms / 1e3) / 1e12
    del kp, vp, q, out
    return {"workload": "P1: 8 causal prompts x 4096 tokens, Qwen2.5-7B attention (28 q / "
                        "4 kv heads, head_dim 128), block 16, per GPU",
            "metric": "paged prefill attention TFLOP/s (causal, useful FLOPs)",
            "kernel_path": PREFILL_PATHS.get(path, path),
            "value": round(w.flops() * world / (ms_job / 1e3) / 1e12, 1), "unit": "TFLOP/s",
            "ms_per_step": round(ms_job, 4), "steps": steps, "scaling": "weak",
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak,
                         "frac": round(tflops / peak, 4),
                         "peak_kind": "measured" if peaks else "fallback"}}


def run_prefill(args):
    """P1: causal prefill of 8 x 4096-token prompts at the Qwen2.5-7B attention
    geometry on the tcgen05 kernel (one launch per step); TFLOP/s of useful
    (causal) FLOPs against the measured bf16 dense peak. Every rank runs its
    own prompts (weak scaling, no collective)."""
    import torch
    import torch.distributed as dist

    from infrared_b200 import dist as irdist
    from infrared_b200 import ops
    from infrared_b200 import workloads as wl

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    w = wl.p1(seed=rank, batch=args.batch or 8)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    slots = w.num_blocks * w.block_size
    kp = (torch.randn(slots, w.num_kv_heads, w.head_dim, generator=g, device=dev) * 0.5
          ).to(torch.bfloat16)
    vp = (torch.randn(slots, w.num_kv_heads, w.head_dim, generator=g, device=dev) * 0.5
          ).to(torch.bfloat16)
    q = (torch.randn(w.total_q, w.num_heads, w.head_dim, generator=g, device=dev) * 0.5
         ).to(torch.bfloat16)
    bt = torch.from_numpy(w.block_tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    qs = torch.from_numpy(w.q_start).to(dev)
    out = torch.empty_like(q)
    ops.set_prefill_path(args.prefill_path)
    path, _ = ops.prefill_plan(q, kp, bt, qs, w.block_size, w.scale)
    flops = w.flops()

    def step():
        ops.paged_prefill(q, kp, vp, bt, ctx, qs, w.scale, w.block_size, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    clocks = ClockSampler(local)
    ev[0].record()
    for _ in range(args.steps):
        step()
    ev[1].record()
    ev[1].synchronize()
    clk = clocks.stop()
    ms = ev[0].elapsed_time(ev[1])
    ms_job = irdist.max_over_ranks(ms, device=dev) if world > 1 else ms
    ops.check_device_errors(dev)
    # e2e: q from pinned host memory in, the output back, every step
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        q_dev.copy_(q_host, non_blocking=True)
        ops.paged_prefill(q_dev, kp, vp, bt, ctx, qs, w.scale, w.block_size, out=out)
        out_host.copy_(out, non_blocking=True)
    torch.cuda.synchronize(dev)
    ev[0].record()
    for _ in range(e2e_steps):
        q_dev.copy_(q_host, non_blocking=True)
        ops.paged_prefill(q_dev, kp, vp, bt, ctx, qs, w.scale, w.block_size, out=out)
        out_host.copy_(out, non_blocking=True)
    ev[1].record()
    ev[1].synchronize()
    e2e_ms = ev[0].elapsed_time(ev[1])
    e2e_ms = irdist.max_over_ranks(e2e_ms, device=dev) if world > 1 else e2e_ms
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    per_step = ms_job / args.steps
    tflops = flops / (ms / args.steps / 1e3) / 1e12
    line = {
        "metric": "paged prefill attention TFLOP/s (causal, useful FLOPs)",
        "value": round(flops * world / (per_step / 1e3) / 1e12, 1), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)*0.5 q/K/V, random block tables",
        "config": {"workload": f"P1: {len(w.q_lens)} prompts x {int(w.q_lens[0])} tokens, "
                               "Qwen2.5-7B attention (28 q / 4 kv heads, head_dim 128), "
                               "block 16, causal",
                   "total_q_rows": w.total_q, "flops_per_step": flops,
                   "kernel_path": PREFILL_PATHS[path],
                   "l2": "q + out = 470 MB per step, larger than L2",
                   "timing": "K back-to-back launches, CUDA events, max over ranks"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tflops / peak, 4),
                     "peak_kind": "measured" if peaks else "fallback", "traffic": None,
                     "scope": "one prefill launch, per GPU"},
        "e2e": {"value": round(flops * world / (e2e_ms / e2e_steps / 1e3) / 1e12, 1),
                "unit": "TFLOP/s", "h2d_bytes_per_step": q.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 2,
                "ms_per_step": round(e2e_ms / e2e_steps, 4)},
        "clocks": clk,
        "gpu_launches": args.steps,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c5" and args.engine:
        run_model_engine(args)
    elif args.config == "c5":
        run_model(args)
    elif args.config == "p1":
        run_prefill(args)
    elif args.config == "kernels":
        run_kernels(args)
    elif args.config == "c4" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_chunked(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
