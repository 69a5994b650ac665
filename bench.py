#!/usr/bin/env python
"""Benchmark of the B200 paged-attention hot path.

Headline workload: paged decode attention at the
Qwen3-8B attention shape (32 query heads, 8 KV heads, head_dim 128, BF16 KV,
block_size 256), 256 sequences of context 4096 per GPU. One step = one decode
attention launch over the batch (plus the split-KV combine when splits > 1).
Multi-GPU runs are weak-scaled: each rank decodes its own 256-sequence shard
(sequences are independent; there is no collective on the data path).

  value    whole-job algorithmic HBM bytes / s (K+V of every context token,
           plus Q, output and page tables), inputs resident in HBM.
  e2e      same metric through the public API with host buffers: per step
           the step's inputs (new-token QKV projections, positions, slots,
           page tables, kv_lens) go H2D from pinned memory, the fused
           norm/RoPE/KV-store kernel writes the new token into the cache,
           decode attention runs, and the output comes back D2H, on three
           streams (a step's download overlaps the next step's upload). It
           can also be pipelined over sequence chunks (--e2e-chunks,
           --e2e-split) so that one chunk's copies overlap another's
           kernels; one chunk measured fastest.
  prefill  varlen causal prefill TFLOP/s on BASELINE config 2 (32 prompts,
           lengths U[64, 2048], 16q/8kv), causal FLOPs of visible keys only;
           `prefill.chunked` is the config's second pass (one 64-token chunk
           per sequence over a cached prefix P ~ U[256, 2048]).

`--impl reference` times the reference's CPU implementation of the path (the
FP32 oracle port; the reference's own CPU oracle is Rust and cannot be built
here) on the host cores with the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn HBM GB/s (% peak) & prefill attn TFLOP/s; tok/s at 1/2/4/8 B200"
BATCH, CTX, QH, KVH, BS, DIM = 256, 4096, 32, 8, 256, 128
WORKLOAD = ("config3: paged decode attention, Qwen3-8B attention shape (32q/8kv, hd128, bf16 KV, block 256), "
            "256 sequences x ctx 4096 per GPU, seeded N(0,1)*0.5, shuffled page table")


def bench_config(batch, world):
    """The `config` object of the JSON line, identical in both arms."""
    kv_gb = batch * CTX * KVH * DIM * 2 * 2 / 1e9
    return {"workload": WORKLOAD if batch == BATCH else WORKLOAD.replace("256 sequences", f"{batch} sequences"),
            "global_batch": batch * world, "seq_len": CTX,
            "parallelism": f"dp{world} (independent sequence shards, no collective)",
            "l2": f"no flush: {kv_gb:.2f} GB of KV per GPU > 126 MB L2"}


def bytes_per_seq(ctx=CTX):
    kv = ctx * KVH * DIM * 2 * 2
    q_out = 2 * QH * DIM * 2
    table = ((ctx + BS - 1) // BS) * 4 + 4
    return kv + q_out + table


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "decode_config3_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler(threading.Thread):
    """Samples SM clock and clock-event reasons through NVML (read-only)."""

    NAMES = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
             0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, device_index):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._halt = threading.Event()
        self.ok = False
        try:
            import pynvml as nv

            nv.nvmlInit()
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            try:
                self.h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.h = nv.nvmlDeviceGetHandleByIndex(device_index)
            self.nv = nv
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clock record
            self.err = str(e)

    def run(self):
        while self.ok and not self._halt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.NAMES.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def stop(self):
        self._halt.set()
        self.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline_sample(budget_s=15.0, seqs_cap=BATCH):
    """The CPU oracle (FP32 port) on a bounded sample of the workload, all host
    threads. Returns (GB/s, threads, sample description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle  # noqa: E402  (CPU baseline leg)
    import torch

    from __graft_entry__ import load_package

    W = load_package().workloads
    threads = os.cpu_count() or 1

    def sample(n, seed):
        case = W.paged_case([CTX] * n, q_heads=QH, kv_heads=KVH, block_size=BS, seed=seed, device="cpu")
        arr = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        return (arr(case.q), arr(case.k), arr(case.v), case.cu_q.numpy(), case.kv_lens.numpy(),
                case.block_table.numpy(), case.num_blocks, case.table_stride)

    def timed(args):
        q, k, v, cu, lens, table, nb, stride = args
        t0 = time.perf_counter()
        oracle.attention_varlen(q, k, v, cu, lens, table, qh=QH, kvh=KVH, bs=BS, blocks=nb, stride=stride,
                                threads=threads)
        return time.perf_counter() - t0

    t1 = timed(sample(max(1, threads // 4), 1000))
    per_seq = t1 / max(1, threads // 4)
    n = int(max(1, min(seqs_cap, budget_s / max(per_seq, 1e-6))))
    dt = timed(sample(n, 1001))
    return n * bytes_per_seq() / dt / 1e9, threads, dt, n


def run_reference(args, rank, world):
    """CPU reference arm: the FP32 oracle port timed on the host cores."""
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle  # noqa: E402
    import torch

    from __graft_entry__ import load_package

    W = load_package().workloads
    threads = os.cpu_count() or 1
    arr = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731

    def make(n, seed):
        c = W.paged_case([CTX] * n, q_heads=QH, kv_heads=KVH, block_size=BS, seed=seed, device="cpu")
        return (arr(c.q), arr(c.k), arr(c.v), c.cu_q.numpy(), c.kv_lens.numpy(), c.block_table.numpy(),
                c.num_blocks, c.table_stride)

    def step(a):
        q, k, v, cu, lens, table, nb, stride = a
        oracle.attention_varlen(q, k, v, cu, lens, table, qh=QH, kvh=KVH, bs=BS, blocks=nb, stride=stride,
                                threads=threads)

    probe = make(max(1, threads // 4), 7)
    t0 = time.perf_counter()
    step(probe)
    per_seq = (time.perf_counter() - t0) / max(1, threads // 4)
    budget = args.ref_budget  # seconds for the whole --warmup + --steps run
    n = int(max(1, min(BATCH, budget / max(1, args.steps + args.warmup) / max(per_seq, 1e-6))))
    data = make(n, 8)
    for _ in range(args.warmup):
        step(data)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(data)
    dt = (time.perf_counter() - t0) / max(1, args.steps)
    gbs = n * bytes_per_seq() / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": bench_config(BATCH, world),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n} of 256 sequences (ctx 4096, 32q/8kv) per step, FP32 oracle port of "
                                   f"src/gpu.rs:1430-1466 / kernels/flash_native/smoke.cu:57-81, {threads} threads"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def long_context_leg(nvb, W, dev, rank, world, stream, steps=50):
    """Qwen3-32B attention shape (64q/8kv), 4 sequences of
    ctx 32768. At N GPUs each rank owns 8/N kv heads (and their query heads),
    runs split-KV decode on its shard, and the combine kernel stores every
    result into all ranks' outputs over NVLink (nvb_paged_decode_gather: one
    launch pair per step, no NCCL). Returns whole-job GB/s of algorithmic
    bytes, timed with CUDA events (max over ranks).

    A rank's KV shard is 537 MB / N, which fits the 126 MB L2 from N = 8
    down to 67 MB: steps rotate over enough independently drawn KV sets that
    the bytes between two uses of one set exceed three L2s. At N > 1 an
    untimed step first checks the fused gather against the NCCL all-gather
    of the same local outputs (decode tolerance, max-abs 2e-2 / mean-abs
    2e-3) and fails the run on a mismatch."""
    import importlib

    import torch
    import torch.distributed as dist

    S = importlib.import_module("nano_vllm_rs_b200.sharding")
    batch, ctx, qh, kvh = 4, 32768, 64, 8
    l2_bytes = 126 * 2**20
    shard = S.HeadShard(rank, world, kv_heads=kvh, q_heads=qh)
    set_bytes = batch * ctx * shard.kv_local * 512
    nsets = max(1, -(-3 * l2_bytes // set_bytes))
    cases = [W.paged_case([ctx] * batch, q_heads=shard.q_local, kv_heads=shard.kv_local, seed=500 + 16 * i + rank,
                          device=dev) for i in range(nsets)]
    c0 = cases[0]
    run = S.KvHeadShardedDecode(nvb, shard, batch=batch, block_size=256, table_stride=c0.table_stride,
                                num_blocks=c0.num_blocks, max_k=ctx, device=dev, fused=world > 1)

    def once(i):
        c = cases[i % nsets]
        if world > 1:
            return run(c.q, c.k, c.v, c.cu_q, c.kv_lens, c.block_table, check=False)
        return run.local(c.q, c.k, c.v, c.cu_q, c.kv_lens, c.block_table, check=False)

    check = None
    if world > 1:
        fused_out = once(0).clone()
        nccl = S.KvHeadShardedDecode(nvb, shard, batch=batch, block_size=256, table_stride=c0.table_stride,
                                     num_blocks=c0.num_blocks, max_k=ctx, device=dev, fused=False,
                                     num_splits=run.splits)
        want = nccl(c0.q, c0.k, c0.v, c0.cu_q, c0.kv_lens, c0.block_table)
        torch.cuda.synchronize()
        err = (fused_out.float() - want.float()).abs()
        t = torch.tensor([err.max().item(), err.mean().item()], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mx, mn = t.tolist()
        check = {"vs": "NCCL all-gather of the same local outputs", "max_abs": mx, "mean_abs": mn,
                 "tolerance": [2e-2, 2e-3]}
        if not (mx <= 2e-2 and mn <= 2e-3):
            run.close()
            raise RuntimeError(f"fused multi-GPU gather differs from the NCCL all-gather: max-abs {mx}, mean-abs {mn}")
    for i in range(5):
        once(i)
    torch.cuda.synchronize()

    # One CUDA graph per KV set: at N > 1 the whole step (decode, combine +
    # peer stores, flag barrier) with its epoch in device memory, at N = 1 the
    # decode and combine; the timed loop replays them in turn.
    graphs = []
    for c in cases:
        if world > 1:
            graphs.append(run.capture(c.q, c.k, c.v, c.cu_q, c.kv_lens, c.block_table))
        else:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                run.local(c.q, c.k, c.v, c.cu_q, c.kv_lens, c.block_table, check=False)
            graphs.append(g)

    def replay(i):
        if world > 1:
            return run.replay(graphs[i % nsets])
        graphs[i % nsets].replay()
        return run.out_local

    def timed(fn, n):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(n):
            fn(i)
        b.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / n], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for i in range(5):
        replay(i)
    ms = timed(replay, steps)
    # Untimed diagnostics of the same step (max over ranks): launched from the
    # host without graphs, and the local decode + combine alone (no exchange).
    breakdown = {"graph_ms": round(ms, 5), "eager_ms": round(timed(once, steps), 5)}
    if world > 1:
        breakdown["local_decode_combine_ms"] = round(
            timed(lambda i: run.local(cases[i % nsets].q, cases[i % nsets].k, cases[i % nsets].v,
                                      cases[i % nsets].cu_q, cases[i % nsets].kv_lens, cases[i % nsets].block_table,
                                      check=False), steps), 5)
    err = nvb.device_error()
    del graphs
    run.close()  # every rank's GPU work is done (the all-reduce above)
    if err:
        raise RuntimeError(f"long-context decode recorded device error {err}")
    total_bytes = batch * ctx * kvh * 512 + 2 * batch * qh * 128 * 2
    return {"value": round(total_bytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 5),
            "splits_per_gpu": run.splits, "kv_heads_per_gpu": shard.kv_local,
            "l2": f"{nsets} KV sets of {set_bytes / 1e6:.0f} MB per GPU, used in turn",
            "gather_check": check, "breakdown": breakdown, "cuda_graph": True,
            "collective": ("combine fused with the all-gather: peer stores over NVLink + epoch-flag barrier "
                           "(nvb_paged_decode_gather)") if world > 1 else None,
            "workload": "config5: 4 seqs x ctx 32768, 64q/8kv, kv-head sharded over the GPUs, split-KV per GPU"}


def long_context_shard_leg(nvb, W, dev, of_gpus, steps):
    """Rank 0's share of config 5 on `of_gpus` GPUs, run on this one GPU: the
    per-rank shard (8 / N kv heads, their 64 / N query heads, 4 x 32768) with
    the step a rank runs at N > 1 - split-KV decode, then the combine fused
    with the gather and its epoch exchange - but over a world of one (the
    exchange is with this rank itself: the kernels' cost without NVLink or
    rank skew). Graph-replayed over KV sets rotated beyond L2, beside the
    local decode + combine alone. A diagnostic for one process (so ncu can
    capture it): no whole-job figure is claimed."""
    import importlib

    import torch

    S = importlib.import_module("nano_vllm_rs_b200.sharding")
    batch, ctx = 4, 32768
    kv, q = 8 // of_gpus, 64 // of_gpus
    shard = S.HeadShard(0, 1, kv_heads=kv, q_heads=q)
    set_bytes = batch * ctx * kv * 512
    nsets = max(2, -(-3 * 126 * 2**20 // set_bytes))
    cases = [W.paged_case([ctx] * batch, q_heads=q, kv_heads=kv, seed=900 + i, device=dev) for i in range(nsets)]
    c0 = cases[0]
    kw = dict(batch=batch, block_size=256, table_stride=c0.table_stride, num_blocks=c0.num_blocks, max_k=ctx,
              device=dev)
    fused = S.KvHeadShardedDecode(nvb, shard, fused=True, **kw)
    local = S.KvHeadShardedDecode(nvb, shard, fused=False, num_splits=fused.splits, **kw)
    args = [(c.q, c.k, c.v, c.cu_q, c.kv_lens, c.block_table) for c in cases]
    for a in args:
        fused(*a)
        local.local(*a)
    torch.cuda.synchronize()
    g_fused = [fused.capture(*a) for a in args]
    g_local = []
    for a in args:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            local.local(*a, check=False)
        g_local.append(g)

    def timed(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    local_ms = timed(lambda i: g_local[i % nsets].replay())
    fused_ms = timed(lambda i: fused.replay(g_fused[i % nsets]))
    err = nvb.device_error()
    del g_fused, g_local
    fused.close()
    if err:
        raise RuntimeError(f"long-context shard step recorded device error {err}")
    return {"emulates": f"rank 0 of config 5 on {of_gpus} GPUs (exchange over a world of one: no NVLink, no rank skew)",
            "kv_heads": kv, "q_heads": q, "splits": fused.splits, "fused_step_ms": round(fused_ms, 5),
            "local_step_ms": round(local_ms, 5), "gather_exchange_ms": round(fused_ms - local_ms, 5),
            "local_gbs": round(set_bytes / (local_ms / 1e3) / 1e9, 1)}


def engine_leg(nvb, dev, rank, world, runs=1, max_tokens=512):
    """the Qwen3-0.6B engine (28 layers, random weights
    N(0, 0.02)) generating for 256 requests with prompt ids uniform over the
    vocabulary, prompt lengths U[128, 1024], max_tokens 512, temperature 0.6
    Gumbel-max with seed 42, ignore_eos; continuous batching (all 256
    admitted at once, prefill chunked at 16384 tokens) with graph-replayed
    decode; one engine replica per GPU, each with its own requests. One
    untimed run captures the decode graphs and warms cuBLAS; the timed runs
    are whole generate() calls, host scheduling included. Returns whole-job
    output tokens per second (sum over ranks / slowest rank)."""
    import torch
    import torch.distributed as dist

    M, E = nvb.model, nvb.engine
    cfg = M.Qwen3Config()
    n_req, lo, hi, max_cap = 256, 128, 1024, 512
    g = torch.Generator().manual_seed(4000 + rank)
    lens = torch.randint(lo, hi + 1, (n_req,), generator=g).tolist()
    reqs = [E.Request(id=i, prompt_token_ids=torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist(),
                      max_tokens=max_tokens, temperature=0.6, ignore_eos=True) for i, n in enumerate(lens)]
    bs = 256
    # Capacities follow config 4 (max_tokens 512) even when a profiling run
    # generates fewer tokens, so the decode geometry is the config's.
    pages = sum(-(-(n + max_cap) // bs) for n in lens)
    sched = E.SchedulerConfig(block_size=bs, num_blocks=pages, max_sequences=n_req, max_model_len=hi + max_cap,
                              max_batch_tokens=16384)
    opts = M.ModelOptions(device=dev.index or 0, block_size=bs, num_blocks=pages, max_batch_tokens=16384,
                          max_sequences=n_req, max_model_len=hi + max_cap, cuda_graphs=True)
    weights = M.random_weights(cfg, seed=0, device=dev)
    model = M.Qwen3Model(cfg, opts, weights)
    engine = E.LlmEngine(sched, model)
    engine.generate(reqs, 42)  # untimed: graph capture, cuBLAS warm-up
    if world > 1:
        dist.barrier()
    best = None
    for _ in range(runs):
        out = engine.generate(reqs, 42)
        st = out.stats
        if best is None or st["elapsed_seconds"] < best["elapsed_seconds"]:
            best = st
    engine.close()
    model.close()
    del weights
    t = torch.tensor([best["elapsed_seconds"], best["output_tokens"], best["decode_seconds"], best["decode_tokens"],
                      best["prefill_seconds"], best["prefill_tokens"]], dtype=torch.float64, device=dev)
    if world > 1:
        tmax, tsum = t.clone(), t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        elapsed, out_tok = tmax[0].item(), tsum[1].item()
        dec_s, dec_tok, pre_s, pre_tok = tmax[2].item(), tsum[3].item(), tmax[4].item(), tsum[5].item()
    else:
        elapsed, out_tok, dec_s, dec_tok, pre_s, pre_tok = t.tolist()
    return {"value": round(out_tok / elapsed, 1), "unit": "output tok/s", "elapsed_s": round(elapsed, 4),
            "output_tokens": int(out_tok), "decode_tok_s": round(dec_tok / dec_s, 1),
            "prefill_tok_s": round(pre_tok / pre_s, 1), "decode_steps": best["decode_steps"],
            "prefill_steps": best["prefill_steps"], "mean_itl_ms": round(best["mean_inter_token_latency_ms"], 4),
            "workload": ("config4: Qwen3-0.6B random init, 256 requests, prompt U[128,1024] uniform ids, "
                         "max_tokens 512, T=0.6 Gumbel seed 42, ignore_eos; one replica per GPU"),
            "path": "LlmEngine (C++ scheduler) -> nvbe_model_run: packed metadata H2D, graph-replayed decode "
                    "(cuBLAS GEMMs, nvb_qkv_rope_cached, nvb_paged_fwd_ex), sampled ids D2H",
            "reference_published": {"native": 1734.4, "flash": 3877.8, "unit": "output tok/s",
                                    "hardware": "RTX 5070 Ti, a different workload (ATTENTION.md:16)"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=1,
                    help="sequence chunks the end-to-end step is pipelined over (copies overlap compute)")
    ap.add_argument("--e2e-split", type=str, default=None,
                    help="comma-separated chunk sizes in sequences (sum = batch); overrides --e2e-chunks")
    ap.add_argument("--no-long-context", action="store_true")
    ap.add_argument("--long-context-shard", type=int, default=0, choices=[0, 1, 2, 4, 8],
                    help="one GPU only: also time rank 0's share of config 5 on N GPUs (diagnostic)")
    ap.add_argument("--no-engine", action="store_true")
    ap.add_argument("--engine-runs", type=int, default=1, help="timed generate() calls of the config-4 engine leg")
    ap.add_argument("--engine-max-tokens", type=int, default=512,
                    help="tokens per request in the engine leg (512 = config 4; fewer only for profiling runs)")
    ap.add_argument("--ref-budget", type=float, default=150.0,
                    help="seconds the reference arm's warm-up and timed steps may take in all")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="sequences per GPU (default 256 = config 3; smaller only for profiler captures)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist

    from __graft_entry__ import load_package

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    nvb = load_package()
    W = nvb.workloads
    hbm_peak, tc_peak, tc_sustained, peak_src = load_peaks()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count

    # ---------------- device-resident decode (value, roofline)
    batch = args.batch
    case = W.config3_decode(device=dev, seed=rank, batch=batch)
    splits = nvb.num_splits(batch, QH, KVH, CTX, sms)
    out = torch.empty_like(case.q)
    lse = torch.empty(batch, QH, 1, dtype=torch.float32, device=dev)
    la, oa = nvb.splitkv_scratch(splits, batch, QH, dev) if splits > 1 else (None, None)
    lib = nvb.library()
    stream = torch.cuda.current_stream()
    raw = [nvb._stream(stream), nvb._ptr(case.q), nvb._ptr(case.k), nvb._ptr(case.v), nvb._ptr(out),
           nvb._ptr(case.cu_q), nvb._ptr(case.kv_lens), nvb._ptr(case.block_table), batch, batch, 1, CTX, QH, KVH,
           BS, case.table_stride, splits, nvb._ptr(lse), nvb._ptr(la), nvb._ptr(oa), case.num_blocks]

    def step():
        rc = lib.nvb_paged_fwd_ex(*raw)
        if rc:
            raise RuntimeError(lib.nvb_last_error().decode())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # an event pair around every launch gives the kernels' own durations
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    clock_rec = clocks.stop()
    ms = t_start.elapsed_time(t_end)
    launch_times = [a.elapsed_time(b) for a, b in ev]
    launch_ms = statistics.mean(launch_times)
    launch_first, launch_last = statistics.mean(launch_times[:10]), statistics.mean(launch_times[-10:])
    if world > 1:
        t = torch.tensor([ms, launch_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, launch_ms = t.tolist()
    ms_per_step = ms / args.steps
    step_bytes = batch * bytes_per_seq()
    value = world * step_bytes / (ms_per_step / 1e3) / 1e9
    achieved = step_bytes / (launch_ms / 1e3) / 1e9
    assert nvb.device_error() == 0, "device pipeline wait timed out"

    # ---------------- end to end through the public API, host buffers
    e2e_value = e2e_ms = None
    e2e_breakdown = None
    e2e_sizes = None
    h2d = d2h = 0
    e2e_steps = 1
    if not args.no_e2e:
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        qkv_h = pin(torch.randn(batch, QH + 2 * KVH, DIM, generator=g, device=dev).bfloat16())
        qw = (1 + 0.02 * torch.randn(DIM, generator=g, device=dev)).bfloat16()
        kw = (1 + 0.02 * torch.randn(DIM, generator=g, device=dev)).bfloat16()
        positions_h = pin((case.kv_lens - 1).to(torch.int32))
        table_cpu = case.block_table.cpu()
        slots_h = pin(torch.tensor([int(table_cpu[i, (CTX - 1) // BS]) * BS + (CTX - 1) % BS for i in range(batch)],
                                   dtype=torch.int32))
        table_h, lens_h, cuq_h = pin(case.block_table), pin(case.kv_lens), pin(case.cu_q)
        out_h = torch.empty(batch, QH, DIM, dtype=torch.bfloat16).pin_memory()
        # All step inputs live in one pinned staging buffer with the same
        # layout on the device (the step metadata first, then the QKV rows;
        # 256-byte aligned fields), so a step uploads with one copy (or one
        # per chunk), as the engine uploads its packed metadata.
        src = {"pos": positions_h, "slots": slots_h, "table": table_h, "lens": lens_h, "cuq": cuq_h, "qkv": qkv_h}
        offs, total = {}, 0
        for n_, t in src.items():
            offs[n_] = total
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        stage_h = torch.empty(total, dtype=torch.uint8).pin_memory()
        stage_d = torch.empty(total, dtype=torch.uint8, device=dev)

        def field_view(buf, n_):
            t = src[n_]
            nb = t.numel() * t.element_size()
            return buf[offs[n_]:offs[n_] + nb].view(t.dtype).view(t.shape)

        host_in = {n_: field_view(stage_h, n_) for n_ in src}
        for n_, t in src.items():
            host_in[n_].copy_(t)
        dev_in = {n_: field_view(stage_d, n_) for n_ in src}
        meta_bytes = offs["qkv"]
        rope = torch.empty(CTX, DIM, dtype=torch.float32, device=dev)
        nvb.rope_cache(rope, CTX, DIM, 1e6)
        q_dev = torch.empty(batch, QH, DIM, dtype=torch.bfloat16, device=dev)
        qkv_bytes = src["qkv"].numel() * src["qkv"].element_size()
        d2h = out_h.numel() * out_h.element_size()

        # The step is pipelined over sequence chunks on three streams: chunk
        # c+1's inputs go H2D while chunk c runs the fused store and decode,
        # and chunk c's output goes D2H while chunk c+1 runs. Every input and
        # output byte of the step still crosses PCIe inside the timed region.
        # Step k+1's uploads wait for step k's compute (the next token's
        # projections depend on this step), and its compute waits for step
        # k's downloads (the output buffer is reused).
        if args.e2e_split:
            sizes = [int(x) for x in args.e2e_split.split(",")]
            if sum(sizes) != batch or min(sizes) < 1:
                raise SystemExit(f"--e2e-split sizes must be positive and sum to the batch ({batch})")
            starts = [sum(sizes[:c]) for c in range(len(sizes))]
            bounds = [(a, a + n) for a, n in zip(starts, sizes)]
        else:
            nch = max(1, min(args.e2e_chunks, batch))
            bounds = [(c * batch // nch, (c + 1) * batch // nch) for c in range(nch)]
        nch = len(bounds)
        e2e_sizes = [b - a for a, b in bounds]
        h2d = total if nch == 1 else meta_bytes + qkv_bytes  # bytes copied per step
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        chunk_cfg = []
        for s0, s1 in bounds:
            n = s1 - s0
            sp = nvb.num_splits(n, QH, KVH, CTX, sms)
            la_c, oa_c = nvb.splitkv_scratch(sp, n, QH, dev) if sp > 1 else (None, None)
            chunk_cfg.append((s0, s1, sp, la_c, oa_c))
        ev_in = [torch.cuda.Event() for _ in bounds]
        ev_done = [torch.cuda.Event() for _ in bounds]

        def e2e_step():
            h2d_s.wait_stream(stream)
            with torch.cuda.stream(h2d_s):
                if len(chunk_cfg) == 1:
                    stage_d.copy_(stage_h, non_blocking=True)
                    ev_in[0].record(h2d_s)
                else:
                    stage_d[:meta_bytes].copy_(stage_h[:meta_bytes], non_blocking=True)
                    for c, (s0, s1, *_r) in enumerate(chunk_cfg):
                        dev_in["qkv"][s0:s1].copy_(host_in["qkv"][s0:s1], non_blocking=True)
                        ev_in[c].record(h2d_s)
            stream.wait_stream(d2h_s)
            for c, (s0, s1, sp, la_c, oa_c) in enumerate(chunk_cfg):
                n = s1 - s0
                stream.wait_event(ev_in[c])
                nvb.qkv_rope_cached(dev_in["qkv"][s0:s1], qw, kw, dev_in["pos"][s0:s1], dev_in["slots"][s0:s1],
                                    q_dev[s0:s1], case.k, case.v, rows=n, q_heads=QH, kv_heads=KVH, head_dim=DIM,
                                    block_size=BS, num_blocks=case.num_blocks, eps=1e-6, rope_cache=rope,
                                    max_positions=CTX)
                nvb.paged_fwd(q_dev[s0:s1], case.k, case.v, out[s0:s1], dev_in["cuq"][:n + 1], dev_in["lens"][s0:s1],
                              dev_in["table"][s0:s1], batch=n, max_q=1, max_k=CTX, q_heads=QH, kv_heads=KVH,
                              block_size=BS, table_stride=case.table_stride, num_blocks=case.num_blocks,
                              num_splits=sp, lse=lse[s0:s1], lse_accum=la_c, out_accum=oa_c)
                ev_done[c].record(stream)
            with torch.cuda.stream(d2h_s):
                for c, (s0, s1, *_r) in enumerate(chunk_cfg):
                    d2h_s.wait_event(ev_done[c])
                    out_h[s0:s1].copy_(out[s0:s1], non_blocking=True)

        e2e_steps = max(10, min(args.steps, 200))
        for _ in range(3):
            e2e_step()
        stream.wait_stream(d2h_s)
        torch.cuda.synchronize()
        # the pipelined step must give the whole-batch result (not timed)
        ref_out = torch.empty_like(out)
        nvb.paged_fwd(q_dev, case.k, case.v, ref_out, dev_in["cuq"], dev_in["lens"], dev_in["table"], batch=batch,
                      max_q=1, max_k=CTX, q_heads=QH, kv_heads=KVH, block_size=BS, table_stride=case.table_stride,
                      num_blocks=case.num_blocks, num_splits=splits, lse=lse, lse_accum=la, out_accum=oa)
        torch.cuda.synchronize()
        e2e_err = (out_h.float() - ref_out.cpu().float()).abs().max().item()
        if not e2e_err <= 2e-2:
            raise RuntimeError(f"pipelined end-to-end step differs from the whole-batch decode: max-abs {e2e_err}")
        del ref_out
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        stream.wait_stream(d2h_s)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = t.item()
        e2e_value = world * step_bytes / (e2e_ms / e2e_steps / 1e3) / 1e9

        # Untimed diagnostics (max over ranks, all ranks at once, as in the
        # timed loop): the step's host-to-device copy alone, its kernels alone
        # (inputs already on the device) and its device-to-host copy alone.
        def alone(s, fn, n=20):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record(s)
            for _ in range(n):
                fn()
            b_.record(s)
            torch.cuda.synchronize()
            t_ = torch.tensor([a_.elapsed_time(b_) / n], device=dev)
            if world > 1:
                dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            return t_.item()

        def kernels_only():
            for (s0, s1, sp, la_c, oa_c) in chunk_cfg:
                n = s1 - s0
                nvb.qkv_rope_cached(dev_in["qkv"][s0:s1], qw, kw, dev_in["pos"][s0:s1], dev_in["slots"][s0:s1],
                                    q_dev[s0:s1], case.k, case.v, rows=n, q_heads=QH, kv_heads=KVH, head_dim=DIM,
                                    block_size=BS, num_blocks=case.num_blocks, eps=1e-6, rope_cache=rope,
                                    max_positions=CTX)
                nvb.paged_fwd(q_dev[s0:s1], case.k, case.v, out[s0:s1], dev_in["cuq"][:n + 1], dev_in["lens"][s0:s1],
                              dev_in["table"][s0:s1], batch=n, max_q=1, max_k=CTX, q_heads=QH, kv_heads=KVH,
                              block_size=BS, table_stride=case.table_stride, num_blocks=case.num_blocks,
                              num_splits=sp, lse=lse[s0:s1], lse_accum=la_c, out_accum=oa_c)

        with torch.cuda.stream(h2d_s):
            h2d_ms = alone(h2d_s, lambda: stage_d.copy_(stage_h, non_blocking=True))
        with torch.cuda.stream(d2h_s):
            d2h_ms = alone(d2h_s, lambda: out_h.copy_(out, non_blocking=True))
        kern_ms = alone(stream, kernels_only)
        e2e_breakdown = {"step_ms": round(e2e_ms / e2e_steps, 5), "h2d_ms": round(h2d_ms, 5),
                         "h2d_gbs": round(total / (h2d_ms / 1e3) / 1e9, 2), "kernels_ms": round(kern_ms, 5),
                         "d2h_ms": round(d2h_ms, 5), "d2h_gbs": round(d2h / (d2h_ms / 1e3) / 1e9, 2)}
        del qkv_h, dev_in

    # ---------------- prefill TFLOP/s (config 2: full prompts, then the
    # chunked pass), rank-local
    def prefill_leg(pc):
        pout = torch.empty_like(pc.q)
        plse = torch.empty(pc.batch, pc.q_heads, pc.max_q, dtype=torch.float32, device=dev)
        kwp = dict(batch=pc.batch, max_q=pc.max_q, max_k=int(pc.kv_lens.max()), q_heads=16, kv_heads=8,
                   block_size=BS, table_stride=pc.table_stride, num_blocks=pc.num_blocks, lse=plse, check=False)

        def pstep():
            nvb.paged_fwd(pc.q, pc.k, pc.v, pout, pc.cu_q, pc.kv_lens, pc.block_table, **kwp)

        for _ in range(3):
            pstep()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        psteps = 10
        p0.record(stream)
        for _ in range(psteps):
            pstep()
        p1.record(stream)
        torch.cuda.synchronize()
        pms = p0.elapsed_time(p1) / psteps
        flops = W.prefill_flops(pc)
        total_flops = flops
        if world > 1:
            # every rank draws its own prompts: sum the work, take the slowest rank's time
            t = torch.tensor([pms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            pms = t.item()
            f = torch.tensor([flops], dtype=torch.float64, device=dev)
            dist.all_reduce(f, op=dist.ReduceOp.SUM)
            total_flops = f.item()
        tflops = total_flops / (pms / 1e3) / 1e12
        return {"value": round(tflops, 2), "unit": "TFLOP/s", "ms_per_step": round(pms, 4),
                "flops_per_step_all_gpus": total_flops, "flops_per_step_rank0": flops, "peak": tc_peak,
                "frac": round(tflops / world / tc_peak, 4)}

    prefill = None
    if not args.no_prefill:
        prefill = prefill_leg(W.config2_prefill(device=dev, seed=rank))
        prefill["workload"] = ("config2: varlen causal prefill, 32 prompts L~U[64,2048] (seed = rank), 16q/8kv, "
                               "FLOPs = 4*128*qh per visible (query, key)")
        prefill["kernel"] = "prefill_kernel"
        cc = W.config2_chunked(device=dev, seed=rank)
        chunked = prefill_leg(cc)
        chunked["workload"] = ("config2 second pass: one 64-token chunk per sequence over a cached prefix "
                               "P~U[256,2048] (32 sequences, seed = rank), 16q/8kv")
        chunked["kernel"] = "prefill_tile_kernel"
        # Per key and kv head a 64-query chunk (16q/8kv) does 64 * 2 * 512
        # FLOPs against 512 B of K/V: 128 FLOP/byte, below the B200's balance
        # (~250), so HBM bounds it. Bytes: every visible K/V row once (512 B
        # per token and kv head), Q in, out back.
        pbytes = cc.kv_bytes() + 2 * cc.q.numel() * cc.q.element_size()
        pgbs = pbytes / (chunked["ms_per_step"] / 1e3) / 1e9  # rank 0's bytes over the slowest rank's time
        chunked.update({"bound": "hbm", "bytes_per_step_per_gpu": pbytes, "hbm_gbs": round(pgbs, 1),
                        "hbm_peak": hbm_peak, "hbm_frac": round(pgbs / hbm_peak, 4)})
        prefill["chunked"] = chunked

    # ---------------- long-context decode (config 5), kv-head sharded for N > 1
    long_ctx = None
    if not args.no_long_context and 8 % world == 0:
        long_ctx = long_context_leg(nvb, W, dev, rank, world, stream)
    shard_probe = None
    if args.long_context_shard and world == 1:
        shard_probe = long_context_shard_leg(nvb, W, dev, args.long_context_shard, max(args.steps, 3))

    # ---------------- config 4 engine, one replica per GPU
    engine = None
    if not args.no_engine:
        engine = engine_leg(nvb, dev, rank, world, runs=args.engine_runs, max_tokens=args.engine_max_tokens)

    # ---------------- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, threads, dt, n = cpu_baseline_sample()
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{n} sequences of ctx 4096 (32q/8kv, hd128) through the FP32 oracle port, {dt:.1f} s"}

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": bench_config(batch, world),
            "num_splits": splits,
            "pct_peak": round(100 * value / world / hbm_peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": profile_traffic(),
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "decode_mma_kernel", "algorithmic_bytes_per_launch": step_bytes,
                         "launch_ms": round(launch_ms, 5), "launch_ms_first10": round(launch_first, 5),
                         "launch_ms_last10": round(launch_last, 5)},
            "tok_s": round(world * batch / (ms_per_step / 1e3), 1),
            "tok_s_note": "decode query tokens per second through one attention layer",
            "prefill": prefill,
            "long_context": long_ctx,
            **({"long_context_shard": shard_probe} if shard_probe else {}),
            "engine": engine,
            "e2e": None if e2e_value is None else {
                "value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / e2e_steps, 5), "chunks": nch, "chunk_sizes": e2e_sizes,
                "breakdown": e2e_breakdown,
                "path": "per sequence chunk: pinned H2D of step inputs -> nvb_qkv_rope_cached -> nvb_paged_fwd_ex -> "
                        "D2H output, chunks pipelined on H2D / compute / D2H streams"},
            "gpu_launches": args.steps * (1 if splits == 1 else 2),
            "gpu_launches_note": "decode_mma_kernel launches (+ combine_kernel when num_splits > 1) in the timed region",
            "clocks": clock_rec,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
