#!/usr/bin/env python
"""bench.py — throughput of the AIHost attention hot path on B200, one JSON line on rank 0.

A step is one call of the fused op (RoPE(q), RoPE(k_new), KV append, attention) through the
library's public C ABI (aihost_attn_forward) on one batch of seeded synthetic inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Default workload: config 2 (causal prefill, Qwen2-0.5B shape, S=2048) -> TFLOP/s (causal-pair
FLOPs) as the line's value, plus one object per other config of the workload list:
`config_1` (fp32 decode, TinyLlama shape; single call, and 256 rotating layer caches),
`config_3` (batched fp16 decode, Llama-3-8B shape), `config_4` (long prefill, S=32768) and
`config_5` (Q8_0 batched decode, Llama-3-70B shape), each with its own value, roofline, e2e and
CPU baseline. N>1 (torchrun, one rank per GPU): configs 1-3 run one independent sequence set per
rank (no data-path collective, weak scaling); configs 4 and 5 split their KV heads over the ranks
and all-gather the head outputs with NCCL (strong scaling). Time = max over ranks.
--impl reference times the CPU restatement of the reference path (oracle/, faithful fp32 mode,
all host threads) on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn tokens/s & KV-read GB/s vs 8 TB/s; prefill attn TFLOP/s vs peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-decode", action="store_true", help="config 2: skip the objects of configs 1, 3, 4 and 5")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU-baseline sample time")
    ap.add_argument("--shard", default="seq", choices=["seq", "heads", "rows", "context"],
                    help="N>1: seq = every rank runs its own sequences (weak scaling); heads = the KV heads "
                         "of one problem are split over the ranks and the head outputs all-gathered (strong); "
                         "rows = prefill configs: the query rows of one sequence are split into causal-balanced "
                         "blocks and the row blocks all-gathered (strong; for Hkv < N); context = decode "
                         "configs: every sequence's cached rows split into N chunks, partial results merged "
                         "(strong; for Hkv < N)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decode configs: also time a CUDA graph of this many layers with distinct caches "
                         "(rotating caches: HBM throughput instead of single-call latency); adds a `layers` object")
    ap.add_argument("--paged", type=int, default=0, metavar="PAGE_ROWS",
                    help="fp16 configs: keep the cache in a shared pool of PAGE_ROWS-row pages (shuffled order) and "
                         "time aihost_attn_forward_paged instead")
    ap.add_argument("--op", default="attention", choices=["attention", "qk-norm-rope"],
                    help="qk-norm-rope: time the Qwen TypeB Q/K prologue kernel alone (one GPU; GB/s of HBM)")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="run N untimed fused calls of --config and exit (the command profiled with ncu)")
    ap.add_argument("--profile-weights", default="",
                    help="with --profile-steps: run that many untimed calls of this weight-product case "
                         "(a name of WEIGHT_CASES) instead of an attention config")
    ap.add_argument("--profile-new", type=int, default=0,
                    help="with --profile-steps: override the config's new rows per sequence (a smaller prefill "
                         "of the same shape, for captures that must stay small)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ workload arithmetic
def work(cfg, lengths):
    """Algorithmic FLOPs and bytes of one step (one fused call)."""
    from aihost_b200 import F16, F32

    B, S, Hq, Hkv, D = cfg.batch, cfg.n_new, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    es = 4 if cfg.q_dtype == F32 else 2
    oes = 4 if cfg.out_dtype == F32 else 2
    kv_row = {F32: 4 * D, F16: 2 * D}.get(cfg.kv_dtype, 34 * (D // 32))
    if S == 1:
        rows = sum(n + 1 for n in lengths)  # every cached row plus the appended one
        flops = 4.0 * Hq * D * rows
        kv_read = 2.0 * Hkv * kv_row * rows
        io = B * Hq * D * (es + oes) + 2.0 * B * Hkv * D * es + 2.0 * B * Hkv * kv_row
        return dict(flops=flops, kernel_bytes=kv_read + B * Hq * D * (es + oes), kv_read=kv_read, bytes=kv_read + io,
                    tokens=B)
    pairs = sum((n + S) * S - S * (S - 1) / 2 for n in lengths)  # causal (query, key) pairs
    flops = 4.0 * Hq * D * pairs
    io = B * S * Hq * D * (es + oes) + 2.0 * B * S * Hkv * D * (es + 2)
    return dict(flops=flops, kernel_bytes=io, bytes=io, tokens=B * S, kv_read=0.0)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,utilization.gpu")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [[c.strip() for c in ln.split(",")] for ln in out.strip().splitlines() if ln.count(",") >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        busy = [r for r in rows if (num(r[9]) or 0) > 0] or rows
        sm = [num(r[1]) for r in busy if num(r[1])]
        mx = [num(r[2]) for r in rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "samples_busy": len(busy),
                "power_w_max": max((num(r[3]) or 0) for r in rows)}


# ------------------------------------------------------------------ CPU (oracle) timing
def _repeat_to(run_once, t_first: float, target_s: float):
    """Repeat a timed run until about target_s of CPU time is spent (at least once, at most 200
    runs). Returns (total seconds, runs)."""
    reps = int(max(1, min(20000, round(target_s / max(t_first, 1e-4)))))
    if reps == 1:
        return t_first, 1
    return sum(run_once() for _ in range(reps)), reps


def cpu_sample_run(cfg, target_s: float):
    """Time the oracle (faithful mode, all threads) on a bounded part of `cfg`: the part grows
    until one run takes about target_s, and a run of the whole workload that is shorter than
    that is repeated. Returns (units, seconds, cores, sample description)."""
    import numpy as np

    from aihost_b200.configs import make_inputs
    from oracle import oracle as orc

    S = cfg.n_new
    if S > 1:  # prefill: whole sequence, a subset of the query heads of one KV head
        G = cfg.n_q_heads // cfg.n_kv_heads
        sub = cfg.scaled(batch=1, n_q_heads=G, n_kv_heads=1)
        inp = make_inputs(sub)
        lengths = inp["lengths"]
        w = work(sub, lengths)
        def run(nh):
            desc = sub.spec(inp["capacity"]).desc()
            kc, vc = inp["k_cache"].numpy().copy(), inp["v_cache"].numpy().copy()
            t = time.perf_counter()
            orc.attn_forward(desc, inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(), kc, vc,
                             inp["seq_len"].numpy(), mode=orc.FAITHFUL, part=(0, 1, 0, nh))
            return time.perf_counter() - t
        t1 = run(1)
        nh = int(max(1, min(G, round(target_s / max(t1, 1e-3)))))
        t = run(nh) if nh > 1 else t1
        t, reps = _repeat_to(lambda: run(nh), t, target_s)
        units = w["flops"] * nh / G * reps
        return dict(units=units, seconds=t, reps=reps, unit="TFLOP/s", scale=1e-12, cores=orc.num_threads(), nh=nh,
                    sample=f"1 sequence x {nh} query head(s) of one KV head (of {cfg.n_q_heads}), S={S}, {reps} "
                           f"run(s) (faithful fp32 oracle)")
    # decode: a subset of sequences, all heads (inputs generated once per subset size)
    lengths_all = cfg.lengths()
    nb = 1
    made = {}
    def run(nb):
        if nb not in made:
            sub = cfg.scaled(batch=nb, cached_range=None, cached=None, cached_list=lengths_all[:nb])
            made[nb] = (sub, make_inputs(sub, capacity=max(lengths_all[:nb]) + 1))
        sub, inp = made[nb]
        desc = sub.spec(inp["capacity"]).desc()
        kc, vc = inp["k_cache"].numpy(), inp["v_cache"].numpy()
        t = time.perf_counter()
        orc.attn_forward(desc, inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(), kc, vc,
                         inp["seq_len"].numpy(), mode=orc.FAITHFUL)
        return time.perf_counter() - t, sub
    t1, sub = run(1)
    # bounded generation: at most ~32 M cache values per tensor in the sample (the timed oracle
    # run is then repeated to fill target_s)
    per_seq = (max(lengths_all) + 1) * cfg.n_kv_heads * cfg.head_dim
    nb_gen = max(1, (32 << 20) // per_seq)
    nb = int(max(1, min(cfg.batch, nb_gen, round(target_s / max(t1, 1e-3)))))
    if nb > 1:
        t1, sub = run(nb)
    t1, reps = _repeat_to(lambda: run(nb)[0], t1, target_s)
    return dict(units=float(nb * reps), seconds=t1, reps=reps, unit="tokens/s", scale=1.0, cores=orc.num_threads(), nb=nb,
                sample=f"{nb}/{cfg.batch} sequences, all {cfg.n_q_heads} query heads, {reps} run(s) "
                       f"(faithful fp32 oracle)")


def cpu_baseline(cfg, target_s):
    r = cpu_sample_run(cfg, target_s)
    return {"value": r["units"] * r["scale"] / r["seconds"], "unit": r["unit"], "cores": r["cores"], "kind": "port",
            "sample": r["sample"], "seconds": round(r["seconds"], 3)}


# ------------------------------------------------------------------ GPU timing
def device_inputs(cfg, device, rank):
    """Seeded inputs generated on the GPU (bit-identical to the CPU generator for integer parts;
    normals may differ in the last bit from CPU-generated ones). Rank r uses seed offset r."""
    import torch

    from aihost_b200.configs import make_inputs

    # Other ranks reseed the data but keep the global lengths (and so the same capacity and the
    # same per-GPU work); a reseeded config would also redraw its lengths.
    c = cfg.scaled(number=cfg.number + 1000 * rank, cached=None, cached_range=None,
                   cached_list=cfg.lengths()) if rank else cfg
    inp = make_inputs(c, device=device)
    assert inp["lengths"] == cfg.lengths() and inp["capacity"] == cfg.capacity()
    return inp


def context_inputs(cfg, device, rank, world):
    """Rank `rank`'s chunk of every sequence's cached rows of `cfg` (the same seeded problem on
    every rank), in a local cache with the same capacity; seq_len = local rows."""
    import torch

    from aihost_b200.ops import row_bytes
    from aihost_b200.shard import ContextShard

    inp = device_inputs(cfg, device, 0)
    sh = ContextShard(rank, world)
    cap = inp["capacity"]
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim) * cfg.n_kv_heads
    local_rows = []
    for name in ("k_cache", "v_cache"):
        full = inp[name].view(cfg.batch, cap, rb)
        local = torch.zeros_like(full)
        local_rows = []
        for b, length in enumerate(inp["lengths"]):
            lo, hi = sh.chunk(length)
            local[b, : hi - lo] = full[b, lo:hi]
            local_rows.append(hi - lo)
        inp[name] = local.reshape(-1)
    inp["global_lengths"] = list(inp["lengths"])
    inp["q_pos"] = inp["seq_len"]
    inp["lengths"] = local_rows
    inp["seq_len"] = torch.tensor(local_rows, dtype=torch.int32, device=device)
    return inp, sh


def shard_inputs(cfg, device, rank, world):
    """This rank's share of `cfg` under KV-head sharding: its Q / new K / V heads and its local
    cache slice (seeded per rank), laid out with the shard's (16-byte padded) token stride."""
    import torch

    from aihost_b200.configs import make_inputs
    from aihost_b200.ops import row_bytes
    from aihost_b200.shard import HeadShard

    shard = HeadShard(cfg.spec(cfg.capacity()), rank, world)
    local = cfg.scaled(number=cfg.number + 1000 * rank, n_q_heads=shard.q_per_rank, n_kv_heads=shard.kv_per_rank,
                       cached=None, cached_range=None, cached_list=cfg.lengths())
    inp = make_inputs(local, device=device)
    assert inp["capacity"] == cfg.capacity()
    spec = shard.local_spec()
    spec.kv_capacity = inp["capacity"]
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim) * shard.kv_per_rank
    if spec.kv_token_stride != rb:  # pad each token row (one Q8_0 head: 136 -> 144 bytes)
        for name in ("k_cache", "v_cache"):
            src = inp[name].view(cfg.batch, inp["capacity"], rb)
            dst = torch.zeros(cfg.batch, inp["capacity"], spec.kv_token_stride, dtype=torch.uint8, device=device)
            dst[:, :, :rb] = src
            inp[name] = dst.reshape(-1)
    inp["lengths"] = cfg.lengths()
    inp["seq_len"] = torch.tensor(inp["lengths"], dtype=torch.int32, device=device)
    return inp, spec, shard, local


def paged_cache(ctx, cfg, inp, page_rows, device):
    """PagedKVCache holding inp's cached rows in shuffled pages of a pool (room for every
    sequence's capacity), plus the step function over it."""
    import numpy as np
    import torch

    from aihost_b200.ops import PagedKVCache, row_bytes

    cap = inp["capacity"]
    max_pages = -(-cap // page_rows)
    n_pages = cfg.batch * max_pages
    cache = PagedKVCache(ctx, cfg.spec(cap), n_pages=n_pages, page_rows=page_rows, batch=cfg.batch, device=device)
    cache.free = [int(p) for p in np.random.default_rng(7).permutation(n_pages)]
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim) * cfg.n_kv_heads
    for b, length in enumerate(inp["lengths"]):
        cache.reserve(b, length + cfg.n_new)
    for name, pool in (("k_cache", cache.k[0]), ("v_cache", cache.v[0])):
        full = inp[name].view(cfg.batch, cap, rb)
        pv = pool.view(-1, rb)
        for b, length in enumerate(inp["lengths"]):
            t = torch.arange(length, device=device)
            pages = torch.tensor(cache.pages[b], device=device)
            pv[pages[t // page_rows] * page_rows + t % page_rows] = full[b, :length]
    cache.seq_len = inp["seq_len"]
    cache.host_len = list(inp["lengths"])
    return cache


def bench_ours(cfg, steps, warmup, device, ctx, flush_bytes, dist_on, shard_mode="seq", paged=0):
    import torch

    import aihost_b200 as A
    from aihost_b200.ops import ComputeOps, KVCache

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rows = None
    ctxs = None
    if shard_mode == "heads":
        inp, spec, shard, local_cfg = shard_inputs(cfg, device, rank, world)
    else:
        shard = None
        if shard_mode == "rows":
            from aihost_b200.shard import RowShard

            if cfg.n_new == 1 or cfg.batch != 1:
                raise SystemExit("--shard rows needs a single-sequence prefill config")
            inp = device_inputs(cfg, device, 0)  # one problem, the same seeded inputs on every rank
            rows = RowShard(cfg.n_new, inp["lengths"][0], rank, world)
        elif shard_mode == "context":
            if cfg.n_new != 1:
                raise SystemExit("--shard context needs a decode config")
            inp, ctxs = context_inputs(cfg, device, rank, world)
        else:
            inp = device_inputs(cfg, device, rank)
        spec, local_cfg = cfg.spec(inp["capacity"]), cfg
    lengths = inp["lengths"]
    if paged:
        cache = paged_cache(ctx, cfg, inp, paged, device)
    else:
        cache = KVCache(ctx, spec, batch=cfg.batch, n_layers=1, device=device)
        cache.k[0], cache.v[0] = inp["k_cache"], inp["v_cache"]
        cache.seq_len, cache.host_len = inp["seq_len"], list(lengths)
    q, kn, vn = inp["q"], inp["k_new"], inp["v_new"]
    ops = ComputeOps(ctx)
    if ctxs is not None:  # every rank serves all B tokens
        out = ctxs.forward(ops, q, kn, vn, cache, inp["q_pos"])
    elif paged:
        out = ops.attention_layer_paged(q, kn, vn, cache)
    else:
        out = ops.attention_layer(q, kn, vn, cache)  # also reserves scratch
    w = work(local_cfg, lengths)  # this rank's work (context mode: its chunk of the rows)
    need_flush = w["bytes"] < 2 * 126e6  # L2 is 126 MB: flush unless the step streams more than 2x that
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=device) if need_flush else None

    nccl = None
    result = out
    if shard is not None:
        # the library's own NCCL communicator: aihost_attn_forward_sharded runs this rank's heads
        # and all-gathers every rank's head outputs (rank-major) in one call
        import torch.distributed as tdist

        from aihost_b200.shard import NcclDist

        idb = [NcclDist.unique_id() if rank == 0 else None]
        if world > 1:
            tdist.broadcast_object_list(idb, src=0)
        nccl = NcclDist(world, rank, idb[0], device.index)
        result = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=device)

    def step():
        if nccl is not None:
            shard.forward(nccl, ops, q, kn, vn, cache, out=result)
        elif rows is not None:
            rows.forward(ops, q, kn, vn, cache, out=result)
        elif ctxs is not None:
            ctxs.forward(ops, q, kn, vn, cache, inp["q_pos"], out=result)
        elif paged:
            ops.attention_layer_paged(q, kn, vn, cache, out=result)
        else:
            ops.attention_layer(q, kn, vn, cache, out=out)

    for _ in range(warmup):
        if flush is not None:
            flush.zero_()
        step()
    torch.cuda.synchronize()
    ctx.sync_status()

    # timed region: K steps, CUDA events per step on the launching stream (flushes excluded).
    # The library's per-launch profiler stays off here: its events between two launches would
    # keep a programmatic launch from overlapping the kernel before it.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if dist_on:
        torch.distributed.barrier()
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    # the same K steps again with the profiler on: per-kernel device times and launch counts
    ctx.profiler_reset()
    ctx.profiler(True)
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        step()
    torch.cuda.synchronize()
    ctx.profiler(False)
    kern = {name: ctx.profiler_read(k) for name, k in
            (("append", A.KERNEL_APPEND), ("decode", A.KERNEL_DECODE), ("combine", A.KERNEL_COMBINE),
             ("prefill", A.KERNEL_PREFILL), ("convert", A.KERNEL_CONVERT))}
    ctx.sync_status()
    launches = sum(n for n, _ in kern.values())
    if rows is not None and world > 1:
        launches += steps  # aihost_rope_full of the new K rows (not timed by the context's profiler)

    # end to end: pinned host inputs -> device, fused call, result -> host, per step
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, kn, vn))
    hout = torch.empty(result.shape, dtype=result.dtype, pin_memory=True)
    e_ms = []
    for i in range(steps + warmup):
        if flush is not None:
            flush.zero_()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        q.copy_(hq, non_blocking=True)
        kn.copy_(hk, non_blocking=True)
        vn.copy_(hv, non_blocking=True)
        step()
        hout.copy_(result, non_blocking=True)
        s1.record()
        s1.synchronize()
        if i >= warmup:
            e_ms.append(s0.elapsed_time(s1))
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()
    if nccl is not None:
        torch.cuda.synchronize()
        nccl.close()
    return dict(ms=ms, wall=wall, kern=kern, launches=launches, e2e_ms=e_ms, h2d=h2d, d2h=d2h, work=w,
                lengths=inp.get("global_lengths", lengths), flushed=need_flush,
                sharded=shard is not None or rows is not None or ctxs is not None,
                rank_flops=(4.0 * cfg.n_q_heads * cfg.head_dim * rows.pairs(rank) if rows is not None else None),
                rank_rows=(rows.rows if rows is not None else None))


def profile_steps(cfg, n, device):
    """n fused calls of `cfg` on device inputs, no timing: the target of ncu captures."""
    import torch

    from aihost_b200.ops import ComputeOps, Context, KVCache

    with Context(device.index) as ctx:
        inp = device_inputs(cfg, device, 0)
        cache = KVCache(ctx, cfg.spec(inp["capacity"]), batch=cfg.batch, n_layers=1, device=device)
        cache.k[0], cache.v[0] = inp["k_cache"], inp["v_cache"]
        cache.seq_len, cache.host_len = inp["seq_len"], list(inp["lengths"])
        ops = ComputeOps(ctx)
        for _ in range(n):
            out = ops.attention_layer(inp["q"], inp["k_new"], inp["v_new"], cache)
        torch.cuda.synchronize()
        ctx.sync_status()
        print(f"profiled config {cfg.number}: {n} calls, mean |out| {out.float().abs().mean().item():.4f}")


def bench_layers(cfg, layers, steps, warmup, device, ctx):
    """Decode throughput with rotating caches: one step is `layers` fused calls, each on its own
    layer's cache (together larger than L2, so the bytes come from HBM), captured once in a CUDA
    graph and replayed. Returns (ms per step, algorithmic bytes per step)."""
    import torch

    from aihost_b200.ops import ComputeOps, KVCache

    inp = device_inputs(cfg, device, 0)
    cache = KVCache(ctx, cfg.spec(inp["capacity"]), batch=cfg.batch, n_layers=layers, device=device)
    for l in range(layers):
        cache.k[l].copy_(inp["k_cache"])
        cache.v[l].copy_(inp["v_cache"])
    cache.seq_len, cache.host_len = inp["seq_len"], list(inp["lengths"])
    q, kn, vn = inp["q"], inp["k_new"], inp["v_new"]
    ops = ComputeOps(ctx)
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = ops.attention_layer(q, kn, vn, cache, layer=0)  # scratch reserved outside the capture
        for l in range(layers):
            ops.attention_layer(q, kn, vn, cache, layer=l, out=out)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(layers):
            ops.attention_layer(q, kn, vn, cache, layer=l, out=out)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        a.record()
        graph.replay()
        b.record()
    torch.cuda.synchronize()
    ctx.sync_status()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    w = work(cfg, inp["lengths"])
    return ms, w["kernel_bytes"] * layers


def time_allgather(nbytes: int, ws: int, device, steps: int, warmup: int, dist_on: bool) -> float:
    """Mean device time (CUDA events, max over ranks) of an NCCL all-gather of `nbytes` per rank
    on the bench's process group: the collective the head-sharded step runs, timed alone."""
    import torch
    import torch.distributed as tdist

    x = torch.empty(nbytes, dtype=torch.uint8, device=device)
    y = torch.empty(ws * nbytes, dtype=torch.uint8, device=device)
    for _ in range(max(warmup, 3)):
        tdist.all_gather_into_tensor(y, x)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        e0.record()
        tdist.all_gather_into_tensor(y, x)
        e1.record()
    torch.cuda.synchronize()
    return max_over_ranks(statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev), dist_on)


def max_over_ranks(x: float, dist_on: bool) -> float:
    if not dist_on:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def decode_kernel_name(cfg) -> str:
    """The decode kernel the library picks for this cache dtype (token-major default strides)."""
    from aihost_b200 import F16, Q8_0

    if cfg.kv_dtype == Q8_0:  # head groups of up to 8 read K straight from the raw tiles
        if cfg.n_q_heads // cfg.n_kv_heads > 8:
            return "decode_q8_kernel"
        # the stream-K schedule for up to 512 sequences
        return "decode_q8s_kernel" if cfg.batch <= 512 else "decode_q8k_kernel"
    return {F16: "decode_mma_kernel"}.get(cfg.kv_dtype, "decode_splitk_kernel")


def summarize(cfg, r, n_gpus, dist_on, pk, pk_kind):
    w = r["work"]
    ms_step = max_over_ranks(statistics.mean(r["ms"]), dist_on)
    e2e_ms = max_over_ranks(statistics.mean(r["e2e_ms"]), dist_on)
    prefill = cfg.n_new > 1
    if prefill:
        unit, per_step = "TFLOP/s", w["flops"] * 1e-12
    else:
        unit, per_step = "tokens/s", float(w["tokens"])
    # FLOPs and bytes add up over ranks under sequence sharding; a sharded problem counts once
    # (head sharding of a decode: every rank serves the same tokens; row sharding: one prefill)
    ranks = 1 if (r.get("sharded") and (not prefill or r.get("rank_flops") is not None)) else n_gpus
    value = ranks * per_step / (ms_step * 1e-3)
    e2e_value = ranks * per_step / (e2e_ms * 1e-3)
    kname = "prefill" if prefill else "decode"
    n_k, tot = r["kern"][kname]
    k_ms = max_over_ranks(tot / max(n_k, 1), dist_on)
    if prefill and r.get("rank_flops") is not None:
        # row sharding: each rank's kernel over its own causal pairs; the slowest rank's rate
        k_local = tot / max(n_k, 1)
        achieved = -max_over_ranks(-r["rank_flops"] / (k_local * 1e-3) * 1e-12, dist_on)
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "traffic": None, "kernel": "prefill_kernel",
                "kernel_ms": k_ms, "algorithmic_per_launch": r["rank_flops"],
                "peak_source": f"{pk_kind} bf16 burst", "note": "min over ranks of (rank's causal-pair FLOPs / "
                "rank's mean prefill launch); algorithmic_per_launch is rank 0's"}
    elif prefill:
        achieved = w["flops"] / (k_ms * 1e-3) * 1e-12
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "traffic": None, "kernel": "prefill_kernel",
                "kernel_ms": k_ms, "algorithmic_per_launch": w["flops"], "peak_source": f"{pk_kind} bf16 burst"}
    else:
        achieved = w["kernel_bytes"] / (k_ms * 1e-3) * 1e-9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": None, "kernel": decode_kernel_name(cfg),
                "kernel_ms": k_ms, "algorithmic_per_launch": w["kernel_bytes"], "peak_source": f"{pk_kind} copy",
                "frac_of_8tbs_spec": achieved / 8000.0}
    roof["traffic"], roof["traffic_source"] = read_traffic(cfg.number)
    other = {k: {"launches": n, "mean_ms": (t / n if n else None)} for k, (n, t) in r["kern"].items()}
    out = dict(value=value, unit=unit, ms_per_step=ms_step, roofline=roof,
               e2e={"value": e2e_value, "unit": unit, "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                    "ms_per_step": e2e_ms},
               kernels=other, gpu_launches=r["launches"])
    if not prefill:
        out["kv_read_gbs"] = n_gpus * w["kv_read"] / (ms_step * 1e-3) * 1e-9
        out["kv_read_frac_of_8tbs"] = out["kv_read_gbs"] / 8000.0
    return out


KERNEL_SOURCE = {1: "decode.cu", 2: "prefill_sm100.cu", 3: "decode_mma.cu", 4: "prefill_sm100.cu", 5: "decode_mma.cu"}


def source_sha16(name: str) -> str:
    import hashlib

    return hashlib.sha256((ROOT / "aihost_b200" / "csrc" / name).read_bytes()).hexdigest()[:16]


def read_traffic(config_number: int):
    """DRAM bytes per launch of the dominant kernel of `config_number` from profiles/traffic.txt
    (one ncu capture each). A line is `configN <bytes> <kernel source file> <sha256[:16] of that
    file when captured>`; a figure whose source has changed since is stale and is not reported.
    Returns (bytes or None, note)."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None, "no capture"
    for ln in p.read_text().splitlines():
        parts = ln.split()
        if len(parts) >= 4 and parts[0] == f"config{config_number}":
            try:
                nbytes = float(parts[1])
            except ValueError:
                return None, "unreadable capture line"
            if source_sha16(parts[2]) != parts[3]:
                return None, f"stale: {parts[2]} changed since the capture ({parts[3]})"
            return nbytes, f"ncu capture of {parts[2]} @ {parts[3]}"
    return None, "no capture"


def needs_flush(cfg, shard_mode="seq", world=1) -> bool:
    """True when one step of this rank streams less than 2x the 126 MB L2, so the bench writes a
    512 MiB buffer between steps (outside the timed events) to start every step cold."""
    w = work(rank_cfg(cfg, shard_mode, world), cfg.lengths())
    return w["bytes"] < 2 * 126e6


def rank_cfg(cfg, shard_mode, world):
    """The share of `cfg` one rank computes: its KV heads under head sharding, else all of it."""
    if shard_mode == "heads" and world > 1:
        return cfg.scaled(n_q_heads=cfg.n_q_heads // world, n_kv_heads=cfg.n_kv_heads // world)
    return cfg


def parallelism(shard_mode, world, rank_rows=None) -> str:
    if world <= 1:
        return "single GPU"
    return {"heads": f"KV heads split over {world} ranks + NCCL all-gather of head outputs",
            "rows": f"query rows split over {world} ranks (causal-balanced 128-row blocks, rank 0 rows {rank_rows}) "
                    f"+ NCCL all-gather of row blocks",
            "context": f"every sequence's cached rows split into {world} chunks (context parallel) + NCCL all-gather "
                       f"of (out, lse) + merge kernel"}.get(shard_mode, "one independent sequence set per rank")


def cfg_desc(cfg, shard_mode="seq", world=1, rank_rows=None):
    """The `config` object of a bench line; the reference arm prints the same one for the same run."""
    return {"workload": f"config {cfg.number}: {cfg.name} ({cfg.note})", "batch": cfg.batch,
            "n_q_heads": cfg.n_q_heads, "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim, "n_new": cfg.n_new,
            "rope_theta": cfg.theta, "cached_rows_total": int(sum(cfg.lengths())),
            "l2": "flushed between steps (write of a 512 MiB buffer, outside the timed events)"
            if needs_flush(cfg, shard_mode, world) else "inputs larger than L2",
            "parallelism": parallelism(shard_mode, world, rank_rows)}


def init_dist(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        return False, 0, 0, 1
    import torch
    import torch.distributed as dist

    rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "ours":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    return True, rank, local, ws


def run_reference(args):
    """CPU restatement of the reference path, timed on the host cores (rank 0 only)."""
    from aihost_b200.configs import CONFIGS

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 per process; the CPU reference uses every host thread
    # (read by the OpenMP runtime when the oracle library loads, which happens below)
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    from oracle import oracle as orc

    orc.set_num_threads(len(os.sched_getaffinity(0)))
    cfg = CONFIGS[args.config]
    per_step = max(1.0, min(6.0, 150.0 / max(1, args.steps + args.warmup)))
    times, units, meta = [], None, None
    for i in range(args.warmup + args.steps):
        r = cpu_sample_run(cfg, per_step) if meta is None else None
        if meta is None:  # the sizing call; later steps repeat one run of the same part
            meta = r
            units = r["units"] / r["reps"]
            times.append(r["seconds"] / r["reps"])
            continue
        t = time.perf_counter()
        _rerun(cfg, meta)
        times.append(time.perf_counter() - t)
    timed = times[args.warmup:] or times
    sec = statistics.mean(timed)
    value = units * meta["scale"] / sec
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": meta["unit"], "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (reference arithmetic on fp16-converted inputs)",
            "data": "synthetic (seeded SplitMix64 + Box-Muller)",
            "config": cfg_desc(cfg, args.shard, int(os.environ.get("WORLD_SIZE", "1"))),
            "cpu_baseline": {"value": value, "unit": meta["unit"], "cores": meta["cores"], "kind": "port",
                             "sample": meta["sample"]},
            "e2e": {"value": value, "unit": meta["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference has no CPU attention and its Vulkan path is unavailable on this box; this is "
                    "the oracle's faithful restatement of the reference shaders"}
    print(json.dumps(line), flush=True)


_RERUN_CACHE = {}


def _rerun(cfg, meta):
    """Repeat the sized CPU sample of cpu_sample_run (same part) for the reference arm's steps."""
    from aihost_b200.configs import make_inputs
    from oracle import oracle as orc

    key = cfg.number
    if key not in _RERUN_CACHE:
        if cfg.n_new > 1:
            nh = meta["nh"]
            sub = cfg.scaled(batch=1, n_q_heads=cfg.n_q_heads // cfg.n_kv_heads, n_kv_heads=1)
            inp = make_inputs(sub)
            _RERUN_CACHE[key] = (sub, inp, (0, 1, 0, nh))
        else:
            nb = meta["nb"]
            ls = cfg.lengths()[:nb]
            sub = cfg.scaled(batch=nb, cached_range=None, cached=None, cached_list=ls)
            inp = make_inputs(sub, capacity=max(ls) + 1)
            _RERUN_CACHE[key] = (sub, inp, None)
    sub, inp, part = _RERUN_CACHE[key]
    desc = sub.spec(inp["capacity"]).desc()
    orc.attn_forward(desc, inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(), inp["k_cache"].numpy(),
                     inp["v_cache"].numpy(), inp["seq_len"].numpy(), mode=orc.FAITHFUL, part=part)


# ------------------------------------------------------------------ weight products
# (name, rows M, k K, n_out N, weight dtype, n_parts of A, description)
WEIGHT_CASES = [
    ("wo_prefill_cfg4", 32768, 4096, 4096, "F16", 1,
     "output projection after config 4's attention: [32768 x 4096] head outputs . Wo [4096 x 4096] fp16"),
    ("wo_decode_cfg3", 64, 4096, 4096, "F16", 1,
     "output projection after config 3's decode step: [64 x 4096] . Wo [4096 x 4096] fp16"),
    ("qkv_q4k_decode_cfg3", 64, 4096, 6144, "Q4_K", 1,
     "Q, K, V projections feeding config 3's decode (Wq|Wk|Wv stacked, 6144 x 4096) as GGUF Q4_K"),
    ("qkv_q6k_prefill_4096", 4096, 4096, 6144, "Q6_K", 1,
     "Q, K, V projections of a 4096-token Llama-3-8B prefill chunk (Wq|Wk|Wv stacked, 6144 x 4096) as GGUF Q6_K"),
]


def weight_bytes(kind: str, n: int, k: int) -> float:
    from aihost_b200.gen import KQUANT_BLOCK_BYTES
    import aihost_b200 as A

    if kind == "F16":
        return 2.0 * n * k
    return n * k / 256 * KQUANT_BLOCK_BYTES[getattr(A, kind)]


def bench_weights(args, device, ctx, pk, pk_kind, cpu_s):
    """aihost_matmul_weights on the projections around the op, fp16 A, fp16 output: the device
    time of a step (weight dequantisation included for K-quant weights: the reference
    dequantises its weights on every call), the dominant kernel's roofline (tensor-bound when
    2MNK / bytes exceeds the peaks' ratio, else HBM-bound over the algorithmic bytes: weight as
    stored + A + output), end to end with A copied in and C copied out, and the oracle's
    MatMulWeights (+ dequantisation) on a bounded sample of rows on the host cores."""
    import torch

    import aihost_b200 as A
    from aihost_b200 import gen
    from aihost_b200.ops import WeightOps

    ops = WeightOps(ctx)
    out = {}
    for name, M, K, N, kind, parts, desc in WEIGHT_CASES:
        t_start = time.perf_counter()
        wt = getattr(A, kind)
        a = gen.normal((M, K), 99, name + ".a", dtype=torch.float16, device=device)
        if kind == "F16":
            w = gen.normal((N, K), 99, name + ".w", std=0.02, dtype=torch.float16, device=device)
        else:
            w = gen.kquant_blocks(wt, N * K // 256, 99, name + ".w", device=device)
        c = ops.mat_mul_weights(a, w, wt, N)
        flops = 2.0 * M * N * K
        nbytes = weight_bytes(kind, N, K) + 2.0 * M * K + 2.0 * M * N
        flush = torch.empty(512 << 20, dtype=torch.uint8, device=device) if nbytes < 2 * 126e6 else None
        for _ in range(args.warmup):
            if flush is not None:
                flush.zero_()
            ops.mat_mul_weights(a, w, wt, N, out=c)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e0, e1 in ev:
            if flush is not None:
                flush.zero_()
            e0.record()
            ops.mat_mul_weights(a, w, wt, N, out=c)
            e1.record()
        torch.cuda.synchronize()
        ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)
        ctx.profiler_reset()
        ctx.profiler(True)
        for _ in range(args.steps):
            if flush is not None:
                flush.zero_()
            ops.mat_mul_weights(a, w, wt, N, out=c)
        torch.cuda.synchronize()
        ctx.profiler(False)
        n_mm, t_mm = ctx.profiler_read(A.KERNEL_MATMUL)
        n_cv, t_cv = ctx.profiler_read(A.KERNEL_CONVERT)
        ctx.sync_status()
        k_ms = t_mm / max(n_mm, 1)
        tensor_bound = flops / nbytes > pk["bf16_tflops"] * 1e12 / (pk["hbm_gbs"] * 1e9)
        if tensor_bound:
            ach = flops / (k_ms * 1e-3) * 1e-12
            roof = {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": ach / pk["bf16_tflops"], "kernel": "gemm_kernel<256>", "kernel_ms": k_ms,
                    "algorithmic_per_launch": flops, "peak_source": f"{pk_kind} bf16 burst", "traffic": None}
        else:
            # the GEMM reads the weight as stored when it dequantises inside (no dequantisation
            # launch), else the fp16 weight (the dequantised copy for K-quants)
            fused = kind != "F16" and n_cv == 0
            wread = weight_bytes(kind, N, K) if fused else 2.0 * N * K
            gbytes = wread + 2.0 * M * K + 2.0 * M * N
            ach = gbytes / (k_ms * 1e-3) * 1e-9
            roof = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                    "kernel": f"gemm_kernel<64> (dequantising {kind})" if fused else "gemm_kernel<64>",
                    "kernel_ms": k_ms, "algorithmic_per_launch": gbytes,
                    "peak_source": f"{pk_kind} copy", "traffic": None,
                    "note": ("bytes of the GEMM launch: weight as stored + A + C" if fused
                             else "bytes of the GEMM launch: fp16 weight + A + C")}
        # end to end: A from pinned host memory, C back, per step
        ha = a.cpu().pin_memory()
        hc = torch.empty(c.shape, dtype=c.dtype, pin_memory=True)
        e_ms = []
        for i in range(args.steps + args.warmup):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            a.copy_(ha, non_blocking=True)
            ops.mat_mul_weights(a, w, wt, N, out=c)
            hc.copy_(c, non_blocking=True)
            e1.record()
            e1.synchronize()
            if i >= args.warmup:
                e_ms.append(e0.elapsed_time(e1))
        res = {"workload": desc, "rows": M, "k": K, "n_out": N, "weight": kind,
               "value": flops / (ms * 1e-3) * 1e-12, "unit": "TFLOP/s", "ms_per_step": ms,
               "weight_bytes_as_stored": weight_bytes(kind, N, K),
               "weight_stream_gbs": weight_bytes(kind, N, K) / (ms * 1e-3) * 1e-9,
               "roofline": roof, "kernels": {"matmul": {"launches": n_mm, "mean_ms": k_ms},
                                             "dequant": {"launches": n_cv, "mean_ms": (t_cv / n_cv if n_cv else None)}},
               "gpu_launches": n_mm + n_cv,
               "e2e": {"value": flops / (statistics.mean(e_ms) * 1e-3) * 1e-12, "unit": "TFLOP/s",
                       "h2d_bytes_per_step": ha.numel() * 2, "d2h_bytes_per_step": hc.numel() * 2,
                       "ms_per_step": statistics.mean(e_ms)},
               "l2": "flushed between steps" if flush is not None else "inputs larger than L2"}
        t_gpu = time.perf_counter()
        if cpu_s > 0:
            res["cpu_baseline"] = cpu_weights_baseline(name, M, K, N, kind, a, w, cpu_s)
        print(f"[bench] weights {name}: gpu {t_gpu - t_start:.1f} s, cpu {time.perf_counter() - t_gpu:.1f} s",
              file=sys.stderr, flush=True)
        out[name] = res
        del a, w, c, flush
    return out


def profile_weights(name, n, device):
    """n untimed calls of one weight-product case: the target of ncu captures."""
    import torch

    import aihost_b200 as A
    from aihost_b200 import gen
    from aihost_b200.ops import Context, WeightOps

    case = {c[0]: c for c in WEIGHT_CASES}[name]
    _, M, K, N, kind, _, _ = case
    with Context(device.index) as ctx:
        ops = WeightOps(ctx)
        a = gen.normal((M, K), 99, name + ".a", dtype=torch.float16, device=device)
        w = (gen.normal((N, K), 99, name + ".w", std=0.02, dtype=torch.float16, device=device) if kind == "F16"
             else gen.kquant_blocks(getattr(A, kind), N * K // 256, 99, name + ".w", device=device))
        for _ in range(n):
            c = ops.mat_mul_weights(a, w, getattr(A, kind), N)
        torch.cuda.synchronize()
        ctx.sync_status()
        print(f"profiled {name}: {n} calls, mean |c| {c.float().abs().mean().item():.4f}")


def cpu_weights_baseline(name, M, K, N, kind, a, w, target_s):
    """The reference's per-call work on the host cores (oracle, faithful fp32): dequantise the
    whole weight (K-quants; ComputeOps.DequantizeInto runs on every call) and MatMulWeights over
    a bounded sample of rows, repeated to about target_s; scaled to the whole product."""
    import numpy as np

    import aihost_b200 as A
    from oracle import oracle as orc

    a_np = a[: min(M, 64)].float().cpu().numpy()
    w_np = w.cpu().numpy()

    def run(rows):
        t = time.perf_counter()
        wf = (w_np.astype(np.float32) if kind == "F16"
              else orc.dequantize(getattr(A, kind), w_np, N * K)).reshape(N, K)
        t_dq = time.perf_counter() - t
        t = time.perf_counter()
        orc.matmul_weights(a_np[:rows], wf, mode=orc.FAITHFUL)
        return t_dq, time.perf_counter() - t

    rows = 1
    t_dq, t_mm = run(rows)
    rows = int(max(1, min(a_np.shape[0], round(target_s / 2 / max(t_mm, 1e-4)))))
    t_dq, t_mm = run(rows)
    per_call = (t_dq if kind != "F16" else 0.0) + t_mm * M / rows
    return {"value": 2.0 * M * N * K / per_call * 1e-12, "unit": "TFLOP/s", "cores": orc.num_threads(), "kind": "port",
            "sample": f"{rows}/{M} rows of MatMulWeights (faithful fp32 oracle) scaled to all rows"
                      + (", plus one full dequantisation of the weight" if kind != "F16" else ""),
            "seconds": round(t_dq + t_mm, 3)}


def bench_qk_norm(args, device, pk, pk_kind):
    """aihost_qk_norm_rope on a Qwen TypeB-shaped Q block larger than L2: 32768 token rows of
    16 heads x 256, fp16, in place. Algorithmic bytes per launch: the block read and written once."""
    import torch

    from aihost_b200.ops import ComputeOps, Context

    seq, heads, d, theta = 32768, 16, 256, 1e7
    g = torch.Generator(device=device).manual_seed(1234)
    x = torch.randn(seq, heads * d, device=device, generator=g).half()
    w = (1.0 + 0.1 * torch.randn(d, device=device, generator=g)).float()
    nbytes = 2 * x.numel() * x.element_size()
    clocks = ClockSampler(device.index).start()
    with Context(device.index) as ctx:
        ops = ComputeOps(ctx)
        for _ in range(args.warmup):
            ops.qk_norm_rope(x, w, 0, heads, d, theta)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in ev:
            a.record()
            ops.qk_norm_rope(x, w, 0, heads, d, theta)
            b.record()
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
        hx = x.cpu().pin_memory()
        e_ms = []
        for i in range(args.steps + args.warmup):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            x.copy_(hx, non_blocking=True)
            ops.qk_norm_rope(x, w, 0, heads, d, theta)
            hx.copy_(x, non_blocking=True)
            b.record()
            b.synchronize()
            if i >= args.warmup:
                e_ms.append(a.elapsed_time(b))
        ctx.sync_status()
    clk = clocks.stop()
    gbs = nbytes / (ms * 1e-3) * 1e-9
    cpu = None
    if not args.no_cpu:
        from oracle import oracle as orc

        rows = 512
        xs = x[:rows].float().cpu().numpy()
        wn = w.cpu().numpy()
        t0 = time.perf_counter()
        runs = 0
        while True:
            orc.qk_norm_rope(xs, wn, 0, heads, d, theta)
            runs += 1
            if time.perf_counter() - t0 > min(args.cpu_seconds, 5.0):
                break
        t = time.perf_counter() - t0
        cpu = {"value": runs * rows * heads * d * 2 * 2 / t * 1e-9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{rows} token rows x {heads} heads x {d}, {runs} run(s) (oracle, single-threaded fp32; "
                         "bytes counted at the fp16 sizes)"}
    line = {"metric": "Qwen TypeB Q/K norm + RoPE prologue, HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 (fp32 math)", "data": "synthetic (torch normal)",
            "config": {"workload": "aihost_qk_norm_rope on x [32768, 16*256] fp16, in place, theta 1e7",
                       "l2": "inputs larger than L2 (268 MB per step)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / pk["hbm_gbs"], "traffic": None, "kernel": "qk_norm_rope_kernel",
                         "kernel_ms": ms, "algorithmic_per_launch": nbytes, "peak_source": f"{pk_kind} copy"},
            "cpu_baseline": cpu,
            "e2e": {"value": nbytes / (statistics.mean(e_ms) * 1e-3) * 1e-9, "unit": "GB/s",
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                    "ms_per_step": statistics.mean(e_ms)},
            "gpu_launches": args.steps, "clocks": clk}
    print(json.dumps(line), flush=True)


def config_object(cfg, shard_mode, args, device, ctx, dist_on, ws, rank, pk, pk_kind, cpu_s, layers=0):
    """One config's measurements as a JSON object: the device-timed value, the dominant kernel's
    roofline, the end-to-end value through the C ABI with host buffers, and (rank 0, N = 1) the
    CPU baseline and, for decode configs with `layers`, the rotating-cache throughput."""
    t_start = time.perf_counter()
    steps = args.steps if cfg.n_new > 1 else max(args.steps, 10)
    r = bench_ours(cfg, steps, args.warmup, device, ctx, 512 << 20, dist_on, shard_mode=shard_mode,
                   paged=args.paged)
    res = summarize(cfg, r, ws, dist_on, pk, pk_kind)
    res["config"] = cfg_desc(cfg, shard_mode, ws, r.get("rank_rows"))
    res["scaling"] = "strong" if (ws > 1 and shard_mode != "seq") else "weak"
    res["dtype"] = "f32" if cfg.q_dtype == 0 else "f16 (fp32 accumulate)"
    kern_ms = sum(v["mean_ms"] or 0.0 for v in res["kernels"].values() if v["launches"])
    if ws > 1 and shard_mode != "seq":
        # the step time this library's kernels do not cover (NCCL plus launch gaps; 0 when the
        # kernels' own overlap hides it), and an all-gather of the same bytes timed alone
        res["step_minus_kernels_ms"] = max(0.0, res["ms_per_step"] - max_over_ranks(kern_ms, dist_on))
        out_elem = 4 if cfg.q_dtype == 0 else 2
        res["collective_ms"] = time_allgather(cfg.batch * cfg.n_new * (cfg.n_q_heads // ws) * cfg.head_dim * out_elem,
                                              ws, device, max(args.steps, 10), args.warmup, dist_on)
    if layers > 0 and cfg.n_new == 1 and ws == 1:
        l_ms, l_bytes = bench_layers(cfg, layers, max(args.steps, 10), args.warmup, device, ctx)
        res["layers"] = {"layers": layers, "ms_per_step": l_ms, "tokens_per_s": cfg.batch * layers / (l_ms * 1e-3),
                         "kv_read_gbs": l_bytes / (l_ms * 1e-3) * 1e-9,
                         "frac_of_measured_hbm": l_bytes / (l_ms * 1e-3) * 1e-9 / pk["hbm_gbs"],
                         "note": "one CUDA graph of `layers` fused calls on distinct caches (together larger than "
                                 "L2, so the bytes come from HBM), replayed per step; bytes = algorithmic bytes of "
                                 "every layer's call"}
    t_gpu = time.perf_counter()
    if rank == 0 and ws == 1 and cpu_s > 0:
        res["cpu_baseline"] = cpu_baseline(cfg, cpu_s)
    if rank == 0:
        print(f"[bench] config {cfg.number} ({shard_mode}): gpu legs {t_gpu - t_start:.1f} s, cpu baseline "
              f"{time.perf_counter() - t_gpu:.1f} s", file=sys.stderr, flush=True)
    return res


def main():
    args = parse_args()
    if args.warmup < 3:
        args.warmup = 3
    dist_on, rank, local, ws = init_dist(args)
    if args.impl == "reference":
        run_reference(args)
        if dist_on:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    import torch

    from aihost_b200.configs import CONFIGS
    from aihost_b200.ops import Context

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.profile_steps and args.profile_weights:
        profile_weights(args.profile_weights, args.profile_steps, device)
        return
    if args.profile_steps:
        pcfg = CONFIGS[args.config]
        if args.profile_new:
            pcfg = pcfg.scaled(n_new=args.profile_new)
        profile_steps(pcfg, args.profile_steps, device)
        return
    pk, pk_kind = peaks()
    if args.op == "qk-norm-rope":
        if ws == 1:
            bench_qk_norm(args, device, pk, pk_kind)
        return
    ctx = Context(local)
    clocks = ClockSampler(local).start()
    cfg = CONFIGS[args.config]
    cpu_main = 0.0 if args.no_cpu else args.cpu_seconds
    main_res = config_object(cfg, args.shard, args, device, ctx, dist_on, ws, rank, pk, pk_kind, cpu_main,
                             layers=args.layers)
    # The default run (config 2 headline) measures every other BASELINE config too: config 1
    # (fp32 decode; with 256 rotating layer caches at N = 1), config 3 (batched fp16 decode), and
    # configs 4 and 5 with their KV heads split over the ranks (one NCCL all-gather of the head
    # outputs) at N > 1, as the workload names them.
    extra = {}
    if args.config == 2 and not args.no_decode:
        cpu_other = 0.0 if args.no_cpu else min(args.cpu_seconds, 6.0)
        plan = [(1, "seq", 256), (3, "seq", 0), (4, "heads" if ws > 1 else "seq", 0),
                (5, "heads" if ws > 1 else "seq", 0)]
        for number, mode, layers in plan:
            extra[f"config_{number}"] = config_object(CONFIGS[number], mode, args, device, ctx, dist_on, ws, rank,
                                                      pk, pk_kind, cpu_other, layers=layers if ws == 1 else 0)
        if ws == 1:  # the weight products around the op (one GPU; they do not shard here)
            extra["weights"] = bench_weights(args, device, ctx, pk, pk_kind, 0.0 if args.no_cpu else 3.0)
    clk = clocks.stop()
    if rank == 0:
        line = {"metric": METRIC, "value": main_res["value"], "unit": main_res["unit"], "n_gpus": ws,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": main_res["ms_per_step"],
                "higher_is_better": True, "scaling": main_res["scaling"], "vs_baseline": None,
                "dtype": main_res["dtype"], "data": "synthetic (seeded SplitMix64 + Box-Muller, no model weights)",
                "config": main_res["config"], "roofline": main_res["roofline"],
                "cpu_baseline": main_res.get("cpu_baseline"), "e2e": main_res["e2e"],
                "kv_layout": (f"paged: {args.paged}-row pages of a shared pool, shuffled order, block table"
                              if args.paged else "contiguous per sequence"),
                "gpu_launches": main_res["gpu_launches"], "clocks": clk, "kernels": main_res["kernels"]}
        for key in ("layers", "collective_ms", "step_minus_kernels_ms", "kv_read_gbs", "kv_read_frac_of_8tbs"):
            if key in main_res:
                line[key] = main_res[key]
        line.update(extra)
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist_on:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
