#!/usr/bin/env python3
"""Benchmark: moe-stream's MoE expert block on B200 -- MoE-block tok/s and
expert-weight HBM GB/s against the measured peak, at 1/2/4/8 GPUs.

Default workload (N=1): a Qwen3-30B-A3B-shape 48-layer expert stack at
batch-1 decode -- 6144 experts in a pinned host store, a 3072-slot HBM pool
with LFU eviction and next-layer router prefetch, Zipf(1.1)-skewed routers.
One step = one decoded token = 48 MoE block calls (router, device slot-table
step, fills, expert kernels), replayed from a CUDA graph with every input
already in HBM. Before the timed steps the pool is brought to its steady
state (untimed tokens until the trailing cache-hit rate reaches 0.97). The
e2e figure replays the same tokens from a checkpoint of the same pool state,
with each token's inputs copied in from pinned host memory and its outputs
copied back.

Every run also measures the sharded configuration -- one gpt-oss layer on
16384 tokens with its 128 experts spread over the N GPUs, NCCL all-to-all
dispatch and combine -- and reports it under "expert_parallel".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank runs its own decode replica (decode does
not shard); value is the sum over replicas of tokens / the slowest rank's
time. ``--impl reference`` times the CPU port of the same decode path on the
host cores (the reference's MLX implementation is not installable here).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-block decode tok/s (Qwen3-30B-A3B shape, 48 layers, batch 1)"
WORKLOAD = ("config1: qwen3 48-layer expert stack, batch-1 decode, 3072 of 6144 experts "
            "resident, LFU, next-layer prefetch (depth 1), Zipf(1.1) router bias")
N_LAYERS, N_SLOTS, SEED = 48, 3072, 0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="host time spent on the CPU baseline sample")
    ap.add_argument("--hit-target", type=float, default=0.97,
                    help="trailing cache-hit rate that ends the untimed pre-roll")
    ap.add_argument("--preroll-max", type=int, default=1024,
                    help="most untimed pre-roll tokens")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the expert-parallel measurement of the default run")
    ap.add_argument("--no-mixed", action="store_true",
                    help="skip the per-expert mixed-precision decode measurement")
    ap.add_argument("--no-fused", action="store_true",
                    help="skip the fused norm + block + residual decode measurement")
    ap.add_argument("--case", choices=["stack", "layer", "prefill", "ep", "fill", "stack3"], default="stack",
                    help="layer: a 2-layer Qwen3 stack with every expert resident (a small "
                         "case for ncu section captures); prints per-call timings only. "
                         "prefill: one MoE layer on a large token batch (qwen3 T=4096, "
                         "gptoss T=512 or 16384), the grouped tcgen05 GEMM path. ep: only "
                         "the expert-parallel measurement (gpt-oss layer, T=16384, experts "
                         "sharded over the ranks under torchrun). fill: host->HBM slot fill "
                         "bandwidth, SM loads (k_fill) against the copy engine. stack3: config 3's "
                         "36-layer gpt-oss decode stack")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1,
                    help="stack case: tokens per decode step (a multi-token verify batch); "
                         "each token its own hidden-state sequence")
    ap.add_argument("--model", choices=["qwen3", "gptoss"], default="qwen3")
    ap.add_argument("--no-replicas", action="store_true",
                    help="expert parallelism: plain sharding, no replicas of hot experts")
    return ap.parse_args()


def layer_case(args):
    """Layer 0 of a 2-layer Qwen3 stack, all 256 experts resident (680 MB
    arena), next-layer prediction on, T tokens per call, repeated block
    calls. For profiling captures."""
    import torch
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    torch.cuda.set_device(0)
    geom = geometry.qwen3(2)
    pool = ExpertPool(geom, geom.n_keys, depths=(1,), max_tokens=max(1, args.tokens or 1))
    st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
    for layer in range(2):
        st[layer * 128:(layer + 1) * 128].copy_(S.make_layer_blobs(geom, SEED, layer))
    blocks = [MoEBlock(pool, l, *S.router_weights(geom, SEED, l, zipf_s=1.1)) for l in range(2)]
    T = args.tokens or 1
    n = args.warmup + args.steps
    x = S.decode_inputs(n * T, 1, geom.d_model, SEED).cuda().reshape(-1, geom.d_model)
    for i in range(args.warmup):
        blocks[0](x[i * T:(i + 1) * T])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.warmup, n):
        blocks[0](x[i * T:(i + 1) * T])
    e1.record()
    torch.cuda.synchronize()
    pool.status()
    print(json.dumps({"case": "layer", "tokens": T, "calls": args.steps,
                      "us_per_call": e0.elapsed_time(e1) * 1e3 / args.steps}))
    pool.close()


def gptoss_stack_case(args):
    """Config 3's decode stack: 36 gpt-oss-shape layers (d = ff = 2880, top-4
    of 128, projection biases, clamped SwiGLU), 2304 of 4608 experts
    resident, LFU, next-layer prefetch, batch 1; Zipf(1.1) router biases and
    the config-1 hidden-state process (the config fixes neither). Same
    method as the default line: steady-state pre-roll, CUDA-graph token
    replay timed with CUDA events, per-layer intervals by events for the
    expert kernels' roofline. 32 GB arena, 65 GB pinned store."""
    import ctypes
    import torch
    from moe_stream_b200 import _lib, geometry, store as S
    from moe_stream_b200.block import DecodeGraph, MoEBlock
    from moe_stream_b200.pool import ExpertPool
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    L, n_slots = 36, 2304
    geom = geometry.gptoss(L)
    pool = ExpertPool(geom, n_slots, evict="lfu", depths=(1,), pf_widen=1, max_tokens=1)
    st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
    t_gen = time.perf_counter()
    for layer in range(L):
        st[layer * 128:(layer + 1) * 128].copy_(S.make_layer_blobs(geom, SEED, layer, device=dev))
    torch.cuda.synchronize()
    t_gen = time.perf_counter() - t_gen
    routers = [S.router_weights(geom, SEED, l, zipf_s=1.1) for l in range(L)]
    blocks = [MoEBlock(pool, l, w, b) for l, (w, b) in enumerate(routers)]
    K, W, PR = args.steps, args.warmup, args.preroll_max
    X = S.decode_inputs(PR + W + K + 16, L, geom.d_model, SEED + 1).to(dev)
    for l, b in enumerate(blocks):
        b(X[0, l:l + 1])
    torch.cuda.synchronize()
    g = DecodeGraph(blocks)
    used, hist, roll = 1, [pool.stats()], 0.0
    while used < PR:
        for t in range(used, min(PR, used + 16)):
            g.step(X[t].unsqueeze(1))
        used = min(PR, used + 16)
        hist.append(pool.stats())
        back = hist[max(0, len(hist) - 3)]
        roll = (hist[-1]["cache"] - back["cache"]) / max(1, hist[-1]["total"] - back["total"])
        if used >= 64 and roll >= args.hit_target:
            break
    for t in range(used, used + W):
        g.step(X[t].unsqueeze(1))
    t0 = used + W
    torch.cuda.synchronize()
    s0 = pool.stats()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(t0, t0 + K):
        g.step(X[t].unsqueeze(1))
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    pool.status()
    s1 = pool.stats()
    d = {k: s1[k] - s0[k] for k in ("total", "prefetch", "cache", "miss")}
    _lib.check(pool._lib.ms_pool_profile(pool._h, 1))
    gp = DecodeGraph(blocks)
    acc = [0.0, 0.0, 0.0]
    buf = (ctypes.c_float * 3)()
    for t in range(t0 + K, t0 + K + 16):
        gp.step(X[t].unsqueeze(1))
        torch.cuda.synchronize()
        for layer in range(L):
            _lib.check(pool._lib.ms_pool_timing(pool._h, layer, buf))
            for i in range(3):
                acc[i] += buf[i] / (16 * L)
    _lib.check(pool._lib.ms_pool_profile(pool._h, 0))
    peaks, peak_kind = measured_peaks()
    bytes_per_layer = geom.top_k * geom.payload_bytes
    achieved = bytes_per_layer / (acc[2] * 1e-3) / 1e9
    print(json.dumps({
        "case": "stack3", "metric": "MoE-block decode tok/s (gpt-oss-120b shape, 36 layers, batch 1)",
        "value": K / (ms / 1e3), "unit": "tok/s", "steps": K, "warmup": W, "ms_per_step": ms / K,
        "config": {"workload": "config3: gpt-oss 36-layer expert stack, batch-1 decode, 2304 of 4608 "
                               "experts resident, LFU, next-layer prefetch, Zipf(1.1) router bias",
                   "n_layers": L, "n_slots": n_slots},
        "hit_rate": {"cache": d["cache"] / max(1, d["total"]),
                     "resident_at_acquire": (d["cache"] + d["prefetch"]) / max(1, d["total"]),
                     "h2d_fill_bytes_per_token": (s1["gb"] - s0["gb"]) * 2 ** 30 / K,
                     "preroll_tokens": used, "preroll_window_cache_hit": roll},
        "expert_bytes_per_token": bytes_per_layer * L,
        "per_layer_us": {"router_table": acc[0] * 1e3, "fill": acc[1] * 1e3, "experts": acc[2] * 1e3},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind,
                     "kernel": "k_up + k_down (expert MLP of one layer)",
                     "algorithmic_bytes_per_launch": bytes_per_layer},
        "setup_s": {"store_generation": t_gen}}))
    del gp, g
    pool.close()


def fill_case(args):
    """Host -> HBM slot fills, the two ways the library has them: k_fill
    (32 CTAs reading the mapped pinned store with SM loads, the path block
    calls use, driven by the device slot table) and cudaMemcpyAsync on the
    copy engine (ms_pool_read, one call per blob, issued by the host). Same
    64 Qwen3 blobs (170 MB) into empty slots each way, CUDA events around
    each batch; prints GB/s for both."""
    import torch
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.pool import ExpertPool
    torch.cuda.set_device(0)
    geom = geometry.qwen3(1)
    n = 64
    out = {"case": "fill", "blobs": n, "blob_bytes": geom.blob_bytes}
    import numpy as np
    # a host array the caller owns, registered (page-locked, mapped) by each pool
    host = np.empty(geom.n_keys * geom.blob_bytes, np.uint8)
    torch.from_numpy(host).view(geom.n_keys, geom.blob_bytes).copy_(S.make_layer_blobs(geom, SEED, 0).cpu())
    res = {"k_fill": [], "copy_engine": []}
    for rep in range(args.warmup + args.steps):
        for how in ("k_fill", "copy_engine"):
            pool = ExpertPool(geom, geom.n_experts, depths=(), max_tokens=1)
            pool.attach_store(host)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if how == "k_fill":
                pool.prefetch(0, list(range(n)))      # one table step + one k_fill of n blobs
            else:
                for e in range(n):
                    pool._read(e, 0, e)
            e1.record()
            torch.cuda.synchronize()
            pool.status()
            if rep >= args.warmup:
                res[how].append(n * geom.blob_bytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
            pool.close()
    for how, v in res.items():
        out[how + "_gbs"] = float(statistics.median(v))
    print(json.dumps(out))


def prefill_case(args):
    """One MoE layer on a large batch on one GPU (Qwen3 T=4096, gpt-oss T=512 or 16384): T tokens routed
    over 128 resident experts (the pool holds the whole layer), grouped
    tcgen05 GEMMs. A step is one block call on T tokens."""
    import ctypes
    import torch
    from moe_stream_b200 import _lib, geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    torch.cuda.set_device(0)
    model = args.model
    T = args.tokens or (4096 if model == "qwen3" else 512)
    geom = geometry.qwen3(1) if model == "qwen3" else geometry.gptoss(1)
    E = geom.n_experts
    pool = ExpertPool(geom, E, depths=(), max_tokens=T)
    st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
    st.copy_(S.make_layer_blobs(geom, SEED, 0).cpu())
    zipf = 1.1 if (model == "qwen3" or T >= 16384) else None
    w, b = S.router_weights(geom, SEED, 0, zipf_s=zipf)
    blk = MoEBlock(pool, 0, w, b)
    W, K = max(3, args.warmup), args.steps
    xs = [S.rms_norm_tokens(T, geom.d_model, seed=SEED + 100 + i, device="cuda") for i in range(2)]
    y = torch.empty_like(xs[0])
    for i in range(W):
        blk(xs[i % 2], out=y)
    torch.cuda.synchronize()
    pool.status()
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        blk(xs[i % 2], out=y)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    pool.status()
    ms = e0.elapsed_time(e1) / K
    # expert phase (scatter, two grouped GEMMs, combine) timed by the
    # library's own events around it
    _lib.check(pool._lib.ms_pool_profile(pool._h, 1))
    buf = (ctypes.c_float * 3)()
    acc = [0.0, 0.0, 0.0]
    n_prof = max(3, min(K, 10))
    for i in range(n_prof):
        blk(xs[i % 2], out=y)
        torch.cuda.synchronize()
        _lib.check(pool._lib.ms_pool_timing(pool._h, 0, buf))
        for j in range(3):
            acc[j] += buf[j] / n_prof
    _lib.check(pool._lib.ms_pool_profile(pool._h, 0))
    flops = 2.0 * T * geom.top_k * 3 * geom.d_model * geom.d_ff
    peaks, peak_kind = measured_peaks()
    achieved = flops / (acc[2] * 1e-3) / 1e12
    # e2e: pinned host tokens in, block, pinned host result out
    xh = xs[0].cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(xs[0])
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        xd.copy_(xh, non_blocking=True)
        blk(xd, out=y)
        yh.copy_(y, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    pool.status()
    cpu = None
    if not args.no_cpu_baseline:
        cpu = prefill_cpu_baseline(geom, st, w, b, xs[0], model, n_tok=16)
    cfg = {"qwen3": "config2: qwen3 layer, 128 experts resident, top-8",
           "gptoss": "config3/4 (1 GPU): gpt-oss layer, 128 experts resident, top-4"}[model]
    line = {
        "metric": "MoE-block prefill tok/s (one layer, grouped tcgen05 GEMM)",
        "value": T / (ms * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u4 weights as exact fp16 hi+lo pairs x fp16 tokens, f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, MLX affine 4-bit g64; N(0,1) RMS-normed tokens)",
        "config": {"workload": cfg, "tokens": T, "top_k": geom.top_k, "d_model": geom.d_model,
                   "d_ff": geom.d_ff, "router_bias": "Zipf(1.1)" if zipf else "none",
                   "l2": "inputs larger than L2: %.0f MB of expert weights" % (E * geom.payload_bytes / 1e6)},
        "per_call_us": {"router_table": acc[0] * 1e3, "fill": acc[1] * 1e3, "experts": acc[2] * 1e3},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": None,
                     "peak_kind": peak_kind,
                     "kernel": "expert phase: scatter + k_gemm<0> + k_gemm<1> + combine",
                     "algorithmic_flops_per_launch": flops,
                     "note": "algorithmic flops count one MMA pass; the exact hi+lo split runs two"},
        "cpu_baseline": cpu,
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": int(xh.numel() * 2), "d2h_bytes_per_step": int(yh.numel() * 2),
                "path": "MoEBlock.__call__ (ms_moe_block), pinned host x in / y out"},
        "gpu_launches": 7 * K,
        "clocks": clk,
    }
    print(json.dumps(line))
    pool.close()


def prefill_cpu_baseline(geom, st, w, b, x, model, n_tok):
    """The oracle on the first n_tok tokens of the batch (routing + every
    routed expert of those tokens), scaled to tok/s."""
    import numpy as np
    from oracle import moe as OM
    comps = [dict(c) for c in geom.components]
    xn = x[:n_tok].float().cpu().numpy()
    t0 = time.perf_counter()
    f = lambda t: None if t is None else t.float().numpy()
    if model == "qwen3":
        inds, scores, _ = OM.route_qwen3(xn, f(w), geom.top_k, True, f(b))
    else:
        inds, scores, _ = OM.route_gptoss(xn, f(w), geom.top_k, f(b))
    blobs = {int(e): st[int(e)].numpy() for e in np.unique(inds)}
    OM.expert_block(xn, inds, scores, blobs, comps, model)
    dt = time.perf_counter() - t0
    return {"value": n_tok / dt, "unit": "tok/s", "cores": len(os.sched_getaffinity(0)), "kind": "port",
            "sample": f"{n_tok} tokens of the batch ({dt:.1f} s): routing and every routed expert"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks/throttle reasons, sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) >= 8 and r[1].replace(".", "").isdigit()]
        if not sm:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 8
                          for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.rows[0][2]),
                "samples": len(sm), "reasons": reasons}


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ---------------------------------------------------------- expert parallel
EP_TOKENS = 16384
EP_WORKLOAD = ("config4: gpt-oss layer (d=ff=2880, top-4 of 128, Zipf(1.1) router bias) on "
               "T=16384 tokens, experts sharded over the ranks, NCCL all-to-all dispatch/combine")


def ep_measure(args, world, rank, dev, steps, warmup):
    """The gpt-oss layer on T tokens (default 16384) with its 128 experts
    sharded over the ranks (one rank: the whole layer on one GPU, the same
    block without the exchange). Every rank routes its T/world tokens; a
    step is one expert-parallel block on every rank (route, pack, all-to-all
    out, local grouped GEMMs, all-to-all back, combine), timed on the device
    as the max over ranks. Returns the measurement dict (every rank)."""
    import torch
    import torch.distributed as dist
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.ep import (DeviceOps, ep_forward, load_local_experts, plan_placement,
                                    routed_counts)
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.gptoss(1)
    T = args.tokens or EP_TOKENS
    if T % world or geom.n_experts % world:
        raise SystemExit(f"T={T} and {geom.n_experts} experts must split over {world} ranks")
    Tr = T // world
    base = geom.n_experts // world
    spare = 0 if (world == 1 or args.no_replicas) else base // 2
    pool = ExpertPool(geom, base + spare, depths=(), max_tokens=T if world == 1 else T)
    st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
    st.copy_(S.make_layer_blobs(geom, SEED, 0, device=dev).cpu())
    w, b = S.router_weights(geom, SEED, 0, zipf_s=1.1)
    block = MoEBlock(pool, 0, w, b)
    xs = [S.rms_norm_tokens(T, geom.d_model, seed=SEED + 200 + i)[rank * Tr:(rank + 1) * Tr]
          .to(dev) for i in range(3)]
    rank_share = 1.0
    if world > 1:
        # placement from a calibration batch (not a timed one): hot experts
        # replicated into the spare slots, replicas balanced over the ranks
        counts = routed_counts(DeviceOps(block, world), xs[2])
        table, slots = plan_placement(counts, world, base + spare)
        load_local_experts(pool, 0, rank, world, slots[rank])
        ops = DeviceOps(block, world, placement=table)
        loads = [float(sum(counts[e] / table[e, 0] for e in r)) for r in slots]
        rank_share = max(loads) / max(1.0, sum(loads))
        fwd = lambda x: ep_forward(x, ops, world)
    else:
        load_local_experts(pool, 0, 0, 1)
        y1 = torch.empty_like(xs[0])
        fwd = lambda x: block(x, out=y1)
    xs = xs[:2]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    W, K = max(3, warmup), max(1, steps)
    for i in range(W):
        fwd(xs[i % 2])
    torch.cuda.synchronize()
    pool.status()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        fwd(xs[i % 2])
    e1.record()
    torch.cuda.synchronize()
    barrier()
    pool.status()
    ms = max_over_ranks(e0.elapsed_time(e1) / K)
    # e2e: pinned host tokens in, pinned host result out, every step
    xh = xs[0].cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(xs[0])
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        xd.copy_(xh, non_blocking=True)
        y = fwd(xd)
        yh.copy_(y, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ems = max_over_ranks(e0.elapsed_time(e1) / K)
    pool.status()
    flops = 2.0 * T * geom.top_k * 3 * geom.d_model * geom.d_ff
    peaks, peak_kind = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    out = {"workload": EP_WORKLOAD, "n_gpus": world, "tokens": T, "tokens_per_rank": Tr,
           "value": T / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms, "steps": K, "warmup": W,
           "scaling": "strong",
           "placement": {"slots_per_gpu": base + spare, "max_rank_share": rank_share},
           "roofline": {"bound": "tensor", "achieved": achieved,
                        "peak": peaks["bf16_tflops"] * world, "unit": "TFLOP/s",
                        "frac": achieved / (peaks["bf16_tflops"] * world), "peak_kind": peak_kind,
                        "algorithmic_flops_per_step": flops},
           "e2e": {"value": T / (ems * 1e-3), "unit": "tok/s",
                   "h2d_bytes_per_step": int(xh.numel() * 2 * world),
                   "d2h_bytes_per_step": int(yh.numel() * 2 * world)},
           "a2a_bytes_per_step": 2 * T * geom.top_k * geom.d_model * 2 if world > 1 else 0}
    if world > 1:
        # phase breakdown of one more step (device events at the phase marks)
        evs = []

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append((name, e))

        barrier()
        torch.cuda.synchronize()
        mark("start")
        ep_forward(xs[0], ops, world, mark=mark)
        torch.cuda.synchronize()
        phases = {evs[i][0]: evs[i - 1][1].elapsed_time(evs[i][1]) for i in range(1, len(evs))}
        ph = torch.tensor([phases[n] for n in phases], device=dev)
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        out["phase_ms_max_over_ranks"] = dict(zip(phases, [round(float(v), 3) for v in ph.tolist()]))
    pool.close()
    del st
    return out


def ep_case(args):
    """--case ep: only the expert-parallel measurement, as its own line."""
    import datetime
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300), device_id=dev)
    clocks = ClockSampler(local)
    clocks.start()
    ep = ep_measure(args, world, rank, dev, args.steps, args.warmup)
    clk = clocks.stop()
    if rank == 0:
        line = {"metric": "MoE-block expert-parallel prefill tok/s (gpt-oss layer, T=%d)" % ep["tokens"],
                "value": ep["value"], "unit": "tok/s", "n_gpus": world, "steps": ep["steps"],
                "warmup": ep["warmup"], "ms_per_step": ep["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "u4 weights as exact fp16 hi+lo pairs x fp16 tokens, f32 accumulate",
                "data": "synthetic (seeded N(0,0.02) weights, MLX affine 4-bit g64; N(0,1) RMS-normed tokens)",
                "config": {"workload": EP_WORKLOAD, "parallelism": f"ep{world}"},
                "roofline": dict(ep["roofline"], traffic=None), "cpu_baseline": None,
                "e2e": ep["e2e"], "gpu_launches": 12 * ep["steps"], "clocks": clk,
                "placement": ep["placement"]}
        if "phase_ms_max_over_ranks" in ep:
            line["phase_ms_max_over_ranks"] = ep["phase_ms_max_over_ranks"]
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------ CPU baseline
def cpu_threads():
    """Host threads the CPU legs use: every core this process may run on."""
    import torch
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return torch.get_num_threads()


def decode_cpu_baseline(geom, blob_of, routers, X, seconds):
    """The CPU port (oracle.torch_port: vectorised fp32 torch with MLX's bf16
    rounding points, the pool simulator and blob fills) on whole 48-layer
    tokens of the same workload, for about `seconds` (at least two tokens);
    tokens/s."""
    import torch
    from oracle.torch_port import DecodeStackCPU
    cores = cpu_threads()
    cpu = DecodeStackCPU(geom, blob_of, routers, N_SLOTS)
    cpu.step(X[0].float())                      # warm-up token
    n, t0 = 0, time.perf_counter()
    while n < 2 or (time.perf_counter() - t0 < seconds and n + 1 < X.shape[0]):
        cpu.step(X[1 + n].float())
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} whole tokens x {geom.n_layers} layers after one warm-up token "
                      f"({dt:.1f} s): router, speculation, pool simulator with blob fills, "
                      f"8 experts per layer (oracle.torch_port, fp32 torch on the host)"}


def _layer_store(geom):
    """blob_of(key) over a store generated layer by layer on first touch:
    the same blobs as the GPU arm (make_layer_blobs on a GPU) when one is
    present; without one (the CPU-only contract test), random 4-bit codes
    with N(0,0.02)-sized scales, which give the same amount of work."""
    import numpy as np
    import torch
    from moe_stream_b200 import store as S
    layers = {}
    gpu = torch.cuda.is_available()

    def cpu_blobs(n=32):
        g = torch.Generator().manual_seed(SEED * 31 + 7)
        out = torch.randint(0, 256, (n, geom.blob_bytes), dtype=torch.uint8, generator=g)
        for c in geom.components:
            if c["dtype"] == "BF16":
                v = (torch.rand(n, c["nbytes"] // 2, generator=g) * 0.01 + 0.001).to(torch.bfloat16)
                out[:, c["offset"]:c["offset"] + c["nbytes"]] = v.view(torch.uint8)
        return out.numpy()

    def blob_of(key):
        layer, e = divmod(int(key), geom.n_experts)
        if gpu:
            if layer not in layers:
                layers[layer] = S.make_layer_blobs(geom, SEED, layer, device="cuda").cpu().numpy()
            return layers[layer][e]
        if "cpu" not in layers:
            layers["cpu"] = cpu_blobs()
        return layers["cpu"][int(key) % layers["cpu"].shape[0]]

    return blob_of, ("the GPU arm's blobs (generated layer by layer on the GPU)" if gpu else
                     "32 random blobs of the same shapes reused for every key (no GPU here to "
                     "generate the GPU arm's blobs; the same work per token)")


def reference_arm(args):
    """--impl reference: the CPU port of the reference's decode block (MLX,
    the reference's own compute path, is not installable here). One step =
    one decoded token through all 48 layers on the host cores."""
    import torch
    from moe_stream_b200 import geometry, store as S
    from oracle.torch_port import DecodeStackCPU
    cores = cpu_threads()
    geom = geometry.qwen3(N_LAYERS)
    routers = [S.router_weights(geom, SEED, l, zipf_s=1.1) for l in range(N_LAYERS)]
    X = S.decode_inputs(args.warmup + args.steps, N_LAYERS, geom.d_model, SEED + 1)
    blob_of, data = _layer_store(geom)
    cpu = DecodeStackCPU(geom, blob_of, routers, N_SLOTS)
    for i in range(args.warmup):
        cpu.step(X[i].float())
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu.step(X[args.warmup + i].float())
    dt = time.perf_counter() - t0
    tok_s = args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 rounding points)",
            "data": "synthetic: " + data,
            "config": {"workload": WORKLOAD, "step": "one decoded token (48 block calls)"},
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} whole tokens after {args.warmup} warm-up tokens "
                                       f"(oracle.torch_port: router, speculation, pool simulator "
                                       f"with blob fills, experts in fp32 torch); MLX itself is not "
                                       f"installable on this image"},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def profile_traffic():
    """DRAM bytes (read + write) of one layer's expert kernels from the
    committed ncu summary, or None."""
    import re
    path = os.path.join(ROOT, "profiles", "expert_kernels_layer_full.md")
    try:
        m = re.search(r"traffic per layer \(k_up \+ k_down[^)]*\):\s*([0-9]+)\s*bytes", open(path).read())
    except OSError:
        return None
    return int(m.group(1)) if m else None


# -------------------------------------------------------------- GPU arm
def fused_measure(pool, blocks, routers, X, t0, K, dev):
    """Decode tokens through the fused block (ms_moe_block_fused: the
    layer's post-attention RMSNorm in the route step, the residual add in
    the combine) against the same block with the norm and the add as torch
    ops around it, both captured as CUDA graphs and replayed on the same
    tokens from the same pool checkpoint; CUDA events."""
    import torch
    from moe_stream_b200.block import MoEBlock
    L, d = len(blocks), X.shape[-1]
    eps = 1e-6
    g = torch.Generator().manual_seed(SEED + 5)
    norm_w = [(1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).to(dev) for _ in range(L)]
    fb = [MoEBlock(pool, l, w, b, norm_weight=norm_w[l], norm_eps=eps) for l, (w, b) in enumerate(routers)]
    h = torch.zeros(L, 1, d, dtype=torch.bfloat16, device=dev)
    out = torch.zeros_like(h)

    def fused_step():
        for l in range(L):
            fb[l].fused(h[l], out=out[l])

    def unfused_step():
        for l in range(L):
            hf = h[l].float()
            xn = ((hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
                  * norm_w[l]).to(torch.bfloat16)
            y = blocks[l](xn)
            out[l].copy_(h[l] + y)

    def capture(fn):
        fn()                                  # eager once (fills, allocations)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        pool.join(torch.cuda.current_stream(dev))
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.graph(graph, stream=s):
            fn()
            pool.join(s)
        torch.cuda.current_stream(dev).wait_stream(s)
        return graph

    res = {}
    snap = pool.save_state(with_arena=True)
    for name, fn in (("fused", fused_step), ("unfused_torch_norm_add", unfused_step)):
        graph = capture(fn)
        pool.load_state(snap, with_arena=True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for t in range(t0, t0 + K):
            h.copy_(X[t], non_blocking=True)
            pool.join(torch.cuda.current_stream(dev))
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        pool.status()
        res[name] = K / (e0.elapsed_time(e1) / 1e3)
        del graph
    pool.load_state(snap, with_arena=True)
    del snap
    torch.cuda.synchronize()
    # the pool's routers back to the main blocks' tensors (fb's go away)
    import ctypes
    from moe_stream_b200 import _lib
    for b in blocks:
        _lib.check(pool._lib.ms_set_router(
            pool._h, b._layer, ctypes.c_void_p(b.gate_weight.data_ptr()),
            ctypes.c_void_p(b.gate_bias.data_ptr()) if b.gate_bias is not None else None))
    return {"tok_s": res["fused"], "tok_s_norm_and_add_as_torch_ops": res["unfused_torch_norm_add"],
            "tokens": K, "what": "out = h + block(rms_norm(h) * w) per layer, 48 layers, CUDA graphs"}


MIXED_CLASSES = ((4, "bf16"), (4, "fp8"), (3, "fp8"), (2, "fp8"))
MIXED_FRACS = (0.30, 0.30, 0.25, 0.15)


def mixed_measure(args, dev, K, W):
    """The config-1 decode stack with per-expert precision classes: each
    (layer, expert) drawn into 4-bit bf16 / 4-bit fp8 / 3-bit fp8 / 2-bit
    fp8 scales with probabilities MIXED_FRACS (a seeded stand-in for the
    sensitivity-keyed allocation the reference plans: the weights here are
    random, so no expert is more sensitive than another). Same weights,
    routers, hidden states, pool size and steady-state pre-roll as the main
    line; reports tok/s and the expert bytes the kernels read per token."""
    import numpy as np
    import torch
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import DecodeGraph, MoEBlock, route
    from moe_stream_b200.pool import ExpertPool

    geom = geometry.qwen3(N_LAYERS)
    classes = [geometry.precision(geom, b, f) for b, f in MIXED_CLASSES]
    sg = geometry.slot_geometry(geom, classes)
    cok = np.random.default_rng(SEED + 77).choice(len(classes), size=geom.n_keys,
                                                  p=MIXED_FRACS).astype(np.uint8)
    pool = ExpertPool(sg, N_SLOTS, evict="lfu", depths=(1,), pf_widen=1, max_tokens=1)
    pool.set_precision(classes, cok)
    store = pool.alloc_store()
    st_t = torch.from_numpy(store).view(geom.n_keys, sg.blob_bytes)
    E = geom.n_experts
    for layer in range(N_LAYERS):
        blobs = S.make_layer_blobs_classes(sg, classes, cok[layer * E:(layer + 1) * E], SEED, layer,
                                           device=dev)
        st_t[layer * E:(layer + 1) * E].copy_(blobs)
        del blobs
    torch.cuda.synchronize()
    routers = [S.router_weights(geom, SEED, l, zipf_s=1.1) for l in range(N_LAYERS)]
    blocks = [MoEBlock(pool, l, w, b) for l, (w, b) in enumerate(routers)]
    PR = args.preroll_max
    X = S.decode_inputs(PR + W + K, N_LAYERS, geom.d_model, SEED + 1000 * 0).to(dev)
    for layer, b in enumerate(blocks):
        b(X[0, layer:layer + 1])
    torch.cuda.synchronize()
    g = DecodeGraph(blocks, T=1)
    used, hist, roll = 1, [pool.stats()], 0.0
    while used < PR:
        n = min(16, PR - used)
        for t in range(used, used + n):
            g.step(X[t].unsqueeze(1))
        used += n
        hist.append(pool.stats())
        back = hist[max(0, len(hist) - 3)]
        roll = (hist[-1]["cache"] - back["cache"]) / max(1, hist[-1]["total"] - back["total"])
        if used >= 64 and roll >= args.hit_target:
            break
    for t in range(used, used + W):
        g.step(X[t].unsqueeze(1))
    t0 = used + W
    torch.cuda.synchronize()
    pool.status()
    s0 = pool.stats()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for t in range(t0, t0 + K):
        g.step(X[t].unsqueeze(1))
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    pool.status()
    s1 = pool.stats()
    # bytes the expert kernels read: the payload of every routed expert's
    # class (routing only: ms_route leaves the pool untouched)
    pay = torch.tensor([classes[c].payload_bytes for c in cok], dtype=torch.float64, device=dev)
    nbytes = torch.zeros((), dtype=torch.float64, device=dev)
    for t in range(t0, t0 + K):
        for layer, b in enumerate(blocks):
            inds, _ = route(b, X[t, layer:layer + 1])
            nbytes += pay[layer * E + inds.long()].sum()
    bpt = float(nbytes.item()) / K
    uniform = N_LAYERS * geom.top_k * geom.payload_bytes
    frac = np.bincount(cok, minlength=len(classes)) / cok.size
    out = {"classes": [f"{b}-bit {f}" for b, f in MIXED_CLASSES],
           "class_fraction": [round(float(v), 4) for v in frac],
           "tok_s": K / (ms / 1e3), "ms_per_token": ms / K, "steps": K,
           "expert_bytes_per_token": bpt,
           "expert_bytes_per_token_uniform_4bit": uniform,
           "bytes_ratio_vs_uniform": bpt / uniform,
           "cache_hit": (s1["cache"] - s0["cache"]) / max(1, s1["total"] - s0["total"]),
           "h2d_fill_bytes_per_token": (s1["gb"] - s0["gb"]) * 2 ** 30 / K,
           "preroll_tokens": used,
           "kernels": "k_up_mx / k_down_mx (per-class decode kernels)"}
    pool.close()
    del store, st_t, X
    torch.cuda.empty_cache()
    return out


def gpu_arm(args):
    import ctypes
    import torch
    import torch.distributed as dist
    from moe_stream_b200 import _lib, geometry, store as S
    from moe_stream_b200.block import DecodeGraph, MoEBlock
    from moe_stream_b200.pool import ExpertPool

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(0)
    dev = torch.device(f"cuda:{torch.cuda.current_device()}")

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    geom = geometry.qwen3(N_LAYERS)
    TB = args.batch
    pool = ExpertPool(geom, N_SLOTS, evict="lfu", depths=(1,), pf_widen=1, max_tokens=TB)
    store = pool.alloc_store()
    st_t = torch.from_numpy(store).view(geom.n_keys, geom.blob_bytes)
    t_gen = time.perf_counter()
    for layer in range(N_LAYERS):
        blobs = S.make_layer_blobs(geom, SEED, layer, device=dev)
        st_t[layer * geom.n_experts:(layer + 1) * geom.n_experts].copy_(blobs)
        del blobs
    torch.cuda.synchronize()
    t_gen = time.perf_counter() - t_gen
    routers = [S.router_weights(geom, SEED, l, zipf_s=1.1) for l in range(N_LAYERS)]
    blocks = [MoEBlock(pool, l, w, b) for l, (w, b) in enumerate(routers)]

    W, K = args.warmup, args.steps
    PR = args.preroll_max
    n_prof = 16
    # [tokens, L, TB, d]: token i of a step follows its own sequence; pre-roll
    # tokens first, then warm-up, timed and profiling tokens
    X_cpu = torch.stack([S.decode_inputs(PR + W + K + n_prof, N_LAYERS, geom.d_model,
                                         SEED + rank + 1000 * i) for i in range(TB)], dim=2)
    X = X_cpu.to(dev)

    # one eager token before capture, then the graph
    for layer, b in enumerate(blocks):
        b(X[0, layer])
    torch.cuda.synchronize()
    pool.status()
    g = DecodeGraph(blocks, T=TB)

    # ---------------------------------------------- steady state pre-roll
    # untimed tokens until the cache-hit rate over a trailing window of 32
    # tokens reaches the target (the pool's steady state), at most PR
    window, used = 32, 1
    hist = [pool.stats()]
    roll_hit = 0.0
    while used < PR:
        n = min(16, PR - used)
        for t in range(used, used + n):
            g.step(X[t])
        used += n
        hist.append(pool.stats())
        back = hist[max(0, len(hist) - 1 - window // 16)]
        tot = hist[-1]["total"] - back["total"]
        roll_hit = (hist[-1]["cache"] - back["cache"]) / max(1, tot)
        if used >= 2 * window and roll_hit >= args.hit_target:
            break
    torch.cuda.synchronize()
    pool.status()
    t0 = used
    for t in range(t0, t0 + W):
        g.step(X[t])
    torch.cuda.synchronize()
    pool.status()
    t0 += W
    barrier()

    # ---------------------------------------------------------- timed
    snap = pool.save_state(with_arena=True)       # e2e replays the same tokens from here
    torch.cuda.synchronize()
    s0 = pool.stats()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for t in range(t0, t0 + K):
        g.step(X[t])
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    pool.status()
    s1 = pool.stats()
    y_value = g.y.clone()
    table_value = pool.table()
    ms_max = max_over_ranks(ms)
    tok_s = world * K * TB / (ms_max / 1e3)
    d = {k: s1[k] - s0[k] for k in ("total", "prefetch", "cache", "miss")}
    hit = {"cache": d["cache"] / max(1, d["total"]),
           "resident_at_acquire": (d["cache"] + d["prefetch"]) / max(1, d["total"]),
           "miss": d["miss"] / max(1, d["total"]),
           "h2d_fill_bytes_per_token": (s1["gb"] - s0["gb"]) * 2 ** 30 / K,
           "preroll_tokens": used, "preroll_window_cache_hit": roll_hit}

    # ------------------------ e2e: the same tokens from the same pool state
    pool.load_state(snap, with_arena=True)
    torch.cuda.synchronize()
    s2 = pool.stats()
    Xh = X_cpu[t0:t0 + K].pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(K):
        y = g.step(Xh[t])
        Yh[t].copy_(y, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ems = max_over_ranks(e0.elapsed_time(e1))
    pool.status()
    s3 = pool.stats()
    same = (torch.equal(Yh[K - 1].to(dev), y_value) and (pool.table() == table_value).all()
            and all(s3[k] - s2[k] == d[k] for k in d))
    del snap
    e2e_tok_s = world * K * TB / (ems / 1e3)
    e2e = {"value": e2e_tok_s, "unit": "tok/s",
           "h2d_bytes_per_step": int(Xh[0].numel() * 2), "d2h_bytes_per_step": int(Yh[0].numel() * 2),
           "path": "DecodeGraph over MoEBlock.__call__ (ms_moe_block), pinned host x in / y out",
           "same_tokens_and_pool_state_as_value": bool(same),
           "e2e_le_value": bool(e2e_tok_s <= tok_s)}

    # ------------------------------------- kernel timing (same kernels, events)
    _lib.check(pool._lib.ms_pool_profile(pool._h, 1))
    gp = DecodeGraph(blocks, T=TB)
    acc = [[0.0, 0.0, 0.0] for _ in range(N_LAYERS)]
    buf = (ctypes.c_float * 3)()
    for t in range(t0 + K, t0 + K + n_prof):
        gp.step(X[t])
        torch.cuda.synchronize()
        for layer in range(N_LAYERS):
            _lib.check(pool._lib.ms_pool_timing(pool._h, layer, buf))
            for i in range(3):
                acc[layer][i] += buf[i]
    _lib.check(pool._lib.ms_pool_profile(pool._h, 0))
    per_layer = [sum(acc[l][i] for l in range(N_LAYERS)) / (N_LAYERS * n_prof) for i in range(3)]
    expert_ms = per_layer[2]
    # the distinct experts a layer reads: top_k at batch 1, the union of the
    # tokens' picks otherwise (every acquired key of the timed steps)
    distinct = d["total"] / (K * N_LAYERS)
    bytes_per_layer = (geom.top_k if TB == 1 else distinct) * geom.payload_bytes
    peaks, peak_kind = measured_peaks()
    achieved = bytes_per_layer / (expert_ms * 1e-3) / 1e9
    del gp
    pool.status()

    # ------------------- the block fused with its layer's norm and residual
    # (same pool state and tokens for both; each layer's hidden state is the
    # residual stream h, out = h + block(rms_norm(h) * w))
    fused = None
    if TB == 1 and not args.no_fused:
        fused = fused_measure(pool, blocks, routers, X, t0, min(K, 64), dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and TB == 1:
        blob_of = lambda key: store[int(key) * geom.blob_bytes:(int(key) + 1) * geom.blob_bytes]
        cpu = decode_cpu_baseline(geom, blob_of, routers, X_cpu[:, :, 0], args.cpu_seconds)
    pool.close()
    del store, st_t, X
    torch.cuda.empty_cache()

    mixed = None
    if not args.no_mixed and TB == 1:
        mixed = mixed_measure(args, dev, max(3, min(K, 64)), max(3, min(W, 8)))

    ep = None
    if not args.no_ep and TB == 1:
        ep = ep_measure(args, world, rank, dev, max(3, min(K, 10)), 3)

    if rank == 0:
        line = {
            "metric": METRIC if TB == 1 else METRIC.replace("batch 1", f"batch {TB}"),
            "value": tok_s, "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u4 weights x f16 MMA, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, MLX affine 4-bit g64, Zipf(1.1) router "
                    "bias, h_{l+1} = h_l + 0.1 N(0,1) hidden states)",
            "config": {"workload": WORKLOAD, "n_layers": N_LAYERS, "n_slots": N_SLOTS,
                       "n_experts_total": geom.n_keys, "top_k": geom.top_k, "batch": TB,
                       "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
                       "steady_state": f"untimed pre-roll until the cache-hit rate over the last "
                                       f"{window} tokens >= {args.hit_target} (at most {PR} tokens)",
                       "l2": "inputs larger than L2: 1.02 GB of expert weights per step"},
            "hit_rate": hit,
            "expert_hbm_gbs": achieved,
            "expert_bytes_per_token": bytes_per_layer * N_LAYERS,
            "per_layer_us": {"router_table": per_layer[0] * 1e3, "fill": per_layer[1] * 1e3,
                             "experts": expert_ms * 1e3},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": profile_traffic() if TB == 1 else None,
                         "peak_kind": peak_kind,
                         "kernel": "k_up + k_down (expert MLP of one layer)",
                         "algorithmic_bytes_per_launch": bytes_per_layer,
                         "distinct_experts_per_layer": geom.top_k if TB == 1 else distinct},
            "cpu_baseline": cpu,
            "e2e": e2e,
            # per layer: route step, demand fill, k_up, k_down, and the
            # side-stream prefetch fill on every layer with a next layer
            "gpu_launches": (4 * N_LAYERS + (N_LAYERS - 1)) * K,
            "clocks": clk,
            "setup_s": {"store_generation": t_gen},
        }
        if fused is not None:
            line["fused_norm_residual"] = fused
        if mixed is not None:
            line["mixed_precision"] = mixed
        if ep is not None:
            line["expert_parallel"] = ep
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        reference_arm(args)
        return
    if args.case == "fill":
        fill_case(args)
        return
    if args.case == "stack3":
        gptoss_stack_case(args)
        return
    if args.case == "layer":
        layer_case(args)
        return
    if args.case == "prefill":
        prefill_case(args)
        return
    if args.case == "ep":
        ep_case(args)
        return
    gpu_arm(args)


if __name__ == "__main__":
    main()
