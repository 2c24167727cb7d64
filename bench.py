#!/usr/bin/env python3
"""Benchmark: moe-stream's MoE expert block on B200 (metric: MoE-block
"MoE-block tok/s and expert-weight HBM GB/s vs peak").

Default workload (N=1, the configuration the metric is quoted on): config 1,
a Qwen3-30B-A3B-shape 48-layer expert stack at batch-1 decode -- 6144 experts
in a pinned host store, a 3072-slot HBM pool with LFU eviction and
next-layer router prefetch, Zipf(1.1)-skewed routers. One step = one decoded
token = 48 MoE block calls (router, device slot-table step, fills, expert
kernels), replayed from a CUDA graph with every input already in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank runs its own replica (decode does not
shard); value is the sum over replicas of tokens / the slowest rank's time.
``--impl reference`` times the CPU restatement of the same path (the
reference's MLX implementation is not installable here) on a bounded sample.
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
    ap.add_argument("--cpu-sample-layers", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", choices=["stack", "layer", "prefill", "ep"], default="stack",
                    help="layer: a 2-layer Qwen3 stack with every expert resident (a small "
                         "case for ncu section captures); prints per-call timings only. "
                         "prefill: one MoE layer on a large token batch (config 2: qwen3, "
                         "T=4096; config 3: gptoss, T=512; config 4 on one GPU: gptoss, "
                         "T=16384), the grouped tcgen05 GEMM path. ep: config 4, the "
                         "gpt-oss layer on T=16384 tokens with its 128 experts sharded over "
                         "the ranks (run under torchrun), NCCL all-to-all dispatch/combine")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1,
                    help="stack case: tokens per decode step (a multi-token verify batch); "
                         "each token its own hidden-state sequence")
    ap.add_argument("--model", choices=["qwen3", "gptoss"], default="qwen3")
    ap.add_argument("--no-replicas", action="store_true",
                    help="ep: plain sharding, no replicas of hot experts")
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


def ep_case(args):
    """Expert parallelism: one gpt-oss layer on T tokens (default 16384), the
    tokens split evenly over the ranks and the 128 experts sharded 128/G per
    GPU; a step is one expert-parallel block (route, pack, all-to-all out,
    local grouped GEMMs, all-to-all back, combine) on every rank. Timed on the
    device, max over ranks."""
    import datetime
    import torch
    import torch.distributed as dist
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.ep import (DeviceOps, ep_forward, load_local_experts, plan_placement,
                                    routed_counts)
    from moe_stream_b200.pool import ExpertPool
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29541")
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300), device_id=dev)
    geom = geometry.gptoss(1)
    T = args.tokens or 16384
    if T % world or geom.n_experts % world:
        raise SystemExit(f"T={T} and {geom.n_experts} experts must split over {world} ranks")
    Tr = T // world
    base = geom.n_experts // world
    spare = 0 if (world == 1 or args.no_replicas) else base // 2
    pool = ExpertPool(geom, base + spare, depths=(), max_tokens=T)
    st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
    st.copy_(S.make_layer_blobs(geom, SEED, 0, device=dev).cpu())
    w, b = S.router_weights(geom, SEED, 0, zipf_s=1.1)
    block = MoEBlock(pool, 0, w, b)
    xs = [S.rms_norm_tokens(T, geom.d_model, seed=SEED + 200 + i)[rank * Tr:(rank + 1) * Tr]
          .to(dev) for i in range(3)]
    # placement from a calibration batch (not a timed one): hot experts
    # replicated into the spare slots, replicas balanced over the ranks
    counts = routed_counts(DeviceOps(block, world), xs[2])
    table, slots = plan_placement(counts, world, base + spare)
    load_local_experts(pool, 0, rank, world, slots[rank])
    ops = DeviceOps(block, world, placement=table)
    rank_load = [float(sum(counts[e] / table[e, 0] for e in r)) for r in slots]
    xs = xs[:2]
    W, K = max(3, args.warmup), args.steps
    for i in range(W):
        ep_forward(xs[i % 2], ops, world)
    torch.cuda.synchronize()
    pool.status()
    clocks = ClockSampler(local)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        ep_forward(xs[i % 2], ops, world)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    pool.status()
    ms = torch.tensor([e0.elapsed_time(e1) / K], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    # e2e: pinned host tokens in, pinned host result out, every step
    xh = xs[0].cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(xs[0])
    dist.barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        xd.copy_(xh, non_blocking=True)
        y = ep_forward(xd, ops, world)
        yh.copy_(y, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    ems = torch.tensor([e0.elapsed_time(e1) / K], device=dev)
    dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    ems = float(ems.item())
    pool.status()
    flops = 2.0 * T * geom.top_k * 3 * geom.d_model * geom.d_ff
    peaks, peak_kind = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    a2a_bytes = 2 * T * geom.top_k * geom.d_model * 2          # rows out and back, whole job
    # phase breakdown of one more step (device events at the phase marks)
    evs = []

    def mark(name):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        evs.append((name, e))

    dist.barrier()
    torch.cuda.synchronize()
    mark("start")
    ep_forward(xs[0], ops, world, mark=mark)
    torch.cuda.synchronize()
    phases = {evs[i][0]: evs[i - 1][1].elapsed_time(evs[i][1]) for i in range(1, len(evs))}
    ph = torch.tensor([phases[n] for n in phases], device=dev)
    dist.all_reduce(ph, op=dist.ReduceOp.MAX)
    phases = dict(zip(phases, [round(float(v), 3) for v in ph.tolist()]))
    if rank == 0:
        line = {
            "metric": "MoE-block expert-parallel prefill tok/s (gpt-oss layer, T=%d)" % T,
            "value": T / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "u4 weights as exact fp16 hi+lo pairs x fp16 tokens, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, MLX affine 4-bit g64; N(0,1) RMS-normed tokens)",
            "config": {"workload": "config4: gpt-oss layer, experts sharded %d per GPU, NCCL "
                                   "all-to-all dispatch/combine" % (geom.n_experts // world),
                       "placement": {"slots_per_gpu": base + spare, "replicas": int(table[:, 0].sum() - geom.n_experts),
                                     "max_rank_share": max(rank_load) / max(1.0, sum(rank_load))},
                       "tokens": T, "tokens_per_rank": Tr, "top_k": geom.top_k,
                       "router_bias": "Zipf(1.1)", "parallelism": f"ep{world}",
                       "l2": "inputs larger than L2: %.1f GB of expert weights per GPU"
                             % (geom.n_experts // world * geom.payload_bytes / 1e9)},
            "roofline": {"bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops"] * world, "unit": "TFLOP/s",
                         "frac": achieved / (peaks["bf16_tflops"] * world), "traffic": None,
                         "peak_kind": peak_kind, "kernel": "whole expert-parallel step",
                         "algorithmic_flops_per_step": flops,
                         "a2a_bytes_per_step": a2a_bytes},
            "cpu_baseline": None,
            "e2e": {"value": T / (ems * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": int(xh.numel() * 2 * world),
                    "d2h_bytes_per_step": int(yh.numel() * 2 * world),
                    "path": "ep.ep_forward on every rank, pinned host tokens in / result out"},
            "gpu_launches": 12 * K,
            "clocks": clk,
            "phase_ms_max_over_ranks": phases,
        }
        print(json.dumps(line))
    pool.close()
    dist.destroy_process_group()


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
    return {"value": n_tok / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
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


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(geom, store, routers, X, n_layers_sample):
    """The oracle (numpy restatement of the reference's block, MLX bf16
    rounding points) on one token over `n_layers_sample` layers, scaled to
    tokens/s of the 48-layer stack. Routing + expert math; the pool is
    irrelevant to the CPU path's arithmetic."""
    import numpy as np
    from oracle import moe as OM
    comps = [dict(c) for c in geom.components]
    t0 = time.perf_counter()
    for layer in range(n_layers_sample):
        x = X[0, layer:layer + 1].float().numpy()
        w, b = routers[layer]
        inds, scores, _ = OM.route_qwen3(x, w.float().numpy(), geom.top_k, True,
                                         b.float().numpy() if b is not None else None)
        base = layer * geom.n_experts
        blobs = {int(e): np.asarray(store[(base + int(e)) * geom.blob_bytes:
                                          (base + int(e) + 1) * geom.blob_bytes])
                 for e in inds[0]}
        OM.expert_block(x, inds, scores, blobs, comps, "qwen3")
    dt = time.perf_counter() - t0
    per_layer = dt / n_layers_sample
    return {"value": 1.0 / (per_layer * geom.n_layers), "unit": "tok/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 token x {n_layers_sample} of {geom.n_layers} layers "
                      f"({dt:.1f} s), scaled to the 48-layer stack"}


def reference_arm(args):
    """--impl reference: the CPU restatement of the reference's block (MLX is
    not installable here). One step = one (token, layer) block call."""
    import torch
    from moe_stream_b200 import geometry, store as S
    from oracle import moe as OM
    import numpy as np
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    geom = geometry.qwen3(N_LAYERS)
    routers = [S.router_weights(geom, SEED, l, zipf_s=1.1) for l in range(N_LAYERS)]
    X = S.decode_inputs(1, N_LAYERS, geom.d_model, SEED)
    comps = [dict(c) for c in geom.components]
    cache = {}

    def blob(layer, e):
        key = (layer, e)
        if key not in cache:
            cache[key] = S.make_blob(geom, SEED, layer, e).numpy()
        return cache[key]

    def step(i):
        layer = i % N_LAYERS
        x = X[0, layer:layer + 1].float().numpy()
        w, b = routers[layer]
        inds, scores, _ = OM.route_qwen3(x, w.float().numpy(), geom.top_k, True, b.float().numpy())
        blobs = {int(e): blob(layer, int(e)) for e in inds[0]}
        OM.expert_block(x, inds, scores, blobs, comps, "qwen3")

    # blobs are generated outside the timed region
    for i in range(args.warmup + args.steps):
        layer = i % N_LAYERS
        x = X[0, layer:layer + 1].float().numpy()
        w, b = routers[layer]
        inds, _, _ = OM.route_qwen3(x, w.float().numpy(), geom.top_k, True, b.float().numpy())
        for e in inds[0]:
            blob(layer, int(e))
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    tok_s = args.steps / (dt * N_LAYERS)
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32/bf16-rounded",
            "data": "synthetic", "config": {"workload": WORKLOAD, "step": "one (token, layer) block call"},
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": "oracle (numpy, MLX bf16 rounding points) block calls; "
                                       "MLX itself is not installable on this image"},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# -------------------------------------------------------------- GPU arm
def gpu_arm(args):
    import torch
    import torch.distributed as dist
    from moe_stream_b200 import geometry, store as S
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
    # [steps, L, TB, d]: token i of a step follows its own sequence
    X_cpu = torch.stack([S.decode_inputs(W + 2 * K + 64, N_LAYERS, geom.d_model, SEED + rank + 1000 * i)
                         for i in range(TB)], dim=2)
    X = X_cpu[:W + K].to(dev)

    # one eager token before capture, then the graph
    for layer, b in enumerate(blocks):
        b(X[0, layer])
    torch.cuda.synchronize()
    pool.status()
    g = DecodeGraph(blocks, T=TB)
    for t in range(1, W):
        g.step(X[t])
    torch.cuda.synchronize()
    pool.status()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---------------------------------------------------------- timed
    s0 = pool.stats()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for t in range(W, W + K):
        g.step(X[t])
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    pool.status()
    s1 = pool.stats()
    ms_max = ms
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt.item())
    tok_s = world * K * TB / (ms_max / 1e3)
    d = {k: s1[k] - s0[k] for k in ("total", "prefetch", "cache", "miss")}
    hit = {"cache": d["cache"] / max(1, d["total"]),
           "resident_at_acquire": (d["cache"] + d["prefetch"]) / max(1, d["total"]),
           "miss": d["miss"] / max(1, d["total"]),
           "h2d_fill_bytes_per_token": (s1["gb"] - s0["gb"]) * 2 ** 30 / K}

    # ------------------------------------- kernel timing (same kernels, events)
    from moe_stream_b200 import _lib
    import ctypes
    _lib.check(pool._lib.ms_pool_profile(pool._h, 1))
    gp = DecodeGraph(blocks, T=TB)
    n_prof = 16
    acc = [[0.0, 0.0, 0.0] for _ in range(N_LAYERS)]
    buf = (ctypes.c_float * 3)()
    Xp = X_cpu[W + K:W + K + n_prof].to(dev)
    for t in range(n_prof):
        gp.step(Xp[t])
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

    # ----------------------------------------------------------- e2e
    Xh = X_cpu[W + K + n_prof:W + 2 * K + n_prof].pin_memory()
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
    ems = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([ems], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ems = float(tt.item())
    e2e = {"value": world * K * TB / (ems / 1e3), "unit": "tok/s",
           "h2d_bytes_per_step": int(Xh[0].numel() * 2), "d2h_bytes_per_step": int(Yh[0].numel() * 2),
           "path": "DecodeGraph over MoEBlock.__call__ (ms_moe_block), pinned host x in / y out"}
    pool.status()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and TB == 1:
        cpu = cpu_baseline(geom, store, routers, X_cpu[:, :, 0], args.cpu_sample_layers)

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
                       "l2": "inputs larger than L2: 1.02 GB of expert weights per step"},
            "hit_rate": hit,
            "expert_hbm_gbs": achieved,
            "per_layer_us": {"router_table": per_layer[0] * 1e3, "fill": per_layer[1] * 1e3,
                             "experts": expert_ms * 1e3},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
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
        print(json.dumps(line))
    pool.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        reference_arm(args)
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
