"""GPU parity at the benchmark configurations' real shapes, and the
reference's own invariants, through the C ABI.

* Pool-size invariance (the reference's verify_quality.py:87-97 check): a
  48-layer Qwen3 decode stack gives bit-identical outputs at 1536 and at 3072
  slots -- the pool decides where experts live, never what a block computes.
* The full-size layers the performance figures are quoted on: Qwen3 at
  T = 4096, gpt-oss with 128 experts at T = 512 and at T = 16384 (the
  expert-parallel layer on one GPU), and an 8-layer gpt-oss decode stack with
  a half-size pool whose slot table must equal the oracle's after every call.
  The oracle is slow, so every token's routing is checked and the outputs on
  a seeded sample of tokens.
* A pool checkpoint (ms_pool_save_state / ms_pool_load_state) replays the
  same tokens to the same outputs, slot table and statistics.
* Batched decode (several tokens per step, the multi-token verify case)
  through a captured decode step, against the oracle.

Router rows that differ from the oracle (allowed only at exact bf16 ties or
within one bf16 ulp of the k-th value) are counted and printed by each test.
"""
import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry, store as S
from oracle import moe as OM
from oracle.pool_sim import PoolSim

from test_gpu_block import MAX_ABS, MEAN_REL, check_topk_sets, mean_rel, to_np_bf16

pytestmark = pytest.mark.gpu


def _stack(geom, n_slots, zipf=1.1, max_tokens=1, seed=0, store=None):
    """Pool + routers for every layer; a store of make_layer_blobs layers
    (generated on the GPU) unless `store` (a pinned store array) is given."""
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    pool = ExpertPool(geom, n_slots, evict="lfu", depths=(1,), max_tokens=max_tokens)
    if store is None:
        st = pool.alloc_store()
        view = torch.from_numpy(st).view(geom.n_keys, geom.blob_bytes)
        for layer in range(geom.n_layers):
            view[layer * geom.n_experts:(layer + 1) * geom.n_experts].copy_(
                S.make_layer_blobs(geom, seed, layer, device="cuda").cpu())
    else:
        st = pool.attach_store(store)
    blocks = [MoEBlock(pool, l, *S.router_weights(geom, seed, l, zipf_s=zipf))
              for l in range(geom.n_layers)]
    return pool, st, blocks


def test_pool_size_invariance_48_layers(lib, cuda):
    """verify_quality.py:87-97: the same tokens through a 48-layer stack at
    1536 and at 3072 slots give the same outputs, bit for bit."""
    from moe_stream_b200.block import DecodeGraph
    geom = geometry.qwen3(48)
    steps = 64
    X = S.decode_inputs(steps, geom.n_layers, geom.d_model, seed=5).cuda()   # [steps, L, d]
    outs = {}
    pool_a, store, blocks_a = _stack(geom, 3072)
    try:
        for n_slots in (3072, 1536):
            if n_slots == 3072:
                pool, blocks = pool_a, blocks_a
            else:
                pool, _, blocks = _stack(geom, n_slots, store=store)
            try:
                g = DecodeGraph(blocks)
                ys = []
                for t in range(steps):
                    ys.append(g.step(X[t].unsqueeze(1)).clone())
                torch.cuda.synchronize()
                pool.status()
                outs[n_slots] = (torch.stack(ys), pool.stats())
                del g
            finally:
                if pool is not pool_a:
                    pool.close()
        (ya, sa), (yb, sb) = outs[3072], outs[1536]
        assert torch.equal(ya, yb)
        # the smaller pool did have to evict: the invariance is not vacuous
        assert sb["miss"] + sb["prefetch"] > sa["miss"] + sa["prefetch"]
    finally:
        pool_a.close()


def _layer_pool(geom, T, zipf, seed=0):
    """One layer, every expert resident in slot e (slot = expert)."""
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    pool = ExpertPool(geom, geom.n_experts, depths=(), max_tokens=T)
    st = pool.alloc_store().reshape(geom.n_keys, geom.blob_bytes)
    torch.from_numpy(st).copy_(S.make_layer_blobs(geom, seed, 0, device="cuda").cpu())
    w, b = S.router_weights(geom, seed, 0, zipf_s=zipf)
    return pool, st, MoEBlock(pool, 0, w, b), w, b


def _wide_layer_case(model, T, zipf, n_check, seed):
    from moe_stream_b200.block import block_debug
    geom = geometry.qwen3(1) if model == "qwen3" else geometry.gptoss(1)
    pool, st, blk, w, b = _layer_pool(geom, T, zipf)
    try:
        x = S.rms_norm_tokens(T, geom.d_model, seed=seed, device="cuda")
        y = blk(x)
        pool.status()
        inds, scores, slots = block_debug(pool, T)
        gi = inds.cpu().numpy()
        gs = to_np_bf16(scores)
        xn = to_np_bf16(x)
        f = lambda t: None if t is None else t.float().numpy()
        k = geom.top_k
        if model == "qwen3":
            _, _, vals = OM.route_qwen3(xn, f(w), k, norm=True, bias=f(b))
        else:
            _, _, vals = OM.route_gptoss(xn, f(w), k, bias=f(b))
        n_diff = check_topk_sets(gi, vals, k)
        print(f"\n{model} T={T}: {n_diff} of {T} router rows differ from the oracle (ties)")
        assert n_diff <= max(2, T // 64)
        # every routed expert's slot holds it
        assert np.all(pool.table()[slots.cpu().numpy()] == gi)
        rng = np.random.default_rng(seed)
        idx = np.sort(rng.choice(T, size=n_check, replace=False))
        blobs = {int(e): st[int(e)] for e in np.unique(gi[idx])}
        comps = [dict(c) for c in geom.components]
        y_mlx = OM.expert_block(xn[idx], gi[idx], gs[idx], blobs, comps, model)
        yn = to_np_bf16(y)[idx]
        assert np.abs(yn - y_mlx).max() <= MAX_ABS
        assert mean_rel(yn, y_mlx) <= MEAN_REL
    finally:
        pool.close()


def test_qwen3_layer_T4096(lib, cuda):
    """The Qwen3 prefill layer at its benchmark size: 4096 tokens, top-8 of
    128 under Zipf(1.1) routing, ~256 tokens per expert."""
    _wide_layer_case("qwen3", 4096, 1.1, 256, seed=41)


def test_gptoss_layer_T512(lib, cuda):
    """The gpt-oss layer with all 128 experts at T = 512."""
    _wide_layer_case("gptoss", 512, None, 16, seed=42)


def test_gptoss_layer_T16384(lib, cuda):
    """The expert-parallel layer's whole batch on one GPU: T = 16384, top-4
    under Zipf(1.1) routing."""
    _wide_layer_case("gptoss", 16384, 1.1, 16, seed=43)


def test_gptoss_decode_stack_8_layers(lib, cuda):
    """An 8-layer gpt-oss decode stack with a half-size pool (512 slots for
    1024 experts), Zipf(1.1) routers and next-layer prefetch: after every
    block call the device slot table equals the oracle pool's driven with the
    same routing; outputs match the oracle block on the first and last step."""
    from moe_stream_b200.block import block_debug, route
    geom = geometry.gptoss(8)
    L, n_slots = geom.n_layers, 512
    pool, st, blocks = _stack(geom, n_slots, seed=3)
    st = st.reshape(geom.n_keys, geom.blob_bytes)
    sim = PoolSim(n_slots, geom.n_experts, "lfu", 1)
    comps = [dict(c) for c in geom.components]
    try:
        g = torch.Generator().manual_seed(17)
        steps = 5
        for step in range(steps):
            h = torch.randn(1, geom.d_model, generator=g)
            for layer in range(L):
                x = (h / h.pow(2).mean().sqrt()).to(torch.bfloat16).cuda()
                pred = None
                if layer + 1 < L:
                    _, _, pred = route(blocks[layer], x, with_pred=True)
                y = blocks[layer](x)
                pool.status()
                inds, scores, _ = block_debug(pool, 1)
                gi = inds.cpu().numpy()
                if pred is not None:
                    sim.prefetch(layer + 1, sorted(set(pred.cpu().numpy().reshape(-1).tolist())))
                sim.acquire(layer, sorted(set(gi.reshape(-1).tolist())))
                assert pool.table().tolist() == sim.table(), (step, layer)
                if step in (0, steps - 1) and layer in (0, L - 1):
                    blobs = {int(e): st[layer * geom.n_experts + int(e)] for e in gi[0]}
                    y_mlx = OM.expert_block(to_np_bf16(x), gi, to_np_bf16(scores), blobs, comps,
                                            "gptoss")
                    yn = to_np_bf16(y)
                    assert np.abs(yn - y_mlx).max() <= MAX_ABS
                    assert mean_rel(yn, y_mlx) <= MEAN_REL
                h = h + 0.1 * torch.randn(1, geom.d_model, generator=g)
        s, ref = pool.stats(), sim.stats()
        assert (s["prefetch"], s["cache"], s["miss"]) == (ref["prefetch"], ref["cache"], ref["miss"])
    finally:
        pool.close()


def test_checkpoint_replays_exactly(lib, cuda):
    """Save a half-size 4-layer pool mid-run, decode 6 tokens, restore and
    decode them again: the same outputs, slot table and statistics."""
    from moe_stream_b200.block import DecodeGraph
    geom = geometry.qwen3(4)
    pool, _, blocks = _stack(geom, geom.n_keys // 2, seed=6)
    try:
        X = S.decode_inputs(16, geom.n_layers, geom.d_model, seed=8).cuda()
        g = DecodeGraph(blocks)
        for t in range(10):
            g.step(X[t].unsqueeze(1))
        snap = pool.save_state(with_arena=True)
        s0 = pool.stats()
        runs = []
        for _ in range(2):
            ys = [g.step(X[t].unsqueeze(1)).clone() for t in range(10, 16)]
            torch.cuda.synchronize()
            pool.status()
            s1 = pool.stats()
            runs.append((torch.stack(ys), pool.table().tolist(),
                         {k: s1[k] - s0[k] for k in ("total", "prefetch", "cache", "miss")}))
            pool.load_state(snap, with_arena=True)
            torch.cuda.synchronize()
        assert torch.equal(runs[0][0], runs[1][0])
        assert runs[0][1] == runs[1][1] and runs[0][2] == runs[1][2]
        assert runs[0][2]["miss"] + runs[0][2]["prefetch"] > 0   # the pool was moving
    finally:
        pool.close()


def test_batched_decode_stack_T4(lib, cuda):
    """Four tokens per decode step (a multi-token verify batch), captured as
    one graph over a 4-layer Qwen3 stack with a half-size pool: the outputs
    of every layer match the oracle block, and the slot table the oracle
    pool's, after each step."""
    from moe_stream_b200.block import DecodeGraph, block_debug, route
    geom = geometry.qwen3(4)
    L, TB, n_slots = geom.n_layers, 4, geom.n_keys // 2
    pool, st, blocks = _stack(geom, n_slots, max_tokens=TB, seed=9)
    st = st.reshape(geom.n_keys, geom.blob_bytes)
    comps = [dict(c) for c in geom.components]
    sim = PoolSim(n_slots, geom.n_experts, "lfu", 1)
    try:
        X = torch.stack([S.decode_inputs(6, L, geom.d_model, seed=30 + i) for i in range(TB)],
                        dim=2).cuda()                                       # [steps, L, TB, d]
        g = DecodeGraph(blocks, T=TB)
        for t in range(X.shape[0]):
            # the routing the graph will use, from the router alone (no table change)
            rts = []
            for layer in range(L):
                if layer + 1 < L:
                    inds, scores, pred = route(blocks[layer], X[t, layer], with_pred=True)
                else:
                    (inds, scores), pred = route(blocks[layer], X[t, layer]), None
                rts.append((inds.cpu().numpy(), to_np_bf16(scores),
                            None if pred is None else pred.cpu().numpy()))
            y = g.step(X[t]).clone()
            torch.cuda.synchronize()
            pool.status()
            for layer in range(L):
                gi, gs, pred = rts[layer]
                if pred is not None:
                    sim.prefetch(layer + 1, sorted(set(pred.reshape(-1).tolist())))
                sim.acquire(layer, sorted(set(gi.reshape(-1).tolist())))
                if t in (0, X.shape[0] - 1):
                    blobs = {int(e): st[layer * geom.n_experts + int(e)] for e in np.unique(gi)}
                    y_mlx = OM.expert_block(to_np_bf16(X[t, layer]), gi, gs, blobs, comps, "qwen3")
                    yn = to_np_bf16(y[layer])
                    assert np.abs(yn - y_mlx).max() <= MAX_ABS, (t, layer)
                    assert mean_rel(yn, y_mlx) <= MEAN_REL, (t, layer)
            assert pool.table().tolist() == sim.table(), t
    finally:
        pool.close()
