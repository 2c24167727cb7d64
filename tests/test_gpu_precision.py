"""GPU parity of per-expert precision classes through the C ABI.

Every expert of a layer is stored in one of eight classes -- 2, 3, 4 or
8-bit codes with bf16 or fp8 scales -- and one block call routes tokens to
experts of all of them. The decode kernels (k_up_mx / k_down_mx), the
grouped tcgen05 GEMM of the wide path and the slot-keyed ms_expert_mlp must
match the oracle's block on the same class blobs (oracle.quant's class
dequantisation, MLX's rounding points) within the parity bar of the other
GPU tests: max-abs 2e-2, mean-rel 1e-2, and error against the fp32
reference no worse than 1.5x the oracle's own MLX-path error. A pool
smaller than the layer checks that fills move each class's payload and the
slots remember their class.
"""
import numpy as np
import pytest
import torch

from moe_stream_b200 import _lib, geometry as G, store as S
from oracle import moe as OM

from test_gpu_block import MAX_ABS, MEAN_REL, mean_rel, to_np_bf16

pytestmark = pytest.mark.gpu

CLASSES = [(b, f) for b in (2, 3, 4, 8) for f in ("bf16", "fp8")]


def _mixed_pool(base, n_slots, layers, depths=(), max_tokens=64, seed=3, assign=None):
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    classes = [G.precision(base, b, f) for b, f in CLASSES]
    slot_geom = G.slot_geometry(base, classes)
    cok = np.array([(k * 5 + 3) % len(classes) if assign is None else assign(k)
                    for k in range(base.n_keys)], np.uint8)
    pool = ExpertPool(slot_geom, n_slots, depths=depths, max_tokens=max_tokens)
    pool.set_precision(classes, cok)
    st = pool.alloc_store()
    S.fill_store_classes(slot_geom, classes, cok, st, seed, layers=layers, device="cuda")
    blocks = [MoEBlock(pool, l, *S.router_weights(base, seed, l, zipf_s=1.1 if base.model == "qwen3" else None,
                                                  bias_std=0.5 if base.model == "gptoss" else None))
              for l in range(base.n_layers)]
    return pool, st.reshape(base.n_keys, slot_geom.blob_bytes), classes, cok, blocks


def _oracle(pool_st, classes, cok, base, layer, xn, gi, gs):
    E = base.n_experts
    keys = sorted(set(gi.reshape(-1).tolist()))
    blobs = {e: pool_st[layer * E + e] for e in keys}
    prec = {}
    for e in keys:
        cg = classes[int(cok[layer * E + e])]
        prec[e] = ([dict(c) for c in cg.components], cg.bits, cg.scale_fmt)
    comps = [dict(c) for c in base.components]
    y_mlx = OM.expert_block(xn, gi, gs, blobs, comps, base.model, prec=prec)
    y_ref = OM.fp32_reference(xn, gi, gs, blobs, comps, base.model, prec=prec)
    return y_mlx, y_ref


def _check(y, y_mlx, y_ref):
    yn = to_np_bf16(y)
    assert np.isfinite(yn).all()
    assert np.abs(yn - y_mlx).max() <= MAX_ABS, np.abs(yn - y_mlx).max()
    assert mean_rel(yn, y_mlx) <= MEAN_REL
    assert OM.rel_err(yn, y_ref) <= 1.5 * max(OM.rel_err(y_mlx, y_ref), 1e-6)


@pytest.mark.parametrize("model,T", [("qwen3", 1), ("qwen3", 6), ("gptoss", 1), ("gptoss", 5)])
def test_decode_block_with_precision_classes(model, T, lib, cuda):
    from moe_stream_b200.block import block_debug
    base = G.qwen3(1) if model == "qwen3" else G.gptoss(1)
    pool, st, classes, cok, blocks = _mixed_pool(base, base.n_experts, [0], max_tokens=8)
    try:
        seen = set()
        for call in range(3):
            x = S.rms_norm_tokens(T, base.d_model, seed=40 + call, device="cuda")
            y = blocks[0](x)
            pool.status()
            inds, scores, _ = block_debug(pool, T)
            gi = inds.cpu().numpy()
            seen |= {int(cok[e]) for e in gi.reshape(-1)}
            y_mlx, y_ref = _oracle(st, classes, cok, base, 0, to_np_bf16(x), gi, to_np_bf16(scores))
            _check(y, y_mlx, y_ref)
        if T > 1:
            assert len(seen) >= 6, seen          # the calls met most classes
    finally:
        pool.close()


@pytest.mark.parametrize("model,T", [("qwen3", 512), ("gptoss", 320)])
def test_prefill_with_precision_classes(model, T, lib, cuda):
    """Wide batches: the grouped GEMM reads every class's codes through its
    own tensor maps; 64 sampled tokens against the oracle."""
    from moe_stream_b200.block import route
    base = G.qwen3(1) if model == "qwen3" else G.gptoss(1)
    pool, st, classes, cok, blocks = _mixed_pool(base, base.n_experts, [0], max_tokens=T)
    try:
        x = S.rms_norm_tokens(T, base.d_model, seed=9, device="cuda")
        inds, scores = route(blocks[0], x)
        y = blocks[0](x)
        pool.status()
        gi = inds.cpu().numpy()
        gs = to_np_bf16(scores)
        assert len({int(cok[e]) for e in gi.reshape(-1)}) == len(CLASSES)
        rows = np.sort(np.random.default_rng(1).choice(T, 64, replace=False))
        y_mlx, y_ref = _oracle(st, classes, cok, base, 0, to_np_bf16(x)[rows], gi[rows], gs[rows])
        _check(y[rows], y_mlx, y_ref)
    finally:
        pool.close()


def test_small_pool_fills_each_class(lib, cuda):
    """Two layers of 128 experts through 48 slots with prefetch: slots are
    refilled with blobs of other classes all along; every output still
    matches the oracle and the table holds what was routed."""
    from moe_stream_b200.block import block_debug
    base = G.qwen3(2)
    pool, st, classes, cok, blocks = _mixed_pool(base, 48, [0, 1], depths=(1,), max_tokens=4)
    try:
        for step in range(6):
            x = S.rms_norm_tokens(2, base.d_model, seed=70 + step, device="cuda")
            for layer in range(2):
                y = blocks[layer](x)
                pool.status()
                inds, scores, slots = block_debug(pool, 2)
                gi = inds.cpu().numpy()
                tab = pool.table()
                assert np.all(tab[slots.cpu().numpy()] == gi + layer * base.n_experts)
                y_mlx, y_ref = _oracle(st, classes, cok, base, layer, to_np_bf16(x), gi,
                                       to_np_bf16(scores))
                _check(y, y_mlx, y_ref)
                x = y
        assert pool.stats()["reads"] > 48
    finally:
        pool.close()


def test_expert_mlp_reads_slot_classes(lib, cuda):
    """ms_expert_mlp on slots filled by ms_pool_read: each slot is read with
    the class of the blob it was given."""
    from moe_stream_b200.block import expert_mlp
    base = G.gptoss(1)
    pool, st, classes, cok, _ = _mixed_pool(base, 16, [0], max_tokens=8)
    try:
        for s in range(16):
            pool._read(s, 0, 8 * (s % 2) + s // 2)   # slot s holds expert e(s)
        e_of = np.array([8 * (s % 2) + s // 2 for s in range(16)])
        rng = np.random.default_rng(4)
        T, k = 3, base.top_k
        slots = np.stack([rng.choice(16, k, replace=False) for _ in range(T)]).astype(np.int32)
        raw = rng.random((T, k)).astype(np.float32) + 0.1
        sc = torch.from_numpy(raw / raw.sum(-1, keepdims=True)).to(torch.bfloat16).float()
        x = S.rms_norm_tokens(T, base.d_model, seed=12, device="cuda")
        y = expert_mlp(pool, torch.from_numpy(slots).cuda(), x, sc.cuda())
        pool.status()
        gs = sc.numpy()
        y_mlx, y_ref = _oracle(st, classes, cok, base, 0, to_np_bf16(x), e_of[slots], gs)
        _check(y, y_mlx, y_ref)
    finally:
        pool.close()


def test_set_precision_is_checked(lib, cuda):
    from moe_stream_b200.pool import ExpertPool
    base = G.make("qwen3", 256, 128, 16, 1, 4)
    classes = [G.precision(base, 2, "fp8"), G.precision(base, 8, "bf16")]
    sg = G.slot_geometry(base, classes)
    pool = ExpertPool(sg, 8, depths=(), max_tokens=2)
    try:
        with pytest.raises(_lib.MoeStreamError) as e:
            pool.set_precision(classes, np.full(16, 2, np.uint8))          # no class 2
        assert e.value.code == _lib.MS_E_INVALID
        small = G.slot_geometry(base, classes[:1])
        pool2 = ExpertPool(small, 8, depths=(), max_tokens=2)
        try:
            with pytest.raises(_lib.MoeStreamError) as e:                  # 8-bit blob > stride
                pool2.set_precision(classes, np.zeros(16, np.uint8))
            assert e.value.code == _lib.MS_E_INVALID
        finally:
            pool2.close()
        pool.set_precision(classes, np.arange(16, dtype=np.uint8) % 2)
        pool.alloc_store()
        pool._read(0, 0, 0)
        with pytest.raises(_lib.MoeStreamError) as e:                      # after a fill
            pool.set_precision(classes, np.zeros(16, np.uint8))
        assert e.value.code == _lib.MS_E_STATE
    finally:
        pool.close()
