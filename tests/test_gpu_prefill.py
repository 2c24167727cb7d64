"""GPU parity tests of the wide-batch (prefill) path through the C ABI: the
tiled router, the expert-order scatter, the two tcgen05 grouped GEMMs and
the combine, against the oracle.

Same bar as the decode tests (the parity bar of this path): routing index sets
bit-exact except at exact bf16 ties (or one ulp, for fp32 accumulation
order); outputs within max-abs 2e-2 and mean-rel 1e-2 of the oracle's
MLX-path restatement; error against the fp32 dequantised reference no worse
than 1.5x the MLX path's (test_kernel.py:95-101).
"""
import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry, store as S
from oracle import moe as OM

from test_gpu_block import (MAX_ABS, MEAN_REL, check_topk_sets, make_pool, mean_rel,
                            to_np_bf16)

pytestmark = pytest.mark.gpu


def _oracle_check(x, gi, gs, blobs, geom, model):
    comps = [dict(c) for c in geom.components]
    xn = to_np_bf16(x)
    y_mlx = OM.expert_block(xn, gi, gs, blobs, comps, model)
    y_ref = OM.fp32_reference(xn, gi, gs, blobs, comps, model)
    return y_mlx, y_ref


def test_wide_router_matches_oracle(lib, cuda):
    """T above the decode scratch: ms_route runs the tiled tensor-core router;
    index sets, scores and the layer-1 speculation match the oracle."""
    from moe_stream_b200.block import route
    geom = geometry.qwen3(n_layers=2)
    T = 300
    pool, _, blocks = make_pool(geom, 4, [], [], zipf=1.1, max_tokens=T)
    try:
        x = S.rms_norm_tokens(T, geom.d_model, seed=12, device="cuda")
        inds, scores, pred = route(blocks[0], x, with_pred=True)
        torch.cuda.synchronize()
        xn = to_np_bf16(x)
        w0, b0 = S.router_weights(geom, 0, 0, zipf_s=1.1)
        w1, b1 = S.router_weights(geom, 0, 1, zipf_s=1.1)
        f = lambda t: None if t is None else t.float().numpy()
        oi, osc, vals = OM.route_qwen3(xn, f(w0), 8, norm=True, bias=f(b0))
        gi = inds.cpu().numpy()
        assert check_topk_sets(gi, vals, 8) <= T // 8
        gs = to_np_bf16(scores)
        for t in range(T):
            if set(gi[t]) == set(oi[t]):
                order = {e: j for j, e in enumerate(oi[t])}
                ref = np.array([osc[t][order[e]] for e in gi[t]], np.float32)
                assert np.all(np.abs(gs[t] - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-6), t
        _, plog = OM.predict(xn, f(w1), 8, f(b1))
        check_topk_sets(pred.cpu().numpy(), plog, 8)
    finally:
        pool.close()


def test_prefill_qwen3_layer(lib, cuda):
    """Config 2 in miniature: one full-shape Qwen3 layer, all 128 experts
    resident, T=512 with a Zipf-skewed router so that the busiest experts
    span several 128-row tiles."""
    from moe_stream_b200.block import block_debug
    geom = geometry.qwen3(n_layers=1)
    T = 512
    pool, st, blocks = make_pool(geom, 128, [0], range(128), zipf=1.1, max_tokens=T, depths=())
    try:
        x = S.rms_norm_tokens(T, geom.d_model, seed=2, device="cuda")
        y = blocks[0](x)
        pool.status()
        inds, scores, slots = block_debug(pool, T)
        gi = inds.cpu().numpy()
        gs = to_np_bf16(scores)
        counts = np.bincount(gi.reshape(-1), minlength=128)
        assert counts.max() > 128, "the case must put more than one tile on an expert"
        tab = pool.table()
        assert np.all(tab[slots.cpu().numpy()] == gi)
        blobs = {e: st[e] for e in range(128)}
        y_mlx, y_ref = _oracle_check(x, gi, gs, blobs, geom, "qwen3")
        yn = to_np_bf16(y)
        assert np.isfinite(yn).all()
        assert np.abs(yn - y_mlx).max() <= MAX_ABS
        assert mean_rel(yn, y_mlx) <= MEAN_REL
        assert OM.rel_err(yn, y_ref) <= 1.5 * max(OM.rel_err(y_mlx, y_ref), 1e-6)
        # a second call on other tokens reuses every buffer
        x2 = S.rms_norm_tokens(T, geom.d_model, seed=3, device="cuda")
        y2 = blocks[0](x2)
        pool.status()
        gi2 = block_debug(pool, T)[0].cpu().numpy()
        gs2 = to_np_bf16(block_debug(pool, T)[1])
        y2_mlx, _ = _oracle_check(x2, gi2, gs2, blobs, geom, "qwen3")
        yn2 = to_np_bf16(y2)
        assert np.abs(yn2 - y2_mlx).max() <= MAX_ABS
        assert mean_rel(yn2, y2_mlx) <= MEAN_REL
    finally:
        pool.close()


def test_prefill_gptoss_layer(lib, cuda):
    """gpt-oss shapes (d = ff = 2880, biases, clamped SwiGLU, top-4 then
    softmax) with 16 experts so the oracle stays quick; T=320 gives ~80
    tokens per expert, the busiest past one tile."""
    from moe_stream_b200.block import block_debug
    geom = geometry.make("gptoss", 2880, 2880, 16, 1, 4, False)
    T = 320
    pool, st, blocks = make_pool(geom, 16, [0], range(16), bias_std=0.5, max_tokens=T, depths=())
    try:
        x = S.rms_norm_tokens(T, geom.d_model, seed=4, device="cuda")
        y = blocks[0](x)
        pool.status()
        inds, scores, _ = block_debug(pool, T)
        gi = inds.cpu().numpy()
        gs = to_np_bf16(scores)
        assert np.bincount(gi.reshape(-1), minlength=16).max() > 128
        blobs = {e: st[e] for e in range(16)}
        y_mlx, y_ref = _oracle_check(x, gi, gs, blobs, geom, "gptoss")
        yn = to_np_bf16(y)
        assert np.isfinite(yn).all()
        assert np.abs(yn - y_mlx).max() <= MAX_ABS
        assert mean_rel(yn, y_mlx) <= MEAN_REL
        assert OM.rel_err(yn, y_ref) <= 1.5 * max(OM.rel_err(y_mlx, y_ref), 1e-6)
    finally:
        pool.close()


@pytest.mark.parametrize("model", ["qwen3", "gptoss"])
def test_wide_and_decode_paths_agree(model, lib, cuda, monkeypatch):
    """The same batch through both expert paths (the threshold moved by
    MS_WIDE_MIN_PAIRS): equal routing, outputs within the parity tolerance."""
    from moe_stream_b200.block import block_debug
    if model == "qwen3":
        geom, T, E = geometry.qwen3(n_layers=1), 160, 128
    else:
        geom, T, E = geometry.make("gptoss", 2880, 2880, 16, 1, 4, False), 200, 16
    ys, routes = [], []
    for thr in ("1", "100000"):
        monkeypatch.setenv("MS_WIDE_MIN_PAIRS", thr)
        pool, st, blocks = make_pool(geom, E, [0], range(E), seed=6, max_tokens=T, depths=(),
                                     bias_std=0.5 if model == "gptoss" else None)
        try:
            x = S.rms_norm_tokens(T, geom.d_model, seed=8, device="cuda")
            ys.append(to_np_bf16(blocks[0](x)))
            pool.status()
            routes.append(block_debug(pool, T)[0].cpu().numpy())
        finally:
            pool.close()
    same = np.all(np.sort(routes[0], 1) == np.sort(routes[1], 1), axis=1)
    assert same.mean() >= 0.97
    a, b = ys[0][same], ys[1][same]
    assert np.abs(a - b).max() <= MAX_ABS
    assert mean_rel(a, b) <= MEAN_REL
