"""The block fused with its decoder layer's post-attention RMSNorm and the
residual add (ms_moe_block_fused): out = h + block(rms_norm(h) * w).

Against the oracle (oracle.moe.rms_norm, mx.fast.rms_norm's rounding, then
the MLX-path block, then the bf16 residual add): routing on the normalised
input (index sets), outputs within the parity bar. The cases take each
path: decode calls of up to 8 tokens normalise inside the route step and
add the residual in the expert kernels' combine; larger decode calls and
the wide path normalise with one kernel first. An in-place call (out = h)
gives the same result.
"""
import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry, store as S
from oracle import bf16 as OB
from oracle import moe as OM

from test_gpu_block import MAX_ABS, MEAN_REL, check_topk_sets, make_pool, mean_rel, to_np_bf16

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _norm_weight(d, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)


def _residual(T, d, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, d, generator=g) * 0.5).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("model,T", [("qwen3", 1), ("qwen3", 5), ("qwen3", 12), ("qwen3", 300),
                                     ("gptoss", 1), ("gptoss", 3)])
def test_fused_block_matches_oracle(model, T, lib, cuda):
    from moe_stream_b200.block import MoEBlock, block_debug
    geom = geometry.qwen3(n_layers=1) if model == "qwen3" else geometry.gptoss(n_layers=1)
    E = geom.n_experts
    pool, st, blocks = make_pool(geom, E, [0], range(E), seed=4, max_tokens=max(T, 16), depths=(),
                                 zipf=1.1 if model == "qwen3" else None,
                                 bias_std=0.5 if model == "gptoss" else None)
    try:
        w = _norm_weight(geom.d_model, 9)
        blk = MoEBlock(pool, 0, blocks[0].gate_weight, blocks[0].gate_bias, norm_weight=w, norm_eps=EPS)
        h = _residual(T, geom.d_model, 13 + T)
        out = blk.fused(h)
        pool.status()
        inds, scores, _ = block_debug(pool, T)
        hn = to_np_bf16(h)
        xn = OM.rms_norm(hn, w.float().numpy(), EPS)
        f = lambda t: None if t is None else t.float().cpu().numpy()
        if model == "qwen3":
            _, _, vals = OM.route_qwen3(xn, f(blk.gate_weight), geom.top_k, norm=True, bias=f(blk.gate_bias))
        else:
            _, _, vals = OM.route_gptoss(xn, f(blk.gate_weight), geom.top_k, f(blk.gate_bias))
        gi = inds.cpu().numpy()
        check_topk_sets(gi, vals, geom.top_k)
        rows = np.arange(T) if T <= 64 else np.sort(np.random.default_rng(2).choice(T, 64, replace=False))
        comps = [dict(c) for c in geom.components]
        blobs = {e: st[e] for e in set(gi[rows].reshape(-1).tolist())}
        y_blk = OM.expert_block(xn[rows], gi[rows], to_np_bf16(scores)[rows], blobs, comps, model)
        want = OB.r(hn[rows] + y_blk)
        got = to_np_bf16(out)[rows]
        assert np.abs(got - want).max() <= MAX_ABS, np.abs(got - want).max()
        assert mean_rel(got - hn[rows], want - hn[rows]) <= MEAN_REL
        # in place: the residual stream updated where it lies
        h2 = h.clone()
        blk.fused(h2, out=h2)
        pool.status()
        assert torch.equal(h2, out)
    finally:
        pool.close()
