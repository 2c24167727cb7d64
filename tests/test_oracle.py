"""CPU tests: the oracle against the reference's golden vectors and
constants, and the host-side data preparation against the oracle."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import bf16 as OB
from oracle import moe as OM
from oracle import quant as OQ
from oracle.pool_sim import PoolExhausted, PoolSim

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "pool_golden.json")))


def replay(sim, sc):
    """Drive a PoolSim through a golden scenario, yielding (op, got, want)."""
    for i, o in enumerate(sc["ops"]):
        if o["op"] == "prefetch":
            sim.prefetch(o["layer"], o["experts"])
            res = None
        else:
            try:
                res = [int(s) for s in sim.acquire(o["layer"], o["experts"])[0]]
            except PoolExhausted:
                res = "exhausted"
        st = sim.stats()
        got = dict(result=res, table=sim.table(),
                   counters=[st["prefetch"], st["cache"], st["miss"], st["bail"], st["issued"],
                             sim.n_reads],
                   clock=sim.clock, use_clock=sim.use_clock)
        want = {k: o[k] for k in got}
        yield i, got, want


@pytest.mark.parametrize("sc", GOLDEN["scenarios"], ids=[s["name"] for s in GOLDEN["scenarios"]])
def test_pool_sim_matches_reference_expertpool(sc):
    """The restated pool bookkeeping reproduces the reference's ExpertPool
    (run unmodified to make the fixture) call by call: returned slots, the
    whole slot table, hit/miss/bail counters and both clocks."""
    sim = PoolSim(sc["n_slots"], sc["n_experts"], sc["evict"], sc["depth"])
    for i, got, want in replay(sim, sc):
        assert got == want, f"call {i}"
    fin = sc["final"]
    assert {str(k): v for k, v in sim.freq.items() if v} == fin["freq"]
    assert {str(k): v for k, v in sim.born.items()} == fin["born"]
    assert {str(k): v for k, v in sim.last_use.items()} == fin["last_use"]
    assert sorted(sim.from_prefetch) == fin["from_prefetch"]
    assert sorted(sim.pinned) == fin["pinned"]


def test_golden_covers_the_interesting_paths():
    names = {s["name"] for s in GOLDEN["scenarios"]}
    assert {"lfu_d1", "lru_d1", "asis_d1", "lfu_d2", "lfu_exhaust"} <= names
    ex = [o for s in GOLDEN["scenarios"] for o in s["ops"] if o["result"] == "exhausted"]
    assert ex, "no exhaustion in the fixture"
    bails = max(s["ops"][-1]["counters"][3] for s in GOLDEN["scenarios"])
    assert bails > 0
    # scenarios where an acquire found a prefetch still pending (double touch)
    wide = [s for s in GOLDEN["scenarios"] if "pending" in s["name"]]
    assert all(s["ops"][-1]["counters"][0] > 0 for s in wide)


def test_planted_mistake_in_the_oracle_is_caught():
    """A pool simulator with the young-window off disagrees with the fixture:
    the golden data constrain the victim choice, not just the counts."""
    sc = next(s for s in GOLDEN["scenarios"] if s["name"] == "lfu_d1")
    sim = PoolSim(sc["n_slots"], sc["n_experts"], sc["evict"], sc["depth"])
    sim.window = 0
    assert any(got != want for _, got, want in replay(sim, sc))


# ------------------------------------------------------------- blob format
def test_qwen3_blob_layout_matches_reference_constants():
    """kernels.py:58-63 LAYOUT_U32 (word offsets) and repack.py:13-14."""
    comps, payload, blob = OM.blob_layout(2048, 768)
    layout_u32 = dict(blob=663552, gate_w=0, gate_s=196608, gate_b=208896, up_w=221184,
                      up_s=417792, up_b=430080, down_w=442368, down_s=638976, down_b=651264)
    got = {c["proj"].replace("_proj", "") + "_" + c["part"][0]: c["offset"] // 4 for c in comps}
    got["blob"] = blob // 4
    assert got == layout_u32
    assert blob == payload == 2_654_208 == 162 * 16384


def test_gptoss_blob_layout_matches_reference_constants():
    """scratchpad/stage_bench.py:11-12: BLOB 14,024,704 and per-projection
    segments [4147200, 259200, 259200, 5760] x 3 + 10624 padding."""
    comps, payload, blob = OM.blob_layout(2880, 2880, proj_bias=True)
    assert blob == 14_024_704 and blob - payload == 10_624
    assert [c["nbytes"] for c in comps] == [4147200, 259200, 259200, 5760] * 3


def test_package_geometry_matches_oracle_layout():
    from moe_stream_b200 import geometry
    for g, args in ((geometry.qwen3(), (2048, 768, 64, 4, False)),
                    (geometry.gptoss(), (2880, 2880, 64, 4, True))):
        comps, payload, blob = OM.blob_layout(*args)
        assert [dict(c) for c in g.components] == comps
        assert (g.payload_bytes, g.blob_bytes) == (payload, blob)


# ------------------------------------------------------------ quantisation
def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], np.float32)
    r = OB.r(x)
    assert r[0] == 1.0 and r[1] == 1.0                   # tie to even
    assert r[2] == np.float32(1.0 + 2 ** -6)             # tie to even (up)
    assert r[3] == -2.5 and r[4] == 0.0
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(OB.to_bits(x), t)


def test_quantizer_roundtrip_and_packing():
    rng = np.random.default_rng(0)
    w = OB.r(rng.standard_normal((64, 256)).astype(np.float32) * 0.02)
    p, s, b = OQ.quantize(w)
    assert p.shape == (64, 32) and s.shape == (64, 4) and b.shape == (64, 4)
    q = OQ.unpack(p)
    assert q.max() <= 15
    # low nibble first (kernels.py:137-139)
    assert np.array_equal(q[:, 0], (p[:, 0] & 0xF).astype(np.uint8))
    assert np.array_equal(q[:, 7], (p[:, 0] >> 28).astype(np.uint8))
    deq = OQ.dequantize_f32(p, s, b)
    step = np.abs(OB.from_bits(s)).repeat(64, axis=1)
    # half a quantisation step plus the bf16 rounding of scale and bias; the
    # edge that snaps the scale (q0 = round(edge/scale)) can push the other
    # edge one code past 15, where it is clipped: one full step there
    gmax = np.abs(w).reshape(64, 4, 64).max(-1).repeat(64, axis=1)
    slack = 16 * step * 2 ** -8 + gmax * 2 ** -8
    err = np.abs(deq - w)
    assert np.all(err <= step + slack)
    assert np.mean(err <= 0.5 * step + slack) > 0.99


@pytest.mark.parametrize("shape", [(96, 2048), (40, 768), (8, 2880)])
def test_torch_quantizer_is_bit_exact_with_oracle(shape):
    """moe_stream_b200.store.quantize (used to build stores, also on the GPU)
    == the oracle's restatement of MLX affine quantisation."""
    from moe_stream_b200 import store
    rng = np.random.default_rng(shape[0])
    w = OB.r(rng.standard_normal(shape).astype(np.float32) * 0.02)
    w[0, :64] = 0.0
    w[1, :64] = 0.01
    w[2, 64:128] = -0.03
    p, s, b = OQ.quantize(w)
    tp, ts, tb = store.quantize(torch.from_numpy(w))
    assert np.array_equal(p, tp.numpy().view(np.uint32))
    assert np.array_equal(s, ts.view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(b, tb.view(torch.int16).numpy().view(np.uint16))


def test_store_blob_is_the_reference_layout():
    from moe_stream_b200 import geometry, store
    g = geometry.make("qwen3", 128, 64, 4, 2, 2)
    blob = store.make_blob(g, seed=3, layer=1, expert=2).numpy()
    w = store.expert_weights(g, 3, 1, 2)
    v = OM.blob_views(blob, [dict(c) for c in g.components])
    p, s, b = OQ.quantize(w["down_proj"].numpy())
    assert np.array_equal(v["down_proj.weight"], p)
    assert np.array_equal(v["down_proj.scales"], s)
    assert np.array_equal(v["down_proj.biases"], b)


# ------------------------------------------------------------------ routers
def test_router_oracles():
    rng = np.random.default_rng(1)
    x = OB.r(rng.standard_normal((5, 256)).astype(np.float32))
    w = OB.r(rng.standard_normal((32, 256)).astype(np.float32) * 0.02)
    inds, scores, g = OM.route_qwen3(x, w, 4, norm=True)
    assert inds.shape == (5, 4)
    assert np.allclose(scores.sum(-1), 1.0, atol=2e-2)
    for t in range(5):                                   # a true top-k set
        kth = np.sort(g[t])[-4]
        assert np.all(g[t][inds[t]] >= kth)
    inds2, sc2, lg = OM.route_gptoss(x, w, 4)
    assert np.allclose(sc2.sum(-1), 1.0, atol=2e-2)
    # softmax is monotone: same selection from the logits up to bf16 ties
    for t in range(5):
        assert set(inds2[t]) == set(OM.topk_desc(lg[t:t + 1], 4)[0])


def test_topk_ties_go_to_lower_index():
    v = np.array([[0.5, 0.7, 0.7, 0.1, 0.7]], np.float32)
    assert OM.topk_desc(v, 2).tolist() == [[1, 2]]


# -------------------------------------------------------------- expert math
@pytest.mark.parametrize("model", ["qwen3", "gptoss"])
def test_oracle_block_close_to_fp32_reference(model):
    """The bf16 MLX-path restatement and the fp32 dequantised reference agree
    to the magnitude the reference measured between them (test_kernel.py:95;
    MLX's error 2.3e-3, kernels.py:31-33)."""
    from moe_stream_b200 import geometry, store
    g = geometry.make(model, 256, 128, 8, 1, 2, True)
    blobs = {e: store.make_blob(g, 0, 0, e).numpy() for e in range(8)}
    rng = np.random.default_rng(2)
    x = OB.r(rng.standard_normal((3, 256)).astype(np.float32))
    inds = np.array([[0, 5], [5, 7], [2, 1]], np.int32)
    scores = OB.r(np.array([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5]], np.float32))
    comps = [dict(c) for c in g.components]
    y = OM.expert_block(x, inds, scores, blobs, comps, model)
    ref = OM.fp32_reference(x, inds, scores, blobs, comps, model)
    err = OM.rel_err(y, ref)
    assert 1e-5 < err < 2e-2, err
