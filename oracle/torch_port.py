"""Vectorised torch-CPU restatement of the decode stack: the timed CPU
baseline (TEST INFRASTRUCTURE ONLY; ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` legs run it, nothing in the library imports it).

MLX itself (the reference's compute path, MLX 0.32 / mlx-lm 0.31) is not
installable on this image, so the CPU baseline is this port of the same
per-token work in float32 torch on the host cores, with MLX's bf16 rounding
points (as in ``oracle.moe``):

  * router, engine_v3.py:467-473 -- bf16 logits (+ bias), softmax over the
    experts, top-k, renormalised scores; and the next layer's speculation,
    engine_v3.py:476-483 / 509-527 (top-k of its raw logits on this x);
  * slot pool, engine_v3.py:383-454 -- ``oracle.pool_sim.PoolSim`` (prefetch
    of the predicted experts, acquire of the routed ones); each fill copies a
    blob from the store into a host arena, as ``_read`` does
    (engine_v3.py:255-290);
  * experts, engine_v3.py:588-600 -- each routed expert's three projections
    dequantised (``w = s*q + b``, kernels.py:129-144) and applied to the
    token, SwiGLU, score-weighted sum, every gather_qmm output in bf16.
"""
import numpy as np
import torch

from .pool_sim import PoolSim


def bfr(t):
    """Round float32 values to bf16 (round to nearest even), kept as float32."""
    return t.to(torch.bfloat16).to(torch.float32)


_SHIFTS = torch.arange(8, dtype=torch.int32) * 4


def dequant(blob, comp_w, comp_s, comp_b, n_out, n_in):
    """float32 [n_out, n_in] weights of one projection of a blob (torch uint8)."""
    w = blob[comp_w["offset"]:comp_w["offset"] + comp_w["nbytes"]].view(torch.int32)
    q = ((w.view(n_out, n_in // 8, 1) >> _SHIFTS) & 0xF).reshape(n_out, n_in).to(torch.float32)
    s = blob[comp_s["offset"]:comp_s["offset"] + comp_s["nbytes"]].view(torch.bfloat16)
    b = blob[comp_b["offset"]:comp_b["offset"] + comp_b["nbytes"]].view(torch.bfloat16)
    g = n_in // 64
    s = s.to(torch.float32).view(n_out, g, 1)
    b = b.to(torch.float32).view(n_out, g, 1)
    return (q.view(n_out, g, 64) * s + b).view(n_out, n_in)


class DecodeStackCPU:
    """The 48-layer Qwen3 decode step of the benchmark on the host: one token
    through every layer's router, slot pool and experts."""

    def __init__(self, geom, blob_of, routers, n_slots, depth=1):
        """blob_of(key) -> numpy uint8 [blob_bytes], the store's blob of key
        layer * n_experts + expert."""
        self.geom = geom
        self.E, self.k = geom.n_experts, geom.top_k
        self.blob = geom.blob_bytes
        self.blob_of = blob_of
        self.w = [w.to(torch.float32) for w, _ in routers]
        self.b = [None if b is None else b.to(torch.float32) for _, b in routers]
        self.sim = PoolSim(n_slots, self.E, "lfu", depth, blob=self.blob)
        self.arena = np.empty((n_slots, self.blob), np.uint8)   # pages touched on fill
        self.comp = {(c["proj"], c["part"]): c for c in geom.components}
        self.depth = depth

    def _fill(self, fills):
        for slot, key in fills:
            self.arena[slot] = self.blob_of(key)

    def _proj(self, blob, proj, n_out, n_in):
        c = self.comp
        return dequant(blob, c[(proj, "weight")], c[(proj, "scales")], c[(proj, "biases")], n_out, n_in)

    def layer(self, layer, x):
        """y [d] for one token x [d] (float32 holding bf16 values)."""
        g = self.geom
        logits = bfr(self.w[layer] @ x + (self.b[layer] if self.b[layer] is not None else 0.0))
        probs = bfr(torch.softmax(logits, dim=-1))
        top = torch.topk(probs, self.k)
        inds = top.indices
        sc = top.values
        sc = bfr(sc / bfr(sc.sum()))
        nxt = layer + self.depth
        if nxt < g.n_layers:
            pl = bfr(self.w[nxt] @ x + (self.b[nxt] if self.b[nxt] is not None else 0.0))
            pred = torch.topk(pl, self.k).indices
            self._fill(self.sim.prefetch(nxt, sorted(set(pred.tolist()))))
        uniq = sorted(set(inds.tolist()))
        slots, fills = self.sim.acquire(layer, uniq)
        self._fill(fills)
        slot_of = dict(zip(uniq, slots))
        y = torch.zeros(g.d_model, dtype=torch.float32)
        for j, e in enumerate(inds.tolist()):
            blob = torch.from_numpy(self.arena[slot_of[e]])
            gate = bfr(self._proj(blob, "gate_proj", g.d_ff, g.d_model) @ x)
            up = bfr(self._proj(blob, "up_proj", g.d_ff, g.d_model) @ x)
            h = bfr(bfr(gate * bfr(torch.sigmoid(gate))) * up)
            yj = bfr(self._proj(blob, "down_proj", g.d_model, g.d_ff) @ h)
            y += bfr(yj * sc[j])
        return bfr(y)

    def step(self, xs):
        """One decoded token: xs [n_layers, d] (float32 holding bf16 values)."""
        return [self.layer(l, xs[l]) for l in range(self.geom.n_layers)]
