"""MoE expert block restated in numpy (test infrastructure only).

Follows, with MLX's bf16 rounding points:
  * blob layout            repack.py:72-82, repack_gptoss.py:139-166
  * Qwen3 router           engine_v3.py:467-473   (softmax over all experts,
                                                   top-k, renormalise)
  * gpt-oss router         engine_120b.py:65-70   (top-k of the logits,
                                                   softmax over the k)
  * speculative top-k      engine_v3.py:476-483, engine_120b.py:73-75
  * Qwen3 expert block     engine_v3.py:588-600   (gather_qmm x3, swiglu,
                                                   weighted sum)
  * gpt-oss expert block   engine_120b.py:130-145 (per-projection bias,
                                                   clamped swiglu)
  * fp32 reference         test_kernel.py:52-65

``mx.argpartition`` returns the top k in an unspecified order and breaks
exact ties in an unspecified way; this restatement orders by value
(descending) and breaks exact ties towards the lower expert index. Tests
therefore compare index SETS and accept differences only at exact ties.
"""
import numpy as np

from . import bf16
from .quant import dequantize_f32, dequantize_bf16, dequantize_class_f32

PAGE = 16384
PROJS = ("gate_proj", "up_proj", "down_proj")


def blob_layout(d_model, d_ff, group_size=64, bits=4, proj_bias=False):
    """Component list of one expert blob, in store order (repack.py:72-82;
    repack_gptoss.py:139-158). Returns (components, payload, blob_bytes)."""
    parts = ("weight", "scales", "biases") + (("bias",) if proj_bias else ())
    comps, off = [], 0
    for proj in PROJS:
        n_out, n_in = (d_ff, d_model) if proj != "down_proj" else (d_model, d_ff)
        for part in parts:
            if part == "weight":
                dt, shape, nb = "U32", [n_out, n_in * bits // 32], n_out * n_in * bits // 8
            elif part == "bias":
                dt, shape, nb = "BF16", [n_out], n_out * 2
            else:
                dt, shape, nb = "BF16", [n_out, n_in // group_size], n_out * (n_in // group_size) * 2
            comps.append(dict(proj=proj, part=part, dtype=dt, shape=shape, offset=off, nbytes=nb))
            off += nb
    blob = -(-off // PAGE) * PAGE
    return comps, off, blob


def blob_views(blob, comps):
    """Split one blob (uint8 bytes) into {'gate_proj.weight': array, ...}."""
    out = {}
    for c in comps:
        raw = blob[c["offset"]:c["offset"] + c["nbytes"]]
        if c["dtype"] == "U32":
            a = np.frombuffer(raw.tobytes(), dtype=np.uint32)
        elif c["dtype"] in ("F8E4M3", "U8"):
            a = np.frombuffer(raw.tobytes(), dtype=np.uint8)
        else:
            a = np.frombuffer(raw.tobytes(), dtype=np.uint16)
        out[f"{c['proj']}.{c['part']}"] = a.reshape(c["shape"])
    return out


# ----------------------------------------------------------------- routers
def linear_bf16(x, w, b=None):
    """MLX Linear on bf16 inputs: fp32 accumulation, bf16 output (one rounding,
    the bias added before it as ``addmm`` does)."""
    acc = (np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32)
    if b is not None:
        acc = acc + np.asarray(b, np.float32)
    return bf16.r(acc)


def softmax_precise(v):
    """``mx.softmax(..., precise=True)`` on bf16 input: fp32 internally, bf16 out."""
    v = np.asarray(v, np.float32)
    m = v.max(axis=-1, keepdims=True)
    e = np.exp(v - m).astype(np.float32)
    return bf16.r(e / e.sum(axis=-1, keepdims=True, dtype=np.float32))


def topk_desc(v, k):
    """Indices of the k largest values per row, descending, exact ties
    broken towards the lower index."""
    order = np.argsort(-np.asarray(v, np.float32), axis=-1, kind="stable")
    return order[..., :k].astype(np.int32)


def route_qwen3(x, w_r, k, norm=True, bias=None):
    """engine_v3.py:467-473. Returns (inds [T,k] int32, scores [T,k] bf16 values,
    probs [T,E] bf16 values)."""
    logits = linear_bf16(x, w_r, bias)
    g = softmax_precise(logits)
    inds = topk_desc(g, k)
    scores = np.take_along_axis(g, inds, axis=-1)
    if norm:
        s = bf16.r(scores.sum(axis=-1, keepdims=True, dtype=np.float32))
        scores = bf16.r(scores / s)
    return inds, scores, g


def route_gptoss(x, w_r, k, bias=None):
    """engine_120b.py:65-70. Returns (inds, scores, logits)."""
    logits = linear_bf16(x, w_r, bias)
    inds = topk_desc(logits, k)
    scores = softmax_precise(np.take_along_axis(logits, inds, axis=-1))
    return inds, scores, logits


def predict(x, w_r_next, kp, bias_next=None):
    """Speculative top-k of the next layer's raw logits on this layer's x
    (engine_v3.py:476-483, 509-514; engine_120b.py:73-75). The engine then
    takes ``np.unique`` of all tokens' predictions (engine_v3.py:523)."""
    logits = linear_bf16(x, w_r_next, bias_next)
    return topk_desc(logits, kp), logits


# ------------------------------------------------------------ expert math
def _deq(v, name, group_size, rounded=False, prec=None):
    """Dequantised weight of projection `name`. prec: None for the default
    4-bit bf16 blob, else (bits, scale_fmt, n_in) of a precision class."""
    if prec is not None:
        bits, fmt, K = prec
        parts = {p: v[f"{name}.{p}"] for p in ("weight", "scales", "biases", "scales_exp", "biases_exp")
                 if f"{name}.{p}" in v}
        parts["weight"] = parts["weight"].view(np.uint8)
        w = dequantize_class_f32(parts, K, bits, fmt, group_size)
        return bf16.r(w) if rounded else w
    f = dequantize_bf16 if rounded else dequantize_f32
    return f(v[f"{name}.weight"], v[f"{name}.scales"], v[f"{name}.biases"], group_size)


def _views_prec(blobs, comps, prec, e, d_model, d_ff):
    """Component views of expert e's blob and a function giving each
    projection's precision argument for _deq (prec: {e: (comps, bits, fmt)}
    for experts stored in a precision class)."""
    if prec is not None and e in prec:
        ce, bits, fmt = prec[e]
        n_in = {"gate_proj": d_model, "up_proj": d_model, "down_proj": d_ff}
        return blob_views(blobs[e], ce), (lambda name: (bits, fmt, n_in[name]))
    return blob_views(blobs[e], comps), (lambda name: None)


def _mm_bf16(inp, w):
    """gather_qmm: fp32-accurate product with the unrounded dequantised
    weight, bf16 output."""
    return bf16.r((np.asarray(inp, np.float64) @ w.astype(np.float64).T).astype(np.float32))


def _sigmoid(v):
    v = np.asarray(v, np.float64)
    return (1.0 / (1.0 + np.exp(-v))).astype(np.float32)


def swiglu_qwen3(g, u):
    """mlx_lm activations.swiglu = silu(gate) * x with silu = x*sigmoid(x),
    every op rounded to bf16 (engine_v3.py:41, 597)."""
    s = bf16.r(_sigmoid(g))
    return bf16.r(bf16.r(g * s) * u)


def swiglu_gptoss(u, g, alpha=1.702, limit=7.0):
    """gpt-oss clamped SwiGLU, argument order (linear, gate) as at
    engine_120b.py:143; each op rounded to bf16, the python-float alpha
    taking the bf16 operand's type (engine_120b.py:27-29)."""
    a = float(bf16.r(np.array([alpha], np.float32))[0])
    g = np.minimum(g, np.float32(limit))
    u = np.clip(u, -np.float32(limit), np.float32(limit))
    gs = bf16.r(np.float32(a) * g)
    og = bf16.r(g * bf16.r(_sigmoid(gs)))
    return bf16.r(og * bf16.r(u + np.float32(1.0)))


def _pairs_by_expert(inds):
    T, K = inds.shape
    by = {}
    for t in range(T):
        for j in range(K):
            by.setdefault(int(inds[t, j]), []).append((t, j))
    return by


def expert_block(x, inds, scores, blobs, comps, model, group_size=64, prec=None):
    """MLX-path block output for tokens x [T,d] (bf16 values).

    inds [T,k] select blobs (blobs[e] is a uint8 blob); scores [T,k] bf16
    values. Returns y [T,d] as bf16 values. Each expert is dequantised once.
    Qwen3: engine_v3.py:588-600. gpt-oss: engine_120b.py:130-145.
    prec: {e: (comps, bits, scale_fmt)} for experts stored in a precision
    class (their products use the class's unrounded s*q + b, as the 4-bit
    path does).
    """
    x = np.asarray(x, np.float32)
    T, K = inds.shape
    d = x.shape[-1]
    parts = np.zeros((T, K, d), np.float32)
    for e, prs in _pairs_by_expert(inds).items():
        d_ff = None
        if prec is not None and e in prec:
            d_ff = [c for c in prec[e][0] if c["proj"] == "down_proj" and c["part"] == "scales"][0]["shape"][1] * group_size
        v, pa = _views_prec(blobs, comps, prec, e, d, d_ff)
        xt = x[[t for t, _ in prs]]
        up = _mm_bf16(xt, _deq(v, "up_proj", group_size, prec=pa("up_proj")))
        gate = _mm_bf16(xt, _deq(v, "gate_proj", group_size, prec=pa("gate_proj")))
        if model == "gptoss":
            up = bf16.r(up + bf16.from_bits(v["up_proj.bias"]))
            gate = bf16.r(gate + bf16.from_bits(v["gate_proj.bias"]))
            h = swiglu_gptoss(up, gate)
            yj = _mm_bf16(h, _deq(v, "down_proj", group_size, prec=pa("down_proj")))
            yj = bf16.r(yj + bf16.from_bits(v["down_proj.bias"]))
        else:
            h = swiglu_qwen3(gate, up)
            yj = _mm_bf16(h, _deq(v, "down_proj", group_size, prec=pa("down_proj")))
        for i, (t, j) in enumerate(prs):
            parts[t, j] = bf16.r(yj[i] * np.float32(scores[t, j]))
    return bf16.r(parts.sum(axis=1, dtype=np.float32))


def rms_norm(h, w, eps):
    """mlx_lm's post-attention RMSNorm (mx.fast.rms_norm, MLX 0.32, a
    third-party dependency outside the reference): r = 1/sqrt(mean(h^2) +
    eps) in fp32, out = bf16(bf16(h * r) * w). h, w: bf16 values."""
    h = np.asarray(h, np.float32)
    ms_ = (h.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(ms_ + np.float32(eps))).astype(np.float32)
    return bf16.r(bf16.r(h * r) * np.asarray(w, np.float32))


def fp32_reference(x, inds, scores, blobs, comps, model, group_size=64, prec=None):
    """test_kernel.py:52-65: dequantise (bf16 weights, as mx.dequantize
    returns them), then the whole MLP in fp32 (float64 here). gpt-oss adds
    its biases and the clamped activation at full precision as well."""
    x = np.asarray(x, np.float64)
    T, K = inds.shape
    y = np.zeros((T, x.shape[-1]), np.float64)
    for e, prs in _pairs_by_expert(inds).items():
        d_ff = None
        if prec is not None and e in prec:
            d_ff = [c for c in prec[e][0] if c["proj"] == "down_proj" and c["part"] == "scales"][0]["shape"][1] * group_size
        v, pa = _views_prec(blobs, comps, prec, e, x.shape[-1], d_ff)
        w = {p: _deq(v, p, group_size, rounded=True, prec=pa(p)).astype(np.float64) for p in PROJS}
        xt = x[[t for t, _ in prs]]
        gate = xt @ w["gate_proj"].T
        up = xt @ w["up_proj"].T
        if model == "gptoss":
            gate = np.minimum(gate + bf16.from_bits(v["gate_proj.bias"]), 7.0)
            up = np.clip(up + bf16.from_bits(v["up_proj.bias"]), -7.0, 7.0)
            h = gate / (1.0 + np.exp(-1.702 * gate)) * (up + 1.0)
            yj = h @ w["down_proj"].T + bf16.from_bits(v["down_proj.bias"])
        else:
            h = gate / (1.0 + np.exp(-gate)) * up
            yj = h @ w["down_proj"].T
        for i, (t, j) in enumerate(prs):
            y[t] += float(scores[t, j]) * yj[i]
    return y


def rel_err(a, ref):
    """test_kernel.py:68-71: max-abs error over max |ref|."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(a - ref).max() / (np.abs(ref).max() + 1e-30))
