"""Synthetic expert stores in the reference's blob format.

There are no checkpoints here, so stores are generated from seeded normal
weights (N(0, 0.02), the configs' distribution) and quantised with MLX's
affine scheme (group 64, 4 bits, bf16 scales/biases). The quantiser runs in
torch so that it can run on the GPU for multi-GB stores; tests check it
bit-exactly against the numpy oracle's restatement.

Random streams: blob (layer, expert) uses its own torch Generator seeded
with ``seed * 1_000_003 + layer * 1009 + expert``, so any subset of blobs can
be regenerated independently and identically on the CPU and on the GPU
(torch's CPU and CUDA generators differ, so the device is part of the
recipe: ``device`` below).
"""
import numpy as np
import torch

from .geometry import PROJS


def quantize(w, group_size=64, bits=4):
    """MLX affine quantisation of w [..., K] (float32, bf16-valued).
    Returns (packed uint32 as int32 tensor [..., K/8], scales bf16, biases bf16)."""
    w = w.to(torch.float32)
    shp = w.shape
    K = shp[-1]
    n_bins = torch.tensor(float((1 << bits) - 1), dtype=torch.float32, device=w.device)
    eps = torch.tensor(1e-7, dtype=torch.float32, device=w.device)
    g = w.reshape(-1, K // group_size, group_size)
    w_max = g.amax(dim=-1, keepdim=True)
    w_min = g.amin(dim=-1, keepdim=True)
    mask = w_min.abs() > w_max.abs()
    scales = torch.maximum((w_max - w_min) / n_bins, eps)
    scales = torch.where(mask, scales, -scales)
    edge = torch.where(mask, w_min, w_max)
    q0 = torch.round(edge / scales)
    scales = torch.where(q0 != 0, edge / q0, scales)
    biases = torch.where(q0 == 0, torch.zeros_like(edge), edge)
    q = torch.clamp(torch.round((g - biases) / scales), 0, float((1 << bits) - 1)).to(torch.int64)
    per = 32 // bits
    q = q.reshape(*shp[:-1], K // per, per)
    shifts = (torch.arange(per, device=w.device, dtype=torch.int64) * bits)
    packed = (q << shifts).sum(dim=-1)                       # < 2**32
    packed = (packed - ((packed >> 31) << 32)).to(torch.int32)  # reinterpret as int32
    sshape = (*shp[:-1], K // group_size)
    return (packed, scales.reshape(sshape).to(torch.bfloat16),
            biases.reshape(sshape).to(torch.bfloat16))


def _affine_params(g, bits):
    """MLX affine scales and biases (float32, unrounded) of groups g [..., gs]."""
    n_bins = torch.tensor(float((1 << bits) - 1), dtype=torch.float32, device=g.device)
    eps = torch.tensor(1e-7, dtype=torch.float32, device=g.device)
    w_max = g.amax(dim=-1, keepdim=True)
    w_min = g.amin(dim=-1, keepdim=True)
    mask = w_min.abs() > w_max.abs()
    scales = torch.maximum((w_max - w_min) / n_bins, eps)
    scales = torch.where(mask, scales, -scales)
    edge = torch.where(mask, w_min, w_max)
    q0 = torch.round(edge / scales)
    scales = torch.where(q0 != 0, edge / q0, scales)
    biases = torch.where(q0 == 0, torch.zeros_like(edge), edge)
    return scales, biases


def fp8_rows(v):
    """Per-row fp8 storage of v [rows, G] (float32): OCP E4M3 codes (uint8)
    of v * 2^(127 - E) and one exponent byte E per row, E the smallest with
    max|v_row| * 2^(127 - E) <= 448 (127 for an all-zero row). Returns
    (codes, exps, decoded float32 values)."""
    amax = v.abs().amax(dim=-1)
    m, e = torch.frexp(amax / 448.0)
    up = torch.where(m > 0.5, e, e - 1)                 # ceil(log2(amax / 448))
    E = torch.where(amax > 0, 127 + up, torch.full_like(up, 127)).clamp(1, 254)
    scaled = torch.ldexp(v, (127 - E).unsqueeze(-1).to(v.dtype))
    codes8 = scaled.to(torch.float8_e4m3fn)
    dec = torch.ldexp(codes8.to(torch.float32), (E - 127).unsqueeze(-1).to(v.dtype))
    return codes8.view(torch.uint8), E.to(torch.uint8), dec


def pack_codes(q, bits, row_bytes):
    """Codes q [..., K] (int64 in [0, 2^bits)) as each row's little-endian
    bit stream (code j at bit bits*j), rows padded to row_bytes: uint8."""
    shp = q.shape
    K = shp[-1]
    if bits == 3:
        q = q.reshape(*shp[:-1], K // 8, 8)
        v = (q << (torch.arange(8, device=q.device, dtype=torch.int64) * 3)).sum(-1)
        by = torch.stack([(v >> (8 * i)) & 0xFF for i in range(3)], dim=-1)
    else:
        per = 8 // bits
        q = q.reshape(*shp[:-1], K // per, per)
        by = (q << (torch.arange(per, device=q.device, dtype=torch.int64) * bits)).sum(-1)
    by = by.reshape(*shp[:-1], -1).to(torch.uint8)
    pad = row_bytes - by.shape[-1]
    if pad:
        by = torch.cat([by, torch.zeros(*shp[:-1], pad, dtype=torch.uint8, device=q.device)], -1)
    return by


def quantize_class(w, group_size=64, bits=4, scale_fmt="bf16"):
    """Affine quantisation of w [..., K] into precision class (bits,
    scale_fmt). bf16: mx.quantize (codes from the unrounded float32 scales,
    scales and biases stored as bf16). fp8: scales and biases stored per row
    as E4M3 times 2^(E - 127) (fp8_rows), and the codes computed against
    those stored values, so the codes fit what the kernels will decode.
    Returns {part: tensor} with weight as uint8 [..., row_bytes]."""
    from .geometry import code_row_bytes
    w = w.to(torch.float32)
    shp = w.shape
    K = shp[-1]
    g = w.reshape(-1, K // group_size, group_size)
    scales, biases = _affine_params(g, bits)
    out = {}
    if scale_fmt == "fp8":
        rows = g.shape[0]
        sc, se, sd = fp8_rows(scales.reshape(rows, -1))
        bc, be, bd = fp8_rows(biases.reshape(rows, -1))
        scales, biases = sd.unsqueeze(-1), bd.unsqueeze(-1)
        out.update(scales=sc.reshape(*shp[:-1], -1), biases=bc.reshape(*shp[:-1], -1),
                   scales_exp=se.reshape(shp[:-1]), biases_exp=be.reshape(shp[:-1]))
        safe = torch.where(scales != 0, scales, torch.ones_like(scales))
        q = torch.where(scales != 0, torch.round((g - biases) / safe), torch.zeros_like(g))
    else:
        sshape = (*shp[:-1], K // group_size)
        out.update(scales=scales.reshape(sshape).to(torch.bfloat16),
                   biases=biases.reshape(sshape).to(torch.bfloat16))
        q = torch.round((g - biases) / scales)
    q = torch.clamp(q, 0, float((1 << bits) - 1)).to(torch.int64).reshape(shp)
    out["weight"] = pack_codes(q, bits, code_row_bytes(K, bits))
    return out


def _gen(seed, layer, expert, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + layer * 1009 + expert)
    return g


def expert_weights(geom, seed, layer, expert, device="cpu", std=0.02):
    """bf16-valued float32 weights of one expert: {proj: [out, in]} plus the
    gpt-oss projection biases {proj + '.bias': [out]}."""
    gen = _gen(seed, layer, expert, device)
    out = {}
    for proj in PROJS:
        n_out, n_in = (geom.d_model, geom.d_ff) if proj == "down_proj" else (geom.d_ff, geom.d_model)
        w = torch.randn(n_out, n_in, generator=gen, device=device, dtype=torch.float32) * std
        out[proj] = w.to(torch.bfloat16).to(torch.float32)
        if geom.proj_bias:
            b = torch.randn(n_out, generator=gen, device=device, dtype=torch.float32) * std
            out[proj + ".bias"] = b.to(torch.bfloat16)
    return out


def pack_blob(geom, weights):
    """One expert's blob (uint8 tensor [blob_bytes]) from its weights."""
    dev = next(iter(weights.values())).device
    blob = torch.zeros(geom.blob_bytes, dtype=torch.uint8, device=dev)
    default = geom.bits == 4 and geom.scale_fmt == "bf16"
    for proj in PROJS:
        if default:
            q, s, b = quantize(weights[proj], geom.group_size, geom.bits)
            parts = {"weight": q, "scales": s, "biases": b}
        else:
            parts = quantize_class(weights[proj], geom.group_size, geom.bits, geom.scale_fmt)
        if geom.proj_bias:
            parts["bias"] = weights[proj + ".bias"]
        for part, t in parts.items():
            c = geom.comp(proj, part)
            raw = t.contiguous().view(torch.uint8).reshape(-1)
            assert raw.numel() == c["nbytes"], (proj, part, raw.numel(), c["nbytes"])
            blob[c["offset"]:c["offset"] + c["nbytes"]] = raw
    return blob


def make_blob(geom, seed, layer, expert, device="cpu"):
    return pack_blob(geom, expert_weights(geom, seed, layer, expert, device))


def fill_store(geom, host_u8, seed, layers=None, experts=None, device="cpu", batch=16):
    """Write blobs into a host uint8 array laid out as the store. layers /
    experts restrict which blobs are generated (others are left as they are)."""
    layers = range(geom.n_layers) if layers is None else layers
    experts = range(geom.n_experts) if experts is None else experts
    view = torch.from_numpy(host_u8) if isinstance(host_u8, np.ndarray) else host_u8
    for layer in layers:
        for e in experts:
            key = layer * geom.n_experts + e
            blob = make_blob(geom, seed, layer, e, device)
            view[key * geom.blob_bytes:(key + 1) * geom.blob_bytes].copy_(blob, non_blocking=False)


def fill_store_classes(slot_geom, classes, class_of_key, host_u8, seed, layers=None, experts=None,
                       device="cpu"):
    """fill_store for a pool with precision classes: blob (layer, expert) is
    make_blob of its class geometry (same seeded weights as the 4-bit
    store), written at the pool's stride slot_geom.blob_bytes."""
    layers = range(slot_geom.n_layers) if layers is None else layers
    experts = range(slot_geom.n_experts) if experts is None else experts
    view = torch.from_numpy(host_u8) if isinstance(host_u8, np.ndarray) else host_u8
    stride = slot_geom.blob_bytes
    for layer in layers:
        for e in experts:
            key = layer * slot_geom.n_experts + e
            cg = classes[int(class_of_key[key])]
            blob = make_blob(cg, seed, layer, e, device)
            view[key * stride:key * stride + cg.blob_bytes].copy_(blob, non_blocking=False)


def router_weights(geom, seed, layer, device="cpu", std=0.02, zipf_s=None, bias_std=None):
    """Router (gate) of one layer: w bf16 [E, d] ~ N(0, std). With zipf_s, a
    bias log(p_{pi(e)}) with p_r ~ r^-s over a seeded permutation pi (the
    skewed-routing configs); with bias_std, a N(0, bias_std) bias (gpt-oss
    routers carry one). Returns (w, b or None) as bf16 tensors."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed * 7_000_003 + layer * 131 + 17)
    w = (torch.randn(geom.n_experts, geom.d_model, generator=g) * std).to(torch.bfloat16)
    b = None
    if zipf_s is not None:
        perm = torch.randperm(geom.n_experts, generator=g)
        r = torch.arange(1, geom.n_experts + 1, dtype=torch.float64)
        p = r ** (-zipf_s)
        p = p / p.sum()
        b = torch.empty(geom.n_experts, dtype=torch.float64)
        b[perm] = torch.log(p)
        b = b.to(torch.bfloat16)
    elif bias_std is not None:
        b = (torch.randn(geom.n_experts, generator=g) * bias_std).to(torch.bfloat16)
    return w.to(device), (None if b is None else b.to(device))


def rms_norm_tokens(T, d, seed, device="cpu"):
    """x ~ N(0,1), RMS-normalised (no weight), bf16 [T, d] (config 0)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed * 3_000_017 + 5)
    x = torch.randn(T, d, generator=g, dtype=torch.float32)
    x = x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + 1e-6)
    return x.to(torch.bfloat16).to(device)


def make_layer_blobs(geom, seed, layer, device="cuda", std=0.02, chunk=32):
    """All n_experts blobs of one layer at once (uint8 [n_experts, blob_bytes]
    on `device`), for multi-GB stores. One generator per (seed, layer); a
    different recipe from make_blob, so the two are not interchangeable."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + layer * 1009 + 977)
    E = geom.n_experts
    out = torch.zeros(E, geom.blob_bytes, dtype=torch.uint8, device=device)
    for e0 in range(0, E, chunk):
        n = min(chunk, E - e0)
        for proj in PROJS:
            n_out, n_in = (geom.d_model, geom.d_ff) if proj == "down_proj" else (geom.d_ff, geom.d_model)
            w = (torch.randn(n, n_out, n_in, generator=g, device=device) * std)
            w = w.to(torch.bfloat16).to(torch.float32)
            q, s, b = quantize(w, geom.group_size, geom.bits)
            parts = {"weight": q, "scales": s, "biases": b}
            if geom.proj_bias:
                parts["bias"] = (torch.randn(n, n_out, generator=g, device=device) * std).to(torch.bfloat16)
            for part, t in parts.items():
                c = geom.comp(proj, part)
                raw = t.contiguous().view(torch.uint8).reshape(n, -1)
                out[e0:e0 + n, c["offset"]:c["offset"] + c["nbytes"]] = raw
            del w, q, s, b, parts
    return out


def make_layer_blobs_classes(geom, classes, cls_of_e, seed, layer, device="cuda", std=0.02,
                             chunk=32):
    """make_layer_blobs for experts stored in precision classes: the same
    weights (same generator and draw order), each expert quantised into
    classes[cls_of_e[e]] and laid out at the start of its row of the result
    (uint8 [n_experts, geom.blob_bytes], geom the pool's slot geometry)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + layer * 1009 + 977)
    E = geom.n_experts
    cls_of_e = torch.as_tensor(np.asarray(cls_of_e, np.int64), device=device)
    out = torch.zeros(E, geom.blob_bytes, dtype=torch.uint8, device=device)
    for e0 in range(0, E, chunk):
        n = min(chunk, E - e0)
        cl = cls_of_e[e0:e0 + n]
        for proj in PROJS:
            n_out, n_in = (geom.d_model, geom.d_ff) if proj == "down_proj" else (geom.d_ff, geom.d_model)
            w = (torch.randn(n, n_out, n_in, generator=g, device=device) * std)
            w = w.to(torch.bfloat16).to(torch.float32)
            bias = None
            if geom.proj_bias:
                bias = (torch.randn(n, n_out, generator=g, device=device) * std).to(torch.bfloat16)
            for c, cg in enumerate(classes):
                idx = torch.nonzero(cl == c).flatten()
                if idx.numel() == 0:
                    continue
                parts = quantize_class(w[idx], cg.group_size, cg.bits, cg.scale_fmt)
                if bias is not None:
                    parts["bias"] = bias[idx]
                rows = e0 + idx
                for part, t in parts.items():
                    comp = cg.comp(proj, part)
                    raw = t.contiguous().view(torch.uint8).reshape(idx.numel(), -1)
                    out[rows, comp["offset"]:comp["offset"] + comp["nbytes"]] = raw
            del w
    return out


def decode_inputs(n_steps, n_layers, d, seed, step_sigma=0.1):
    """Config-1 hidden states: per decode step an i.i.d. h_0 ~ N(0,1), then
    h_{l+1} = h_l + step_sigma * N(0,1); the block input of layer l is
    RMS-normalised h_l in bf16. Returns bf16 [n_steps, n_layers, d] (CPU)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed * 5_000_011 + 23)
    h = torch.randn(n_steps, 1, d, generator=g)
    steps = torch.randn(n_steps, n_layers - 1, d, generator=g) * step_sigma
    hs = torch.cat([h, h + torch.cumsum(steps, dim=1)], dim=1)
    x = hs * torch.rsqrt(hs.pow(2).mean(dim=-1, keepdim=True) + 1e-6)
    return x.to(torch.bfloat16)
