"""MLX affine quantisation, restated in numpy (test infrastructure only).

The reference never quantises on its hot path: its store holds the codes that
``mlx_lm`` produced with ``mx.quantize`` (affine mode, group 64, 4 bits), and
its tests dequantise with ``mx.dequantize`` (test_kernel.py:57-60;
subspace_q1b.py:73-76, 89-91). MLX itself is not vendored, so this module
restates MLX 0.32's published affine scheme:

  per group of ``group_size`` consecutive input elements
    scale = max((w_max - w_min) / (2**bits - 1), 1e-7), signed so that the
            edge of larger magnitude is representable exactly,
    bias  = that edge (0 when it rounds to code 0),
    q     = clip(round((w - bias) / scale), 0, 2**bits - 1)   (ties to even)
  scales and biases are stored in the weight dtype (bf16); q is packed eight
  nibbles per uint32, element j of a row in bits 4*(j % 8) of word j // 8,
  low nibble first (kernels.py:129-139).

Dequantisation is ``w = scale * q + bias`` (kernels.py:104-112).
"""
import numpy as np

from . import bf16


def quantize(w, group_size=64, bits=4):
    """w: float [..., K] -> (packed uint32 [..., K*bits/32],
    scales bf16-bits uint16 [..., K/group_size], biases bf16-bits uint16)."""
    w = np.asarray(w, dtype=np.float32)
    shp = w.shape
    K = shp[-1]
    if K % group_size or K % (32 // bits):
        raise ValueError("last dim must be a multiple of the group size")
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    g = w.reshape(-1, K // group_size, group_size)
    w_max = g.max(axis=-1, keepdims=True)
    w_min = g.min(axis=-1, keepdims=True)
    mask = np.abs(w_min) > np.abs(w_max)
    scales = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
    scales = np.where(mask, scales, -scales).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.round(edge / scales).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        scales = np.where(q0 != 0, edge / q0, scales).astype(np.float32)
    biases = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    q = np.clip(np.round((g - biases) / scales), 0, n_bins).astype(np.uint32)
    per = 32 // bits
    q = q.reshape(*shp[:-1], K // per, per)
    packed = np.zeros(q.shape[:-1], dtype=np.uint32)
    for i in range(per):
        packed |= q[..., i] << np.uint32(bits * i)
    sshape = (*shp[:-1], K // group_size)
    return packed, bf16.to_bits(scales.reshape(sshape)), bf16.to_bits(biases.reshape(sshape))


def unpack(packed, bits=4):
    """packed uint32 [..., W] -> codes uint8 [..., W*32/bits]."""
    packed = np.asarray(packed, dtype=np.uint32)
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    q = np.stack([(packed >> np.uint32(bits * i)) & mask for i in range(per)], axis=-1)
    return q.reshape(*packed.shape[:-1], packed.shape[-1] * per).astype(np.uint8)


def dequantize_f32(packed, scales_bits, biases_bits, group_size=64, bits=4):
    """Unrounded dequantisation, as the quantised matmul uses it: float32
    ``scale*q + bias`` per element (MLX's qmm never materialises bf16 weights)."""
    q = unpack(packed, bits).astype(np.float32)
    s = bf16.from_bits(scales_bits)
    b = bf16.from_bits(biases_bits)
    K = q.shape[-1]
    q = q.reshape(*q.shape[:-1], K // group_size, group_size)
    w = q * s[..., None] + b[..., None]
    return w.reshape(*w.shape[:-2], K).astype(np.float32)


def dequantize_bf16(packed, scales_bits, biases_bits, group_size=64, bits=4):
    """``mx.dequantize`` on bf16 scales: the weight comes back as bf16
    (test_kernel.py:57-60), returned here as float32 values."""
    return bf16.r(dequantize_f32(packed, scales_bits, biases_bits, group_size, bits))


# ------------------------------------------------------ precision classes
# Per-expert precision (the kernels' classes): 2-, 3-, 4- or 8-bit codes as
# each row's little-endian bit stream (code j at bit bits*j, rows padded to
# 16 bytes), scales and biases in bf16 (mx.quantize) or fp8: OCP FP8 E4M3
# codes times a per-row 2^(E - 127). E4M3 here is restated from the OCP
# 8-bit floating point specification: sign, 4 exponent bits (bias 7), 3
# mantissa bits; exponent field 0 is subnormal (m/8 * 2^-6); the all-ones
# pattern S.1111.111 is NaN; largest finite 448; no infinities.

def _e4m3_table():
    vals = np.zeros(128, np.float64)
    for code in range(128):
        e, m = code >> 3, code & 7
        vals[code] = (m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
    vals[127] = np.nan
    return vals


E4M3 = _e4m3_table()


def e4m3_decode(codes):
    """uint8 E4M3 codes -> float32 values (exact)."""
    c = np.asarray(codes, np.uint8).astype(np.int64)
    v = E4M3[c & 0x7F]
    return np.where(c & 0x80, -v, v).astype(np.float32)


def e4m3_encode(x):
    """float32 -> E4M3 codes, round to nearest, ties to the even code;
    magnitudes above 448 saturate to 448."""
    x = np.asarray(x, np.float64)
    a = np.minimum(np.abs(x), 448.0)
    finite = E4M3[:127]
    hi = np.clip(np.searchsorted(finite, a, side="left"), 0, 126)   # finite[hi] >= a
    lo = np.maximum(hi - 1, 0)
    dlo, dhi = a - finite[lo], finite[hi] - a
    pick = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(hi % 2 == 0, hi, lo)))
    pick = np.where(a == finite[hi], hi, pick)
    return (pick | np.where(x < 0, 0x80, 0)).astype(np.uint8)


def fp8_rows(v):
    """v [rows, G] float32 -> (codes uint8, exps uint8 [rows], decoded
    float32): E = 127 + ceil(log2(max|v_row| / 448)) (127 for a zero row),
    clamped to [1, 254]; code = e4m3(v * 2^(127 - E))."""
    v = np.asarray(v, np.float32)
    amax = np.abs(v).max(axis=-1).astype(np.float64)
    E = np.full(amax.shape, 127, np.int64)
    nz = amax > 0
    m, e = np.frexp(amax[nz] / 448.0)
    E[nz] = 127 + np.where(m > 0.5, e, e - 1)
    E = np.clip(E, 1, 254)
    scaled = v.astype(np.float64) * np.exp2(127 - E)[:, None]
    codes = e4m3_encode(scaled)
    dec = (e4m3_decode(codes).astype(np.float64) * np.exp2(E - 127)[:, None]).astype(np.float32)
    return codes, E.astype(np.uint8), dec


def code_row_bytes(K, bits):
    return -(-(K * bits // 8) // 16) * 16


def pack_bits(q, bits, row_bytes):
    """codes [..., K] -> uint8 [..., row_bytes], each row a little-endian bit
    stream (code j at bit bits*j), zero padded."""
    q = np.asarray(q, np.uint64)
    K = q.shape[-1]
    out = np.zeros((*q.shape[:-1], row_bytes), np.uint8)
    for j in range(K):
        bit = bits * j
        v = q[..., j] << np.uint64(bit % 8)
        for b in range((bit % 8 + bits + 7) // 8):
            out[..., bit // 8 + b] |= ((v >> np.uint64(8 * b)) & np.uint64(0xFF)).astype(np.uint8)
    return out


def unpack_bits(packed, K, bits):
    """uint8 [..., row_bytes] rows -> codes uint8 [..., K]."""
    p = np.asarray(packed, np.uint8).astype(np.uint64)
    q = np.zeros((*p.shape[:-1], K), np.uint8)
    mask = np.uint64((1 << bits) - 1)
    for j in range(K):
        bit = bits * j
        v = np.zeros(p.shape[:-1], np.uint64)
        for b in range((bit % 8 + bits + 7) // 8):
            v |= p[..., bit // 8 + b] << np.uint64(8 * b)
        q[..., j] = ((v >> np.uint64(bit % 8)) & mask).astype(np.uint8)
    return q


def quantize_class(w, group_size=64, bits=4, scale_fmt="bf16"):
    """Affine quantisation into a precision class. bf16: mx.quantize's
    scales, biases and codes (codes from the unrounded float32 scales);
    fp8: the same float32 scales and biases stored per row by fp8_rows, and
    the codes computed against the stored (decoded) values. Returns a dict:
    weight uint8 [..., row_bytes]; scales / biases (bf16 bits uint16, or
    E4M3 codes uint8) [..., K/group_size]; fp8 also scales_exp / biases_exp
    uint8 [...]."""
    w = np.asarray(w, dtype=np.float32)
    shp = w.shape
    K = shp[-1]
    n_bins = np.float32((1 << bits) - 1)
    g = w.reshape(-1, K // group_size, group_size)
    w_max = g.max(axis=-1, keepdims=True)
    w_min = g.min(axis=-1, keepdims=True)
    mask = np.abs(w_min) > np.abs(w_max)
    scales = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7)).astype(np.float32)
    scales = np.where(mask, scales, -scales).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.round(edge / scales).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        scales = np.where(q0 != 0, edge / q0, scales).astype(np.float32)
    biases = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    out = {}
    sshape = (*shp[:-1], K // group_size)
    if scale_fmt == "fp8":
        rows = g.shape[0]
        sc, se, sd = fp8_rows(scales.reshape(rows, -1))
        bc, be, bd = fp8_rows(biases.reshape(rows, -1))
        out.update(scales=sc.reshape(sshape), biases=bc.reshape(sshape),
                   scales_exp=se.reshape(shp[:-1]), biases_exp=be.reshape(shp[:-1]))
        s_use, b_use = sd[..., None], bd[..., None]
        with np.errstate(divide="ignore", invalid="ignore"):
            q = np.where(s_use != 0, np.round((g - b_use) / np.where(s_use != 0, s_use, 1)), 0)
    else:
        out.update(scales=bf16.to_bits(scales.reshape(sshape)), biases=bf16.to_bits(biases.reshape(sshape)))
        q = np.round((g - biases) / scales)
    q = np.clip(q, 0, n_bins).astype(np.uint8).reshape(shp)
    out["weight"] = pack_bits(q, bits, code_row_bytes(K, bits))
    return out


def dequantize_class_f32(parts, K, bits, scale_fmt, group_size=64):
    """Unrounded float32 s*q + b of a precision-class matrix from its stored
    parts (quantize_class's dict, or blob views of the same)."""
    q = unpack_bits(parts["weight"], K, bits).astype(np.float32)
    if scale_fmt == "fp8":
        s = e4m3_decode(parts["scales"]) * np.exp2(
            parts["scales_exp"].astype(np.float64) - 127).astype(np.float32)[..., None]
        b = e4m3_decode(parts["biases"]) * np.exp2(
            parts["biases_exp"].astype(np.float64) - 127).astype(np.float32)[..., None]
    else:
        s = bf16.from_bits(parts["scales"])
        b = bf16.from_bits(parts["biases"])
    q = q.reshape(*q.shape[:-1], K // group_size, group_size)
    w = q * s[..., None] + b[..., None]
    return w.reshape(*w.shape[:-2], K).astype(np.float32)
