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
