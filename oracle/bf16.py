"""bfloat16 emulation on float32 numpy arrays (test infrastructure only).

MLX carries bf16 between operations, so every op output is rounded to bf16
(round to nearest, ties to even). bf16 is the upper half of an IEEE float32
bit pattern (kernels.py:66-72 reads it the same way).
"""
import numpy as np


def to_bits(a):
    """float32 array -> uint16 bf16 bit patterns, round-to-nearest-even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + r) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.uint16(0x7FC0)
    return out


def from_bits(b):
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def r(a):
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return from_bits(to_bits(a))


def ulp(a):
    """Spacing of bf16 values at |a| (float32 result), for tie tolerances."""
    a = np.abs(np.asarray(a, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(1e-38))))
    return np.exp2(e - 7).astype(np.float32)
