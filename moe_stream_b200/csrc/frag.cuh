// Tensor-core dequant-dot for 4-bit affine weights (mma.sync m16n8k16, f16
// inputs, f32 accumulate).
//
// A (weights) never goes through a dequantised copy. A 32-bit word holds the
// codes q0..q7 of 8 consecutive inputs of one row (low nibble first,
// kernels.py:137-139). One LOP3 per register ORs two nibbles into the
// mantissas of an f16x2 whose exponent is that of 1024:
//   R0 = (u & 0x000F000F) | 0x64006400 -> {1024 + q0,    1024 + q4}
//   R1 = (u & 0x00F000F0) | 0x64006400 -> {1024 + 16*q1, 1024 + 16*q5}
//   R2 = R0 of (u >> 8)                -> {1024 + q2,    1024 + q6}
//   R3 = R1 of (u >> 8)                -> {1024 + 16*q3, 1024 + 16*q7}
// The activation operand is stored pre-divided by 16 at the odd positions,
// so an MMA over a 64-input quantisation group g gives
//   acc_g = 1024 * X'_g + sum_k q_k x_k,     X'_g = sum_k x'_k,
// and the row output is sum_g s_g * (acc_g - 1024 X'_g) + b_g * X_g with
// X_g = sum_k x_k -- the scale/bias factoring of kernels.py:104-112, applied
// once per group instead of once per weight.
//
// Activation layout ("frag" layout, f16): per (row of activations r, group
// kg) 64 halves = 128 B, ordered [p][c][8] where word w = 2c + p of the
// group and the 8 halves are the B-operand registers {MMA1.b0, MMA1.b1,
// MMA2.b0, MMA2.b1} of lane c: element i of word w lands at half index
// ((i & 3) << 1) | (i >> 2), divided by 16 when i is odd. Per (r, kg) two
// floats X_g, X'_g are kept beside it.
#pragma once
#include "ms_common.cuh"

namespace ms {

__device__ __forceinline__ uint32_t lop_or(uint32_t u, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(u), "r"(mask), "r"(0x64006400u));
  return r;
}

// Not volatile: the MMA is a pure function of its operands, so the compiler
// may interleave the independent accumulation chains of different groups.
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One quantisation group of a 16-row tile: words ra (row g) and rb (row g+8)
// of this lane (uint2 = words 2c and 2c+1 of the group), activation
// fragments b0 (p = 0) and b1 (p = 1). Accumulates into c[4].
__device__ __forceinline__ void mma_group(float* c, uint2 ra, uint2 rb, uint4 b0, uint4 b1) {
  const uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u;
  {
    const uint32_t u = ra.x, v = rb.x, us = u >> 8, vs = v >> 8;
    mma16816(c, lop_or(u, M0), lop_or(v, M0), lop_or(u, M1), lop_or(v, M1), b0.x, b0.y);
    mma16816(c, lop_or(us, M0), lop_or(vs, M0), lop_or(us, M1), lop_or(vs, M1), b0.z, b0.w);
  }
  {
    const uint32_t u = ra.y, v = rb.y, us = u >> 8, vs = v >> 8;
    mma16816(c, lop_or(u, M0), lop_or(v, M0), lop_or(u, M1), lop_or(v, M1), b1.x, b1.y);
    mma16816(c, lop_or(us, M0), lop_or(vs, M0), lop_or(us, M1), lop_or(vs, M1), b1.z, b1.w);
  }
}

// Offset (in halves) of input element k of activation row r in frag layout.
__device__ __forceinline__ long long frag_off(long long r, int G, int k) {
  const int kg = k >> 6, w = (k >> 3) & 7, i = k & 7;
  const int p = w & 1, cc = w >> 1, hidx = ((i & 3) << 1) | (i >> 2);
  return ((r * G + kg) * 2 + p) * 32 + cc * 8 + hidx;
}

// Frag layout of activation row r, quantisation group kg, word w (inputs
// 8w..8w+7 of the group) from 8 bf16 values: the 8 halves are exactly the
// 16-byte B-operand block of lane w>>1, pass w&1, so one thread writes one
// uint4. The group's sums (X, X') are reduced over the 8 lanes that handle
// words 0..7 (aligned octet of the warp, all active) and written by word 0.
// Returns true when one of the 8 values lies beyond the fp16 range. (Values
// below fp16's normal range, 2^-14, or 2^-10 at the odd positions, keep an
// absolute precision of 2^-24 (2^-20 before the division by 16): far below
// a bf16 output ulp, so they are not flagged.)
__device__ __forceinline__ bool frag_write_word(const uint16_t* src8, __half* frag, float* sums,
                                                long long r, int G, int kg, int w, bool valid) {
  float xs = 0.f, xp = 0.f;
  bool over = false;
  if (valid) {
    const uint4 v = *reinterpret_cast<const uint4*>(src8);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    __half h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint16_t b = (uint16_t)((w4[i >> 1] >> ((i & 1) * 16)) & 0xffffu);
      const float xf = bf2f(b);
      over |= fabsf(xf) > F16_MAX;
      const __half x = __float2half_rn(xf);
      const __half xs_ = (i & 1) ? __hmul(x, __float2half(0.0625f)) : x;
      xs += __half2float(x);
      xp += __half2float(xs_);
      h[((i & 3) << 1) | (i >> 2)] = xs_;
    }
    uint4 out;
    out.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
    out.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
    out.z = (uint32_t)__half_as_ushort(h[4]) | ((uint32_t)__half_as_ushort(h[5]) << 16);
    out.w = (uint32_t)__half_as_ushort(h[6]) | ((uint32_t)__half_as_ushort(h[7]) << 16);
    *reinterpret_cast<uint4*>(frag + (r * G + kg) * 64 + ((w & 1) * 4 + (w >> 1)) * 8) = out;
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    xs += __shfl_xor_sync(MS_FULL, xs, o);
    xp += __shfl_xor_sync(MS_FULL, xp, o);
  }
  if (valid && w == 0) {
    sums[(r * G + kg) * 2] = xs;
    sums[(r * G + kg) * 2 + 1] = xp;
  }
  return over;
}

// Frag layout of rows [0, T) of x (bf16 [T, d]) by the calling threads:
// thread index `tid` of `nthreads` (a multiple of 32), grid-stride.
// Records ST_E_RANGE in *status (first error wins) when a value of x lies
// beyond the fp16 range.
__device__ __forceinline__ void frag_write_rows(const uint16_t* x, int T, int d, __half* frag,
                                                float* sums, int tid, int nthreads, int* status) {
  const int G = d / 64;
  const int tasks = T * G * 8;
  const int rounded = (tasks + 31) & ~31;
  bool over = false;
  for (int i = tid; i < rounded; i += nthreads) {
    const bool valid = i < tasks;
    const int grp = valid ? (i >> 3) : 0, w = i & 7;
    const int t = grp / G, kg = grp % G;
    over |= frag_write_word(x + (long long)t * d + kg * 64 + w * 8, frag, sums, t, G, kg, w, valid);
  }
  if (over) atomicCAS(status, 0, ST_E_RANGE);
}

}  // namespace ms
