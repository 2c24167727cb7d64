// Per-expert precision classes: the weight codes of an expert are 2, 3, 4 or
// 8 bits wide and its scales and biases are bf16 or fp8 (the reference's
// stated purpose for owning the expert kernel, kernels.py:25-29: per-expert
// mixed precision, which gather_qmm cannot express because it takes one
// `bits` per call; fp8 scales, its lossless-axis note on the blob's scales).
//
// Codes. A row's codes form one little-endian bit stream: code j of the row
// occupies bits [b*j, b*j + b) of the row's bytes, so a quantisation group
// of 64 codes is 8*b bytes (mx.quantize's packing for 2, 3, 4 and 8 bits).
//
// fp8 scales. scales and biases are OCP FP8 E4M3 codes, [out, in/64] bytes,
// times a per-row power of two: scales_exp / biases_exp hold one byte E per
// row and the value is e4m3(code) * 2^(E - 127). Every such value is exactly
// a float (and a bf16 inside bf16's range), so the kernels' arithmetic after
// the decode is the bf16-scale arithmetic.
//
// A class is a component table like ms_geom's: comp_offset[proj][part] with
// parts weight, scales, biases, bias (gpt-oss), scales_exp, biases_exp.
#pragma once
#include "ms_common.cuh"
#include "frag.cuh"

#ifndef MS_MAX_CLASSES
#define MS_MAX_CLASSES 8
#endif

namespace ms {

constexpr int SF_BF16 = 0, SF_FP8 = 1;
constexpr int P_W = 0, P_S = 1, P_B = 2, P_BIAS = 3, P_SE = 4, P_BE = 5;

struct PrecDev {
  int bits, fmt;
  long long off[3][6];
};

struct ClassTab {
  int n;
  PrecDev c[MS_MAX_CLASSES];
};

// e4m3 byte -> float, exact (cvt.rn.f16x2.e4m3x2: every e4m3 value is an
// f16 value)
__device__ __forceinline__ float e4m3_to_f(uint8_t v) {
  uint32_t h2;
  const uint16_t pair = v;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(pair));
  return __half2float(__ushort_as_half((uint16_t)(h2 & 0xffffu)));
}

// 2^(E - 127) for a row exponent byte (1..254 by construction)
__device__ __forceinline__ float exp_factor(uint8_t e) {
  return __uint_as_float(((uint32_t)e) << 23);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (t & m) | c in one LOP3
__device__ __forceinline__ uint32_t and_or(uint32_t t, uint32_t m, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(t), "r"(m), "r"(c));
  return r;
}

// The MMA A registers of lane quad position c for one row and one
// quantisation group, in the activation frag layout's k order: R[p][0..3]
// for the lane's words w = 2c + p (group elements 8w..8w+7), each
//   R0 = {e(q0), e(q4)}, R1 = {o(q1), o(q5)}, R2 = {e(q2), e(q6)},
//   R3 = {o(q3), o(q7)}
// with e(q) = 1024 + q and o(q) = 1024 + 16 q (2, 3, 4 bits; the odd
// positions of the activation are stored divided by 16), or o(q) = 16384 +
// 16 q (8 bits, whose 16 q does not fit the 1024 exponent). The MMA over a
// group then gives 1024 X' + sum q x (2, 3, 4 bits) or 1024 X + sum q x (8
// bits); see corr_sum.
// rowgrp: the row's first byte of the group, 8*BITS bytes.
template <int BITS>
__device__ __forceinline__ void group_regs(const uint8_t* rowgrp, int c, uint32_t R[2][4]);

template <>
__device__ __forceinline__ void group_regs<4>(const uint8_t* rowgrp, int c, uint32_t R[2][4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(rowgrp + 8 * c);
  const uint32_t w[2] = {u.x, u.y};
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    R[p][0] = lop_or(w[p], 0x000F000Fu);
    R[p][1] = lop_or(w[p], 0x00F000F0u);
    R[p][2] = lop_or(w[p] >> 8, 0x000F000Fu);
    R[p][3] = lop_or(w[p] >> 8, 0x00F000F0u);
  }
}

template <>
__device__ __forceinline__ void group_regs<2>(const uint8_t* rowgrp, int c, uint32_t R[2][4]) {
  // bytes B0..B3 of the lane's word hold codes 0-3, 4-7, 8-11, 12-15;
  // v = [B0, B2, B1, B3] puts codes i and i+4 of each 8-code half 16 bits apart
  const uint32_t v = prmt(*reinterpret_cast<const uint32_t*>(rowgrp + 4 * c), 0u, 0x3120u);
  const uint32_t E = 0x00030003u, O = 0x00300030u, C = 0x64006400u;
  R[0][0] = and_or(v, E, C);
  R[0][1] = and_or(v << 2, O, C);
  R[0][2] = and_or(v >> 4, E, C);
  R[0][3] = and_or(v >> 2, O, C);
  R[1][0] = and_or(v >> 8, E, C);
  R[1][1] = and_or(v >> 6, O, C);
  R[1][2] = and_or(v >> 12, E, C);
  R[1][3] = and_or(v >> 10, O, C);
}

template <>
__device__ __forceinline__ void group_regs<8>(const uint8_t* rowgrp, int c, uint32_t R[2][4]) {
  const uint4 u = *reinterpret_cast<const uint4*>(rowgrp + 16 * c);
  const uint32_t a[2] = {u.x, u.z}, b[2] = {u.y, u.w};
  // K: byte 4 = 0x64 (exponent of 1024), byte 5 = 0x74 (exponent of 16384)
  const uint32_t K = 0x00007464u;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const uint32_t t0 = prmt(a[p], b[p], 0x5140u);   // [q0, q4, q1, q5]
    const uint32_t t1 = prmt(a[p], b[p], 0x7362u);   // [q2, q6, q3, q7]
    R[p][0] = prmt(t0, K, 0x4140u);
    R[p][1] = prmt(t0, K, 0x5352u);
    R[p][2] = prmt(t1, K, 0x4140u);
    R[p][3] = prmt(t1, K, 0x5352u);
  }
}

template <>
__device__ __forceinline__ void group_regs<3>(const uint8_t* rowgrp, int c, uint32_t R[2][4]) {
  // the lane's 16 codes are bits [48c, 48c + 48) of the group: bytes 6c..6c+5,
  // read as two aligned words and shifted into place
  const int b0 = 6 * c, base = b0 & ~3, sh = (b0 & 3) * 8;
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(rowgrp + base);
  const uint32_t hi = *reinterpret_cast<const uint32_t*>(rowgrp + base + 4);
  const uint32_t a = sh ? __funnelshift_r(lo, hi, 16) : lo;        // bits 0..31
  const uint32_t bb = sh ? (hi >> 16) : hi;                        // bits 32..47
  const uint32_t t[2] = {a, __funnelshift_r(a, bb, 24)};            // codes 0-7, 8-15
  const uint32_t C = 0x64006400u;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const uint32_t x = t[p];   // code i at bits 3i
    R[p][0] = and_or(x << 4, 0x00070000u, and_or(x, 0x7u, C));
    R[p][1] = and_or(x << 5, 0x00700000u, and_or(x << 1, 0x70u, C));
    R[p][2] = and_or(x >> 2, 0x00070000u, and_or(x >> 6, 0x7u, C));
    R[p][3] = and_or(x >> 1, 0x00700000u, and_or(x >> 5, 0x70u, C));
  }
}

// Which activation sum the 1024 offset multiplies: X' (frag layout's
// divided odd positions) for 2, 3 and 4 bits, X for 8 bits.
template <int BITS>
__device__ __forceinline__ float corr_sum(float2 sums) {
  return BITS == 8 ? sums.x : sums.y;
}

// Scale and bias of (row, group) of a staged tile: bf16 [rows][G] halves,
// or fp8 [rows][G] bytes with the row's factor.
struct SBTile {
  const uint8_t* s;   // scales of the tile's first row
  const uint8_t* b;   // biases
  const uint8_t* se;  // fp8: per-row exponent bytes (tile rows), else null
  const uint8_t* be;
  int G;
  bool fp8;
  __device__ __forceinline__ float scale(int row, int kg) const {
    if (!fp8) return bf2f(reinterpret_cast<const uint16_t*>(s)[row * G + kg]);
    return e4m3_to_f(s[row * G + kg]) * exp_factor(se[row]);
  }
  __device__ __forceinline__ float bias(int row, int kg) const {
    if (!fp8) return bf2f(reinterpret_cast<const uint16_t*>(b)[row * G + kg]);
    return e4m3_to_f(b[row * G + kg]) * exp_factor(be[row]);
  }
};

// Bytes of a row of codes: K*bits/8 rounded up to 16 bytes, so that every
// row starts on a 16-byte boundary (a bulk copy or a tensor map can address
// it; only 3-bit rows of K not a multiple of 128 carry padding).
__host__ __device__ constexpr int code_row_bytes(int K, int bits) {
  return ((K / 8 * bits) + 15) & ~15;
}

// Shared-memory stride of a staged row of codes: padded so that the 8 rows a
// warp reads at once fall on distinct bank groups. A quad reads 2*bits words
// of a row per group (6 for 3 bits, padded to 8: strides step by 4 words),
// so the stride is that many words mod 32.
__host__ __device__ inline int mx_stride(int K, int bits) {
  const int want = bits == 3 ? 8 : (2 * bits) & 31;
  int s = code_row_bytes(K, bits);
  for (int i = 0; i < 8 && ((s >> 2) & 31) != want; ++i) s += 16;
  return s;
}

}  // namespace ms
