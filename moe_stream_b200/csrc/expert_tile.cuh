// Pieces of the decode expert kernels (expert.cu: k_up / k_down): the
// 16-row tile dot product on tensor cores from shared memory, the
// activations with MLX's rounding points, and the shared-memory layouts of
// the weight tiles.
#pragma once
#include "ms_common.cuh"
#include "frag.cuh"

namespace ms {

constexpr int EX_THREADS = 256;
constexpr int EX_WARPS = EX_THREADS / 32;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The activations keep MLX's rounding points: gather_qmm returns bf16, and
// every elementwise op of the SwiGLU rounds its result to bf16
// (engine_v3.py:592-597, engine_120b.py:136-143), so the block tracks the
// reference's arithmetic, not a more precise variant of it.
// 1/(1+e^-v); __frcp_rn is the correctly rounded reciprocal, i.e. 1.f / x
__device__ __forceinline__ float sigm(float v) { return __frcp_rn(1.f + expf(-v)); }

__device__ __forceinline__ float silu_mul(float g, float u) {
  // activations.swiglu(gate, x) = silu(gate) * x, silu(v) = v * sigmoid(v)
  return bfr(bfr(g * bfr(sigm(g))) * u);
}

__device__ __forceinline__ float clamped_swiglu(float g, float u) {
  // gpt_oss.swiglu(x_linear=u, x_glu=g): alpha 1.702 (a bf16 1.703125 once it
  // meets a bf16 operand), limit 7, (linear + 1) (engine_120b.py:27-29)
  g = fminf(g, 7.f);
  u = fminf(fmaxf(u, -7.f), 7.f);
  const float og = bfr(g * bfr(sigm(bfr(1.703125f * g))));
  return bfr(og * bfr(u + 1.f));
}

// Padded shared-memory row stride for a weight row of `row_bytes`: a stride
// of 8 (mod 32) words puts the 8 rows a warp reads at once on disjoint bank
// octets, so the 8-byte fragment loads take the minimum two wavefronts.
__host__ __device__ constexpr int padded_stride(int row_bytes) {
  int s = row_bytes;
  while (((s >> 2) & 31) != 8) s += 16;
  return s;
}

// Activation fragments (frag layout, written before the launch, so read by
// the read-only path) of quantisation groups [kg0, kg1) for lane quad
// position c; zeros past kg1 or without activations.
template <int KPW>
__device__ __forceinline__ void load_frags(uint4* b0, uint4* b1, const __half* frag_b, int kg0,
                                           int kg1, int c) {
#pragma unroll
  for (int q = 0; q < KPW; ++q) {
    b0[q] = make_uint4(0, 0, 0, 0);
    b1[q] = b0[q];
    const int kg = kg0 + q;
    if (frag_b && kg < kg1) {
      const uint4* fb = reinterpret_cast<const uint4*>(frag_b + kg * 64);
      b0[q] = __ldg(fb + c);
      b1[q] = __ldg(fb + 4 + c);
    }
  }
}

// Per-group activation sums (X, X') of the two columns of this lane for
// groups [kg0, kg1), into registers (zeros where a column is absent).
template <int KPW>
__device__ __forceinline__ void load_sums(float2* v0, float2* v1, const float* sum_c0,
                                          const float* sum_c1, int kg0, int kg1) {
#pragma unroll
  for (int q = 0; q < KPW; ++q) {
    const int kg = kg0 + q;
    v0[q] = make_float2(0.f, 0.f);
    v1[q] = v0[q];
    if (kg < kg1) {
      if (sum_c0) v0[q] = *reinterpret_cast<const float2*>(sum_c0 + kg * 2);
      if (sum_c1) v1[q] = *reinterpret_cast<const float2*>(sum_c1 + kg * 2);
    }
  }
}

// Offset of lane (g4, c)'s 8 weight bytes of quantisation group kg in a
// 16-row tile at At, rows g4 (hi = 0) or g4 + 8 (hi = 1). Padded layout:
// rows `stride` bytes apart. Swizzled layout (a 128-byte-swizzled tensor
// map box of whole rows, [chunk][row][128 B]): `stride` is the chunk stride
// and the 16-byte unit u of row r sits at u ^ (r mod 8); At is the tile's
// first row, a multiple of 8 rows into the box.
template <bool SWZ>
__device__ __forceinline__ const uint8_t* wrow(const uint8_t* At, int stride, int g4, int hi, int kg, int c) {
  if (!SWZ) return At + (g4 + 8 * hi) * stride + kg * 32 + 8 * c;
  return At + (kg >> 2) * stride + (g4 + 8 * hi) * 128 + (((((kg & 3) << 1) | (c >> 1)) ^ g4) << 4) +
         ((c & 1) << 3);
}

// The dot product with fragments and sums already in registers.
template <int KPW, bool SWZ = false>
__device__ __forceinline__ void tile_dot_regs(float* tot, const uint8_t* At, int stride, int G,
                                              int kg0, int kg1, int g4, int c, const uint16_t* sS,
                                              const uint16_t* sB, const uint4* b0, const uint4* b1,
                                              const float2* v0, const float2* v1) {
#pragma unroll
  for (int q = 0; q < KPW; ++q) {
    const int kg = kg0 + q;
    if (kg >= kg1) continue;
    const uint2 ra = *reinterpret_cast<const uint2*>(wrow<SWZ>(At, stride, g4, 0, kg, c));
    const uint2 rb = *reinterpret_cast<const uint2*>(wrow<SWZ>(At, stride, g4, 1, kg, c));
    float cc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_group(cc, ra, rb, b0[q], b1[q]);
    const float xs0 = v0[q].x, xp0 = v0[q].y, xs1 = v1[q].x, xp1 = v1[q].y;
    const float s0 = bf2f(sS[g4 * G + kg]), s1 = bf2f(sS[(g4 + 8) * G + kg]);
    const float q0 = bf2f(sB[g4 * G + kg]), q1 = bf2f(sB[(g4 + 8) * G + kg]);
    tot[0] += s0 * (cc[0] - 1024.f * xp0) + q0 * xs0;
    tot[1] += s0 * (cc[1] - 1024.f * xp1) + q0 * xs1;
    tot[2] += s1 * (cc[2] - 1024.f * xp0) + q1 * xs0;
    tot[3] += s1 * (cc[3] - 1024.f * xp1) + q1 * xs1;
  }
}

// tile_dot_regs with each group's sums read from sum_c0 / sum_c1 (shared
// memory) as the loop reaches it: fewer live registers than load_sums up
// front, the same arithmetic in the same order.
template <int KPW, bool SWZ = false>
__device__ __forceinline__ void tile_dot_frags(float* tot, const uint8_t* At, int stride, int G,
                                               int kg0, int kg1, int g4, int c, const uint16_t* sS,
                                               const uint16_t* sB, const uint4* b0, const uint4* b1,
                                               const float* sum_c0, const float* sum_c1) {
#pragma unroll
  for (int q = 0; q < KPW; ++q) {
    const int kg = kg0 + q;
    if (kg >= kg1) continue;
    const uint2 ra = *reinterpret_cast<const uint2*>(wrow<SWZ>(At, stride, g4, 0, kg, c));
    const uint2 rb = *reinterpret_cast<const uint2*>(wrow<SWZ>(At, stride, g4, 1, kg, c));
    float cc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_group(cc, ra, rb, b0[q], b1[q]);
    float xs0 = 0.f, xp0 = 0.f, xs1 = 0.f, xp1 = 0.f;
    if (sum_c0) { const float2 v = *reinterpret_cast<const float2*>(sum_c0 + kg * 2); xs0 = v.x; xp0 = v.y; }
    if (sum_c1) { const float2 v = *reinterpret_cast<const float2*>(sum_c1 + kg * 2); xs1 = v.x; xp1 = v.y; }
    const float s0 = bf2f(sS[g4 * G + kg]), s1 = bf2f(sS[(g4 + 8) * G + kg]);
    const float q0 = bf2f(sB[g4 * G + kg]), q1 = bf2f(sB[(g4 + 8) * G + kg]);
    tot[0] += s0 * (cc[0] - 1024.f * xp0) + q0 * xs0;
    tot[1] += s0 * (cc[1] - 1024.f * xp1) + q0 * xs1;
    tot[2] += s1 * (cc[2] - 1024.f * xp0) + q1 * xs0;
    tot[3] += s1 * (cc[3] - 1024.f * xp1) + q1 * xs1;
  }
}

struct UpSmem {
  static __host__ __device__ int stride(int K) { return padded_stride(K / 2); }
  static __host__ __device__ int a_bytes(int K) { return 16 * stride(K); }
  static __host__ __device__ int sb_bytes(int G) { return 16 * G * 2; }
  // tma: dense rows in 128-byte-swizzled boxes, 1 KB of alignment slack
  static __host__ __device__ int total(int K, bool tma) {
    const int G = K / 64;
    const int a = tma ? 16 * (K / 2) : a_bytes(K);
    return 2 * a + 4 * sb_bytes(G) + EX_WARPS * 2 * 4 * 32 * 4 + 16 + (tma ? 1024 : 0);
  }
};

struct DownSmem {
  static __host__ __device__ int stride(int F) { return padded_stride(F / 2); }
  static __host__ __device__ int a_bytes(int F, int RT) { return RT * 16 * stride(F); }
  static __host__ __device__ int sb_bytes(int GF, int RT) { return RT * 16 * GF * 2; }
  static __host__ __device__ int total(int F, int RT, bool tma) {
    const int GF = F / 64;
    const int a = tma ? RT * 16 * (F / 2) : a_bytes(F, RT);
    return a + 2 * sb_bytes(GF, RT) + EX_WARPS * 4 * 32 * 4 + 8 * GF * 2 * 4 + 16 + (tma ? 1024 : 0);
  }
};

}  // namespace ms
