// K3: 4-bit expert MLP for decode and small batches (tokens per expert <= a
// few dozen): the batched replacement of the three gather_qmm calls, the
// SwiGLU and the weighted sum (engine_v3.py:588-600, engine_120b.py:130-145;
// kernels.py:87-186 is the reference's own fused attempt).
//
//   k_up   one CTA per (16-row tile of d_ff, group of pairs sharing a slot):
//          gate and up rows of the tile for up to 8 tokens per MMA pass,
//          the input dimension split over the CTA's 8 warps, SwiGLU (or
//          gpt-oss's clamped SwiGLU with the projection biases) in the
//          epilogue; h goes out in frag layout, ready to be the next
//          kernel's MMA operand, with its per-group sums.
//   k_down one CTA per (16-row tile of d_model, group): down rows, bias,
//          then the weighted combine over each token's k experts is done
//          by the last CTA to finish a row tile (arrival counter, fixed j
//          order, so the sum is deterministic), writing bf16 y.
//
// Weights stream straight from the slot arena with 8-byte non-allocating
// loads; every lane's 32 bytes of a quantisation group are one sector.
#include "ms_common.cuh"
#include "frag.cuh"
#include "kernels.h"

namespace ms {

constexpr int EX_THREADS = 256;
constexpr int EX_WARPS = EX_THREADS / 32;

__device__ __forceinline__ uint2 ldw(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

__device__ __forceinline__ float clamped_swiglu(float g, float u) {
  // gpt_oss.swiglu(x_linear=u, x_glu=g): alpha 1.702, limit 7 (engine_120b.py:27-29)
  g = fminf(g, 7.f);
  u = fminf(fmaxf(u, -7.f), 7.f);
  return g / (1.f + expf(-1.702f * g)) * (u + 1.f);
}

// Partial dot products of a 16-row tile over quantisation groups [kg0, kg1)
// for the 8 activation columns of this pass. Returns the lane's C fragment
// (rows g4, g4+8 x columns 2c, 2c+1) with scales and biases applied.
__device__ __forceinline__ void tile_dot(float* tot, const uint32_t* W, const uint16_t* S,
                                         const uint16_t* B, int WPR, int G, int r0, int r1,
                                         int kg0, int kg1, const __half* frag, long long rb,
                                         const float* sums, long long rc0, long long rc1,
                                         int c) {
  for (int kg = kg0; kg < kg1; ++kg) {
    const uint2 a0 = ldw(W + (long long)r0 * WPR + kg * 8 + 2 * c);
    const uint2 a1 = ldw(W + (long long)r1 * WPR + kg * 8 + 2 * c);
    uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
    if (rb >= 0) {
      const uint4* fb = reinterpret_cast<const uint4*>(frag + (rb * G + kg) * 64);
      b0 = fb[c];
      b1 = fb[4 + c];
    }
    float cc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_group(cc, a0, a1, b0, b1);
    float xs0 = 0.f, xp0 = 0.f, xs1 = 0.f, xp1 = 0.f;
    if (rc0 >= 0) { xs0 = sums[(rc0 * G + kg) * 2]; xp0 = sums[(rc0 * G + kg) * 2 + 1]; }
    if (rc1 >= 0) { xs1 = sums[(rc1 * G + kg) * 2]; xp1 = sums[(rc1 * G + kg) * 2 + 1]; }
    const float s0 = bf2f(S[(long long)r0 * G + kg]), s1 = bf2f(S[(long long)r1 * G + kg]);
    const float q0 = bf2f(B[(long long)r0 * G + kg]), q1 = bf2f(B[(long long)r1 * G + kg]);
    tot[0] += s0 * (cc[0] - 1024.f * xp0) + q0 * xs0;
    tot[1] += s0 * (cc[1] - 1024.f * xp1) + q0 * xs1;
    tot[2] += s1 * (cc[2] - 1024.f * xp0) + q1 * xs0;
    tot[3] += s1 * (cc[3] - 1024.f * xp1) + q1 * xs1;
  }
}

template <int MODEL>
__global__ void __launch_bounds__(EX_THREADS) k_up(ExpArgs A) {
  const int g = blockIdx.y;
  if (g >= *A.grp.n_groups) return;
  const int slot = A.grp.grp_slot[g];
  const int m = A.grp.grp_count[g], start = A.grp.grp_start[g];
  const int rt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int K = A.geo.d_model, G = K / 64, WPR = K / 8, F = A.geo.d_ff, GF = F / 64;
  const int k = A.geo.top_k;
  const int kg0 = warp * G / EX_WARPS, kg1 = (warp + 1) * G / EX_WARPS;
  const int r0 = rt * 16 + g4, r1 = r0 + 8;
  __shared__ float red[EX_WARPS][2][4][32];

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  const uint32_t* Wg = reinterpret_cast<const uint32_t*>(blob + A.geo.off[0][0]);
  const uint16_t* Sg = reinterpret_cast<const uint16_t*>(blob + A.geo.off[0][1]);
  const uint16_t* Bg = reinterpret_cast<const uint16_t*>(blob + A.geo.off[0][2]);
  const uint32_t* Wu = reinterpret_cast<const uint32_t*>(blob + A.geo.off[1][0]);
  const uint16_t* Su = reinterpret_cast<const uint16_t*>(blob + A.geo.off[1][1]);
  const uint16_t* Bu = reinterpret_cast<const uint16_t*>(blob + A.geo.off[1][2]);

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = A.grp.grp_pairs + start + n0;
    const int nn = min(8, m - n0);
    const long long pb = (g4 < nn) ? pairs[g4] : -1;
    const long long pc0 = (2 * c < nn) ? pairs[2 * c] : -1;
    const long long pc1 = (2 * c + 1 < nn) ? pairs[2 * c + 1] : -1;
    const long long tb = pb >= 0 ? pb / k : -1;
    const long long tc0 = pc0 >= 0 ? pc0 / k : -1, tc1 = pc1 >= 0 ? pc1 / k : -1;
    float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0) {
      tile_dot(tg, Wg, Sg, Bg, WPR, G, r0, r1, kg0, kg1, A.xfrag, tb, A.xsum, tc0, tc1, c);
      tile_dot(tu, Wu, Su, Bu, WPR, G, r0, r1, kg0, kg1, A.xfrag, tb, A.xsum, tc0, tc1, c);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      red[warp][0][i][lane] = tg[i];
      red[warp][1][i][lane] = tu[i];
    }
    __syncthreads();
    if (warp == 0) {
      float hs[2] = {0.f, 0.f}, hp[2] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float gv = 0.f, uv = 0.f;
        for (int w = 0; w < EX_WARPS; ++w) { gv += red[w][0][i][lane]; uv += red[w][1][i][lane]; }
        const int row = (i < 2) ? r0 : r1;
        const int col = 2 * c + (i & 1);
        const long long pc = (i & 1) ? pc1 : pc0;
        if (col < nn && slot >= 0) {
          float h;
          if (MODEL == 1) {
            const uint16_t* bgp = reinterpret_cast<const uint16_t*>(blob + A.geo.off[0][3]);
            const uint16_t* bup = reinterpret_cast<const uint16_t*>(blob + A.geo.off[1][3]);
            h = clamped_swiglu(gv + bf2f(bgp[row]), uv + bf2f(bup[row]));
          } else {
            h = silu_mul(gv, uv);
          }
          const __half hh = __float2half_rn(h);
          const __half hsc = (row & 1) ? __hmul(hh, __float2half(0.0625f)) : hh;
          A.hfrag[frag_off(pc, GF, row)] = hsc;
          hs[i & 1] += __half2float(hh);
          hp[i & 1] += __half2float(hsc);
        } else if (col < nn) {
          A.hfrag[frag_off(pc, GF, row)] = __float2half(0.f);
        }
      }
      // sums over the 16 rows of the tile, per column
#pragma unroll
      for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          hs[q] += __shfl_xor_sync(MS_FULL, hs[q], o);
          hp[q] += __shfl_xor_sync(MS_FULL, hp[q], o);
        }
      }
      if (g4 == 0) {
        const int nt = F / 16;
        if (2 * c < nn) {
          A.hpart[(pc0 * nt + rt) * 2] = hs[0];
          A.hpart[(pc0 * nt + rt) * 2 + 1] = hp[0];
        }
        if (2 * c + 1 < nn) {
          A.hpart[(pc1 * nt + rt) * 2] = hs[1];
          A.hpart[(pc1 * nt + rt) * 2 + 1] = hp[1];
        }
      }
    }
    __syncthreads();
  }
}

template <int MODEL>
__global__ void __launch_bounds__(EX_THREADS) k_down(ExpArgs A) {
  const int g = blockIdx.y;
  const int n_groups = *A.grp.n_groups;
  if (g >= n_groups) return;
  const int slot = A.grp.grp_slot[g];
  const int m = A.grp.grp_count[g], start = A.grp.grp_start[g];
  const int rt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int K = A.geo.d_ff, G = K / 64, WPR = K / 8, D = A.geo.d_model;
  const int k = A.geo.top_k;
  const int kg0 = warp * G / EX_WARPS, kg1 = (warp + 1) * G / EX_WARPS;
  const int r0 = rt * 16 + g4, r1 = r0 + 8;
  const int nt_ff = K / 16;
  __shared__ float red[EX_WARPS][4][32];
  __shared__ float s_sums[8][64][2];     // per column: X_g, X'_g for every group of d_ff
  __shared__ int s_last;

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  const uint32_t* Wd = reinterpret_cast<const uint32_t*>(blob + A.geo.off[2][0]);
  const uint16_t* Sd = reinterpret_cast<const uint16_t*>(blob + A.geo.off[2][1]);
  const uint16_t* Bd = reinterpret_cast<const uint16_t*>(blob + A.geo.off[2][2]);

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = A.grp.grp_pairs + start + n0;
    const int nn = min(8, m - n0);
    // per-group sums of h for the columns of this pass (4 row tiles each)
    for (int i = threadIdx.x; i < nn * G; i += EX_THREADS) {
      const int col = i / G, kg = i % G;
      const long long p = pairs[col];
      float xs = 0.f, xp = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        xs += A.hpart[(p * nt_ff + kg * 4 + q) * 2];
        xp += A.hpart[(p * nt_ff + kg * 4 + q) * 2 + 1];
      }
      s_sums[col][kg][0] = xs;
      s_sums[col][kg][1] = xp;
    }
    __syncthreads();
    const long long pb = (g4 < nn) ? pairs[g4] : -1;
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0) {
      for (int kg = kg0; kg < kg1; ++kg) {
        const uint2 a0 = ldw(Wd + (long long)r0 * WPR + kg * 8 + 2 * c);
        const uint2 a1 = ldw(Wd + (long long)r1 * WPR + kg * 8 + 2 * c);
        uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
        if (pb >= 0) {
          const uint4* fb = reinterpret_cast<const uint4*>(A.hfrag + (pb * G + kg) * 64);
          b0 = fb[c];
          b1 = fb[4 + c];
        }
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group(cc, a0, a1, b0, b1);
        float xs0 = 0.f, xp0 = 0.f, xs1 = 0.f, xp1 = 0.f;
        if (2 * c < nn) { xs0 = s_sums[2 * c][kg][0]; xp0 = s_sums[2 * c][kg][1]; }
        if (2 * c + 1 < nn) { xs1 = s_sums[2 * c + 1][kg][0]; xp1 = s_sums[2 * c + 1][kg][1]; }
        const float s0 = bf2f(Sd[(long long)r0 * G + kg]), s1 = bf2f(Sd[(long long)r1 * G + kg]);
        const float q0 = bf2f(Bd[(long long)r0 * G + kg]), q1 = bf2f(Bd[(long long)r1 * G + kg]);
        tot[0] += s0 * (cc[0] - 1024.f * xp0) + q0 * xs0;
        tot[1] += s0 * (cc[1] - 1024.f * xp1) + q0 * xs1;
        tot[2] += s1 * (cc[2] - 1024.f * xp0) + q1 * xs0;
        tot[3] += s1 * (cc[3] - 1024.f * xp1) + q1 * xs1;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][i][lane] = tot[i];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = 0.f;
        for (int w = 0; w < EX_WARPS; ++w) v += red[w][i][lane];
        const int row = (i < 2) ? r0 : r1;
        const int col = 2 * c + (i & 1);
        if (col < nn) {
          if (MODEL == 1 && slot >= 0) {
            const uint16_t* bdp = reinterpret_cast<const uint16_t*>(blob + A.geo.off[2][3]);
            v += bf2f(bdp[row]);
          }
          A.ypart[(long long)pairs[col] * D + row] = (slot >= 0) ? v : 0.f;
        }
      }
    }
    __syncthreads();
  }

  // ---- arrival: the last CTA of this row tile combines all tokens' k parts
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&A.cnt[rt], 1u);
    s_last = (prev == (unsigned)n_groups - 1u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < A.T * 16; i += EX_THREADS) {
    const int t = i >> 4, row = rt * 16 + (i & 15);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const long long p = (long long)t * k + j;
      acc += A.scores[p] * __ldcg(A.ypart + p * D + row);
    }
    A.y[(long long)t * D + row] = f2bf(acc);
  }
  if (threadIdx.x == 0) A.cnt[rt] = 0u;
}

cudaError_t launch_expert(const ExpArgs& a, int max_groups, cudaStream_t s) {
  if (max_groups <= 0) return cudaSuccess;
  dim3 gu(a.geo.d_ff / 16, max_groups), gd(a.geo.d_model / 16, max_groups);
  if (a.geo.model == 1) {
    k_up<1><<<gu, EX_THREADS, 0, s>>>(a);
    k_down<1><<<gd, EX_THREADS, 0, s>>>(a);
  } else {
    k_up<0><<<gu, EX_THREADS, 0, s>>>(a);
    k_down<0><<<gd, EX_THREADS, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace ms
