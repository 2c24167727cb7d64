// The decode expert kernels for pools whose experts come in precision
// classes (prec.cuh): 2-, 3-, 4- or 8-bit codes, bf16 or fp8 scales, chosen
// per expert. They do what k_up / k_down (expert.cu) do -- gate and up with
// the SwiGLU, then down with the weighted combine -- and each CTA reads the
// class of the slot it serves and runs that class's code path:
//
//   k_up_mx   one CTA per (16-row tile of d_ff, group of pairs sharing a
//             slot), the input dimension over 8 warps, SwiGLU in the
//             epilogue, h in the frag layout with its per-tile sums.
//   k_down_mx one CTA per (RT 16-row tiles of d_model, group); the last CTA
//             of a row tile combines each token's k expert rows in a fixed
//             order.
//
// A tile's bytes shrink with its class (16 rows x d*bits/8 codes, rows
// padded to 16 bytes), and the copies move exactly those bytes, one per row
// into padded shared-memory rows. The uniform 4-bit bf16 pools keep the
// tuned kernels of expert.cu.
#include "ms_common.cuh"
#include "frag.cuh"
#include "tma.cuh"
#include "kernels.h"
#include "expert_tile.cuh"
#include "prec.cuh"

namespace ms {

namespace {

// Shared-memory plan of a tile of `rows` rows of K inputs at the widest
// class of the pool: codes, then scales and biases (bf16-sized, fp8 uses
// half), then the fp8 row exponents.
struct MxTile {
  static __host__ __device__ int a_bytes(int K, int bits, int rows) { return rows * mx_stride(K, bits); }
  static __host__ __device__ int sb_bytes(int K, int rows) { return rows * (K / 64) * 2; }
};

// 16-row tile dot product of one class: rows g4 and g4 + 8 of the tile at
// At (row stride `stride`), groups [kg0, kg1), activation fragments b0/b1
// and column sums v0/v1 in registers (frag.cuh's correction, applied per
// group: s * (acc - 1024 X') + b X, with X for 8-bit codes).
template <int KPW, int BITS>
__device__ __forceinline__ void tile_dot_mx(float* tot, const uint8_t* At, int stride, int kg0,
                                            int kg1, int g4, int c, const SBTile& sb,
                                            const uint4* b0, const uint4* b1, const float2* v0,
                                            const float2* v1) {
#pragma unroll
  for (int q = 0; q < KPW; ++q) {
    const int kg = kg0 + q;
    if (kg >= kg1) continue;
    uint32_t Ra[2][4], Rb[2][4];
    group_regs<BITS>(At + g4 * stride + kg * 8 * BITS, c, Ra);
    group_regs<BITS>(At + (g4 + 8) * stride + kg * 8 * BITS, c, Rb);
    float cc[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(cc, Ra[0][0], Rb[0][0], Ra[0][1], Rb[0][1], b0[q].x, b0[q].y);
    mma16816(cc, Ra[0][2], Rb[0][2], Ra[0][3], Rb[0][3], b0[q].z, b0[q].w);
    mma16816(cc, Ra[1][0], Rb[1][0], Ra[1][1], Rb[1][1], b1[q].x, b1[q].y);
    mma16816(cc, Ra[1][2], Rb[1][2], Ra[1][3], Rb[1][3], b1[q].z, b1[q].w);
    const float c0 = corr_sum<BITS>(v0[q]), c1 = corr_sum<BITS>(v1[q]);
    const float s0 = sb.scale(g4, kg), s1 = sb.scale(g4 + 8, kg);
    const float q0 = sb.bias(g4, kg), q1 = sb.bias(g4 + 8, kg);
    tot[0] += s0 * (cc[0] - 1024.f * c0) + q0 * v0[q].x;
    tot[1] += s0 * (cc[1] - 1024.f * c1) + q0 * v1[q].x;
    tot[2] += s1 * (cc[2] - 1024.f * c0) + q1 * v0[q].x;
    tot[3] += s1 * (cc[3] - 1024.f * c1) + q1 * v1[q].x;
  }
}

// Copies of a tile of `rows` rows (from row r0 of projection proj) into
// shared memory, issued by the lanes of warp 0: this lane copies code row
// `row` (when in [0, rows)) into its padded row, and copy `sbc` (0 scales,
// 1 biases, fp8: 2 and 3 their row exponents) when in [0, 4). Lane 0 of the
// warp has armed `bar` for stage_bytes.
template <int BITS>
__device__ __forceinline__ void stage_rows(uint8_t* sA, uint8_t* sS, uint8_t* sB, uint8_t* sE,
                                           const uint8_t* blob, const PrecDev& pc, int proj,
                                           int r0, int rows, int K, uint64_t* bar, uint64_t pol,
                                           int row, int sbc) {
  const int rb = code_row_bytes(K, BITS), stride = mx_stride(K, BITS), G = K / 64;
  const uint8_t* W = blob + pc.off[proj][P_W] + (long long)r0 * rb;
  if (row >= 0 && row < rows) bulk_g2s_hint(sA + row * stride, W + (long long)row * rb, rb, bar, pol);
  const int esz = pc.fmt == SF_FP8 ? 1 : 2;
  const unsigned sbn = (unsigned)(rows * G * esz);
  if (sbc == 0) bulk_g2s_hint(sS, blob + pc.off[proj][P_S] + (long long)r0 * G * esz, sbn, bar, pol);
  if (sbc == 1) bulk_g2s_hint(sB, blob + pc.off[proj][P_B] + (long long)r0 * G * esz, sbn, bar, pol);
  if (pc.fmt == SF_FP8) {
    if (sbc == 2) bulk_g2s_hint(sE, blob + pc.off[proj][P_SE] + r0, (unsigned)rows, bar, pol);
    if (sbc == 3) bulk_g2s_hint(sE + rows, blob + pc.off[proj][P_BE] + r0, (unsigned)rows, bar, pol);
  }
}

template <int BITS>
__host__ __device__ __forceinline__ unsigned stage_bytes(int K, int rows, int fmt) {
  const int G = K / 64, esz = fmt == SF_FP8 ? 1 : 2;
  return (unsigned)(rows * code_row_bytes(K, BITS) + 2 * rows * G * esz + (fmt == SF_FP8 ? 2 * rows : 0));
}

template <int MODEL, int KPW, int BITS>
__device__ __forceinline__ void up_body(const ExpArgs& A, const PrecDev& pc, int g, int slot, int m,
                                        int start, uint8_t* smem, int a_cap) {
  const int rt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int K = A.geo.d_model, G = K / 64, F = A.geo.d_ff, GF = F / 64;
  const int k = A.geo.top_k;
  const int stride = mx_stride(K, BITS);
  const int kg0 = min(G, warp * KPW), kg1 = min(G, kg0 + KPW);
  // [gate codes | up codes | gate s | gate b | up s | up b | exps | red | bar]
  uint8_t* sA[2] = {smem, smem + a_cap};
  uint8_t* sb0 = smem + 2 * a_cap;
  const int sbb = MxTile::sb_bytes(K, 16);
  uint8_t* sS[2] = {sb0, sb0 + 2 * sbb};
  uint8_t* sB[2] = {sb0 + sbb, sb0 + 3 * sbb};
  uint8_t* sE = sb0 + 4 * sbb;                 // [proj][s/b][16]
  float* red = reinterpret_cast<float*>(sE + 64);
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + EX_WARPS * 2 * 4 * 32);

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  if (warp == 0 && slot >= 0) {
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
      mbar_expect_tx(bar, 2u * stage_bytes<BITS>(K, 16, pc.fmt));
    }
    __syncwarp();
    const uint64_t pol = l2_evict_first();
    // gate: rows on lanes 0-15, its scale copies on lanes 16-19; up: rows
    // on lanes 16-31, its scale copies on lanes 0-3
    stage_rows<BITS>(sA[0], sS[0], sB[0], sE, blob, pc, 0, rt * 16, 16, K, bar, pol,
                     lane < 16 ? lane : -1, lane - 16);
    stage_rows<BITS>(sA[1], sS[1], sB[1], sE + 32, blob, pc, 1, rt * 16, 16, K, bar, pol,
                     lane >= 16 ? lane - 16 : -1, lane);
  }
  __syncthreads();
  bool ok = true, waited = false;
  const SBTile sbg{sS[0], sB[0], sE, sE + 16, G, pc.fmt == SF_FP8};
  const SBTile sbu{sS[1], sB[1], sE + 32, sE + 48, G, pc.fmt == SF_FP8};

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = A.grp.grp_pairs + start + n0;
    const int nn = min(8, m - n0);
    const int pb = (g4 < nn) ? pairs[g4] : -1;
    const int pc0 = (2 * c < nn) ? pairs[2 * c] : -1;
    const int pc1 = (2 * c + 1 < nn) ? pairs[2 * c + 1] : -1;
    const __half* fb = pb >= 0 ? A.xfrag + (long long)(pb / k) * G * 64 : nullptr;
    const float* s0 = pc0 >= 0 ? A.xsum + (long long)(pc0 / k) * G * 2 : nullptr;
    const float* s1 = pc1 >= 0 ? A.xsum + (long long)(pc1 / k) * G * 2 : nullptr;
    uint4 b0[KPW], b1[KPW];
    float2 v0[KPW], v1[KPW];
    load_frags<KPW>(b0, b1, (slot >= 0) ? fb : nullptr, kg0, kg1, c);
    load_sums<KPW>(v0, v1, s0, s1, kg0, kg1);
    if (!waited) {
      if (slot >= 0) ok = mbar_wait(bar, 0, A.status);
      waited = true;
    }
    float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0 && ok && kg0 < kg1) {
      tile_dot_mx<KPW, BITS>(tg, sA[0], stride, kg0, kg1, g4, c, sbg, b0, b1, v0, v1);
      tile_dot_mx<KPW, BITS>(tu, sA[1], stride, kg0, kg1, g4, c, sbu, b0, b1, v0, v1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      red[((warp * 2 + 0) * 4 + i) * 32 + lane] = tg[i];
      red[((warp * 2 + 1) * 4 + i) * 32 + lane] = tu[i];
    }
    __syncthreads();
    if (threadIdx.x < 128) {
      const int r = threadIdx.x & 15, col = threadIdx.x >> 4;
      const int src = (r & 7) * 4 + (col >> 1), e = ((r >> 3) << 1) | (col & 1);
      const int row = rt * 16 + r;
      float hh_f = 0.f, hsc_f = 0.f;
      const int pcol = col < nn ? pairs[col] : -1;
      if (col < nn) {
        __half hsc = __float2half(0.f);
        if (slot >= 0 && ok) {
          float gv = 0.f, uv = 0.f;
#pragma unroll
          for (int w = 0; w < EX_WARPS; ++w) {
            gv += red[((w * 2 + 0) * 4 + e) * 32 + src];
            uv += red[((w * 2 + 1) * 4 + e) * 32 + src];
          }
          gv = bfr(gv);
          uv = bfr(uv);
          float h;
          if (MODEL == 1) {
            const uint16_t* bgp = reinterpret_cast<const uint16_t*>(blob + pc.off[0][P_BIAS]);
            const uint16_t* bup = reinterpret_cast<const uint16_t*>(blob + pc.off[1][P_BIAS]);
            h = clamped_swiglu(bfr(gv + bf2f(bgp[row])), bfr(uv + bf2f(bup[row])));
          } else {
            h = silu_mul(gv, uv);
          }
          if (fabsf(h) > F16_MAX) atomicCAS(A.status, 0, ST_E_RANGE);
          const __half hh = __float2half_rn(h);
          hsc = (row & 1) ? __hmul(hh, __float2half(0.0625f)) : hh;
          hh_f = __half2float(hh);
          hsc_f = __half2float(hsc);
        }
        A.hfrag[frag_off(pcol, GF, row)] = hsc;
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        hh_f += __shfl_xor_sync(MS_FULL, hh_f, o);
        hsc_f += __shfl_xor_sync(MS_FULL, hsc_f, o);
      }
      if (r == 0 && col < nn)
        *reinterpret_cast<float2*>(A.hpart + ((long long)pcol * (F / 16) + rt) * 2) =
            make_float2(hh_f, hsc_f);
    }
    __syncthreads();
  }
}

// Qwen3 shapes: three CTAs per SM, so a batch-1 layer's 384 tiles fit one
// wave (as k_up).
template <int MODEL, int KPW>
__global__ void __launch_bounds__(EX_THREADS, (MODEL == 0 && KPW == 4) ? 3 : 2)
    k_up_mx(ExpArgs A, const __grid_constant__ ClassTab C, int a_cap) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.y;
  const int n_groups = *A.grp.n_groups;
  const int slot = A.grp.grp_slot[g];
  const int m = A.grp.grp_count[g], start = A.grp.grp_start[g];
  if (g >= n_groups) return;
  const int cls = slot >= 0 ? min((int)A.slot_class[slot], C.n - 1) : 0;
  const PrecDev& pc = C.c[cls];
  switch (pc.bits) {
    case 2: up_body<MODEL, KPW, 2>(A, pc, g, slot, m, start, smem, a_cap); break;
    case 3: up_body<MODEL, KPW, 3>(A, pc, g, slot, m, start, smem, a_cap); break;
    case 8: up_body<MODEL, KPW, 8>(A, pc, g, slot, m, start, smem, a_cap); break;
    default: up_body<MODEL, KPW, 4>(A, pc, g, slot, m, start, smem, a_cap); break;
  }
}

template <int MODEL, int KPW, int RT, int BITS>
__device__ __forceinline__ void down_body(const ExpArgs& A, const PrecDev& pc, int slot, int m,
                                          int start, uint8_t* smem, int a_cap) {
  constexpr int WPT = EX_WARPS / RT;            // warps per row tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int sub = warp / WPT, wk = warp % WPT;
  const int rt = blockIdx.x * RT + sub;
  const int K = A.geo.d_ff, G = K / 64, D = A.geo.d_model;
  const int stride = mx_stride(K, BITS);
  const int kg0 = min(G, wk * KPW), kg1 = min(G, kg0 + KPW);
  const int nt_ff = K / 16;
  const int esz = pc.fmt == SF_FP8 ? 1 : 2;
  // [codes | scales | biases | exps (s, b) | red | sums | bar]
  uint8_t* sA = smem;
  const int sbb = MxTile::sb_bytes(K, RT * 16);
  uint8_t* sS = smem + a_cap;
  uint8_t* sB = sS + sbb;
  uint8_t* sE = sB + sbb;
  float* red = reinterpret_cast<float*>(sE + 32 * RT);
  float* s_sums = red + EX_WARPS * 4 * 32;      // [8][G][2]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_sums + 8 * G * 2);

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  if (warp == 0 && slot >= 0) {
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
      mbar_expect_tx(bar, stage_bytes<BITS>(K, RT * 16, pc.fmt));
    }
    __syncwarp();
    // the RT*16 rows one or two per lane, the scale copies on lanes 0-3
    const uint64_t pol = l2_evict_first();
    for (int r = lane; r < RT * 16; r += 32)
      stage_rows<BITS>(sA, sS, sB, sE, blob, pc, 2, blockIdx.x * RT * 16, RT * 16, K, bar, pol, r,
                       r == lane ? lane : -1);
  }
  pdl_wait();                                   // h and its sums come from k_up_mx
  __syncthreads();
  bool ok = true;
  if (slot >= 0) ok = mbar_wait(bar, 0, A.status);
  const SBTile sb{sS + sub * 16 * G * esz, sB + sub * 16 * G * esz, sE + sub * 16, sE + RT * 16 + sub * 16,
                  G, pc.fmt == SF_FP8};

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = A.grp.grp_pairs + start + n0;
    const int nn = min(8, m - n0);
    const int pb = (g4 < nn) ? pairs[g4] : -1;
    uint4 b0[KPW], b1[KPW];
    load_frags<KPW>(b0, b1, (pb >= 0 && slot >= 0) ? A.hfrag + (long long)pb * G * 64 : nullptr,
                    kg0, kg1, c);
    for (int i = threadIdx.x; i < nn * G; i += EX_THREADS) {
      const int col = i / G, kg = i % G;
      const float4* hp4 = reinterpret_cast<const float4*>(
          A.hpart + ((long long)pairs[col] * nt_ff + kg * 4) * 2);
      const float4 a = hp4[0], b = hp4[1];
      s_sums[(col * G + kg) * 2] = (a.x + a.z) + (b.x + b.z);
      s_sums[(col * G + kg) * 2 + 1] = (a.y + a.w) + (b.y + b.w);
    }
    __syncthreads();
    float2 v0[KPW], v1[KPW];
    load_sums<KPW>(v0, v1, (2 * c < nn) ? s_sums + (2 * c) * G * 2 : nullptr,
                   (2 * c + 1 < nn) ? s_sums + (2 * c + 1) * G * 2 : nullptr, kg0, kg1);
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0 && ok && kg0 < kg1)
      tile_dot_mx<KPW, BITS>(tot, sA + sub * 16 * stride, stride, kg0, kg1, g4, c, sb, b0, b1, v0, v1);
#pragma unroll
    for (int i = 0; i < 4; ++i) red[(warp * 4 + i) * 32 + lane] = tot[i];
    __syncthreads();
    if (wk == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < WPT; ++w) v += red[((sub * WPT + w) * 4 + i) * 32 + lane];
        const int row = rt * 16 + g4 + ((i < 2) ? 0 : 8);
        const int col = 2 * c + (i & 1);
        if (col < nn) {
          v = bfr(v);
          if (MODEL == 1 && slot >= 0) {
            const uint16_t* bdp = reinterpret_cast<const uint16_t*>(blob + pc.off[2][P_BIAS]);
            v = bfr(v + bf2f(bdp[row]));
          }
          A.ypart[(long long)pairs[col] * D + row] = (slot >= 0 && ok) ? v : 0.f;
        }
      }
    }
    __syncthreads();
  }
}

template <int MODEL, int KPW, int RT>
__global__ void __launch_bounds__(EX_THREADS, 2) k_down_mx(ExpArgs A, const __grid_constant__ ClassTab C,
                                                            int a_cap) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_last[RT];
  const int g = blockIdx.y;
  const int n_groups = *A.grp.n_groups;
  const int slot = A.grp.grp_slot[g];
  const int m = A.grp.grp_count[g], start = A.grp.grp_start[g];
  if (g >= n_groups) {
    pdl_wait();
    return;
  }
  const int cls = slot >= 0 ? min((int)A.slot_class[slot], C.n - 1) : 0;
  const PrecDev& pc = C.c[cls];
  switch (pc.bits) {
    case 2: down_body<MODEL, KPW, RT, 2>(A, pc, slot, m, start, smem, a_cap); break;
    case 3: down_body<MODEL, KPW, RT, 3>(A, pc, slot, m, start, smem, a_cap); break;
    case 8: down_body<MODEL, KPW, RT, 8>(A, pc, slot, m, start, smem, a_cap); break;
    default: down_body<MODEL, KPW, RT, 4>(A, pc, slot, m, start, smem, a_cap); break;
  }
  pdl_trigger();
  // ---- arrival: the last CTA of a row tile combines all tokens' k parts
  const int D = A.geo.d_model, k = A.geo.top_k;
  __threadfence();
  __syncthreads();
  if (threadIdx.x < RT) {
    const unsigned prev = atomicAdd(&A.cnt[blockIdx.x * RT + threadIdx.x], 1u);
    s_last[threadIdx.x] = (prev == (unsigned)n_groups - 1u);
  }
  __syncthreads();
  bool any = false;
  for (int r = 0; r < RT; ++r) any |= s_last[r] != 0;
  if (!any) return;
  __threadfence();
  for (int r = 0; r < RT; ++r) {
    if (!s_last[r]) continue;
    const int rtile = blockIdx.x * RT + r;
    for (int i = threadIdx.x; i < A.T * 16; i += EX_THREADS) {
      const int t = i >> 4, row = rtile * 16 + (i & 15);
      float acc = 0.f;
      for (int j = 0; j < k; ++j) {
        const long long p = (long long)t * k + j;
        acc += bfr(A.scores[p] * __ldcg(A.ypart + p * D + row));
      }
      // the block's bf16 output; the fused block adds it to the residual
      A.y[(long long)t * D + row] =
          A.resid ? f2bf(bf2f(A.resid[(long long)t * D + row]) + bfr(acc)) : f2bf(acc);
    }
    if (threadIdx.x == 0) A.cnt[rtile] = 0u;
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_mx(Kern kern, dim3 grid, int smem, cudaStream_t s, const Args&... args) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(EX_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int MODEL, int KPW_UP, int KPW_DN, int RT>
cudaError_t launch_mx_pair(const ExpArgs& a, const ClassTab& C, int max_bits, int max_groups,
                           cudaStream_t s) {
  const int K = a.geo.d_model, F = a.geo.d_ff;
  const int cap_u = MxTile::a_bytes(K, max_bits, 16), cap_d = MxTile::a_bytes(F, max_bits, RT * 16);
  // rounded so that every region after the codes stays 16-byte aligned
  const int cu = (cap_u + 15) & ~15, cd = (cap_d + 15) & ~15;
  const int su = 2 * cu + 4 * MxTile::sb_bytes(K, 16) + 64 + EX_WARPS * 2 * 4 * 32 * 4 + 16;
  const int sd = cd + 2 * MxTile::sb_bytes(F, RT * 16) + 32 * RT + EX_WARPS * 4 * 32 * 4 +
                 8 * (F / 64) * 2 * 4 + 16;
  cudaError_t e = launch_mx(k_up_mx<MODEL, KPW_UP>, dim3(F / 16, max_groups), su, s, a, C, cu);
  if (e != cudaSuccess) return e;
  return launch_mx(k_down_mx<MODEL, KPW_DN, RT>, dim3(K / (16 * RT), max_groups), sd, s, a, C, cd);
}

}  // namespace

int mx_max_bits(const ClassTab& C) {
  int b = 0;
  for (int i = 0; i < C.n; ++i) b = b > C.c[i].bits ? b : C.c[i].bits;
  return b;
}

cudaError_t launch_expert_mx(const ExpArgs& a, const ClassTab& C, int max_groups, cudaStream_t s) {
  if (max_groups <= 0) return cudaSuccess;
  if (!expert_shape_ok(a.geo.model, a.geo.d_model, a.geo.d_ff)) return cudaErrorInvalidValue;
  const int mb = mx_max_bits(C);
  const int G = a.geo.d_model / 64, GF = a.geo.d_ff / 64;
  cudaError_t e;
  if (a.geo.model == 1) {
    e = launch_mx_pair<1, 6, 6, 1>(a, C, mb, max_groups, s);
  } else if (G <= 32 && GF <= 12 && (a.geo.d_model / 16) % 2 == 0) {
    // Qwen3 2048/768: two 16-row tiles of down rows per CTA, 4 warps x 3 groups each
    e = launch_mx_pair<0, 4, 3, 2>(a, C, mb, max_groups, s);
  } else {
    e = launch_mx_pair<0, 8, 8, 1>(a, C, mb, max_groups, s);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ms
