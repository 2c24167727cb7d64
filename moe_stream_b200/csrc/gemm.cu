// K4/K5/K6: the prefill / large-batch expert path on the 5th-generation
// tensor cores (tcgen05 + TMEM), for token batches where every routed expert
// sees many tokens (the reference runs these through the same gather_qmm
// calls, engine_v3.py:588-600 / engine_120b.py:130-145, batched by MLX).
//
// Exactness. gather_qmm multiplies by the unrounded dequantised weight
// w = s*q + b (fp32 math). A bf16 copy of w would round it (2^-9 relative),
// enough to flip bf16 output roundings wherever |y| is large. Here every
// weight is carried exactly as the sum of two fp16 values, hi = fp16(w) and
// lo = w - hi (a few bits, exact for any scale above ~1e-5), and each K step
// runs two MMAs, A*hi and A*lo, into the same fp32 accumulator. The
// activations enter as fp16, which holds every bf16 value of magnitude
// 2^-17 .. 65504 exactly. The products are therefore exact and only the fp32
// accumulation order differs from the reference.
//
//   k_scatter  token rows copied into expert order (X_perm, one fp16 row
//              per token/expert pair), each 8-column block stored in the
//              order (0,4,1,5,2,6,3,7) that the nibble unpacking gives the
//              weights, so A and B agree on k; with the per-row score and
//              the pair -> row map. The groups and their 128-row tiles come
//              from the wide router (route.cu).
//   k_gemm<0>  H = SwiGLU(X_perm W_gate^T, X_perm W_up^T) per (M tile, 128/96
//              features): B = [gate rows ; up rows] dequantised in shared
//              memory, tcgen05.mma (M=128, N=256/192, K=16) x {hi, lo} per
//              16 columns, fp32 accumulator in TMEM, SwiGLU in the epilogue,
//              h written as fp16 in the same column order.
//   k_gemm<1>  Y = H W_down^T (+bias), times the routing score, per (M tile,
//              256/192 features).
//   k_combine  y[t] = sum_j Y[inv(t, j)] in a fixed j order.
//
// One CTA = 12 warps: warp 0 issues the TMA loads, warp 1 issues the MMAs,
// warp 2 owns the TMEM allocation, warps 4-11 dequantise each K tile's
// weights and then run the epilogue. Three mbarrier rings hand the tiles
// over: activations + codes (TMA -> dequant/MMA, 4 deep), dequantised
// operands (dequant -> MMA, 2 deep), and the accumulator (MMA -> epilogue).
// Every wait is bounded and reports MS_E_TIMEOUT instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "ms_common.cuh"
#include "tma.cuh"
#include "kernels.h"

namespace ms {

constexpr int GM_THREADS = 384;
constexpr int GM_AP_STAGES = 4;               // activation + code tiles
constexpr int GM_B_STAGES = 2;                // dequantised operand tiles
constexpr int GM_A_BYTES = 128 * 128;         // 128 rows x 64 fp16
constexpr int GM_P_BYTES = 256 * 32;          // up to 256 rows x 64 nibbles
constexpr int GM_B_BYTES = 256 * 128;         // up to 256 rows x 64 fp16 (one of hi / lo)
constexpr int GM_AP_BYTES = GM_A_BYTES + GM_P_BYTES;                   // 24 KB
constexpr int GM_OFF_B = GM_AP_STAGES * GM_AP_BYTES;                   // 96 KB
constexpr int GM_OFF_BAR = GM_OFF_B + GM_B_STAGES * 2 * GM_B_BYTES;    // 224 KB
constexpr int GM_SMEM = GM_OFF_BAR + 256 + 1024;
static_assert(GM_AP_BYTES % 1024 == 0 && GM_B_BYTES % 1024 == 0, "1 KB aligned tiles");

// ------------------------------------------------------------- PTX helpers
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// K-major, 128-byte-swizzled operand tile: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp16 A and B (both K-major), f32 D,
// M=128, N.
__host__ __device__ constexpr uint32_t idesc_f16(int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  const uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m0), "r"(m1), "r"(m2), "r"(m3));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- numerics
// Same rounding points as the decode kernels (MLX's): gather_qmm output bf16,
// each SwiGLU op rounded to bf16.
__device__ __forceinline__ float g_sigm(float v) { return 1.f / (1.f + expf(-v)); }
__device__ __forceinline__ float g_swiglu(int model, float g, float u) {
  if (model == 1) {
    g = fminf(g, 7.f);
    u = fminf(fmaxf(u, -7.f), 7.f);
    const float og = bfr(g * bfr(g_sigm(bfr(1.703125f * g))));
    return bfr(og * bfr(u + 1.f));
  }
  return bfr(bfr(g * bfr(g_sigm(g))) * u);
}

// position of column k (mod 8) inside its 8-column block: (0,4,1,5,2,6,3,7)
__device__ __forceinline__ int kperm_pos(int k) { return ((k & 3) << 1) | (k >> 2); }

__device__ __forceinline__ uint32_t h2_bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 consecutive bf16 (natural order) -> 8 fp16 in the (0,4,1,5,2,6,3,7)
// order; exact for |x| in [2^-17, 65504] (and x = 0).
__device__ __forceinline__ uint4 kperm8_f16(uint4 v) {
  uint4 o;
  o.x = h2_bits(__uint_as_float(v.x << 16), __uint_as_float(v.z << 16));
  o.y = h2_bits(__uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.z & 0xffff0000u));
  o.z = h2_bits(__uint_as_float(v.y << 16), __uint_as_float(v.w << 16));
  o.w = h2_bits(__uint_as_float(v.y & 0xffff0000u), __uint_as_float(v.w & 0xffff0000u));
  return o;
}

// ------------------------------------------------------------------ K5
// One warp per pair: its row goes to the next free row of its group.
// Rows inside a group end up in arrival order; every row is computed on its
// own, so the order changes nothing in the output.
__global__ void __launch_bounds__(256) k_scatter(ScatterArgs a) {
  const int P = a.T * a.k;
  const int warps = gridDim.x * 8;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int chunks = a.d / 8;
  for (int p = gw; p < P; p += warps) {
    int pos = 0;
    if (lane == 0) {
      const int g = a.grp.map[a.inds[p]];
      pos = a.grp.grp_start[g] + atomicAdd(&a.cursor[g], 1);
      a.perm_score[pos] = a.scores_f[p];
      a.inv[p] = pos;
      if (a.pair_slot) a.pair_slot[p] = a.grp.grp_slot[g];
    }
    pos = __shfl_sync(MS_FULL, pos, 0);
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)(p / a.k) * a.d);
    uint4* dst = reinterpret_cast<uint4*>(a.xperm + (long long)pos * a.d);
    for (int c = lane; c < chunks; c += 32) dst[c] = kperm8_f16(__ldg(src + c));
  }
}

// ------------------------------------------------------------------ K4
// PHASE 0: N = 2*NT (gate rows then up rows); PHASE 1: N = NT (down rows).
template <int PHASE, int NT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW0,
           const __grid_constant__ CUtensorMap tmW1, GemmArgs a) {
  constexpr int N = PHASE == 0 ? 2 * NT : NT;
  static_assert(N % 16 == 0 && N <= 256, "MMA N");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.y, nt = blockIdx.x;
  if (tile >= *a.n_tiles || timed_out(a.status)) return;   // uniform: before any barrier
  const GemmTile t = a.tiles[tile];
  const int slot = a.grp_slot[t.g];
  const int KT = a.K / 64, G = a.K / 64;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GM_OFF_BAR);
  uint64_t* full = bars;                                   // [AP]  TMA landed
  uint64_t* empty_ap = bars + GM_AP_STAGES;                // [AP]  MMA done with A (and P)
  uint64_t* deq = bars + 2 * GM_AP_STAGES;                 // [B]   operands written
  uint64_t* empty_b = deq + GM_B_STAGES;                   // [B]   MMA done with them
  uint64_t* accf = empty_b + GM_B_STAGES;                  // accumulator complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  auto sA = [&](int s) { return smem + s * GM_AP_BYTES; };
  auto sP = [&](int s) { return smem + s * GM_AP_BYTES + GM_A_BYTES; };
  auto sBh = [&](int s) { return smem + GM_OFF_B + s * 2 * GM_B_BYTES; };
  auto sBl = [&](int s) { return smem + GM_OFF_B + s * 2 * GM_B_BYTES + GM_B_BYTES; };

  if (slot < 0) {                              // exhausted pool: this tile contributes zeros
    const int cols = PHASE == 0 ? NT : N;
    for (int i = threadIdx.x; i < t.rows * cols; i += GM_THREADS) {
      const int m = i / cols, c = i % cols;
      if (PHASE == 0) a.H[(long long)(t.row0 + m) * a.ld_out + nt * NT + c] = 0;
      else a.Y[(long long)(t.row0 + m) * a.ld_out + nt * NT + c] = 0;
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < GM_AP_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty_ap[s], 1);
    }
    for (int s = 0; s < GM_B_STAGES; ++s) {
      mbar_init(&deq[s], 8);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {                           // ---- TMA producer
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % GM_AP_STAGES;
        if (kt >= GM_AP_STAGES &&
            !mbar_wait(&empty_ap[s], ((kt / GM_AP_STAGES) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&full[s], GM_A_BYTES + N * 32);
        tma_load_2d(sA(s), &tmA, kt * 64, t.row0, &full[s]);
        tma_load_3d(sP(s), &tmW0, kt * 32, nt * NT, slot, &full[s]);
        if (PHASE == 0) tma_load_3d(sP(s) + NT * 32, &tmW1, kt * 32, nt * NT, slot, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {                           // ---- MMA issuer
      constexpr uint32_t idesc = idesc_f16(N);
      for (int kt = 0; kt < KT; ++kt) {
        const int sa = kt % GM_AP_STAGES, sb = kt % GM_B_STAGES;
        if (!mbar_wait(&deq[sb], (kt / GM_B_STAGES) & 1, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(sA(sa)), bh = sw128_desc(sBh(sb)), bl = sw128_desc(sBl(sb));
#pragma unroll
        for (int j = 0; j < 4; ++j) {          // K = 16 per MMA: +32 bytes in the atom
          mma_f16(tmem, ad + 2 * j, bh + 2 * j, idesc, (kt | j) != 0);
          mma_f16(tmem, ad + 2 * j, bl + 2 * j, idesc, 1u);
        }
        mma_commit(&empty_b[sb]);
        mma_commit(&empty_ap[sa]);
      }
      mma_commit(accf);
    }
  } else if (warp >= 4) {
    // ---- dequantise: one weight row per thread, into hi and lo
    const int r = threadIdx.x - 128;
    const int proj = PHASE == 0 ? (r < NT ? 0 : 1) : 2;
    const int orow = nt * NT + (PHASE == 0 ? (r % NT) : r);
    const uint8_t* blob = a.arena + (long long)slot * a.blob;
    const uint16_t* Sc = reinterpret_cast<const uint16_t*>(blob + a.off[proj][1]) + (long long)orow * G;
    const uint16_t* Bi = reinterpret_cast<const uint16_t*>(blob + a.off[proj][2]) + (long long)orow * G;
    const bool active = r < N;
    uint16_t s_next = active ? Sc[0] : 0, b_next = active ? Bi[0] : 0;
    const __half2 h1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    for (int kt = 0; kt < KT; ++kt) {
      const int sa = kt % GM_AP_STAGES, sb = kt % GM_B_STAGES;
      const float sc = bf2f(s_next), bi = bf2f(b_next);
      if (active && kt + 1 < KT) {
        s_next = Sc[kt + 1];
        b_next = Bi[kt + 1];
      }
      // every lane waits; the warp goes on only if all of them saw the stage
      bool got = mbar_wait(&full[sa], (kt / GM_AP_STAGES) & 1, a.status);
      if (got && kt >= GM_B_STAGES)
        got = mbar_wait(&empty_b[sb], ((kt / GM_B_STAGES) - 1) & 1, a.status);
      if (!__all_sync(MS_FULL, got)) {
        ok = false;
        break;
      }
      if (active) {
        const uint4* pk = reinterpret_cast<const uint4*>(sP(sa) + r * 32);
        const uint4 p0 = pk[0], p1 = pk[1];
        const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        uint8_t* rh = sBh(sb) + r * 128;
        uint8_t* rl = sBl(sb) + r * 128;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t u = words[i];
          uint32_t wh[4], wl[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // {q_j, q_j+4} exactly, as fp16 1024+q minus 1024
            const uint32_t m = ((u >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
            const float2 q = __half22float2(__hsub2(*reinterpret_cast<const __half2*>(&m), h1024));
            const float w0 = fmaf(sc, q.x, bi), w1 = fmaf(sc, q.y, bi);   // exact in fp32
            const __half2 hi = __floats2half2_rn(w0, w1);
            const float2 hf = __half22float2(hi);
            wh[j] = *reinterpret_cast<const uint32_t*>(&hi);
            wl[j] = h2_bits(w0 - hf.x, w1 - hf.y);
          }
          const int c = (i ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(rh + c) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
          *reinterpret_cast<uint4*>(rl + c) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
        }
      }
      fence_proxy_async();                     // generic writes -> async (MMA) reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq[sb]);
    }
    // ---- epilogue
    const int ew = warp - 4, quarter = ew & 3, half = ew >> 2;
    const int m = quarter * 32 + lane;
    const bool row_ok = m < t.rows;
    const long long orow_g = t.row0 + m;
    if (ok) ok = __all_sync(MS_FULL, mbar_wait(accf, 0, a.status));
    tc_fence_after();
    const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16);
    if (PHASE == 0) {
      constexpr int HALF = NT / 2;
      const uint16_t* gbias = reinterpret_cast<const uint16_t*>(blob + a.off[0][3]);
      const uint16_t* ubias = reinterpret_cast<const uint16_t*>(blob + a.off[1][3]);
      for (int c0 = half * HALF; c0 < (half + 1) * HALF; c0 += 16) {
        uint32_t gv[16], uv[16];
        tmem_ld16(tbase + c0, gv);
        tmem_ld16(tbase + NT + c0, uv);
        // h (gpt-oss: projection biases first), fp16, in (0,4,1,5,2,6,3,7)
        // order per 8 columns: the next GEMM's A operand
        float hv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float g = bfr(__uint_as_float(gv[j])), u = bfr(__uint_as_float(uv[j]));
          if (a.model == 1) {
            const int f = nt * NT + c0 + j;
            g = bfr(g + bf2f(gbias[f]));
            u = bfr(u + bf2f(ubias[f]));
          }
          hv[(j & 8) | kperm_pos(j & 7)] = g_swiglu(a.model, g, u);
        }
        uint32_t out[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = h2_bits(hv[2 * j], hv[2 * j + 1]);
        if (row_ok && ok) {
          uint4* dst = reinterpret_cast<uint4*>(a.H + orow_g * a.ld_out + nt * NT + c0);
          dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
          dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
        }
      }
    } else {
      constexpr int HALF = N / 2;
      const float score = row_ok ? a.perm_score[orow_g] : 0.f;
      const uint16_t* dbias = reinterpret_cast<const uint16_t*>(blob + a.off[2][3]);
      for (int c0 = half * HALF; c0 < (half + 1) * HALF; c0 += 16) {
        uint32_t acc[16];
        tmem_ld16(tbase + c0, acc);
        uint32_t out[8];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          float v0 = bfr(__uint_as_float(acc[j])), v1 = bfr(__uint_as_float(acc[j + 1]));
          if (a.model == 1) {
            v0 = bfr(v0 + bf2f(dbias[nt * NT + c0 + j]));
            v1 = bfr(v1 + bf2f(dbias[nt * NT + c0 + j + 1]));
          }
          // (y * scores) is a bf16 product (engine_v3.py:600)
          out[j / 2] = (uint32_t)f2bf(score * v0) | ((uint32_t)f2bf(score * v1) << 16);
        }
        if (row_ok && ok) {
          uint4* dst = reinterpret_cast<uint4*>(a.Y + orow_g * a.ld_out + nt * NT + c0);
          dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
          dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ K6
__global__ void __launch_bounds__(256) k_combine(CombineArgs a) {
  const int chunks = a.d / 8;
  const long long total = (long long)a.T * chunks;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const int t = (int)(i / chunks), c = (int)(i % chunks);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < a.k; ++j) {
      const int row = a.inv[t * a.k + j];
      const uint4 v = *reinterpret_cast<const uint4*>(a.Y + (long long)row * a.d + c * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += __uint_as_float(w[q] << 16);
        acc[2 * q + 1] += __uint_as_float(w[q] & 0xffff0000u);
      }
    }
    uint4 o;
    o.x = (uint32_t)f2bf(acc[0]) | ((uint32_t)f2bf(acc[1]) << 16);
    o.y = (uint32_t)f2bf(acc[2]) | ((uint32_t)f2bf(acc[3]) << 16);
    o.z = (uint32_t)f2bf(acc[4]) | ((uint32_t)f2bf(acc[5]) << 16);
    o.w = (uint32_t)f2bf(acc[6]) | ((uint32_t)f2bf(acc[7]) << 16);
    *reinterpret_cast<uint4*>(a.y + (long long)t * a.d + c * 8) = o;
  }
}

// ------------------------------------------------------------- tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// fp16 activations [rows, K]: 64 x 128 boxes, 128-byte swizzle (the
// canonical K-major layout the MMA descriptors describe).
int encode_act_map(CUtensorMap* m, const void* base, int K, long long rows) {
  auto fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -2;
}

// 4-bit weight codes of one projection across all slots, as bytes
// [n_slots][rows_out][K/2]: boxes of 32 bytes (one group of 64 codes) x
// box_rows rows x 1 slot, unswizzled.
int encode_weight_map(CUtensorMap* m, const void* base, int K, int rows_out, int n_slots,
                      long long blob, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[3] = {(cuuint64_t)(K / 2), (cuuint64_t)rows_out, (cuuint64_t)n_slots};
  const cuuint64_t strides[2] = {(cuuint64_t)(K / 2), (cuuint64_t)blob};
  const cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -2;
}

int gemm_col_tile(int phase, int n) {
  static const int p0[] = {128, 96, 64};
  static const int p1[] = {256, 192, 128, 64};
  if (phase == 0) {
    for (int c : p0)
      if (n % c == 0) return c;
  } else {
    for (int c : p1)
      if (n % c == 0) return c;
  }
  return 0;
}

// ---------------------------------------------------------------- launchers
cudaError_t launch_scatter(const ScatterArgs& a, int grid, cudaStream_t s) {
  k_scatter<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_combine(const CombineArgs& a, int grid, cudaStream_t s) {
  k_combine<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

template <int PHASE, int NT>
static cudaError_t launch_gemm_t(const CUtensorMap& tA, const CUtensorMap& tW0,
                                 const CUtensorMap& tW1, const GemmArgs& a, int n_col_tiles,
                                 int max_tiles, cudaStream_t s) {
  auto kern = k_gemm<PHASE, NT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_SMEM);
  if (e != cudaSuccess) return e;
  kern<<<dim3(n_col_tiles, max_tiles), GM_THREADS, GM_SMEM, s>>>(tA, tW0, tW1, a);
  return cudaGetLastError();
}

cudaError_t launch_gemm(int phase, int nt, const CUtensorMap& tA, const CUtensorMap& tW0,
                        const CUtensorMap& tW1, const GemmArgs& a, int n_col_tiles, int max_tiles,
                        cudaStream_t s) {
  if (phase == 0 && nt == 128) return launch_gemm_t<0, 128>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 0 && nt == 96) return launch_gemm_t<0, 96>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 0 && nt == 64) return launch_gemm_t<0, 64>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 1 && nt == 256) return launch_gemm_t<1, 256>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 1 && nt == 192) return launch_gemm_t<1, 192>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 1 && nt == 128) return launch_gemm_t<1, 128>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  if (phase == 1 && nt == 64) return launch_gemm_t<1, 64>(tA, tW0, tW1, a, n_col_tiles, max_tiles, s);
  return cudaErrorInvalidValue;
}

}  // namespace ms
