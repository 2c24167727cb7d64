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
// runs two MMAs, hi*X and lo*X, into the same fp32 accumulator. The
// activations enter as fp16, which holds every bf16 value of magnitude
// 2^-17 .. 65504 exactly. The products are therefore exact and only the fp32
// accumulation order differs from the reference.
//
// Shape. Weights are the MMA's A operand and live in tensor memory: each
// dequantising thread owns one weight row = one TMEM lane and writes its hi
// and lo halves there with tcgen05.st, so the dequantised operand never
// touches shared memory. Tokens are the B operand: up to 256 rows of X per
// CTA, TMA-loaded into shared memory (128-byte swizzle). D[weight row, token]
// accumulates in TMEM. Each dequantised weight thus serves up to 256 tokens.
//
//   k_scatter  token rows copied into expert order (X_perm, one fp16 row
//              per token/expert pair), each 8-column block stored in the
//              order (0,4,1,5,2,6,3,7) that the nibble unpacking gives the
//              weights, so both operands agree on k; with the per-row score
//              and the pair -> row map. The groups and their 256-row tiles
//              come from the wide router (route.cu).
//   k_gemm<0>  per (64 features, token tile): A = [64 gate rows; 64 up rows],
//              D lanes 0-63 gate, 64-127 up; SwiGLU in the epilogue; h
//              written as fp16 in the k-permuted column order.
//   k_gemm<1>  per (128 output features, token tile): A = down rows;
//              Y = bf16(acc) (+bias), times the routing score.
//   k_combine  y[t] = sum_j Y[inv(t, j)] in a fixed j order.
//
// One CTA = 12 warps: warp 0 issues the TMA loads, warp 1 issues the MMAs,
// warp 2 owns the TMEM allocation, warps 4-11 dequantise (two warps per
// TMEM lane quarter, each taking half of a K tile's columns) and then run
// the epilogue. mbarrier rings hand the tiles over: tokens + codes (TMA ->
// dequant/MMA, 4 deep), weights in TMEM (dequant -> MMA, 2 deep), and the
// accumulator (MMA -> epilogue). Every wait is bounded and reports
// MS_E_TIMEOUT instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "ms_common.cuh"
#include "tma.cuh"
#include "kernels.h"

namespace ms {

constexpr int GM_THREADS = 384;
constexpr int GM_STAGES = 4;                  // token + code tiles
constexpr int GM_A_STAGES = 4;                // weight tiles in TMEM
constexpr int GM_TOK = GEMM_TILE_ROWS;        // tokens per CTA (MMA N, at most)
constexpr int GM_X_BYTES = GM_TOK * 128;      // 256 tokens x 64 fp16
constexpr int GM_P_BYTES = 128 * 32;          // 128 weight rows x 64 nibbles
constexpr int GM_OFF_P = GM_STAGES * GM_X_BYTES;                   // 128 KB
constexpr int GM_OFF_BAR = GM_OFF_P + GM_STAGES * GM_P_BYTES;      // 144 KB
constexpr int GM_SMEM = GM_OFF_BAR + 256 + 1024;
// TMEM columns: accumulator [0, 256), weight stage s at 256 + 64 s (hi, then lo)
constexpr uint32_t TM_ACC = 0, TM_A = 256, TM_COLS = 512;
static_assert(TM_A + GM_A_STAGES * 64 <= TM_COLS, "weight stages fit in TMEM");
static_assert(GM_X_BYTES % 1024 == 0 && GM_P_BYTES % 1024 == 0, "1 KB aligned tiles");
// epilogue staging, in the (then idle) token ring: 256 tokens x 128 fp32
static_assert(GM_TOK * 128 * 4 <= GM_OFF_P, "epilogue staging fits in the token ring");
constexpr int SCALE_AHEAD = 4;                // scale/bias loads issued this many K tiles early

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
// M=128, N (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t idesc_f16(int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((128u >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T (A: M=128 rows x K=16, one row per lane).
__device__ __forceinline__ void mma_ts_f16(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  const uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m0), "r"(m1), "r"(m2), "r"(m3));
}

// 16 consecutive columns of this thread's lane <- v[0..16)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// barrier 1 among the 256 epilogue threads (warps 4-11)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

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
// PHASE 0: blockIdx.x = 64-feature tile of d_ff (A rows: gate f0..f0+63,
// then up f0..f0+63). PHASE 1: 128-feature tile of d_model (down rows).
template <int PHASE>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW0,
           const __grid_constant__ CUtensorMap tmW1, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.y;
  if (tile >= *a.n_tiles || timed_out(a.status)) return;   // uniform: before any barrier
  const GemmTile t = a.tiles[tile];
  const int slot = a.grp_slot[t.g];
  const int KT = a.K / 64, G = a.K / 64;
  const int n_out = a.n_out;                   // rows of this projection's output
  const int f0 = blockIdx.x * (PHASE == 0 ? 64 : 128);
  const int ntok = (t.rows + 15) & ~15;        // MMA N: the tile's rows, rounded up to 16

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GM_OFF_BAR);
  uint64_t* full = bars;                                   // [S]  TMA landed
  uint64_t* empty_x = bars + GM_STAGES;                    // [S]  MMA done with X (and P)
  uint64_t* deq = bars + 2 * GM_STAGES;                    // [A]  weights in TMEM
  uint64_t* empty_a = deq + GM_A_STAGES;                   // [A]  MMA done with them
  uint64_t* accf = empty_a + GM_A_STAGES;                  // accumulator complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  auto sX = [&](int s) { return smem + s * GM_X_BYTES; };
  auto sP = [&](int s) { return smem + GM_OFF_P + s * GM_P_BYTES; };

  if (slot < 0) {                              // exhausted pool: this tile contributes zeros
    const int cols = PHASE == 0 ? 64 : min(128, n_out - f0);
    uint16_t* out = PHASE == 0 ? a.H : a.Y;
    for (int i = threadIdx.x; i < t.rows * cols; i += GM_THREADS) {
      const int m = i / cols, c = i % cols;
      out[(long long)(t.row0 + m) * a.ld_out + f0 + c] = 0;
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < GM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < GM_A_STAGES; ++s) {
      mbar_init(&deq[s], 8);
      mbar_init(&empty_a[s], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, TM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {                           // ---- TMA producer
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % GM_STAGES;
        if (kt >= GM_STAGES && !mbar_wait(&empty_x[s], ((kt / GM_STAGES) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&full[s], GM_X_BYTES + GM_P_BYTES);
        tma_load_2d(sX(s), &tmX, kt * 64, t.row0, &full[s]);
        if (PHASE == 0) {
          tma_load_3d(sP(s), &tmW0, kt * 32, f0, slot, &full[s]);
          tma_load_3d(sP(s) + 64 * 32, &tmW1, kt * 32, f0, slot, &full[s]);
        } else {
          tma_load_3d(sP(s), &tmW0, kt * 32, f0, slot, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {                           // ---- MMA issuer
      const uint32_t idesc = idesc_f16(ntok);
      for (int kt = 0; kt < KT; ++kt) {
        const int sx = kt % GM_STAGES, sa = kt % GM_A_STAGES;
        if (!mbar_wait(&deq[sa], (kt / GM_A_STAGES) & 1, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bd = sw128_desc(sX(sx));
        const uint32_t ahi = tmem + TM_A + sa * 64, alo = ahi + 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {          // K = 16 per MMA: 8 TMEM columns, 32 smem bytes
          mma_ts_f16(tmem + TM_ACC, ahi + 8 * j, bd + 2 * j, idesc, (kt | j) != 0);
          mma_ts_f16(tmem + TM_ACC, alo + 8 * j, bd + 2 * j, idesc, 1u);
        }
        mma_commit(&empty_a[sa]);
        mma_commit(&empty_x[sx]);
      }
      mma_commit(accf);
    }
  } else if (warp >= 4) {
    // ---- dequantise: TMEM lane r = weight row r; this warp takes columns
    // [16*half, 16*half + 16) of each K tile (32 codes)
    const int quarter = warp & 3, half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;
    int proj, orow;
    if (PHASE == 0) {
      proj = r < 64 ? 0 : 1;
      orow = f0 + (r & 63);
    } else {
      proj = 2;
      orow = f0 + r;
    }
    const bool active = orow < n_out;
    const uint8_t* blob = a.arena + (long long)slot * a.blob;
    const uint16_t* Sc = reinterpret_cast<const uint16_t*>(blob + a.off[proj][1]) + (long long)orow * G;
    const uint16_t* Bi = reinterpret_cast<const uint16_t*>(blob + a.off[proj][2]) + (long long)orow * G;
    // (scale | bias << 16) of K tiles kt .. kt + SCALE_AHEAD - 1, a shifting ring
    uint32_t sb[SCALE_AHEAD];
#pragma unroll
    for (int i = 0; i < SCALE_AHEAD; ++i)
      sb[i] = (active && i < KT) ? ((uint32_t)Sc[i] | ((uint32_t)Bi[i] << 16)) : 0u;
    const float2 magic_off = make_float2(-8388608.f, -8388608.f);
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    for (int kt = 0; kt < KT; ++kt) {
      const int sx = kt % GM_STAGES, sa = kt % GM_A_STAGES;
      const float sc = __uint_as_float(sb[0] << 16), bi = __uint_as_float(sb[0] & 0xffff0000u);
#pragma unroll
      for (int i = 0; i + 1 < SCALE_AHEAD; ++i) sb[i] = sb[i + 1];
      const int kn = kt + SCALE_AHEAD;
      sb[SCALE_AHEAD - 1] = (active && kn < KT) ? ((uint32_t)Sc[kn] | ((uint32_t)Bi[kn] << 16)) : 0u;
      // every lane waits; the warp goes on only if all of them saw the stage
      bool got = mbar_wait(&full[sx], (kt / GM_STAGES) & 1, a.status);
      if (got && kt >= GM_A_STAGES)
        got = mbar_wait(&empty_a[sa], ((kt / GM_A_STAGES) - 1) & 1, a.status);
      if (!__all_sync(MS_FULL, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t wh[16], wl[16];
      if (active) {
        const uint4 pw = *reinterpret_cast<const uint4*>(sP(sx) + r * 32 + half * 16);
        const uint32_t words[4] = {pw.x, pw.y, pw.z, pw.w};
        const float2 s2 = make_float2(sc, sc), b2 = make_float2(bi, bi);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t u = words[i];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // q_j and q_j+4 as exact floats (2^23 + q, minus 2^23)
            const uint32_t m = (u >> (4 * j)) & 0x000F000Fu;
            const float2 q = __fadd2_rn(make_float2(__uint_as_float((m & 0xFu) | 0x4B000000u),
                                                    __uint_as_float((m >> 16) | 0x4B000000u)),
                                        magic_off);
            const float2 w = __ffma2_rn(q, s2, b2);             // exact: s*q + b
            const __half2 hi = __floats2half2_rn(w.x, w.y);
            const float2 hf = __half22float2(hi);
            const float2 lo = __fadd2_rn(w, make_float2(-hf.x, -hf.y));
            wh[i * 4 + j] = *reinterpret_cast<const uint32_t*>(&hi);
            wl[i * 4 + j] = h2_bits(lo.x, lo.y);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) wh[i] = wl[i] = 0u;
      }
      const uint32_t col = TM_A + sa * 64 + half * 16;
      tmem_st16(lane_base + col, wh);
      tmem_st16(lane_base + col + 32, wl);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq[sa]);
    }
    // ---- epilogue. Each warp reads lanes [32*quarter, +32) and token
    // columns [128*half, +128) of the accumulator into the staging area S
    // (the token ring, idle once the accumulator is complete), as fp32
    // S[token][lane]; then the 256 threads write whole 16-byte chunks.
    if (ok) ok = __all_sync(MS_FULL, mbar_wait(accf, 0, a.status));
    tc_fence_after();
    float* S = reinterpret_cast<float*>(smem);
    const int c_lo = half * 128, c_hi = min(ntok, c_lo + 128);
    const int et = threadIdx.x - 128;          // 0..255
    if (PHASE == 0) {
      // lanes 0-63: gate + bias, 64-127: up + bias, both bf16-rounded
      const int fg = f0 + (r & 63);
      const float bias = a.model == 1 ? bf2f(reinterpret_cast<const uint16_t*>(
                                                blob + a.off[r < 64 ? 0 : 1][3])[fg])
                                      : 0.f;
      for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + TM_ACC + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float g = bfr(__uint_as_float(v[j]));
          if (a.model == 1) g = bfr(g + bias);
          S[(c0 + j) * 128 + r] = g;
        }
      }
      epi_sync();
      // h for 8 consecutive features of one token per task, k-permuted, fp16
      for (int task = et; task < t.rows * 8; task += 256) {
        const int m = task >> 3, c8 = (task & 7) * 8;
        const float4* gs = reinterpret_cast<const float4*>(S + m * 128 + c8);
        const float4 g0 = gs[0], g1 = gs[1], u0 = gs[16], u1 = gs[17];
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float hv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) hv[kperm_pos(j)] = g_swiglu(a.model, gv[j], uv[j]);
        if (ok)
          *reinterpret_cast<uint4*>(a.H + (long long)(t.row0 + m) * a.ld_out + f0 + c8) =
              make_uint4(h2_bits(hv[0], hv[1]), h2_bits(hv[2], hv[3]), h2_bits(hv[4], hv[5]),
                         h2_bits(hv[6], hv[7]));
      }
    } else {
      const int fo = f0 + r;                   // output feature
      const float bias = (a.model == 1 && fo < n_out)
                             ? bf2f(reinterpret_cast<const uint16_t*>(blob + a.off[2][3])[fo]) : 0.f;
      for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + TM_ACC + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = bfr(__uint_as_float(v[j]));
          if (a.model == 1) y = bfr(y + bias);
          S[(c0 + j) * 128 + r] = y;
        }
      }
      epi_sync();
      // (y * scores) is a bf16 product (engine_v3.py:600); 8 features per task
      const int nf = min(128, n_out - f0);     // a multiple of 8 (d_model % 64 == 0)
      const int chunks = nf >> 3;
      for (int task = et; task < t.rows * chunks; task += 256) {
        const int m = task / chunks, c8 = (task % chunks) * 8;
        const float sc = a.perm_score[t.row0 + m];
        const float4* y4 = reinterpret_cast<const float4*>(S + m * 128 + c8);
        const float4 y0 = y4[0], y1 = y4[1];
        const float ys[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = (uint32_t)f2bf(sc * ys[2 * j]) | ((uint32_t)f2bf(sc * ys[2 * j + 1]) << 16);
        if (ok)
          *reinterpret_cast<uint4*>(a.Y + (long long)(t.row0 + m) * a.ld_out + f0 + c8) =
              make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
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

// fp16 activations [rows, K]: 64 x 256 boxes, 128-byte swizzle (the
// canonical K-major layout the MMA descriptors describe).
int encode_act_map(CUtensorMap* m, const void* base, int K, long long rows) {
  auto fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)GM_TOK};
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

// ---------------------------------------------------------------- launchers
cudaError_t launch_scatter(const ScatterArgs& a, int grid, cudaStream_t s) {
  k_scatter<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_combine(const CombineArgs& a, int grid, cudaStream_t s) {
  k_combine<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

template <int PHASE>
static cudaError_t launch_gemm_t(const CUtensorMap& tX, const CUtensorMap& tW0,
                                 const CUtensorMap& tW1, const GemmArgs& a, int n_col_tiles,
                                 int max_tiles, cudaStream_t s) {
  auto kern = k_gemm<PHASE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_SMEM);
  if (e != cudaSuccess) return e;
  kern<<<dim3(n_col_tiles, max_tiles), GM_THREADS, GM_SMEM, s>>>(tX, tW0, tW1, a);
  return cudaGetLastError();
}

cudaError_t launch_gemm(int phase, const CUtensorMap& tX, const CUtensorMap& tW0,
                        const CUtensorMap& tW1, const GemmArgs& a, int n_col_tiles, int max_tiles,
                        cudaStream_t s) {
  if (phase == 0) return launch_gemm_t<0>(tX, tW0, tW1, a, n_col_tiles, max_tiles, s);
  return launch_gemm_t<1>(tX, tW0, tW1, a, n_col_tiles, max_tiles, s);
}

}  // namespace ms
