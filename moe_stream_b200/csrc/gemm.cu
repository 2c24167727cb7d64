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
// touches shared memory. Tokens are the B operand: up to 128 rows of X per
// work item, TMA-loaded into shared memory (128-byte swizzle). D[weight row,
// token] accumulates in TMEM.
//
//   k_scatter  token rows copied into expert order (X_perm, one fp16 row
//              per token/expert pair), each 8-column block stored in the
//              order (0,4,1,5,2,6,3,7) that the nibble unpacking gives the
//              weights, so both operands agree on k; with the per-row score
//              and the pair -> row map. The groups and their 128-row tiles
//              come from the wide router (route.cu).
//   k_gemm<0>  per (64 features, token tile): A = 64 gate and 64 up rows,
//              arranged so that lane 32q + l holds gate feature 16q + l and
//              lane 32q + 16 + l the up row of the same feature; SwiGLU in
//              the epilogue pairs them with one shuffle; h written as fp16
//              in the k-permuted column order.
//   k_gemm<1>  per (128 output features, token tile): A = down rows;
//              Y = bf16(acc) (+bias), times the routing score.
//   k_combine  y[t] = sum_j Y[inv(t, j)] in a fixed j order.
//
// Persistent CTAs, one per SM, each looping over (token tile, feature tile)
// work items with 24 warps in fixed roles: warp 0 issues the TMA loads,
// warp 1 the MMAs, warp 2 owns the TMEM allocation, warps 4-19 dequantise
// (four per TMEM lane quarter, each taking a quarter of a K tile's columns),
// warps 20-23 drain finished accumulators (one per lane quarter). mbarrier
// rings hand the work over: tokens + codes (TMA -> dequant/MMA, 8 deep),
// weights in TMEM (dequant -> MMA, 4 deep) and two accumulators (MMA <->
// epilogue), so one item's epilogue overlaps the next item's main loop.
// Every wait is bounded and reports MS_E_TIMEOUT instead of hanging.
#include <algorithm>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "ms_common.cuh"
#include "tma.cuh"
#include "kernels.h"

namespace ms {

constexpr int GM_THREADS = 768;              // 24 warps, see the role list above
constexpr int GM_STAGES = 8;                  // token + code tiles
constexpr int GM_A_STAGES = 4;                // weight tiles in TMEM
constexpr int GM_TOK = GEMM_TILE_ROWS;        // tokens per tile (MMA N, at most)
constexpr int GM_X_BYTES = GM_TOK * 128;      // 128 tokens x 64 fp16
constexpr int GM_P_BYTES = 128 * 64;          // 128 weight rows x 64 codes of up to 8 bits
constexpr int GM_OFF_P = GM_STAGES * GM_X_BYTES;                   // 128 KB
constexpr int GM_OFF_BAR = GM_OFF_P + GM_STAGES * GM_P_BYTES;      // 192 KB (> half an SM:
constexpr int GM_SMEM = GM_OFF_BAR + 256 + 1024;                   //  one CTA per SM)
// TMEM columns: accumulators [0, 128) and [128, 256); weight stage s at
// 256 + 64 s (hi, then lo)
constexpr uint32_t TM_ACC = 0, TM_A = 256, TM_COLS = 512;
static_assert(2 * GM_TOK <= (int)TM_A && TM_A + GM_A_STAGES * 64 <= TM_COLS, "TMEM budget");
static_assert(GM_X_BYTES % 1024 == 0 && GM_P_BYTES % 1024 == 0, "1 KB aligned tiles");
static_assert(GM_SMEM > 232448 / 2, "one CTA per SM: the whole of TMEM is allocated");
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

// 8 consecutive columns of this thread's lane <- v[0..8)
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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
// 1/(1+e^-v); __frcp_rn is the correctly rounded reciprocal, i.e. 1.f / x
__device__ __forceinline__ float g_sigm(float v) { return __frcp_rn(1.f + expf(-v)); }
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

// Either bf16 of a pair beyond the fp16 range: |v| > 65504 <=> magnitude
// bits above 0x477f (65280, the largest bf16 below 65504), inf and NaN
// included.
__device__ __forceinline__ bool bf16x2_beyond_f16(uint32_t v) {
  return (v & 0x7fffu) > 0x477fu || ((v >> 16) & 0x7fffu) > 0x477fu;
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
    bool over = false;
    for (int c = lane; c < chunks; c += 32) {
      const uint4 v = __ldg(src + c);
      over |= bf16x2_beyond_f16(v.x) | bf16x2_beyond_f16(v.y) | bf16x2_beyond_f16(v.z) |
              bf16x2_beyond_f16(v.w);
      dst[c] = kperm8_f16(v);
    }
    if (__any_sync(MS_FULL, over) && lane == 0) atomicCAS(a.status, 0, ST_E_RANGE);
  }
}

// ------------------------------------------------------------------ K4
// Work item w: token tile w / n_ft, feature tile w % n_ft. PHASE 0 feature
// tiles are 64 features of d_ff (gate and up rows), PHASE 1 tiles 128
// features of d_model (down rows). Items whose group has no slot (pool
// exhausted) run with zero weights and write zeros.
// The class of an item's slot (MIXED pools; 0 for a missing slot, whose
// codes read as zeros through class 0's maps).
template <bool MIXED>
__device__ __forceinline__ int item_class(const GemmArgs& a, int slot) {
  if (!MIXED || slot < 0) return 0;
  return min((int)a.slot_class[slot], a.C.n - 1);
}

// Codes j and j + 4 (j in 0..3) of 8-code block b of the 16 codes a
// dequantising lane takes from a staged K tile, as exact floats. r: the raw
// bits (see load_codes).
template <int BITS>
__device__ __forceinline__ float2 code_pair(const uint32_t* r, int b, int j) {
  uint32_t q0, q1;
  if (BITS == 2) {
    q0 = (r[0] >> (16 * b + 2 * j)) & 3u;
    q1 = (r[0] >> (16 * b + 2 * j + 8)) & 3u;
  } else if (BITS == 8) {
    q0 = (r[2 * b] >> (8 * j)) & 0xFFu;
    q1 = (r[2 * b + 1] >> (8 * j)) & 0xFFu;
  } else {                                     // 3: r[b] holds codes 8b..8b+7 at bits 3i
    q0 = (r[b] >> (3 * j)) & 7u;
    q1 = (r[b] >> (3 * j + 12)) & 7u;
  }
  return make_float2(__uint_as_float(q0 | 0x4B000000u) - 8388608.f,
                     __uint_as_float(q1 | 0x4B000000u) - 8388608.f);
}

// The raw bits of a lane's 16 codes (part `part` of a 64-code K tile) from
// its staged row: 2 bits one word, 8 bits four, 3 bits two words of codes
// 0-7 and 8-15 (the tile starts o3 bytes into the staged row).
template <int BITS>
__device__ __forceinline__ void load_codes(const uint8_t* row, int part, int o3, uint32_t* r) {
  if (BITS == 2) {
    r[0] = *reinterpret_cast<const uint32_t*>(row + 4 * part);
  } else if (BITS == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + 16 * part);
    r[0] = u.x; r[1] = u.y; r[2] = u.z; r[3] = u.w;
  } else {
    const int b0 = o3 + 6 * part, base = b0 & ~3, sh = (b0 & 3) * 8;
    const uint32_t lo = *reinterpret_cast<const uint32_t*>(row + base);
    const uint32_t hi = *reinterpret_cast<const uint32_t*>(row + base + 4);
    const uint32_t aa = __funnelshift_r(lo, hi, sh);
    const uint32_t bb = hi >> sh;
    r[0] = aa;
    r[1] = __funnelshift_r(aa, bb, 24);
  }
}

template <int PHASE, bool MIXED>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ GemmMaps mm, GemmArgs a) {
  constexpr int FT = PHASE == 0 ? 64 : 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = a.n_out;
  const int n_ft = (n_out + FT - 1) / FT;
  const int total = *a.n_tiles * n_ft;
  if (blockIdx.x >= total || timed_out(a.status)) return;   // uniform: before any barrier
  const int KT = a.K / 64, G = a.K / 64;
  const int step = gridDim.x;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GM_OFF_BAR);
  uint64_t* full = bars;                                   // [S]  TMA landed
  uint64_t* empty_x = full + GM_STAGES;                    // [S]  MMA done with X (and P)
  uint64_t* deq = empty_x + GM_STAGES;                     // [A]  weights in TMEM
  uint64_t* empty_a = deq + GM_A_STAGES;                   // [A]  MMA done with them
  uint64_t* acc_full = empty_a + GM_A_STAGES;              // [2]  accumulator complete
  uint64_t* acc_empty = acc_full + 2;                      // [2]  accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  auto sX = [&](int s) { return smem + s * GM_X_BYTES; };
  auto sP = [&](int s) { return smem + GM_OFF_P + s * GM_P_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < GM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < GM_A_STAGES; ++s) {
      mbar_init(&deq[s], 16);
      mbar_init(&empty_a[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, TM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {                           // ---- TMA producer
      int it = 0;
      bool ok = true;
      GemmTile tn = a.tiles[blockIdx.x / n_ft];          // tile records: one item ahead
      for (int w = blockIdx.x; w < total && ok; w += step) {
        const GemmTile t = tn;
        if (w + step < total) tn = a.tiles[(w + step) / n_ft];
        const int f0 = (w % n_ft) * FT;
        const int cls = item_class<MIXED>(a, t.slot);
        const int bits = MIXED ? a.C.c[cls].bits : 4;
        const int cb = gemm_tile_row_bytes(bits);   // staged bytes per row of a K tile
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % GM_STAGES;
          if (it >= GM_STAGES && !mbar_wait(&empty_x[s], ((it / GM_STAGES) - 1) & 1, a.status)) {
            ok = false;
            break;
          }
          // the K tile's codes start 8*bits*kt bytes into the row (3 bits:
          // from the 16-byte boundary below, the rest is read past it)
          const int xc = bits == 3 ? ((24 * kt) & ~15) : 8 * bits * kt;
          mbar_expect_tx(&full[s], GM_X_BYTES + 128 * cb);
          tma_load_2d(sX(s), &tmX, kt * 64, t.row0, &full[s]);
          // a slot of -1 reads outside the tensor: the codes arrive as zeros
          if (PHASE == 0) {
            tma_load_3d(sP(s), &mm.w[0][cls], xc, f0, t.slot, &full[s]);
            tma_load_3d(sP(s) + 64 * cb, &mm.w[1][cls], xc, f0, t.slot, &full[s]);
          } else {
            tma_load_3d(sP(s), &mm.w[0][cls], xc, f0, t.slot, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {                           // ---- MMA issuer
      int it = 0, ai = 0;
      bool ok = true;
      GemmTile tn = a.tiles[blockIdx.x / n_ft];
      for (int w = blockIdx.x; w < total && ok; w += step, ++ai) {
        const GemmTile t = tn;
        if (w + step < total) tn = a.tiles[(w + step) / n_ft];
        const uint32_t idesc = idesc_f16((t.rows + 15) & ~15);
        const int b = ai & 1;
        if (ai >= 2 && !mbar_wait(&acc_empty[b], ((ai >> 1) - 1) & 1, a.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + TM_ACC + b * GM_TOK;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int sx = it % GM_STAGES, sa = it % GM_A_STAGES;
          if (!mbar_wait(&deq[sa], (it / GM_A_STAGES) & 1, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = sw128_desc(sX(sx));
          const uint32_t ahi = tmem + TM_A + sa * 64, alo = ahi + 32;
#pragma unroll
          for (int j = 0; j < 4; ++j) {        // K = 16 per MMA: 8 TMEM columns, 32 smem bytes
            mma_ts_f16(d, ahi + 8 * j, bd + 2 * j, idesc, (kt | j) != 0);
            mma_ts_f16(d, alo + 8 * j, bd + 2 * j, idesc, 1u);
          }
          mma_commit(&empty_a[sa]);
          mma_commit(&empty_x[sx]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 4 && warp < 20) {
    // ---- dequantise: TMEM lane L = one weight row; this warp takes columns
    // [8*part, 8*part + 8) of each K tile (16 codes)
    const int quarter = warp & 3, part = (warp - 4) >> 2;
    const int L = quarter * 32 + lane;
    // this lane's row inside the tile of codes (PHASE 0: gate rows 0-63,
    // then up rows 64-127 of the shared-memory tile)
    const int prow = PHASE == 0 ? ((lane < 16 ? 0 : 64) + 16 * quarter + (lane & 15)) : L;
    const int proj = PHASE == 0 ? (lane < 16 ? 0 : 1) : 2;
    // scale/bias prefetch cursor: item pw, K tile pkt, SCALE_AHEAD K tiles
    // ahead of the work and running across item boundaries. Every load
    // address is valid (rows without weights read row 0 of slot 0 and are
    // masked when consumed), so no load is ever waited on early: a ring
    // entry keeps the raw scale and bias (bf16 bits, or fp8 codes) in the
    // registers the loads write, untouched until the entry is consumed, and
    // a word with whether the row is active plus (MIXED) the item's code
    // width and fp8 row exponents, so the consumer needs no per-item lookups
    // of its own.
    int pw = blockIdx.x, pkt = 0;
    const uint8_t *psc = nullptr, *pbi = nullptr;
    uint32_t pmeta = 0;                        // active | fp8 << 1 | bits << 2 | es << 8 | eb << 16
    int pesz = 2;
    GemmTile pnext = a.tiles[pw / n_ft];
    auto enter = [&](int w) {                  // the cursor enters item w (pnext = its tile)
      const GemmTile tt = pnext;
      if (w + step < total) pnext = a.tiles[(w + step) / n_ft];
      const int orow = (w % n_ft) * FT + (PHASE == 0 ? 16 * quarter + (lane & 15) : L);
      const bool act = tt.slot >= 0 && orow < n_out;
      const uint8_t* blob = a.arena + (long long)(act ? tt.slot : 0) * a.blob;
      const long long ro = act ? orow : 0;
      if (!MIXED) {
        psc = blob + a.off[proj][1] + ro * G * 2;
        pbi = blob + a.off[proj][2] + ro * G * 2;
        pmeta = (act ? 1u : 0u) | (4u << 2);
      } else {
        const PrecDev& pc = a.C.c[item_class<MIXED>(a, tt.slot)];
        pesz = pc.fmt == SF_FP8 ? 1 : 2;
        psc = blob + pc.off[proj][P_S] + ro * G * pesz;
        pbi = blob + pc.off[proj][P_B] + ro * G * pesz;
        uint32_t es = 0, eb = 0;
        if (pc.fmt == SF_FP8) {
          es = blob[pc.off[proj][P_SE] + ro];
          eb = blob[pc.off[proj][P_BE] + ro];
        }
        pmeta = (act ? 1u : 0u) | ((pc.fmt == SF_FP8 ? 1u : 0u) << 1) | ((uint32_t)pc.bits << 2) |
                (es << 8) | (eb << 16);
      }
    };
    auto fetch = [&](uint32_t& sv, uint32_t& bv, uint32_t& meta) {
      meta = pw < total ? pmeta : 0u;
      if (!MIXED || pesz == 2) {
        sv = reinterpret_cast<const uint16_t*>(psc)[pkt];
        bv = reinterpret_cast<const uint16_t*>(pbi)[pkt];
      } else {
        sv = psc[pkt];
        bv = pbi[pkt];
      }
      if (++pkt == KT) {
        pkt = 0;
        pw += step;
        if (pw < total) enter(pw);
      }
    };
    enter(pw);
    uint32_t rs[SCALE_AHEAD], rb[SCALE_AHEAD], rmeta[SCALE_AHEAD];
#pragma unroll
    for (int i = 0; i < SCALE_AHEAD; ++i) fetch(rs[i], rb[i], rmeta[i]);
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const int n_it = ((total - (int)blockIdx.x + step - 1) / step) * KT;   // K tiles of this CTA
    bool ok = true;
    // one flat loop over this CTA's K tiles, unrolled so that every ring
    // entry is a fixed register
    for (int it0 = 0; it0 < n_it && ok; it0 += SCALE_AHEAD) {
#pragma unroll
      for (int j = 0; j < SCALE_AHEAD; ++j) {
        const int it = it0 + j;
        if (it >= n_it || !ok) continue;
        const uint32_t meta = rmeta[j];
        float sc = 0.f, bi = 0.f;
        if (meta & 1u) {
          if (MIXED && (meta & 2u)) {
            sc = e4m3_to_f((uint8_t)rs[j]) * exp_factor((uint8_t)((meta >> 8) & 0xFFu));
            bi = e4m3_to_f((uint8_t)rb[j]) * exp_factor((uint8_t)((meta >> 16) & 0xFFu));
          } else {
            sc = bf2f((uint16_t)rs[j]);
            bi = bf2f((uint16_t)rb[j]);
          }
        }
        const int bits = MIXED ? (int)((meta >> 2) & 0xFu) : 4;
        fetch(rs[j], rb[j], rmeta[j]);
        const int sx = it % GM_STAGES, sa = it % GM_A_STAGES;
        // every lane waits; the warp goes on only if all of them saw the stage
        bool got = mbar_wait(&full[sx], (it / GM_STAGES) & 1, a.status);
        if (got && it >= GM_A_STAGES)
          got = mbar_wait(&empty_a[sa], ((it / GM_A_STAGES) - 1) & 1, a.status);
        if (!__all_sync(MS_FULL, got)) {
          ok = false;
          continue;
        }
        tc_fence_after();
        uint32_t wh[8], wl[8];
        const float2 s2 = make_float2(sc, sc), b2 = make_float2(bi, bi);
        // the weight pair (q, q') -> hi and lo halves: exact s*q + b split
        auto put = [&](int idx, float2 q) {
          const float2 wv = __ffma2_rn(q, s2, b2);            // exact: s*q + b
          const __half2 hi = __floats2half2_rn(wv.x, wv.y);
          const float2 hf = __half22float2(hi);
          const float2 lo = __fadd2_rn(wv, make_float2(-hf.x, -hf.y));
          wh[idx] = *reinterpret_cast<const uint32_t*>(&hi);
          wl[idx] = h2_bits(lo.x, lo.y);
        };
        if (!MIXED || bits == 4) {
          // One LOP3 turns two nibbles into the f16x2 {1024 + q, 1024 + q'}
          // (1024 + 16 q at the odd nibbles), and
          //   s*q + b = s*(1024 + q) + (b - 1024 s) = (s/16)*(1024 + 16 q) + (b - 64 s):
          // one FFMA2 on the converted pair gives the same correctly rounded
          // float as fma(q, s, b) (1024 s and s/16 are exact, and so is the
          // shifted bias for any scale/bias within 2^15 of each other), with
          // the integer work of the unpacking cut to one LOP3 per pair.
          const float2 s_ev = s2, b_ev = make_float2(bi - 1024.f * sc, bi - 1024.f * sc);
          const float so = sc * 0.0625f, bo = bi - 64.f * sc;
          const float2 s_od = make_float2(so, so), b_od = make_float2(bo, bo);
          auto put_h = [&](int idx, uint32_t h, float2 sv, float2 bv) {
            const float2 q = __half22float2(*reinterpret_cast<const __half2*>(&h));
            const float2 wv = __ffma2_rn(q, sv, bv);
            const __half2 hi = __floats2half2_rn(wv.x, wv.y);
            const float2 hf = __half22float2(hi);
            const float2 lo = __fadd2_rn(wv, make_float2(-hf.x, -hf.y));
            wh[idx] = *reinterpret_cast<const uint32_t*>(&hi);
            wl[idx] = h2_bits(lo.x, lo.y);
          };
          const uint2 pw2 = *reinterpret_cast<const uint2*>(sP(sx) + prow * 32 + part * 8);
          const uint32_t words[2] = {pw2.x, pw2.y};
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint32_t u = words[i], us = u >> 8;
            put_h(i * 4 + 0, lop_or(u, 0x000F000Fu), s_ev, b_ev);    // q0, q4
            put_h(i * 4 + 1, lop_or(u, 0x00F000F0u), s_od, b_od);    // q1, q5
            put_h(i * 4 + 2, lop_or(us, 0x000F000Fu), s_ev, b_ev);   // q2, q6
            put_h(i * 4 + 3, lop_or(us, 0x00F000F0u), s_od, b_od);   // q3, q7
          }
        } else {
          const uint8_t* row = sP(sx) + prow * gemm_tile_row_bytes(bits);
          const int kt = it % KT;
          uint32_t r[4];
          if (bits == 2) {
            load_codes<2>(row, part, 0, r);
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) put(i * 4 + q4, code_pair<2>(r, i, q4));
          } else if (bits == 8) {
            load_codes<8>(row, part, 0, r);
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) put(i * 4 + q4, code_pair<8>(r, i, q4));
          } else {
            load_codes<3>(row, part, (24 * kt) & 15, r);
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) put(i * 4 + q4, code_pair<3>(r, i, q4));
          }
        }
        const uint32_t col = TM_A + sa * 64 + part * 8;
        tmem_st8(lane_base + col, wh);
        tmem_st8(lane_base + col + 32, wl);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[sa]);
      }
    }
  } else if (warp >= 20) {
    // ---- epilogue: lanes [32*quarter, +32) of each finished accumulator
    const int quarter = warp & 3;
    const int L = quarter * 32 + lane;
    int ai = 0;
    GemmTile tn = a.tiles[blockIdx.x / n_ft];
    for (int w = blockIdx.x; w < total; w += step, ++ai) {
      const GemmTile t = tn;
      if (w + step < total) tn = a.tiles[(w + step) / n_ft];
      const int f0 = (w % n_ft) * FT;
      const int b = ai & 1;
      const int ntok = (t.rows + 15) & ~15;
      // routing scores of the item's tokens, lane l holding tokens l + 32 i
      float sc4[GM_TOK / 32];
#pragma unroll
      for (int i = 0; i < GM_TOK / 32; ++i)
        sc4[i] = (PHASE == 1 && i * 32 + lane < t.rows) ? a.perm_score[t.row0 + i * 32 + lane] : 0.f;
      if (!__all_sync(MS_FULL, mbar_wait(&acc_full[b], (ai >> 1) & 1, a.status))) break;
      tc_fence_after();
      const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + TM_ACC + b * GM_TOK;
      const uint8_t* blob = a.arena + (long long)(t.slot >= 0 ? t.slot : 0) * a.blob;
      if (PHASE == 0) {
        const bool is_up = lane >= 16;
        const int fg = f0 + 16 * quarter + (lane & 15);     // feature index in d_ff
        const int pos = (fg & ~7) | kperm_pos(fg & 7);      // its k-permuted h column
        const long long boff = MIXED ? a.C.c[item_class<MIXED>(a, t.slot)].off[is_up ? 1 : 0][P_BIAS]
                                     : a.off[is_up ? 1 : 0][3];
        const float bias = (a.model == 1 && t.slot >= 0)
                               ? bf2f(reinterpret_cast<const uint16_t*>(blob + boff)[fg])
                               : 0.f;
        uint16_t* hrow = a.H + (long long)t.row0 * a.ld_out + pos;
        for (int c0 = 0; c0 < ntok; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(lane_base + c0, v);
          float vf[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float x = bfr(__uint_as_float(v[j]));
            if (a.model == 1) x = bfr(x + bias);
            vf[j] = x;
          }
          // gate lane l and up lane l + 16 hold the same feature: the gate
          // lane forms tokens c0..c0+7, the up lane tokens c0+8..c0+15
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float other = __shfl_xor_sync(MS_FULL, is_up ? vf[j] : vf[8 + j], 16);
            const float g = is_up ? other : vf[j];
            const float u = is_up ? vf[8 + j] : other;
            const int m = c0 + (is_up ? 8 : 0) + j;
            const float h = t.slot >= 0 ? g_swiglu(a.model, g, u) : 0.f;
            if (m < t.rows) {
              if (fabsf(h) > F16_MAX) atomicCAS(a.status, 0, ST_E_RANGE);
              hrow[(long long)m * a.ld_out] = __half_as_ushort(__float2half_rn(h));
            }
          }
        }
      } else {
        const int fo = f0 + L;                 // output feature
        const bool f_ok = fo < n_out;
        const long long boff = MIXED ? a.C.c[item_class<MIXED>(a, t.slot)].off[2][P_BIAS] : a.off[2][3];
        const float bias = (a.model == 1 && f_ok && t.slot >= 0)
                               ? bf2f(reinterpret_cast<const uint16_t*>(blob + boff)[fo]) : 0.f;
#pragma unroll
        for (int c0 = 0; c0 < GM_TOK; c0 += 16) {
          if (c0 >= ntok) continue;
          uint32_t v[16];
          tmem_ld16(lane_base + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c0 + j;
            const float score = __shfl_sync(MS_FULL, sc4[m >> 5], m & 31);
            if (m < t.rows && f_ok) {
              float y = bfr(__uint_as_float(v[j]));
              if (a.model == 1) y = bfr(y + bias);
              // (y * scores) is a bf16 product (engine_v3.py:600)
              const uint16_t o = t.slot >= 0 ? f2bf(score * y) : (uint16_t)0;
              a.Y[(long long)(t.row0 + m) * a.ld_out + fo] = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
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
    if (a.resid) {
      // the fused block: residual + the block's bf16 output
      const uint4 hv = *reinterpret_cast<const uint4*>(a.resid + (long long)t * a.d + c * 8);
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = __uint_as_float(hw[q] << 16) + bfr(acc[2 * q]);
        acc[2 * q + 1] = __uint_as_float(hw[q] & 0xffff0000u) + bfr(acc[2 * q + 1]);
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

// ------------------------------------------------- slot-keyed grouping
// ms_expert_mlp on a wide batch (kernels.py:231-252 generalised to many
// tokens): pairs are grouped by the slot they read, groups in ascending slot
// order, each cut into GEMM tiles. Pass 1 counts pairs per slot; pass 2 (one
// CTA) lays the groups out: every thread takes a contiguous range of slots,
// a CTA scan turns the ranges' group/row/tile totals into offsets.
__global__ void __launch_bounds__(256) k_mlp_count(MlpWideArgs a) {
  for (int p = blockIdx.x * 256 + threadIdx.x; p < a.P; p += gridDim.x * 256) {
    int s = a.slots[p];
    if (s < 0 || s >= a.n_slots) {             // its group reads nothing and yields zeros
      s = a.n_slots;
      atomicCAS(a.status, 0, ST_E_INVALID);
    }
    a.keys[p] = s;
    atomicAdd(&a.cnt[s], 1);
  }
}

__device__ __forceinline__ int cta_exclusive_scan(int v, int* s_tmp, int* total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(MS_FULL, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < 8 ? s_tmp[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int u = __shfl_up_sync(MS_FULL, wi, o);
      if (lane >= o) wi += u;
    }
    if (lane < 8) s_tmp[8 + lane] = wi - w;
    if (lane == 7) s_tmp[16] = wi;
  }
  __syncthreads();
  const int ex = s_tmp[8 + warp] + incl - v;
  *total = s_tmp[16];
  __syncthreads();
  return ex;
}

__global__ void __launch_bounds__(256) k_mlp_groups(MlpWideArgs a) {
  __shared__ int s_tmp[32];
  const int nk = a.n_slots + 1;
  const int chunk = (nk + 255) / 256;
  const int k0 = threadIdx.x * chunk, k1 = min(nk, k0 + chunk);
  int ng = 0, nr = 0, nt = 0;
  for (int key = k0; key < k1; ++key) {
    const int c = a.cnt[key];
    if (c) {
      ++ng;
      nr += c;
      nt += (c + GEMM_TILE_ROWS - 1) / GEMM_TILE_ROWS;
    }
  }
  int tot_g, tot_r, tot_t;
  int g = cta_exclusive_scan(ng, s_tmp, &tot_g);
  int row = cta_exclusive_scan(nr, s_tmp, &tot_r);
  int tl = cta_exclusive_scan(nt, s_tmp, &tot_t);
  for (int key = k0; key < k1; ++key) {
    const int c = a.cnt[key];
    if (!c) continue;
    a.cnt[key] = 0;
    a.grp.grp_key[g] = key;
    a.grp.grp_slot[g] = key < a.n_slots ? key : -1;
    a.grp.grp_start[g] = row;
    a.grp.grp_count[g] = c;
    a.grp.map[key] = g;
    a.w.cursor[g] = 0;
    for (int j = 0; j * GEMM_TILE_ROWS < c; ++j, ++tl) {
      if (tl >= a.w.max_tiles) continue;
      GemmTile t;
      t.g = g;
      t.row0 = row + j * GEMM_TILE_ROWS;
      t.rows = min(GEMM_TILE_ROWS, c - j * GEMM_TILE_ROWS);
      t.slot = key < a.n_slots ? key : -1;
      a.w.tiles[tl] = t;
    }
    row += c;
    ++g;
  }
  if (threadIdx.x == 0) {
    *a.grp.n_groups = tot_g;
    *a.w.n_tiles = min(tot_t, a.w.max_tiles);
  }
}

cudaError_t launch_mlp_wide_prep(const MlpWideArgs& a, int sms, cudaStream_t s) {
  k_mlp_count<<<std::max(1, std::min((a.P + 255) / 256, sms * 4)), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_mlp_groups<<<1, 256, 0, s>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------ expert-parallel dispatch
// Pairs are packed destination-major; inside a destination in arrival
// order, which changes nothing in the result (every row is computed on its
// own and returns to pair_pos). Pair p of expert e goes to replica
// p % n_rep(e) of e under a placement table, else to rank e / e_local.
__device__ __forceinline__ int2 ep_dest(const EpPackArgs& a, int p, int e) {
  if (!a.placement) {
    const int r = e / a.e_local;
    return make_int2(r, e - r * a.e_local);
  }
  const int* row = a.placement + (long long)e * (1 + 2 * a.max_rep);
  const int j = p % row[0];
  return make_int2(row[1 + 2 * j], row[2 + 2 * j]);
}

__global__ void __launch_bounds__(256) k_ep_count(EpPackArgs a) {
  const int P = a.T * a.k;
  for (int p = blockIdx.x * 256 + threadIdx.x; p < P; p += gridDim.x * 256)
    atomicAdd(&a.counts[ep_dest(a, p, a.inds[p]).x], 1);
}

__global__ void __launch_bounds__(256) k_ep_pack(EpPackArgs a) {
  __shared__ int s_start[64];
  if (threadIdx.x < 32) {
    int run = 0;
    for (int base = 0; base < a.world; base += 32) {
      const int r = base + threadIdx.x;
      const int c = r < a.world ? a.counts[r] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(MS_FULL, incl, o);
        if ((int)threadIdx.x >= o) incl += u;
      }
      if (r < a.world) s_start[r] = run + incl - c;
      run += __shfl_sync(MS_FULL, incl, 31);
    }
  }
  __syncthreads();
  const int P = a.T * a.k;
  const int warps = gridDim.x * 8;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int chunks = a.d / 8;
  for (int p = gw; p < P; p += warps) {
    int pos = 0;
    if (lane == 0) {
      const int2 ds = ep_dest(a, p, a.inds[p]);
      pos = s_start[ds.x] + atomicAdd(&a.cursor[ds.x], 1);
      a.send_meta[2 * pos] = ds.y;
      a.send_meta[2 * pos + 1] = __float_as_int(bf2f(a.scores[p]));
      a.pair_pos[p] = pos;
    }
    pos = __shfl_sync(MS_FULL, pos, 0);
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)(p / a.k) * a.d);
    uint4* dst = reinterpret_cast<uint4*>(a.send_x + (long long)pos * a.d);
    for (int c = lane; c < chunks; c += 32) dst[c] = __ldg(src + c);
  }
}

cudaError_t launch_ep_pack(const EpPackArgs& a, int sms, cudaStream_t s) {
  const int P = a.T * a.k;
  k_ep_count<<<std::max(1, std::min((P + 255) / 256, sms * 4)), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_ep_pack<<<std::max(1, std::min((P + 7) / 8, sms * 8)), 256, 0, s>>>(a);
  return cudaGetLastError();
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

// Weight codes of one projection across all slots, as bytes
// [n_slots][rows_out][row_bytes]: boxes of box_bytes (one K tile of codes)
// x box_rows rows x 1 slot, unswizzled.
int encode_codes_map(CUtensorMap* m, const void* base, int row_bytes, int rows_out, int n_slots,
                     long long blob, int box_bytes, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)rows_out, (cuuint64_t)n_slots};
  const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)blob};
  const cuuint32_t box[3] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -2;
}

// 4-bit weight rows of one projection across all slots, for the decode
// kernels: dims (innermost first) 128 bytes, rows_out rows (stride
// row_bytes), row_bytes / 128 chunks (stride 128 B), n_slots slots (stride
// blob); boxes of box_rows whole rows, 128-byte swizzled, so a tile lands in
// shared memory as [chunk][row][128 B] with the 16-byte units of row r XORed
// with r mod 8 (bank-conflict-free fragment reads).
int encode_rows_map(CUtensorMap* m, const void* base, int row_bytes, int rows_out, int n_slots,
                    long long blob, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return -1;
  if (row_bytes % 128 || row_bytes / 128 > 256 || box_rows > 256 || rows_out % box_rows) return -3;
  const cuuint64_t dims[4] = {128, (cuuint64_t)rows_out, (cuuint64_t)(row_bytes / 128),
                              (cuuint64_t)n_slots};
  const cuuint64_t strides[3] = {(cuuint64_t)row_bytes, 128, (cuuint64_t)blob};
  const cuuint32_t box[4] = {128, (cuuint32_t)box_rows, (cuuint32_t)(row_bytes / 128), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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

template <int PHASE, bool MIXED>
static cudaError_t launch_gemm_t(const CUtensorMap& tX, const GemmMaps& maps, const GemmArgs& a,
                                 int grid, cudaStream_t s) {
  auto kern = k_gemm<PHASE, MIXED>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_SMEM);
  if (e != cudaSuccess) return e;
  kern<<<grid, GM_THREADS, GM_SMEM, s>>>(tX, maps, a);
  return cudaGetLastError();
}

cudaError_t launch_gemm(int phase, const CUtensorMap& tX, const GemmMaps& maps, const GemmArgs& a,
                        bool mixed, int max_items, int sms, cudaStream_t s) {
  const int grid = std::max(1, std::min(max_items, sms));
  if (phase == 0)
    return mixed ? launch_gemm_t<0, true>(tX, maps, a, grid, s) : launch_gemm_t<0, false>(tX, maps, a, grid, s);
  return mixed ? launch_gemm_t<1, true>(tX, maps, a, grid, s) : launch_gemm_t<1, false>(tX, maps, a, grid, s);
}

}  // namespace ms
