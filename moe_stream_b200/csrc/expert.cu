// K3: 4-bit expert MLP for decode and small batches: the batched replacement
// of the three gather_qmm calls, the SwiGLU and the weighted sum
// (engine_v3.py:588-600, engine_120b.py:130-145; kernels.py:87-186 is the
// reference's own fused attempt).
//
//   k_up   one CTA per (16-row tile of d_ff, group of pairs sharing a slot):
//          gate and up rows for up to 8 tokens per MMA pass, the input
//          dimension split over 8 warps, SwiGLU (or gpt-oss's clamped SwiGLU
//          with the projection biases) in the epilogue; h leaves in the frag
//          layout, ready to be k_down's MMA operand, with per-tile sums.
//   k_down one CTA per (RT row tiles of d_model, group): down rows and bias;
//          the last CTA to finish a row tile then does the weighted combine
//          over each token's k experts in a fixed order (deterministic).
//
// Staging: one thread per CTA issues TMA bulk copies (cp.async.bulk) of the
// tile's weight rows -- each row to a padded shared-memory row, so the MMA
// fragment reads are bank-conflict free -- and of its scales/biases, all
// completing on one mbarrier. A CTA therefore has its whole tile (37-60 KB)
// in flight from its first instructions, whatever its register budget.
// k_down is launched as a programmatic dependent of k_up: its weights are
// copied while k_up is still running, and only the h reads wait.
#include "ms_common.cuh"
#include "frag.cuh"
#include "tma.cuh"
#include "kernels.h"
#include "expert_tile.cuh"

namespace ms {

// Qwen3 shapes (KPW 4): three CTAs per SM, so a batch-1 layer's 384 tiles
// fit one wave; the wider rows of the other shapes keep two.
// TMA: the gate and up rows of the tile come as two tensor-map boxes
// (128-byte swizzled, see encode_rows_map) instead of 32 row copies.
template <int MODEL, int KPW, bool TMA>
__global__ void __launch_bounds__(EX_THREADS, (MODEL == 0 && KPW == 4) ? 3 : 2)
    k_up(ExpArgs A, const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmU) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // swizzled boxes need a 1 KB aligned destination
  uint8_t* smem = smem_raw + (TMA ? ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : 0u);
  pdl_wait();                                   // slots and groups come from the route step
  pdl_trigger();
  const int g = blockIdx.y;
  // the group's metadata in one round trip with the group count (every g
  // of the grid lies inside the group arrays; past n_groups it is unused)
  const int n_groups = *A.grp.n_groups;
  const int slot = A.grp.grp_slot[g];
  const int m = A.grp.grp_count[g], start = A.grp.grp_start[g];
  if (g >= n_groups) return;
  const int rt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int K = A.geo.d_model, G = K / 64, F = A.geo.d_ff, GF = F / 64;
  const int k = A.geo.top_k;
  const int row_bytes = K / 2;
  const int stride = TMA ? 16 * 128 : UpSmem::stride(K);   // chunk stride when swizzled
  const int a_bytes = TMA ? 16 * row_bytes : UpSmem::a_bytes(K);
  const int kg0 = min(G, warp * KPW), kg1 = min(G, kg0 + KPW);

  uint8_t* sA[2] = {smem, smem + a_bytes};
  uint16_t* sSB = reinterpret_cast<uint16_t*>(smem + 2 * a_bytes);
  const int sbn = 16 * G;                       // elements per staged [16][G] block
  float* red = reinterpret_cast<float*>(smem + 2 * a_bytes + 4 * UpSmem::sb_bytes(G));
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + EX_WARPS * 2 * 4 * 32);

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  if (warp == 0 && slot >= 0) {
    // warp 0 issues the tile's 36 copies, one or two per lane: gate rows
    // 0..15 and up rows 0..15, then the gate and up scales and biases
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
      mbar_expect_tx(bar, 2u * 16u * row_bytes + 4u * UpSmem::sb_bytes(G));
    }
    __syncwarp();
    const uint64_t pol = l2_evict_first();     // the weights stream through L2
    if (TMA) {
      if (lane == 0) tma_load_4d_hint(sA[0], &tmG, 0, rt * 16, 0, slot, bar, pol);
      if (lane == 1) tma_load_4d_hint(sA[1], &tmU, 0, rt * 16, 0, slot, bar, pol);
    } else {
      const int p = lane >> 4, r = lane & 15;
      bulk_g2s_hint(sA[p] + r * stride, blob + A.geo.off[p][0] + (long long)(rt * 16 + r) * row_bytes,
                    row_bytes, bar, pol);
    }
    if (lane < 4)
      bulk_g2s_hint(sSB + lane * sbn, blob + A.geo.off[lane >> 1][1 + (lane & 1)] + (long long)rt * 16 * G * 2,
                    UpSmem::sb_bytes(G), bar, pol);
  }
  __syncthreads();
  bool ok = true, waited = false;

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = A.grp.grp_pairs + start + n0;
    const int nn = min(8, m - n0);
    const int pb = (g4 < nn) ? pairs[g4] : -1;
    const int pc0 = (2 * c < nn) ? pairs[2 * c] : -1;
    const int pc1 = (2 * c + 1 < nn) ? pairs[2 * c + 1] : -1;
    const __half* fb = pb >= 0 ? A.xfrag + (long long)(pb / k) * G * 64 : nullptr;
    const float* s0 = pc0 >= 0 ? A.xsum + (long long)(pc0 / k) * G * 2 : nullptr;
    const float* s1 = pc1 >= 0 ? A.xsum + (long long)(pc1 / k) * G * 2 : nullptr;
    // the activations come in while the tile's weights are still in flight
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
      tile_dot_regs<KPW, TMA>(tg, sA[0], stride, G, kg0, kg1, g4, c, sSB, sSB + sbn, b0, b1, v0, v1);
      tile_dot_regs<KPW, TMA>(tu, sA[1], stride, G, kg0, kg1, g4, c, sSB + 2 * sbn, sSB + 3 * sbn, b0,
                              b1, v0, v1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      red[((warp * 2 + 0) * 4 + i) * 32 + lane] = tg[i];
      red[((warp * 2 + 1) * 4 + i) * 32 + lane] = tu[i];
    }
    __syncthreads();
    // epilogue: thread t < 128 owns (row r, column col) of the tile
    if (threadIdx.x < 128) {
      const int r = threadIdx.x & 15, col = threadIdx.x >> 4;
      const int src = (r & 7) * 4 + (col >> 1), e = ((r >> 3) << 1) | (col & 1);
      const int row = rt * 16 + r;
      float hh_f = 0.f, hsc_f = 0.f;
      const int pc = col < nn ? pairs[col] : -1;
      if (col < nn) {
        __half hsc = __float2half(0.f);
        if (slot >= 0 && ok) {
          float gv = 0.f, uv = 0.f;
#pragma unroll
          for (int w = 0; w < EX_WARPS; ++w) {
            gv += red[((w * 2 + 0) * 4 + e) * 32 + src];
            uv += red[((w * 2 + 1) * 4 + e) * 32 + src];
          }
          gv = bfr(gv);                          // gather_qmm outputs are bf16
          uv = bfr(uv);
          float h;
          if (MODEL == 1) {
            const uint16_t* bgp = reinterpret_cast<const uint16_t*>(blob + A.geo.off[0][3]);
            const uint16_t* bup = reinterpret_cast<const uint16_t*>(blob + A.geo.off[1][3]);
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
        A.hfrag[frag_off(pc, GF, row)] = hsc;
      }
      // sums over the 16 rows of the tile, per column (16 consecutive threads)
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        hh_f += __shfl_xor_sync(MS_FULL, hh_f, o);
        hsc_f += __shfl_xor_sync(MS_FULL, hsc_f, o);
      }
      if (r == 0 && col < nn)
        *reinterpret_cast<float2*>(A.hpart + ((long long)pc * (F / 16) + rt) * 2) =
            make_float2(hh_f, hsc_f);
    }
    __syncthreads();
  }
}


// Largest cluster of k_down's one-token combine (the portable cluster size).
constexpr int CL_MAX = 8;

// TMA: the RT*16 down rows of the unit come as one tensor-map box.
// CL (one token, launched as clusters of the k CTAs that share a row tile,
// one per expert): each CTA writes its rows into the shared memory of the
// cluster's first CTA, which combines them after one cluster barrier --
// instead of the global partials, fence and arrival counter of the general
// path. Same values, same j order.
template <int MODEL, int KPW, int RT, bool TMA, bool CL>
__global__ void __launch_bounds__(EX_THREADS) k_down(ExpArgs A, const __grid_constant__ CUtensorMap tmD) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + (TMA ? ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : 0u);
  // the route step finished before k_up started, so the groups and the
  // filled slots can be read now; only h (k_up's output) needs pdl_wait
  const int g = blockIdx.y;
  const int n_groups = *A.grp.n_groups;
  // (CL: a CTA past the groups -- never launched so by the block call --
  // still reaches the cluster barrier, with no slot and no pairs)
  const bool live = g < n_groups;
  const int slot = live ? A.grp.grp_slot[g] : -1;   // one round trip, as in k_up
  const int m = live ? A.grp.grp_count[g] : 0, start = A.grp.grp_start[g];
  // CL: the cluster's y extent is the token's k experts, one group each
  __shared__ float s_y[CL ? CL_MAX : 1][RT * 16];
  if (!CL && !live) {
    pdl_wait();
    return;
  }
  const bool cl_ok = !CL || n_groups == (int)gridDim.y;
  constexpr int WPT = EX_WARPS / RT;            // warps per row tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, c = lane & 3;
  const int sub = warp / WPT, wk = warp % WPT;
  const int rt = blockIdx.x * RT + sub;
  const int K = A.geo.d_ff, G = K / 64, D = A.geo.d_model;
  const int k = A.geo.top_k;
  const int row_bytes = K / 2;
  const int stride = TMA ? RT * 16 * 128 : DownSmem::stride(K);   // chunk stride when swizzled
  const int a_bytes = TMA ? RT * 16 * row_bytes : DownSmem::a_bytes(K, RT);
  const int kg0 = min(G, wk * KPW), kg1 = min(G, kg0 + KPW);
  const int nt_ff = K / 16;

  uint8_t* sA = smem;
  uint16_t* sS = reinterpret_cast<uint16_t*>(smem + a_bytes);
  uint16_t* sB = sS + RT * 16 * G;
  float* red = reinterpret_cast<float*>(smem + a_bytes + 2 * DownSmem::sb_bytes(G, RT));
  float* s_sums = red + EX_WARPS * 4 * 32;      // [8][G][2]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_sums + 8 * G * 2);
  __shared__ int s_last[RT];

  const uint8_t* blob = A.arena + (long long)(slot < 0 ? 0 : slot) * A.geo.blob;
  if (warp == 0 && slot >= 0) {
    // warp 0 issues the tile's copies, about one per lane: the RT*16 rows,
    // then the scales and biases
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
      mbar_expect_tx(bar, (unsigned)(RT * 16 * row_bytes + 2 * DownSmem::sb_bytes(G, RT)));
    }
    __syncwarp();
    const uint64_t pol = l2_evict_first();     // the weights stream through L2
    if (TMA) {
      if (lane == 0) tma_load_4d_hint(sA, &tmD, 0, blockIdx.x * RT * 16, 0, slot, bar, pol);
    } else {
      const uint8_t* W = blob + A.geo.off[2][0] + (long long)blockIdx.x * RT * 16 * row_bytes;
      for (int r = lane; r < RT * 16; r += 32)
        bulk_g2s_hint(sA + r * stride, W + (long long)r * row_bytes, row_bytes, bar, pol);
    }
    if (lane < 2)
      bulk_g2s_hint(lane ? sB : sS, blob + A.geo.off[2][1 + lane] + (long long)blockIdx.x * RT * 16 * G * 2,
                    DownSmem::sb_bytes(G, RT), bar, pol);
  }
  // the first pass's pairs come from the route step, so they are read
  // before the wait for k_up: after it, h is one round trip away, not two
  __shared__ int s_pairs[8];
  if (threadIdx.x < 8) s_pairs[threadIdx.x] = (int)threadIdx.x < m ? A.grp.grp_pairs[start + threadIdx.x] : -1;
  __syncthreads();                              // (also the mbarrier's init)
  pdl_wait();                                   // h and its sums come from k_up
  bool ok = true, waited = false;

  for (int n0 = 0; n0 < m; n0 += 8) {
    const int* pairs = s_pairs;
    const int nn = min(8, m - n0);
    const int pb = (g4 < nn) ? pairs[g4] : -1;
    // h fragments requested before the sums' round trip, so the two overlap
    uint4 b0[KPW], b1[KPW];
    load_frags<KPW>(b0, b1, (pb >= 0 && slot >= 0) ? A.hfrag + (long long)pb * G * 64 : nullptr,
                       kg0, kg1, c);
    // per-group sums of h for this pass's columns: 4 row-tile partials each
    for (int i = threadIdx.x; i < nn * G; i += EX_THREADS) {
      const int col = i / G, kg = i % G;
      const float4* hp4 = reinterpret_cast<const float4*>(
          A.hpart + ((long long)pairs[col] * nt_ff + kg * 4) * 2);
      const float4 a = hp4[0], b = hp4[1];
      s_sums[(col * G + kg) * 2] = (a.x + a.z) + (b.x + b.z);
      s_sums[(col * G + kg) * 2 + 1] = (a.y + a.w) + (b.y + b.w);
    }
    // the weights (copied since the kernel's start) after h was requested
    if (!waited) {
      if (slot >= 0) ok = mbar_wait(bar, 0, A.status);
      waited = true;
    }
    __syncthreads();
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0 && ok && kg0 < kg1) {
      tile_dot_frags<KPW, TMA>(tot, sA + sub * 16 * (TMA ? 128 : stride), stride, G, kg0, kg1, g4, c,
                         sS + sub * 16 * G, sB + sub * 16 * G, b0, b1,
                         (2 * c < nn) ? s_sums + (2 * c) * G * 2 : nullptr,
                         (2 * c + 1 < nn) ? s_sums + (2 * c + 1) * G * 2 : nullptr);
    }
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
          v = bfr(v);                            // gather_qmm output
          if (MODEL == 1 && slot >= 0) {
            const uint16_t* bdp = reinterpret_cast<const uint16_t*>(blob + A.geo.off[2][3]);
            v = bfr(v + bf2f(bdp[row]));
          }
          v = (slot >= 0 && ok) ? v : 0.f;
          if (CL) {
            const int j = pairs[col];            // one token: the pair is its j
            if (cl_ok && j >= 0 && j < (int)gridDim.y)
              st_cluster_f32(cluster_map(&s_y[j][row - blockIdx.x * RT * 16], 0), v);
          } else {
            A.ypart[(long long)pairs[col] * D + row] = v;
          }
        }
      }
    }
    __syncthreads();
    if (n0 + 8 < m) {                           // the next pass's pairs
      if (threadIdx.x < 8)
        s_pairs[threadIdx.x] = n0 + 8 + (int)threadIdx.x < m ? A.grp.grp_pairs[start + n0 + 8 + threadIdx.x] : -1;
      __syncthreads();
    }
  }

  // the next kernel in the stream (the next layer's route step) may launch
  // while the arrivals and combines finish; it waits for this grid itself
  pdl_trigger();
  if (CL) {
    // every CTA of the cluster has written its rows into the first one's
    // s_y; that CTA adds them in j order
    cluster_sync();
    if (cluster_rank() != 0) return;
    if (!cl_ok && threadIdx.x == 0) atomicCAS(A.status, 0, ST_E_INVALID);
    for (int i = threadIdx.x; i < RT * 16; i += EX_THREADS) {
      const int row = blockIdx.x * RT * 16 + i;
      float acc = 0.f;
      for (int j = 0; j < (int)gridDim.y; ++j)
        acc += cl_ok ? bfr(A.scores[j] * s_y[j][i]) : 0.f;   // engine_v3.py:600
      A.y[row] = A.resid ? f2bf(bf2f(A.resid[row]) + bfr(acc)) : f2bf(acc);
    }
    return;
  }
  // ---- arrival: the last CTA of a row tile combines all tokens' k parts
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
        // (y * scores) is a bf16 product before the sum (engine_v3.py:600)
        acc += bfr(A.scores[p] * __ldcg(A.ypart + p * D + row));
      }
      // the block's bf16 output; the fused block adds it to the residual
      A.y[(long long)t * D + row] =
          A.resid ? f2bf(bf2f(A.resid[(long long)t * D + row]) + bfr(acc)) : f2bf(acc);
    }
    if (threadIdx.x == 0) A.cnt[rtile] = 0u;
  }
}

// cluster_y > 0: clusters of (1, cluster_y, 1) CTAs
template <typename Kern, typename... Args>
static cudaError_t launch_pdl(Kern kern, dim3 grid, int smem, cudaStream_t s, int cluster_y,
                              const Args&... args) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(EX_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_y > 0) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = cluster_y;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

bool expert_shape_ok(int model, int d_model, int d_ff) {
  if (d_model <= 0 || d_ff <= 0 || d_model % 64 || d_ff % 64) return false;
  // gpt-oss: 6 quantisation groups per warp, at most 48 groups each way;
  // Qwen3 and other shapes: at most 64 groups each way
  const int G = d_model / 64, GF = d_ff / 64;
  return model == 1 ? (G <= 48 && GF <= 48) : (G <= 64 && GF <= 64);
}

// The Qwen3 kernels: 2048/768 (up 32 groups, 4 per warp; down 12 groups, 2
// row tiles per CTA with 4 warps x 3 groups each).
static bool qwen3_shape(int model, int d_model, int d_ff) {
  return model == 0 && d_model / 64 <= 32 && d_ff / 64 <= 12 && (d_model / 16) % 2 == 0;
}

int expert_down_rows(int model, int d_model, int d_ff) {
  return qwen3_shape(model, d_model, d_ff) ? 32 : 16;
}

template <int MODEL, int KPW_UP, int KPW_DN, int RT>
static cudaError_t launch_pair(const ExpArgs& a, int max_groups, cudaStream_t s, const CUtensorMap* maps) {
  const int K = a.geo.d_model, F = a.geo.d_ff;
  const dim3 gu(F / 16, max_groups), gd(K / (16 * RT), max_groups);
  const int su = UpSmem::total(K, maps != nullptr), sd = DownSmem::total(F, RT, maps != nullptr);
  // one-token block call: the k CTAs of a row tile combine as a cluster
  const int cl = (a.cl_k > 0 && a.cl_k <= CL_MAX && max_groups == a.cl_k) ? a.cl_k : 0;
  cudaError_t e;
  if (maps) {
    e = launch_pdl(k_up<MODEL, KPW_UP, true>, gu, su, s, 0, a, maps[0], maps[1]);
    if (e != cudaSuccess) return e;
    if (cl) return launch_pdl(k_down<MODEL, KPW_DN, RT, true, true>, gd, sd, s, cl, a, maps[2]);
    return launch_pdl(k_down<MODEL, KPW_DN, RT, true, false>, gd, sd, s, 0, a, maps[2]);
  }
  CUtensorMap none{};
  e = launch_pdl(k_up<MODEL, KPW_UP, false>, gu, su, s, 0, a, none, none);
  if (e != cudaSuccess) return e;
  if (cl) return launch_pdl(k_down<MODEL, KPW_DN, RT, false, true>, gd, sd, s, cl, a, none);
  return launch_pdl(k_down<MODEL, KPW_DN, RT, false, false>, gd, sd, s, 0, a, none);
}

cudaError_t launch_expert(const ExpArgs& a, int max_groups, cudaStream_t s, const CUtensorMap* maps) {
  if (max_groups <= 0) return cudaSuccess;
  if (!expert_shape_ok(a.geo.model, a.geo.d_model, a.geo.d_ff)) return cudaErrorInvalidValue;
  cudaError_t e;
  if (a.geo.model == 1) {
    // gpt-oss 2880/2880: 45 groups both ways, 6 per warp (rows of 1440 B
    // are not whole 128-byte chunks: row copies)
    e = launch_pair<1, 6, 6, 1>(a, max_groups, s, nullptr);
  } else if (qwen3_shape(a.geo.model, a.geo.d_model, a.geo.d_ff)) {
    e = launch_pair<0, 4, 3, 2>(a, max_groups, s, maps);
  } else {
    // other shapes: up to 64 groups, 8 per warp
    e = launch_pair<0, 8, 8, 1>(a, max_groups, s, maps);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ms
