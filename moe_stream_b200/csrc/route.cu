// K1: router + slot-table step, one launch per MoE block call.
//
// Phase 1 (every CTA): router logits x . W_r^T (+ bias) for this layer and
// for each prefetch target layer (engine_v3.py:507-514), one warp per router
// row, fp32 accumulation; and the frag-layout copy of x that the expert
// kernels read.
// Phase 2 (the last CTA to finish phase 1, picked by an arrival counter; no
// CTA ever waits on another): per-token softmax / top-k in the reference's
// bf16 rounding order, the sorted unions of routed and predicted experts,
// the device slot-table step (prefetch each target layer, then acquire this
// layer's experts, engine_v3.py:522-548) and the grouping of token/expert
// pairs by slot for the expert kernels.
#include "ms_common.cuh"
#include "pool_table.cuh"
#include "groups.cuh"
#include "frag.cuh"
#include "tma.cuh"
#include "kernels.h"

namespace ms {

constexpr int MAX_E = 256;
constexpr int RT_THREADS = 256;
constexpr int SMALL_P = 256;     // pairs grouped inside one warp up to this many

__device__ __forceinline__ uint32_t mono_key(uint16_t b) {
  // order-preserving map of bf16 bits to unsigned
  return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(MS_FULL, v, o);
  return v;
}

// top-k of vals[0..E) (bf16 bit patterns, one warp): descending, exact ties
// to the lower index. A candidate is the 32-bit key (value << 16 | ~index),
// so one redux.sync per round finds the winner. Writes out[0..k).
// PER candidates per lane (E <= 32 * PER); every winner search takes a max
// over them, so the decode-sized E <= 128 uses PER = 4.
template <int PER>
__device__ void warp_topk_n(const uint16_t* vals, int E, int k, int* out, int lane) {
  uint32_t key[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    key[i] = (e < E) ? ((mono_key(vals[e]) << 16) | (uint32_t)(0xffff - e)) : 0u;
  }
  for (int r = 0; r < k; ++r) {
    uint32_t best = 0u;
#pragma unroll
    for (int i = 0; i < PER; ++i) best = max(best, key[i]);
    const uint32_t w = __reduce_max_sync(MS_FULL, best);
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (key[i] == w) key[i] = 0u;          // keys are unique (they carry the index)
    if (lane == 0) out[r] = 0xffff - (int)(w & 0xffffu);
  }
  __syncwarp();
}

__device__ void warp_topk(const uint16_t* vals, int E, int k, int* out, int lane) {
  if (E <= 128) warp_topk_n<4>(vals, E, k, out, lane);
  else warp_topk_n<MAX_E / 32>(vals, E, k, out, lane);
}

// Routes one token from its fp32 logits lg[0..E) (one warp; vals/sel are the
// warp's scratch). Leaves the selected experts in sel[0..k) and returns lane
// j's score for j < k (0 elsewhere).
__device__ __forceinline__ float route_token(const float* lg, const Geo& geo, uint16_t* vals, int* sel,
                                             int lane) {
  const int E = geo.n_experts, k = geo.top_k;
  // logits rounded to bf16 as the Linear's output (engine_v3.py:468)
  float lmax = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    const uint16_t b = f2bf(lg[e]);
    vals[e] = b;
    lmax = fmaxf(lmax, bf2f(b));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(MS_FULL, lmax, o));
  __syncwarp();
  float sc = 0.f;
  if (geo.model == 0) {
    // softmax(precise) over all experts, bf16 out (engine_v3.py:468)
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) sum += expf(bf2f(vals[e]) - lmax);
    sum = warp_sum(sum);
    for (int e = lane; e < E; e += 32) vals[e] = f2bf(expf(bf2f(vals[e]) - lmax) / sum);
    __syncwarp();
    warp_topk(vals, E, k, sel, lane);
    // scores of the k selected, renormalised (engine_v3.py:469-472)
    const float p = (lane < k) ? bf2f(vals[sel[lane]]) : 0.f;
    const float den = bfr(warp_sum(p));
    sc = geo.norm_topk ? bfr(p / den) : p;
  } else {
    // gpt-oss: top-k of the logits, softmax over the k (engine_120b.py:67-70)
    warp_topk(vals, E, k, sel, lane);
    const float m = bf2f(vals[sel[0]]);     // descending: the first is the max
    const float ex = (lane < k) ? expf(bf2f(vals[sel[lane]]) - m) : 0.f;
    sc = bfr(ex / warp_sum(ex));
  }
  return sc;
}

// Speculation for one token: top-(k*widen) of a target layer's raw logits
// lg[0..E) into sel[0..kp) (engine_v3.py:476-483, 509-514).
__device__ __forceinline__ void predict_token(const float* lg, int E, int kp, uint16_t* vals, int* sel,
                                              int lane) {
  for (int e = lane; e < E; e += 32) vals[e] = f2bf(lg[e]);
  __syncwarp();
  warp_topk(vals, E, kp, sel, lane);
}

// The slot-table step of one block call, by one warp: register every key,
// load all their state in one round, then ExpertPool.prefetch for each
// target layer and acquire of this layer (engine_v3.py:522-526, 548).
// np.unique makes both lists sorted and distinct; so are s_pred / s_acq.
__device__ __forceinline__ void warp_pool_step(const RouteArgs& A, int (*s_pred)[MAX_E],
                                               const int* s_n_pred, const int* s_acq, int n_acq,
                                               int* s_slots, int* s_waits, OpCtx* s_op, KeyCache* s_kc,
                                               int (*s_ci)[MAX_E], int lane) {
  const DevTable& Tb = A.tab;
  if (A.n_pred <= 1) {
    // the common case (no key needs a slot) in one round of loads
    int* keys = s_ci[0];                       // [0, np): predicted keys, [32, 32 + na): acquired
    const int np_ = A.n_pred ? s_n_pred[0] : 0;
    for (int i = lane; i < np_ && i < 32; i += 32) keys[i] = A.pred_layer[0] * Tb.n_experts + s_pred[0][i];
    for (int i = lane; i < n_acq && i < 32; i += 32) keys[32 + i] = A.layer * Tb.n_experts + s_acq[i];
    __syncwarp();
    if (warp_table_fast(Tb, keys, np_, keys + 32, n_acq, s_slots, lane)) {
      if (A.pf_ring && lane == 0) *A.pf_cnt = 0;
      __syncwarp();
      return;
    }
  }
  op_load(Tb, s_op, lane);
  if (lane == 0) s_kc->n = 0;
  __syncwarp();
  Req rp[MS_MAX_DEPTHS], ra;
  for (int dd = 0; dd < A.n_pred; ++dd) {
    rp[dd].ci = s_ci[dd];
    kc_add(Tb, s_kc, rp[dd], A.pred_layer[dd], s_pred[dd], s_n_pred[dd], false, lane);
  }
  ra.ci = s_ci[MS_MAX_DEPTHS];
  kc_add(Tb, s_kc, ra, A.layer, s_acq, n_acq, false, lane);
  kc_load(Tb, s_op, s_kc, lane);
  for (int dd = 0; dd < A.n_pred; ++dd) warp_prefetch(Tb, s_op, s_kc, rp[dd], lane);
  __syncwarp();
  if (lane == 0) s_op->n_fill_pf = s_op->n_fill;
  __syncwarp();
  warp_acquire(Tb, s_op, s_kc, ra, s_slots, s_waits, lane);
  op_store(Tb, s_op, lane);
  if (A.pf_ring) {
    // the prefetch fills leave the per-call list for this call's ring half,
    // which the side-stream fill reads while later calls rewrite the list
    const int n = min(s_op->n_fill_pf, Tb.max_fills);
    for (int i = lane; i < n; i += 32) A.pf_ring[i] = Tb.fills[i];
    if (lane == 0) *A.pf_cnt = n;
    __syncwarp();
  }
}

__global__ void __launch_bounds__(RT_THREADS) k_route_step(RouteArgs A) {
  const int E = A.geo.n_experts, d = A.geo.d_model, T = A.T, k = A.geo.top_k;
  const int rows = E * (1 + A.n_pred);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps_total = gridDim.x * (RT_THREADS / 32);
  const int gw = blockIdx.x * (RT_THREADS / 32) + warp;
  const int nchunk = d / 8;  // 16-byte chunks of a row

  // a programmatic dependent of the previous kernel in the stream (the
  // previous layer's k_down triggers once its dot products are done): wait
  // for that grid before touching anything
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // fused post-attention norm (A.norm_w): the block input is
  // rms_norm(h) * w of the residual stream h = A.x, computed by every CTA
  // into shared memory, as mlx's fast rms_norm rounds it: bf16(bf16(h * r) * w)
  // with r = 1/sqrt(mean(h^2) + eps)
  extern __shared__ __align__(16) uint16_t s_xn[];   // [T][d] when A.norm_w
  const uint16_t* xin = A.x;
  if (A.norm_w) {
    __shared__ float s_red[32];
    for (int t = 0; t < T; ++t) {
      const uint16_t* h = A.x + (long long)t * d;
      const float rn = cta_rms_factor(h, d, A.norm_eps, s_red);
      for (int i = threadIdx.x; i < d; i += RT_THREADS)
        s_xn[t * d + i] = f2bf(bfr(bf2f(h[i]) * rn) * bf2f(A.norm_w[i]));
    }
    __syncthreads();
    xin = s_xn;
  }
  // ---------------------------------------------------------------- phase 1
  for (int r = gw; r < rows; r += nwarps_total) {
    const int which = r / E, e = r % E;
    const uint16_t* w = (which == 0 ? A.w_r : A.w_p[which - 1]) + (long long)e * d;
    const uint16_t* b = (which == 0 ? A.b_r : A.b_p[which - 1]);
    const float bias = b ? bf2f(b[e]) : 0.f;
    for (int t = 0; t < T; ++t) {
      const uint16_t* x = xin + (long long)t * d;
      float acc = 0.f;
#pragma unroll 8
      for (int ch = lane; ch < nchunk; ch += 32) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + ch);
        const uint4 xv = A.norm_w ? reinterpret_cast<const uint4*>(x)[ch]
                                  : __ldg(reinterpret_cast<const uint4*>(x) + ch);
        const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc = fmaf(__uint_as_float(wa[q] << 16), __uint_as_float(xa[q] << 16), acc);
          acc = fmaf(__uint_as_float(wa[q] & 0xffff0000u), __uint_as_float(xa[q] & 0xffff0000u), acc);
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) A.logits[(long long)t * rows + r] = acc + bias;
    }
  }
  if (A.xfrag)
    frag_write_rows(xin, T, d, A.xfrag, A.xsum, blockIdx.x * RT_THREADS + threadIdx.x,
                    gridDim.x * RT_THREADS, &A.tab.ctr->status);

  // ----------------------------------------------------- arrival: last CTA
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(A.ticket, 1u);
    s_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---------------------------------------------------------------- phase 2
  __shared__ unsigned s_acq_mask[MAX_E / 32];
  __shared__ unsigned s_pred_mask[MS_MAX_DEPTHS][MAX_E / 32];
  __shared__ uint16_t s_vals[RT_THREADS / 32][MAX_E];
  __shared__ int s_sel[RT_THREADS / 32][MAX_E];
  __shared__ int s_acq[MAX_E];
  __shared__ int s_pred[MS_MAX_DEPTHS][MAX_E];
  __shared__ int s_n_pred[MS_MAX_DEPTHS];
  __shared__ int s_slots[MAX_E];
  __shared__ int s_waits[MAX_E];
  __shared__ int s_cnt[MAX_E], s_run[MAX_E];
  __shared__ int s_rank[MAX_E];
  __shared__ int s_inds[SMALL_P];
  __shared__ int s_n_acq;
  __shared__ OpCtx s_op;
  __shared__ KeyCache s_kc;
  __shared__ int s_ci[MS_MAX_DEPTHS + 1][MAX_E];

  for (int i = threadIdx.x; i < MAX_E / 32; i += RT_THREADS) {
    s_acq_mask[i] = 0;
    for (int dd = 0; dd < MS_MAX_DEPTHS; ++dd) s_pred_mask[dd][i] = 0;
  }
  __syncthreads();

  const int kp = A.kp;
  const bool small = T * k <= SMALL_P;
  // one token: its k experts and each speculation's kp experts are distinct,
  // so the routing warps sort them into the acquire / prefetch lists
  // directly (a lane's rank = how many of the selection are smaller), and a
  // lane's rank is its expert's group -- no masks, no list building
  const bool one = T == 1 && k <= 32 && kp <= 32;
  __shared__ int s_rank1[32];
  // one task per (token, router): task part 0 routes the token, part d >= 1
  // is the speculation of prefetch depth d-1 -- top-(k*widen) of the target
  // layer's raw logits (engine_v3.py:476-483, 509-514). Tasks go to warps
  // round-robin, so a token's routing and its predictions run side by side.
  const int parts = 1 + A.n_pred;
  for (int task = warp; task < T * parts; task += RT_THREADS / 32) {
    const int t = task / parts, part = task % parts;
    const float* lg = A.logits + (long long)t * rows;
    uint16_t* vals = s_vals[warp];
    int* sel = s_sel[warp];
    if (part == 0) {
      const float sc = route_token(lg, A.geo, vals, sel, lane);
      const int e = lane < k ? sel[lane] : 0x7fffffff;
      if (lane < k) {
        A.inds[t * k + lane] = e;
        A.scores[t * k + lane] = f2bf(sc);
        A.scores_f[t * k + lane] = sc;
        if (small) s_inds[t * k + lane] = e;
        if (!one) atomicOr(&s_acq_mask[e >> 5], 1u << (e & 31));
      }
      if (one) {
        int rank = 0;
        for (int j = 0; j < k; ++j) rank += __shfl_sync(MS_FULL, e, j) < e;
        if (lane < k) {
          s_acq[rank] = e;
          s_rank1[lane] = rank;
        }
      }
    } else {
      const int dd = part - 1;
      predict_token(lg + part * E, E, kp, vals, sel, lane);
      if (one) {
        const int e = lane < kp ? sel[lane] : 0x7fffffff;
        int rank = 0;
        for (int j = 0; j < kp; ++j) rank += __shfl_sync(MS_FULL, e, j) < e;
        if (lane < kp) {
          s_pred[dd][rank] = e;
          if (dd == 0 && A.pred_out) A.pred_out[lane] = e;
        }
      } else {
        for (int j = lane; j < kp; j += 32) {
          atomicOr(&s_pred_mask[dd][sel[j] >> 5], 1u << (sel[j] & 31));
          if (dd == 0 && A.pred_out) A.pred_out[t * kp + j] = sel[j];
        }
      }
    }
    __syncwarp();
  }
  __syncthreads();

  if (warp == 0) {
    int n_acq;
    if (one) {
      n_acq = k;
      if (lane == 0) {
        s_n_acq = k;
        for (int dd = 0; dd < A.n_pred; ++dd) s_n_pred[dd] = kp;
      }
    } else {
      n_acq = warp_small_mask_to_list(s_acq_mask, (E + 31) / 32, s_acq, lane);
      if (lane == 0) s_n_acq = n_acq;
      for (int dd = 0; dd < A.n_pred; ++dd) {
        const int n = warp_small_mask_to_list(s_pred_mask[dd], (E + 31) / 32, s_pred[dd], lane);
        if (lane == 0) s_n_pred[dd] = n;
      }
    }
    __syncwarp();
    if (A.do_pool) {
      warp_pool_step(A, s_pred, s_n_pred, s_acq, n_acq, s_slots, s_waits, &s_op, &s_kc, s_ci, lane);
    } else {
      for (int i = lane; i < n_acq; i += 32) s_slots[i] = -1;
    }
    __syncwarp();
    if (A.do_groups && one) {
      // one token: its k experts are distinct, so group g is the g-th
      // smallest of them with that one pair; g is the expert's rank
      if (lane < k) {
        const int e = s_inds[lane];
        const int g = s_rank1[lane];
        A.grp.grp_start[g] = g;
        A.grp.grp_count[g] = 1;
        A.grp.grp_key[g] = e;
        A.grp.grp_slot[g] = s_slots[g];
        A.grp.grp_pairs[g] = lane;
        if (A.pair_slot) A.pair_slot[lane] = s_slots[g];
      }
      if (lane == 0) *A.grp.n_groups = k;
    } else if (A.do_groups && small) {
      // pairs grouped by expert in one warp: everything is computed in
      // shared memory first and written out once at the end
      const int P = T * k;
      for (int g = lane; g < n_acq; g += 32) {
        s_rank[s_acq[g]] = g;
        s_cnt[g] = 0;
      }
      __syncwarp();
      for (int p = lane; p < P; p += 32) atomicAdd(&s_cnt[s_rank[s_inds[p]]], 1);
      __syncwarp();
      int run = 0;
      for (int base = 0; base < n_acq; base += 32) {
        const int g = base + lane;
        const int cnt = (g < n_acq) ? s_cnt[g] : 0;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(MS_FULL, incl, o);
          if (lane >= o) incl += v;
        }
        if (g < n_acq) s_run[g] = run + incl - cnt;
        run += __shfl_sync(MS_FULL, incl, 31);
      }
      __syncwarp();
      for (int g = lane; g < n_acq; g += 32) s_waits[g] = s_run[g];   // group starts
      for (int base = 0; base < P; base += 32) {
        const int p = base + lane;
        const int g = (p < P) ? s_rank[s_inds[p]] : -1;
        const unsigned same = __match_any_sync(MS_FULL, g);
        const int rank = __popc(same & ((1u << lane) - 1u));
        __syncwarp();
        if (g >= 0) {
          s_sel[0][s_run[g] + rank] = p;         // stable: ascending pair order
          if (rank == 0) s_run[g] += __popc(same);
        }
        __syncwarp();
      }
      for (int g = lane; g < n_acq; g += 32) {
        A.grp.grp_start[g] = s_waits[g];
        A.grp.grp_count[g] = s_cnt[g];
        A.grp.grp_key[g] = s_acq[g];
        A.grp.grp_slot[g] = s_slots[g];
      }
      for (int i = lane; i < P; i += 32) {
        A.grp.grp_pairs[i] = s_sel[0][i];
        if (A.pair_slot) A.pair_slot[i] = s_slots[s_rank[s_inds[i]]];
      }
      if (lane == 0) *A.grp.n_groups = n_acq;
    }
  }
  __syncthreads();

  if (A.do_groups && !small) {
    cta_build_groups(A.inds, T * k, s_acq, s_n_acq, A.grp, s_cnt, s_run,
                     [&](int g) { return s_slots[g]; });
    if (A.pair_slot)
      for (int p = threadIdx.x; p < T * k; p += RT_THREADS)
        A.pair_slot[p] = s_slots[A.grp.map[A.inds[p]]];
  }
  if (threadIdx.x == 0) *A.ticket = 0u;
}

// ------------------------------------------------------------ wide batches
// K1 for prefill and large batches. Each CTA owns RW_TOK tokens and computes
// every router row for them (this layer's and each prefetch target's) on the
// tensor cores, so the per-token softmax / top-k follows in the same CTA from
// shared memory; per-expert pair counts and predicted-expert masks are then
// merged in global memory. The last CTA to arrive runs the slot-table step,
// lays the groups out (ascending expert id, each a contiguous run of rows)
// and cuts them into the token tiles of the grouped GEMM.
constexpr int RW_TOK = 32;

__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__global__ void __launch_bounds__(RT_THREADS) k_route_wide(RouteArgs A, WideArgs W) {
  extern __shared__ float s_lg[];   // [RW_TOK][rows] logits (+ bias)
  const int E = A.geo.n_experts, d = A.geo.d_model, T = A.T, k = A.geo.top_k;
  const int rows = E * (1 + A.n_pred);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * RW_TOK;
  const int ntok = min(RW_TOK, T - t0);
  const int g8 = lane >> 2, c4 = lane & 3;

  __shared__ int s_hist[MAX_E];
  __shared__ unsigned s_pm[MS_MAX_DEPTHS][MAX_E / 32];
  __shared__ uint16_t s_vals[RT_THREADS / 32][MAX_E];
  __shared__ int s_sel[RT_THREADS / 32][MAX_E];
  for (int i = threadIdx.x; i < MAX_E; i += RT_THREADS) s_hist[i] = 0;
  for (int i = threadIdx.x; i < MS_MAX_DEPTHS * (MAX_E / 32); i += RT_THREADS) (&s_pm[0][0])[i] = 0;

  // ---- logits: mma.sync m16n8k16 over 16-row chunks of the router rows.
  // Lane (g8, c4) loads 16 contiguous bytes of its rows per 32-column chunk
  // (columns 8*c4 .. 8*c4+7): the first four feed k slots (2c, 2c+1, 2c+8,
  // 2c+9) of one MMA, the last four those of a second. A and B use the same
  // assignment, so the two MMAs sum the chunk's 32 products exactly once.
  const uint4* xr[2][2];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = min(t0 + m * 16 + h * 8 + g8, T - 1);   // rows past T: computed, never used
      xr[m][h] = reinterpret_cast<const uint4*>(A.x + (long long)t * d) + c4;
    }
  for (int rc = warp; rc * 16 < rows; rc += RT_THREADS / 32) {
    const uint4* wr[2];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int r = min(rc * 16 + n * 8 + g8, rows - 1);
      const int which = r / E, e = r % E;
      wr[n] = reinterpret_cast<const uint4*>((which == 0 ? A.w_r : A.w_p[which - 1]) +
                                             (long long)e * d) + c4;
    }
    float acc[2][2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[m][n][q] = 0.f;
#pragma unroll 4
    for (int kc = 0; kc < d / 8; kc += 4) {     // 32 columns per step
      uint4 av[2][2], bv[2];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) av[m][h] = __ldg(xr[m][h] + kc);
#pragma unroll
      for (int n = 0; n < 2; ++n) bv[n] = __ldg(wr[n] + kc);
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const uint32_t a0[4] = {av[m][0].x, av[m][1].x, av[m][0].y, av[m][1].y};
          const uint32_t b0[2] = {bv[n].x, bv[n].y};
          mma_bf16_16816(acc[m][n], a0, b0);
          const uint32_t a1[4] = {av[m][0].z, av[m][1].z, av[m][0].w, av[m][1].w};
          const uint32_t b1[2] = {bv[n].z, bv[n].w};
          mma_bf16_16816(acc[m][n], a1, b1);
        }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int r = rc * 16 + n * 8 + 2 * c4 + q;
        if (r >= rows) continue;
        const int which = r / E, e = r % E;
        const uint16_t* b = which == 0 ? A.b_r : A.b_p[which - 1];
        const float bias = b ? bf2f(b[e]) : 0.f;
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) s_lg[(m * 16 + h * 8 + g8) * rows + r] = acc[m][n][h * 2 + q] + bias;
      }
  }
  __syncthreads();

  // ---- per token: route, predictions
  const int kp = A.kp;
  for (int tt = warp; tt < ntok; tt += RT_THREADS / 32) {
    const int t = t0 + tt;
    const float* lg = s_lg + tt * rows;
    const float sc = route_token(lg, A.geo, s_vals[warp], s_sel[warp], lane);
    if (lane < k) {
      const int e = s_sel[warp][lane];
      A.inds[t * k + lane] = e;
      A.scores[t * k + lane] = f2bf(sc);
      A.scores_f[t * k + lane] = sc;
      atomicAdd(&s_hist[e], 1);
    }
    __syncwarp();
    for (int dd = 0; dd < A.n_pred; ++dd) {
      predict_token(lg + (dd + 1) * E, E, kp, s_vals[warp], s_sel[warp], lane);
      for (int j = lane; j < kp; j += 32) {
        const int e = s_sel[warp][j];
        atomicOr(&s_pm[dd][e >> 5], 1u << (e & 31));
        if (dd == 0 && A.pred_out) A.pred_out[t * kp + j] = e;
      }
      __syncwarp();
    }
  }
  if (!A.do_pool) return;                      // routing only (ms_route)
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += RT_THREADS)
    if (s_hist[e]) atomicAdd(&W.cnt_e[e], s_hist[e]);
  for (int i = threadIdx.x; i < A.n_pred * (MAX_E / 32); i += RT_THREADS)
    if ((&s_pm[0][0])[i]) atomicOr(&W.pmask[i], (&s_pm[0][0])[i]);

  // ---- arrival: the last CTA goes on
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(A.ticket, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  __shared__ int s_cnt[MAX_E], s_acq[MAX_E], s_slots[MAX_E], s_waits[MAX_E];
  __shared__ int s_pred[MS_MAX_DEPTHS][MAX_E];
  __shared__ int s_n_pred[MS_MAX_DEPTHS];
  __shared__ unsigned s_am[MAX_E / 32];
  __shared__ OpCtx s_op;
  __shared__ KeyCache s_kc;
  __shared__ int s_ci[MS_MAX_DEPTHS + 1][MAX_E];
  for (int e = threadIdx.x; e < MAX_E; e += RT_THREADS) {
    s_cnt[e] = e < E ? __ldcg(&W.cnt_e[e]) : 0;
    if (e < E) W.cnt_e[e] = 0;
  }
  for (int i = threadIdx.x; i < MS_MAX_DEPTHS * (MAX_E / 32); i += RT_THREADS) {
    (&s_pm[0][0])[i] = __ldcg(&W.pmask[i]);
    W.pmask[i] = 0u;
  }
  __syncthreads();
  if (warp == 0) {
    for (int base = 0; base < MAX_E; base += 32) {
      const unsigned bits = __ballot_sync(MS_FULL, s_cnt[base + lane] > 0);
      if (lane == 0) s_am[base >> 5] = bits;
    }
    __syncwarp();
    const int nw = (E + 31) / 32;
    const int n_acq = warp_mask_to_list(s_am, nw, s_acq, lane);
    for (int dd = 0; dd < A.n_pred; ++dd) {
      const int n = warp_mask_to_list(s_pm[dd], nw, s_pred[dd], lane);
      if (lane == 0) s_n_pred[dd] = n;
    }
    __syncwarp();
    warp_pool_step(A, s_pred, s_n_pred, s_acq, n_acq, s_slots, s_waits, &s_op, &s_kc, s_ci, lane);
    __syncwarp();
    // groups in ascending expert order, and their token tiles
    int run = 0, trun = 0;
    for (int base = 0; base < n_acq; base += 32) {
      const int gi = base + lane;
      const int e = gi < n_acq ? s_acq[gi] : 0;
      const int cnt = gi < n_acq ? s_cnt[e] : 0;
      const int nt = (cnt + GEMM_TILE_ROWS - 1) / GEMM_TILE_ROWS;
      int ic = cnt, itl = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(MS_FULL, ic, o);
        const int u = __shfl_up_sync(MS_FULL, itl, o);
        if (lane >= o) {
          ic += v;
          itl += u;
        }
      }
      if (gi < n_acq) {
        const int start = run + ic - cnt;
        A.grp.grp_start[gi] = start;
        A.grp.grp_count[gi] = cnt;
        A.grp.grp_key[gi] = e;
        A.grp.grp_slot[gi] = s_slots[gi];
        A.grp.map[e] = gi;
        W.cursor[gi] = 0;
        const int first = trun + itl - nt;
        for (int j = 0; j < nt && first + j < W.max_tiles; ++j) {
          GemmTile tl;
          tl.g = gi;
          tl.row0 = start + j * GEMM_TILE_ROWS;
          tl.rows = min(GEMM_TILE_ROWS, cnt - j * GEMM_TILE_ROWS);
          tl.slot = s_slots[gi];
          W.tiles[first + j] = tl;
        }
      }
      run += __shfl_sync(MS_FULL, ic, 31);
      trun += __shfl_sync(MS_FULL, itl, 31);
    }
    if (lane == 0) {
      *A.grp.n_groups = n_acq;
      *W.n_tiles = min(trun, W.max_tiles);
    }
  }
  if (threadIdx.x == 0) *A.ticket = 0u;
}

// Host API table operation (ExpertPool.prefetch / .acquire called directly):
// one warp, the request passed by value.
__global__ void k_pool_op(DevTable Tb, PoolReq R, int* slots_out, int* op_status) {
  __shared__ OpCtx s_op;
  __shared__ KeyCache s_kc;
  __shared__ int s_exp[MS_MAX_REQ];
  __shared__ int s_ci[MS_MAX_REQ];
  __shared__ int s_slots[MS_MAX_REQ];
  __shared__ int s_waits[MS_MAX_REQ];
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  for (int i = lane; i < R.n; i += 32) s_exp[i] = R.experts[i];
  if (lane == 0) s_kc.n = 0;
  __syncwarp();
  op_load(Tb, &s_op, lane);
  Req r;
  r.ci = s_ci;
  kc_add(Tb, &s_kc, r, R.layer, s_exp, R.n, true, lane);   // callers may repeat experts
  kc_load(Tb, &s_op, &s_kc, lane);
  int st = 0;
  if (R.op == 0) {
    warp_prefetch(Tb, &s_op, &s_kc, r, lane);
    __syncwarp();
    if (lane == 0) s_op.n_fill_pf = s_op.n_fill;
  } else {
    st = warp_acquire(Tb, &s_op, &s_kc, r, s_slots, s_waits, lane);
    for (int i = lane; i < R.n; i += 32) slots_out[i] = s_slots[i];
  }
  op_store(Tb, &s_op, lane);
  if (lane == 0) *op_status = st;
}

// Store -> arena copy of the fills the last table step produced. The store
// is mapped pinned host memory read directly by the SMs, so the fill list
// never has to travel to the host.
__global__ void __launch_bounds__(256) k_fill(FillArgs F) {
  if (F.pdl) {
    // a programmatic dependent of the route step: let the expert kernels
    // launch now; the fill list is read once the route step has finished
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }
  if (F.l2_next_bytes && threadIdx.x == 0) {
    // the next block call's router rows that are not in L2 yet (read-only
    // weights, so this may run before the wait): one slice per CTA
    const unsigned slice = ((F.l2_next_bytes / gridDim.x) + 15u) & ~15u;
    const unsigned off = slice * blockIdx.x;
    if (off < F.l2_next_bytes) {
      const unsigned n = min(slice, F.l2_next_bytes - off);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                       static_cast<const uint8_t*>(F.l2_next) + off),
                   "r"(n)
                   : "memory");
    }
  }
  if (F.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
  const int2* list;
  int first, n;
  int* err;
  if (F.ring) {
    list = F.ring;
    first = 0;
    n = min(*F.ring_cnt, F.max_fills);
    err = F.ring_err;
  } else {
    list = F.fills;
    n = min(F.ctr->n_fill, F.max_fills);
    first = F.acquire_only ? min(F.ctr->n_fill_pf, n) : 0;
    err = &F.ctr->status;
  }
  const long long chunks = F.blob / 16384;
  const long long total = (long long)(n - first) * chunks;
  for (long long i = blockIdx.x; i < total; i += gridDim.x) {
    const int2 f = list[first + i / chunks];
    const long long part = i % chunks;
    if (f.y < 0 || (long long)f.y >= F.store_keys) {
      if (threadIdx.x == 0) atomicCAS(err, 0, -7);
      continue;
    }
    // a blob of a smaller precision class copies only its own chunks; the
    // slot records the class of what it now holds
    const int cls = F.class_of_key ? F.class_of_key[f.y] : 0;
    if (part == 0 && threadIdx.x == 0 && F.slot_class) F.slot_class[f.x] = (uint8_t)cls;
    if (F.class_of_key && part >= F.cls_chunks[cls]) continue;
    const uint4* src = reinterpret_cast<const uint4*>(F.store + (long long)f.y * F.blob + part * 16384);
    uint4* dst = reinterpret_cast<uint4*>(F.arena + (long long)f.x * F.blob + part * 16384);
    uint4 v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = src[threadIdx.x + q * 256];
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[threadIdx.x + q * 256] = v[q];
  }
}

// ms_expert_mlp preparation: frag layout of x and groups keyed by slot.
__global__ void __launch_bounds__(RT_THREADS) k_mlp_prep(MlpPrepArgs A) {
  __shared__ int s_uniq[MS_MLP_MAX_PAIRS];
  __shared__ int s_cnt[MS_MLP_MAX_PAIRS], s_run[MS_MLP_MAX_PAIRS];
  extern __shared__ unsigned s_mask[];
  frag_write_rows(A.x, A.T, A.d_model, A.xfrag, A.xsum, threadIdx.x, RT_THREADS, &A.ctr->status);
  // key n_slots collects out-of-range slots: its group reads nothing and
  // yields zeros, and the pool status records MS_E_INVALID
  const int nw = (A.n_slots + 1 + 31) / 32;
  for (int i = threadIdx.x; i < nw; i += RT_THREADS) s_mask[i] = 0;
  __syncthreads();
  const int P = A.T * A.k;
  for (int p = threadIdx.x; p < P; p += RT_THREADS) {
    int s = A.slots[p];
    if (s < 0 || s >= A.n_slots) {
      s = A.n_slots;
      atomicCAS(&A.ctr->status, 0, ST_E_INVALID);
    }
    A.keys[p] = s;
    atomicOr(&s_mask[s >> 5], 1u << (s & 31));
  }
  __syncthreads();
  __shared__ int s_n;
  if (threadIdx.x < 32) {
    const int n = warp_mask_to_list(s_mask, nw, s_uniq, threadIdx.x);
    if (threadIdx.x == 0) s_n = n;
  }
  __syncthreads();
  cta_build_groups(A.keys, P, s_uniq, s_n, A.grp, s_cnt, s_run,
                   [&](int g) { return s_uniq[g] < A.n_slots ? s_uniq[g] : -1; });
}

// ----------------------------------------------------------------- launchers
// The kernels that run beside the expert kernels (the route step before
// them, the fills on the pool's side stream) ask for the largest
// shared-memory carveout: an SM can only change its L1/shared split once it
// has drained, so a long fill CTA on a small-shared configuration would keep
// the expert kernels' CTAs off that SM until the fill ends.
cudaError_t route_prefer_shared() {
  const void* fns[] = {reinterpret_cast<const void*>(k_route_step),
                       reinterpret_cast<const void*>(k_fill),
                       reinterpret_cast<const void*>(k_mlp_prep)};
  for (const void* f : fns) {
    const cudaError_t e =
        cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Self-test of the bounded waits: an mbarrier that expects two arrivals gets
// one, so its phase never completes; every thread waits on it with the
// bounded wait the kernels use (a limit of limit_ns), which must give up,
// record MS_E_TIMEOUT in *status and return. No copy is in flight, so
// nothing is left pending when the CTA exits.
__global__ void k_wait_selftest(unsigned long long limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
  mbar_wait_ns(&bar, 0, status, limit_ns);
}

cudaError_t launch_wait_selftest(unsigned long long limit_ns, int* status, cudaStream_t s) {
  k_wait_selftest<<<1, 32, 0, s>>>(limit_ns, status);
  return cudaGetLastError();
}

cudaError_t route_step_attributes(cudaFuncAttributes* attr) {
  return cudaFuncGetAttributes(attr, k_route_step);
}

cudaError_t launch_route_step(const RouteArgs& a, int grid, cudaStream_t s) {
  // the fused norm's input rows in dynamic shared memory, beside the
  // kernel's static arrays
  const int smem = a.norm_w ? a.T * a.geo.d_model * 2 : 0;
  if (smem > 0) {
    cudaError_t e = cudaFuncSetAttribute(k_route_step, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(RT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_route_step, a);
}

// rms_norm(h) * w for the fused block's wide path: one CTA per token row.
__global__ void __launch_bounds__(256) k_rmsnorm(const uint16_t* h, const uint16_t* w, float eps, int d,
                                                 uint16_t* out) {
  __shared__ float s_red[32];
  const uint16_t* hr = h + (long long)blockIdx.x * d;
  const float rn = cta_rms_factor(hr, d, eps, s_red);
  uint16_t* o = out + (long long)blockIdx.x * d;
  for (int i = threadIdx.x; i < d; i += 256) o[i] = f2bf(bfr(bf2f(hr[i]) * rn) * bf2f(w[i]));
}

cudaError_t launch_rmsnorm(const uint16_t* h, const uint16_t* w, float eps, int T, int d, uint16_t* out,
                           cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  k_rmsnorm<<<T, 256, 0, s>>>(h, w, eps, d, out);
  return cudaGetLastError();
}
cudaError_t launch_route_wide(const RouteArgs& a, const WideArgs& w, cudaStream_t s) {
  const int rows = a.geo.n_experts * (1 + a.n_pred);
  const size_t smem = (size_t)RW_TOK * rows * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(k_route_wide, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  k_route_wide<<<(a.T + RW_TOK - 1) / RW_TOK, RT_THREADS, smem, s>>>(a, w);
  return cudaGetLastError();
}
cudaError_t launch_pool_op(const DevTable& t, const PoolReq& r, int* slots_out, int* st,
                           cudaStream_t s) {
  k_pool_op<<<1, 32, 0, s>>>(t, r, slots_out, st);
  return cudaGetLastError();
}
cudaError_t launch_fill(const FillArgs& f, int grid, cudaStream_t s) {
  if (!f.pdl) {
    k_fill<<<grid, 256, 0, s>>>(f);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_fill, f);
}
cudaError_t launch_mlp_prep(const MlpPrepArgs& a, cudaStream_t s) {
  const size_t smem = ((a.n_slots + 1 + 31) / 32) * sizeof(unsigned);
  k_mlp_prep<<<1, RT_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace ms
