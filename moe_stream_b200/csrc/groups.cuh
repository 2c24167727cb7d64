// Pair grouping shared by the routed path (key = expert id) and the
// ms_expert_mlp path (key = slot id): one CTA turns the keys of P pairs into
// groups ordered by ascending key, with the pairs of each group in ascending
// pair order. This replaces the reference's np.unique(..., return_inverse)
// bookkeeping (engine_v3.py:530-552).
#pragma once
#include "ms_common.cuh"

namespace ms {

// Sorted list of the set bits of mask[0..nw) (nw <= 32*32), by one warp.
// The same for a few mask words (an expert mask, nw <= 8): lane l handles
// bit l of every word, so the list is a handful of independent steps
// instead of a scan and a per-lane bit loop.
__device__ __forceinline__ int warp_small_mask_to_list(const unsigned* mask, int nw, int* out, int lane) {
  int total = 0;
  for (int w = 0; w < nw; ++w) {
    const unsigned m = mask[w];
    if ((m >> lane) & 1u) out[total + __popc(m & ((1u << lane) - 1u))] = w * 32 + lane;
    total += __popc(m);
  }
  __syncwarp();
  return total;
}

__device__ __forceinline__ int warp_mask_to_list(const unsigned* mask, int nw, int* out, int lane) {
  int total = 0;
  for (int base = 0; base < nw; base += 32) {
    const int w = base + lane;
    const unsigned bits = (w < nw) ? mask[w] : 0u;
    const int cnt = __popc(bits);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(MS_FULL, incl, o);
      if (lane >= o) incl += v;
    }
    int pos = total + incl - cnt;
    unsigned b = bits;
    while (b) {
      const int i = __ffs(b) - 1;
      out[pos++] = w * 32 + i;
      b &= b - 1;
    }
    total += __shfl_sync(MS_FULL, incl, 31);
  }
  __syncwarp();
  return total;
}

// Build the groups of pairs keyed by keys[0..P). uniq[0..n_uniq) is the
// sorted distinct key list (shared memory), slot_of_group(g) gives the slot of
// group g. s_cnt / s_run: shared scratch of n_uniq ints each. All threads of
// the CTA must call it.
template <typename SlotFn>
__device__ void cta_build_groups(const int* keys, int P, const int* uniq, int n_uniq,
                                 const Groups& G, int* s_cnt, int* s_run, SlotFn slot_of_group) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int g = tid; g < n_uniq; g += nt) {
    G.map[uniq[g]] = g;
    s_cnt[g] = 0;
  }
  __syncthreads();
  for (int p = tid; p < P; p += nt) atomicAdd(&s_cnt[G.map[keys[p]]], 1);
  __syncthreads();
  if (tid < 32) {
    const int lane = tid;
    int run = 0;
    for (int base = 0; base < n_uniq; base += 32) {
      const int g = base + lane;
      const int cnt = (g < n_uniq) ? s_cnt[g] : 0;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(MS_FULL, incl, o);
        if (lane >= o) incl += v;
      }
      if (g < n_uniq) {
        const int st = run + incl - cnt;
        s_run[g] = st;
        G.grp_start[g] = st;
        G.grp_count[g] = cnt;
        G.grp_key[g] = uniq[g];
        G.grp_slot[g] = slot_of_group(g);
      }
      run += __shfl_sync(MS_FULL, incl, 31);
    }
    __syncwarp();
    // stable scatter: pairs in ascending order, 32 at a time
    for (int base = 0; base < P; base += 32) {
      const int p = base + lane;
      const int g = (p < P) ? G.map[keys[p]] : -1;
      const unsigned same = __match_any_sync(MS_FULL, g);
      const int rank = __popc(same & ((1u << lane) - 1u));
      const int pos = (g >= 0) ? s_run[g] + rank : 0;
      __syncwarp();
      if (g >= 0) {
        G.grp_pairs[pos] = p;
        if (rank == 0) s_run[g] += __popc(same);
      }
      __syncwarp();
    }
    if (lane == 0) *G.n_groups = n_uniq;
  }
  __syncthreads();
}

}  // namespace ms
