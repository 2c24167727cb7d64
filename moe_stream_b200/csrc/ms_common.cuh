// Shared device-side structures of libmoestream (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#define MS_FULL 0xffffffffu

namespace ms {

// ------------------------------------------------------------ slot table
// Per-key flags (key = layer * n_experts + expert).
constexpr uint8_t KF_PENDING = 1;   // ExpertPool.pending   (engine_v3.py:219)
constexpr uint8_t KF_FROMPF = 2;    // ExpertPool.from_prefetch (:220)

constexpr int EVICT_LFU = 0, EVICT_LRU = 1, EVICT_ASIS = 2;
constexpr int SAMPLE = 24;                    // engine_v3.py:322
constexpr long long STRIDE = 7919;            // engine_v3.py:336
constexpr long long YOUNG = 1LL << 30;        // engine_v3.py:349

// Device-side status codes (the same values as MS_E_* of the C ABI).
constexpr int ST_E_INVALID = -1, ST_E_TIMEOUT = -4, ST_E_RANGE = -8;
// Largest finite fp16. An activation beyond it would enter the fp16
// tensor-core operands as inf; its writer records ST_E_RANGE instead of
// passing the overflow on silently.
constexpr float F16_MAX = 65504.f;

// stats slots (ms_stats order minus totals)
enum { ST_PREFETCH = 0, ST_CACHE, ST_MISS, ST_BAIL, ST_ISSUED, ST_READS, ST_EXPOSED, ST_N };

// Mutable scalars of the table, resident in device memory.
struct TableCtr {
  long long clock;       // allocation counter (engine_v3.py:222)
  long long use_clock;   // access counter (:225)
  int n_free;            // free list is [0, n_free): pop() takes n_free-1 (:218, 325)
  int n_pend;            // pend_list length
  int n_pin;             // pin_list length
  int n_fill;            // fills produced by the current call
  int status;            // sticky error code (0 / negative MS_E_*)
  int n_fill_pf;         // fills[0, n_fill_pf) of the current call came from its prefetches
  long long st[ST_N];
};

struct DevTable {
  int n_slots, n_keys, n_experts, evict, window;
  int* key_of;           // [n_slots]  key or -1   (engine_v3.py:216)
  int* slot_of;          // [n_keys]   slot or -1  (:215)
  int* freq;             // [n_keys]               (:217)
  long long* born;       // [n_keys]               (:223)
  long long* last_use;   // [n_keys]               (:224)
  uint8_t* kflags;       // [n_keys]   KF_*
  uint8_t* pinned;       // [n_slots]              (:221)
  int* pin_list;         // [n_slots]  slots with pinned=1
  int* pend_list;        // [n_slots]  keys that went pending, in issue order
  int2* fills;           // [max_fills] (slot, key) to copy store -> arena
  int max_fills;
  TableCtr* ctr;
};

// ---------------------------------------------------------------- groups
// Token/expert pairs p = t*k + j grouped by the slot they read. Groups are
// ordered by ascending key (expert id on the routed path, slot id on the
// ms_expert_mlp path); pairs inside a group by ascending p.
struct Groups {
  int* n_groups;         // [1]
  int* grp_key;          // [max_groups]
  int* grp_slot;         // [max_groups]  -1 when the pool could not place it
  int* grp_start;        // [max_groups]
  int* grp_count;        // [max_groups]
  int* grp_pairs;        // [max_pairs]
  int* map;              // [key_range] scratch: key -> group
};

// Geometry as the kernels need it.
struct Geo {
  int model;             // 0 qwen3, 1 gpt-oss
  int d_model, d_ff, n_experts, top_k, group_size;
  int norm_topk, proj_bias;
  long long blob;
  long long off[3][4];
};

__device__ __forceinline__ float bf2f(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

// 1/sqrt(mean(h^2) + eps) of a bf16 row of d values, by the whole CTA
// (blockDim.x a multiple of 32); red: >= 32 floats of shared scratch. As
// mlx's RMSNorm (mx.fast.rms_norm): fp32 sum of squares, correctly rounded
// sqrt and division.
__device__ __forceinline__ float cta_rms_factor(const uint16_t* h, int d, float eps, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = __uint_as_float(((uint32_t)h[i]) << 16);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w];
  __syncthreads();
  return 1.f / sqrtf(tot / (float)d + eps);
}
// round-to-nearest-even float -> bf16 bits (the hardware conversion)
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bfr(float f) { return bf2f(f2bf(f)); }

}  // namespace ms
