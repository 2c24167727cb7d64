// Bulk-copy (TMA, cp.async.bulk) staging with mbarrier completion, and the
// bounded waits every spin in this library must use.
#pragma once
#include "ms_common.cuh"

namespace ms {

// Spin limit of an mbarrier wait: ~2^26 polls (far beyond any legitimate
// copy); on expiry the waiter records MS_E_TIMEOUT and gives up.
constexpr unsigned MBAR_SPIN_LIMIT = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read once and not again soon (a decode step streams
// ~1 GB of expert weights through a 126 MB L2): its lines go first, so the
// router rows, the slot table and the kernels' code stay resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache policy (l2_evict_first).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled 4-D tensor copy global -> this CTA's shared memory (no multicast),
// completing on `bar`, with an L2 cache policy.
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const void* tmap, int x, int y, int z, int w,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Wall-clock limit of one mbarrier wait (ns), checked on %globaltimer.
constexpr unsigned long long MBAR_WAIT_NS = 1000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// try_wait that may suspend the thread until the phase completes, for at
// most hint_ns: a waiting warp then leaves its issue slots to the others.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, unsigned phase, unsigned hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `phase` of `bar`: suspending polls, at most
// MBAR_SPIN_LIMIT of them and MBAR_WAIT_NS of wall time. Returns false (and
// sets *status to MS_E_TIMEOUT once) if either limit ran out.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, unsigned phase, int* status,
                                             unsigned long long limit_ns) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned i = 0; i < MBAR_SPIN_LIMIT; ++i) {
    if (mbar_try_wait_sleep(bar, phase, 100000u)) return true;
    if (global_ns() - t0 > limit_ns) break;
  }
  if (status) atomicCAS(status, 0, -4);
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned phase, int* status) {
  return mbar_wait_ns(bar, phase, status, MBAR_WAIT_NS);
}

// True once any wait of this call chain has timed out: later CTAs then skip
// their work instead of waiting out the same limit again.
__device__ __forceinline__ bool timed_out(const int* status) {
  return status && *reinterpret_cast<const volatile int*>(status) == -4;
}

// Thread-block clusters (distributed shared memory within one GPU).
// DSMEM address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* p, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// every thread of every CTA of the cluster: writes before it (shared
// memory of any CTA of the cluster included) are visible after it
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

}  // namespace ms
