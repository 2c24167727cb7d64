// Device-resident slot table: ExpertPool's bookkeeping (engine_v3.py:303-454)
// executed by ONE warp. Every decision is sequential, as in the reference,
// because each victim choice depends on the previous one; the only parallel
// part is the victim scan, where 32 lanes score 32 consecutive candidates of
// the stride-7919 walk at once and a warp prefix scan recovers exactly the
// candidate the sequential loop would have stopped at.
//
// Timing rule (shared with the CPU oracle and the golden fixtures): a
// prefetched key stays pending until an acquire waits on it or until the end
// of the next acquire call.
#pragma once
#include "ms_common.cuh"

namespace ms {

// Scalar state of one table operation, held in shared memory and owned by
// lane 0; other lanes read it after a __syncwarp().
struct OpCtx {
  long long clock, use_clock;
  int n_free, n_pend, n_pin, n_fill;
  int status;
  long long st[ST_N];
};

__device__ __forceinline__ void op_load(const DevTable& T, OpCtx* c, int lane) {
  if (lane == 0) {
    const TableCtr* g = T.ctr;
    c->clock = g->clock; c->use_clock = g->use_clock;
    c->n_free = g->n_free; c->n_pend = g->n_pend; c->n_pin = g->n_pin;
    c->n_fill = 0; c->status = 0;
    for (int i = 0; i < ST_N; ++i) c->st[i] = g->st[i];
  }
  __syncwarp();
}

__device__ __forceinline__ void op_store(const DevTable& T, OpCtx* c, int lane) {
  __syncwarp();
  if (lane == 0) {
    TableCtr* g = T.ctr;
    g->clock = c->clock; g->use_clock = c->use_clock;
    g->n_free = c->n_free; g->n_pend = c->n_pend; g->n_pin = c->n_pin;
    g->n_fill = c->n_fill;
    if (c->status && !g->status) g->status = c->status;
    for (int i = 0; i < ST_N; ++i) g->st[i] = c->st[i];
  }
  __syncwarp();
}

// _alloc (engine_v3.py:313-374). All 32 lanes call it; returns the slot or
// -1 when every slot is empty/pinned/pending ("pool exhausted"). The clock
// advances even on failure, as in the reference (:323).
__device__ int warp_alloc(const DevTable& T, OpCtx* c, int key, int lane) {
  __syncwarp();
  if (lane == 0) c->clock += 1;
  __syncwarp();
  const long long clock = c->clock;
  const int n_free = c->n_free;
  __syncwarp();
  int slot;
  if (n_free > 0) {
    slot = n_free - 1;                       // free.pop() from the end (:325)
    if (lane == 0) c->n_free = n_free - 1;
  } else {
    const int n = T.n_slots;
    const long long start = clock % n;
    int carry_cnt = 0;
    unsigned long long carry_best = ~0ull, best = ~0ull;
    bool found = false;
    for (int base = 0; base < n && !found; base += 32) {
      const int j = base + lane;
      bool valid = false;
      unsigned long long packed = ~0ull;
      if (j < n) {
        const int sidx = (int)((start + (long long)j * STRIDE) % n);
        const int k = T.key_of[sidx];
        if (k >= 0 && !T.pinned[sidx] && !(T.kflags[k] & KF_PENDING)) {
          const long long young = (clock - T.born[k] < T.window) ? YOUNG : 0;
          long long b = 0;
          if (T.evict == EVICT_LRU) b = T.last_use[k];
          else if (T.evict == EVICT_LFU) b = T.freq[k];
          // first-seen strict minimum == min over (score, walk position)
          packed = ((unsigned long long)(b + young) << 20) | (unsigned long long)j;
          valid = true;
        }
      }
      const unsigned vb = __ballot_sync(MS_FULL, valid);
      const int cnt = carry_cnt + __popc(vb & (MS_FULL >> (31 - lane)));
      unsigned long long pm = packed;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(MS_FULL, pm, o);
        if (lane >= o && v < pm) pm = v;
      }
      if (carry_best < pm) pm = carry_best;
      // the reference stops after a SEEN candidate once SAMPLE were seen and
      // the best so far is not young (:352-354)
      const bool stop = valid && cnt >= SAMPLE && (long long)(pm >> 20) < YOUNG;
      const unsigned sb = __ballot_sync(MS_FULL, stop);
      if (sb) {
        best = __shfl_sync(MS_FULL, pm, __ffs(sb) - 1);
        found = true;
      } else {
        carry_cnt += __popc(vb);
        carry_best = __shfl_sync(MS_FULL, pm, 31);
      }
    }
    if (!found) best = carry_best;
    if (best == ~0ull) return -1;
    const int j = (int)(best & 0xFFFFFull);
    slot = (int)((start + (long long)j * STRIDE) % n);
    if (lane == 0) {                         // evict (:357-362)
      const int vk = T.key_of[slot];
      T.kflags[vk] &= (uint8_t)~KF_FROMPF;
      T.born[vk] = 0;
      T.last_use[vk] = 0;
      T.freq[vk] = 0;
      T.slot_of[vk] = -1;
    }
  }
  if (lane == 0) {                           // (:364-366)
    T.key_of[slot] = key;
    T.slot_of[key] = slot;
    T.born[key] = clock;
  }
  __syncwarp();
  return slot;
}

// _touch (engine_v3.py:376-380). Lane 0 only.
__device__ __forceinline__ void touch0(const DevTable& T, OpCtx* c, int key) {
  c->use_clock += 1;
  T.last_use[key] = c->use_clock;
  T.freq[key] += 1;
}

__device__ __forceinline__ void pin0(const DevTable& T, OpCtx* c, int slot) {
  if (!T.pinned[slot]) {
    T.pinned[slot] = 1;
    T.pin_list[c->n_pin++] = slot;
  }
}

__device__ __forceinline__ void add_fill0(const DevTable& T, OpCtx* c, int slot, int key) {
  if (c->n_fill < T.max_fills) T.fills[c->n_fill] = make_int2(slot, key);
  c->n_fill++;
}

// prefetch (engine_v3.py:383-396): experts in caller order; stops at the
// first exhaustion and counts one bail.
__device__ void warp_prefetch(const DevTable& T, OpCtx* c, int layer, const int* experts,
                              int n, int lane) {
  for (int i = 0; i < n; ++i) {
    const int key = layer * T.n_experts + experts[i];
    __syncwarp();
    const bool skip = T.slot_of[key] >= 0 || (T.kflags[key] & KF_PENDING);
    __syncwarp();
    if (skip) continue;
    const int slot = warp_alloc(T, c, key, lane);
    if (slot < 0) {
      if (lane == 0) c->st[ST_BAIL] += 1;
      __syncwarp();
      return;
    }
    if (lane == 0) {
      c->st[ST_ISSUED] += 1;
      T.kflags[key] |= KF_PENDING;
      T.pend_list[c->n_pend++] = key;
      add_fill0(T, c, slot, key);
    }
    __syncwarp();
  }
}

// Completion of every read still pending (end of an acquire call).
__device__ void warp_drain(const DevTable& T, OpCtx* c, int lane) {
  __syncwarp();
  if (lane == 0) {
    for (int i = 0; i < c->n_pend; ++i) {
      const int key = T.pend_list[i];
      if (T.kflags[key] & KF_PENDING) {
        T.kflags[key] = (uint8_t)((T.kflags[key] & ~KF_PENDING) | KF_FROMPF);
        c->st[ST_READS] += 1;
      }
    }
    c->n_pend = 0;
  }
  __syncwarp();
}

// acquire (engine_v3.py:398-454). slots_out[i] receives the slot of
// experts[i] (-1 if exhausted before it was placed). waits: scratch of n
// ints (shared or global). Returns 0 or MS_E_EXHAUSTED (-3).
__device__ int warp_acquire(const DevTable& T, OpCtx* c, int layer, const int* experts,
                            int n, int* slots_out, int* waits, int lane) {
  int n_wait = 0, n_issue = 0, status = 0;
  for (int i = 0; i < n; ++i) {
    const int key = layer * T.n_experts + experts[i];
    __syncwarp();
    const bool pend = (T.kflags[key] & KF_PENDING) != 0;
    int slot = T.slot_of[key];
    __syncwarp();
    bool issued_now = false;
    if (!pend && slot < 0) {
      slot = warp_alloc(T, c, key, lane);
      if (slot < 0) { status = -3; break; }
      if (lane == 0) {
        pin0(T, c, slot);
        touch0(T, c, key);
        add_fill0(T, c, slot, key);
      }
      ++n_issue;
      issued_now = true;
    } else if (slot >= 0) {
      if (lane == 0) { pin0(T, c, slot); touch0(T, c, key); }
    }
    if (lane == 0) {
      if (pend) {
        waits[n_wait] = i;
        slots_out[i] = -1;
      } else if (slot >= 0 && !issued_now) {
        const bool early = (T.kflags[key] & KF_FROMPF) != 0;
        T.kflags[key] &= (uint8_t)~KF_FROMPF;
        c->st[early ? ST_PREFETCH : ST_CACHE] += 1;
        slots_out[i] = slot;
      }
      if (issued_now) slots_out[i] = slot;
    }
    if (pend) ++n_wait;
  }
  __syncwarp();
  if (status == 0) {
    if (lane == 0) {
      c->st[ST_EXPOSED] += n_issue;
      c->st[ST_READS] += n_issue;
      for (int w = 0; w < n_wait; ++w) {            // (:438-446)
        const int i = waits[w];
        const int key = layer * T.n_experts + experts[i];
        if (T.kflags[key] & KF_PENDING) c->st[ST_READS] += 1;
        T.kflags[key] &= (uint8_t)~(KF_PENDING | KF_FROMPF);
        const int slot = T.slot_of[key];
        slots_out[i] = slot;
        pin0(T, c, slot);
        touch0(T, c, key);
        c->st[ST_PREFETCH] += 1;
      }
      c->st[ST_MISS] += n_issue;
      // pinned = set(slots) (:452-453)
      for (int i = 0; i < c->n_pin; ++i) T.pinned[T.pin_list[i]] = 0;
      c->n_pin = 0;
      for (int i = 0; i < n; ++i) {
        const int s = slots_out[i];
        if (s >= 0) pin0(T, c, s);
      }
    }
  } else if (lane == 0) {
    c->status = status;
  }
  __syncwarp();
  warp_drain(T, c, lane);
  return status;
}

}  // namespace ms
