// Device-resident slot table: ExpertPool's bookkeeping (engine_v3.py:303-454)
// executed by ONE warp. Every decision is sequential, as in the reference,
// because each victim choice depends on the previous one. Two things are
// parallel: the victim scan, where 32 lanes score 32 consecutive candidates
// of the stride-7919 walk at once and a warp prefix scan recovers exactly the
// candidate the sequential loop would have stopped at; and the loading of the
// request's per-key state into shared memory ("key cache") before lane 0
// walks the request, so the walk itself never waits on a global load. Every
// update goes to the shared copy and straight through to global memory.
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
  int n_fill_pf;            // n_fill when the call's prefetch requests were done
  int status;
  int victim_key;           // key evicted by the last warp_alloc, -1 if none
  int n_pend0;              // pending keys left by earlier calls (0 on the fused path)
  long long st[ST_N];
};

__device__ __forceinline__ void op_load(const DevTable& T, OpCtx* c, int lane) {
  if (lane == 0) {
    const TableCtr g = *T.ctr;                 // all loads issued before any store
    c->clock = g.clock; c->use_clock = g.use_clock;
    c->n_free = g.n_free; c->n_pend = g.n_pend; c->n_pin = g.n_pin;
    c->n_fill = 0; c->n_fill_pf = 0; c->status = 0; c->victim_key = -1; c->n_pend0 = g.n_pend;
    for (int i = 0; i < ST_N; ++i) c->st[i] = g.st[i];
  }
  __syncwarp();
}

__device__ __forceinline__ void op_store(const DevTable& T, OpCtx* c, int lane) {
  __syncwarp();
  if (lane == 0) {
    TableCtr g;
    g.clock = c->clock; g.use_clock = c->use_clock;
    g.n_free = c->n_free; g.n_pend = c->n_pend; g.n_pin = c->n_pin;
    g.n_fill = c->n_fill;
    const int prev = T.ctr->status;            // sticky: the first error stays
    g.status = prev ? prev : c->status;
    g.n_fill_pf = c->n_fill_pf;
    for (int i = 0; i < ST_N; ++i) g.st[i] = c->st[i];
    *T.ctr = g;
  }
  __syncwarp();
}

// _alloc (engine_v3.py:313-374). All 32 lanes call it; returns the slot or
// -1 when every slot is empty/pinned/pending ("pool exhausted"). The clock
// advances even on failure, as in the reference (:323). The evicted key, if
// any, is left in c->victim_key.
__device__ __forceinline__ int warp_alloc(const DevTable& T, OpCtx* c, int key, int lane) {
  __syncwarp();
  if (lane == 0) { c->clock += 1; c->victim_key = -1; }
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
      c->victim_key = vk;
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

// ---------------------------------------------------------------- key cache
constexpr int KC_MAX = 640;   // >= n_experts * (1 + prefetch depths), checked at create

struct KeyCache {
  int n;
  int key[KC_MAX];
  int slot[KC_MAX];
  int freq[KC_MAX];
  uint8_t flags[KC_MAX];
  uint8_t pin[KC_MAX];      // pinned[slot[i]] when slot[i] >= 0
  int n_prev_pin;           // the pin list left by the previous acquire
  int prev_pin[KC_MAX];     // (valid when n_prev_pin <= KC_MAX)
};

// A request: items i = 0..n-1 map to cache entries ci[i] (distinct keys get
// distinct entries; a repeated expert reuses its entry).
struct Req {
  int n;
  int base;                 // first cache entry of this request
  int n_uniq;               // entries [base, base + n_uniq)
  int* ci;                  // [n] shared scratch
};

// Register keys layer*E + experts[i] as cache entries (all lanes); no
// global memory is read here. With may_repeat == false the caller
// guarantees distinct experts.
__device__ __forceinline__ void kc_add(const DevTable& T, KeyCache* kc, Req& r, int layer, const int* experts,
                       int n, bool may_repeat, int lane) {
  __syncwarp();
  r.n = n;
  r.base = kc->n;
  if (!may_repeat) {
    const int base = r.base;
    for (int i = lane; i < n; i += 32) {
      r.ci[i] = base + i;
      kc->key[base + i] = layer * T.n_experts + experts[i];
    }
    r.n_uniq = n;
    __syncwarp();
    if (lane == 0) kc->n = base + n;
    __syncwarp();
    return;
  } else {
    // first occurrence of each expert (n is small on this path)
    for (int i = lane; i < n; i += 32) {
      int first = i;
      for (int j = 0; j < i; ++j)
        if (experts[j] == experts[i]) { first = j; break; }
      r.ci[i] = -1 - first;                  // provisional: index of first occurrence
    }
    __syncwarp();
    if (lane == 0) {
      int m = 0;
      for (int i = 0; i < n; ++i) {
        const int f = -1 - r.ci[i];
        r.ci[i] = (f == i) ? r.base + m++ : r.ci[f];
      }
      r.n_uniq = m;
    }
    __syncwarp();
    r.n_uniq = __shfl_sync(MS_FULL, r.n_uniq, 0);
  }
  __syncwarp();
  for (int i = lane; i < n; i += 32)
    kc->key[r.ci[i]] = layer * T.n_experts + experts[i];   // repeats write the same key
  __syncwarp();
  if (lane == 0) kc->n = r.base + r.n_uniq;
  __syncwarp();
}

// Load the state of every registered entry and the previous pin list in one
// round of independent loads (all lanes). The pinned-ness of an entry's slot
// is membership in that pin list (pinned[] and the list are kept equal).
__device__ __forceinline__ void kc_load(const DevTable& T, const OpCtx* c, KeyCache* kc, int lane) {
  __syncwarp();
  const int n = kc->n;
  const int np = c->n_pin;
  for (int i = lane; i < n; i += 32) {
    const int key = kc->key[i];
    const int sl = T.slot_of[key];             // three independent loads, then the stores
    const uint8_t fl = T.kflags[key];
    const int fr = T.freq[key];
    kc->slot[i] = sl;
    kc->flags[i] = fl;
    kc->freq[i] = fr;
  }
  if (np <= KC_MAX)
    for (int i = lane; i < np; i += 32) {
      const int v = T.pin_list[i];
      kc->prev_pin[i] = v;
    }
  if (lane == 0) kc->n_prev_pin = np;
  __syncwarp();
  for (int i = lane; i < n; i += 32) {
    const int sl = kc->slot[i];
    uint8_t pin = 0;
    if (sl >= 0) {
      if (np <= KC_MAX) {
        for (int j = 0; j < np; ++j) pin |= (kc->prev_pin[j] == sl);
      } else {
        pin = T.pinned[sl];
      }
    }
    kc->pin[i] = pin;
  }
  __syncwarp();
}

// _alloc for cache entry ci, keeping the copies coherent (all lanes).
__device__ __forceinline__ int kc_alloc(const DevTable& T, OpCtx* c, KeyCache* kc, int ci, int lane) {
  const int slot = warp_alloc(T, c, kc->key[ci], lane);
  if (slot < 0) return -1;
  const int vk = c->victim_key;
  if (vk >= 0) {
    for (int i = lane; i < kc->n; i += 32)
      if (kc->key[i] == vk) {
        kc->slot[i] = -1;
        kc->flags[i] &= (uint8_t)~KF_FROMPF;
        kc->freq[i] = 0;
        kc->pin[i] = 0;
      }
  }
  __syncwarp();
  if (lane == 0) {
    kc->slot[ci] = slot;
    kc->pin[ci] = 0;                         // a victim or free slot is never pinned
  }
  __syncwarp();
  return slot;
}

// _touch (engine_v3.py:376-380). Lane 0 only.
__device__ __forceinline__ void touch0(const DevTable& T, OpCtx* c, KeyCache* kc, int ci) {
  const int key = kc->key[ci];
  c->use_clock += 1;
  T.last_use[key] = c->use_clock;
  kc->freq[ci] += 1;
  T.freq[key] = kc->freq[ci];
}

__device__ __forceinline__ void pin0(const DevTable& T, OpCtx* c, KeyCache* kc, int ci) {
  if (!kc->pin[ci]) {
    const int slot = kc->slot[ci];
    kc->pin[ci] = 1;
    T.pinned[slot] = 1;
    T.pin_list[c->n_pin++] = slot;
  }
}

__device__ __forceinline__ void setflags0(const DevTable& T, KeyCache* kc, int ci, uint8_t f) {
  kc->flags[ci] = f;
  T.kflags[kc->key[ci]] = f;
}

__device__ __forceinline__ void add_fill0(const DevTable& T, OpCtx* c, int slot, int key) {
  if (c->n_fill < T.max_fills) T.fills[c->n_fill] = make_int2(slot, key);
  c->n_fill++;
}

// prefetch (engine_v3.py:383-396) of request r in caller order; stops at the
// first exhaustion and counts one bail.
// The items are visited in order as in the reference, but 32 at a time: the
// lanes test their items at once and the warp jumps to the next one that
// needs a slot (usually none). An allocation may evict the key of a later
// item (kc_alloc updates its cache entry), so the test is repeated after
// each one, for the items after it only.
__device__ __forceinline__ void warp_prefetch(const DevTable& T, OpCtx* c, KeyCache* kc, const Req& r,
                              int lane) {
  for (int base = 0; base < r.n; base += 32) {
    int next = base;                         // first item not visited yet
    while (true) {
      const int i = base + lane;
      bool need = false;
      if (i < r.n && i >= next) {
        const int ci = r.ci[i];
        need = kc->slot[ci] < 0 && !(kc->flags[ci] & KF_PENDING);
      }
      const unsigned m = __ballot_sync(MS_FULL, need);
      if (!m) break;
      const int i0 = base + __ffs(m) - 1;
      const int ci = r.ci[i0];
      __syncwarp();                          // lane 0's writes before the collective scan
      const int slot = kc_alloc(T, c, kc, ci, lane);
      if (slot < 0) {
        if (lane == 0) c->st[ST_BAIL] += 1;
        __syncwarp();
        return;
      }
      if (lane == 0) {
        c->st[ST_ISSUED] += 1;
        setflags0(T, kc, ci, (uint8_t)(kc->flags[ci] | KF_PENDING));
        T.pend_list[c->n_pend++] = kc->key[ci];
        add_fill0(T, c, slot, kc->key[ci]);
      }
      __syncwarp();
      next = i0 + 1;
    }
  }
  __syncwarp();
}

// Completion of every read still pending (end of an acquire call). Pending
// keys are distinct, so the lanes take them in parallel.
__device__ __forceinline__ void warp_drain(const DevTable& T, OpCtx* c, KeyCache* kc, int lane) {
  __syncwarp();
  const int n = c->n_pend;
  int done = 0;
  if (c->n_pend0 == 0) {
    // every pending key went pending in this call, so it is in the cache
    for (int i = lane; i < kc->n; i += 32) {
      const uint8_t f = kc->flags[i];
      if (f & KF_PENDING) {
        T.kflags[kc->key[i]] = (uint8_t)((f & ~KF_PENDING) | KF_FROMPF);
        ++done;
      }
    }
  } else {
    for (int i = lane; i < n; i += 32) {
      const int key = T.pend_list[i];
      const uint8_t f = T.kflags[key];
      if (f & KF_PENDING) {
        T.kflags[key] = (uint8_t)((f & ~KF_PENDING) | KF_FROMPF);
        ++done;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) done += __shfl_xor_sync(MS_FULL, done, o);
  __syncwarp();
  for (int i = lane; i < kc->n; i += 32)
    if (kc->flags[i] & KF_PENDING) kc->flags[i] = (uint8_t)((kc->flags[i] & ~KF_PENDING) | KF_FROMPF);
  if (lane == 0) {
    c->st[ST_READS] += done;
    c->n_pend = 0;
  }
  __syncwarp();
}

// acquire without allocation: when every key of a request of distinct keys
// is resident or pending, no slot changes hands, so the items are
// independent and the warp takes them 32 at a time. The one serial part of
// the reference loop, the use clock, is reproduced by ranking: every item is
// touched in item order (a pending key already has its slot), then each
// waited-on pending key is touched again, in item order
// (engine_v3.py:412-446). Pins are left to the caller's pinned = set(slots)
// step, which is all they amount to when nothing is allocated. Returns
// false (and changes nothing) when some key needs a slot.
__device__ __forceinline__ bool warp_acquire_resident(const DevTable& T, OpCtx* c, KeyCache* kc,
                                                      const Req& r, int* slots_out, int lane) {
  const int n = r.n;
  if (r.n_uniq != n) return false;
  bool miss = false;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    bool m = false;
    if (i < n) {
      const int ci = r.ci[i];
      m = !(kc->flags[ci] & KF_PENDING) && kc->slot[ci] < 0;
    }
    miss = __any_sync(MS_FULL, m) || miss;
  }
  if (miss) return false;
  const long long uc0 = c->use_clock;
  const unsigned lt = (1u << lane) - 1u;
  int waits_before = 0;
  int n_pf = 0, n_cache = 0, n_reads = 0;         // per call: at most n each
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const int ci = i < n ? r.ci[i] : 0;
    const bool pend = i < n && (kc->flags[ci] & KF_PENDING) != 0;
    const unsigned pb = __ballot_sync(MS_FULL, pend);
    if (i < n) {
      const int key = kc->key[ci];
      uint8_t f = kc->flags[ci];
      long long uc = uc0 + i + 1;              // the in-order touch
      int uses = 1;
      if (!pend) {
        if (f & KF_FROMPF) {                   // first use of a prefetched key (:431-435)
          f = (uint8_t)(f & ~KF_FROMPF);
          kc->flags[ci] = f;
          T.kflags[key] = f;
          ++n_pf;
        } else {
          ++n_cache;
        }
      } else {                                 // waited on, touched again (:438-446)
        uc = uc0 + n + waits_before + __popc(pb & lt) + 1;
        uses = 2;
        f = (uint8_t)(f & ~(KF_PENDING | KF_FROMPF));
        kc->flags[ci] = f;
        T.kflags[key] = f;
        ++n_reads;
        ++n_pf;
      }
      T.last_use[key] = uc;                    // _touch (:376-380)
      kc->freq[ci] += uses;
      T.freq[key] = kc->freq[ci];
      slots_out[i] = kc->slot[ci];
    }
    waits_before += __popc(pb);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    n_pf += __shfl_xor_sync(MS_FULL, n_pf, o);
    n_cache += __shfl_xor_sync(MS_FULL, n_cache, o);
    n_reads += __shfl_xor_sync(MS_FULL, n_reads, o);
  }
  if (lane == 0) {
    c->use_clock = uc0 + n + waits_before;
    c->st[ST_PREFETCH] += n_pf;
    c->st[ST_CACHE] += n_cache;
    c->st[ST_READS] += n_reads;
  }
  __syncwarp();
  return true;
}

// The whole table step of a block call -- prefetch of `np_` keys (one
// prefetch depth), then acquire of `na` keys, both sorted and distinct -- in
// the common case where no key needs a slot: every predicted key is resident
// or pending and every acquired key too. Then no slot changes hands and the
// reference's loops (prefetch engine_v3.py:383-396, acquire :398-454, the
// completion of the earlier prefetches at the end of the acquire) reduce to
// independent per-key updates: one round of loads (key states, counters, the
// previous pin list, the pending list), then stores. The use clock is
// reproduced by rank, as in warp_acquire_resident. Returns false, having
// written nothing, when some key needs a slot (or a list is longer than a
// warp): the caller then runs the sequential walk.
__device__ __forceinline__ bool warp_table_fast(const DevTable& T, const int* pkeys, int np_,
                                                const int* akeys, int na, int* slots_out,
                                                int lane) {
  if (np_ > 32 || na > 32) return false;
  // ---- one round of independent loads
  int ps = 0, as = -1, afr = 0, pin = -1, pend = -1;
  uint8_t pf = 0, af = 0;
  const int pk = lane < np_ ? pkeys[lane] : -1;
  const int ak = lane < na ? akeys[lane] : -1;
  if (pk >= 0) {
    ps = T.slot_of[pk];
    pf = T.kflags[pk];
  }
  if (ak >= 0) {
    as = T.slot_of[ak];
    af = T.kflags[ak];
    afr = T.freq[ak];
  }
  if (lane < T.n_slots) {
    pin = T.pin_list[lane];
    pend = T.pend_list[lane];
  }
  long long uc0 = 0;
  int n_pin = 0, n_pend = 0;
  if (lane == 0) {
    uc0 = T.ctr->use_clock;
    n_pin = T.ctr->n_pin;
    n_pend = T.ctr->n_pend;
  }
  uc0 = __shfl_sync(MS_FULL, uc0, 0);
  n_pin = __shfl_sync(MS_FULL, n_pin, 0);
  n_pend = __shfl_sync(MS_FULL, n_pend, 0);
  // ---- the common case?
  const bool p_need = pk >= 0 && ps < 0 && !(pf & KF_PENDING);
  const bool a_pend = ak >= 0 && (af & KF_PENDING) != 0;
  const bool a_need = ak >= 0 && !a_pend && as < 0;
  if (__any_sync(MS_FULL, p_need || a_need) || n_pin > 32 || n_pend > 32) return false;
  // ---- acquire: every item touched in item order, then each waited-on
  // pending item once more, in item order (engine_v3.py:412-446)
  const unsigned lt = (1u << lane) - 1u;
  const unsigned pb = __ballot_sync(MS_FULL, a_pend);
  const int n_wait = __popc(pb);
  int n_pf = 0, n_cache = 0, n_reads = 0;
  if (ak >= 0) {
    long long uc = uc0 + lane + 1;
    uint8_t f = af;
    int uses = 1;
    if (!a_pend) {
      if (f & KF_FROMPF) {                     // first use of a prefetched key (:431-435)
        f = (uint8_t)(f & ~KF_FROMPF);
        ++n_pf;
      } else {
        ++n_cache;
      }
    } else {                                   // waited on, touched again (:438-446)
      uc = uc0 + na + __popc(pb & lt) + 1;
      uses = 2;
      f = (uint8_t)(f & ~(KF_PENDING | KF_FROMPF));
      ++n_reads;
      ++n_pf;
    }
    if (f != af) T.kflags[ak] = f;
    T.last_use[ak] = uc;                       // _touch (:376-380)
    T.freq[ak] = afr + uses;
    slots_out[lane] = as;
  }
  // ---- pinned = set(slots) (:452-453): the previous pins go, this call's
  // slots come (distinct keys, distinct slots)
  if (lane < n_pin) T.pinned[pin] = 0;
  __syncwarp();
  if (ak >= 0) {
    T.pinned[as] = 1;
    T.pin_list[lane] = as;
  }
  // ---- the earlier prefetches that were not waited on complete now:
  // pending -> from_prefetch (a pending key's flags are exactly PENDING)
  bool waited = false;
  for (int i = 0; i < na; ++i) {
    const int ki = __shfl_sync(MS_FULL, ak, i);
    waited |= (ki == pend) && ((pb >> i) & 1u);
  }
  int n_done = 0;
  if (lane < n_pend && !waited) {
    T.kflags[pend] = KF_FROMPF;
    n_done = 1;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    n_pf += __shfl_xor_sync(MS_FULL, n_pf, o);
    n_cache += __shfl_xor_sync(MS_FULL, n_cache, o);
    n_reads += __shfl_xor_sync(MS_FULL, n_reads, o);
    n_done += __shfl_xor_sync(MS_FULL, n_done, o);
  }
  if (lane == 0) {
    TableCtr* c = T.ctr;
    c->use_clock = uc0 + na + n_wait;
    c->n_pend = 0;
    c->n_pin = na;
    c->n_fill = 0;
    c->n_fill_pf = 0;
    c->st[ST_PREFETCH] += n_pf;
    c->st[ST_CACHE] += n_cache;
    c->st[ST_READS] += n_reads + n_done;
  }
  __syncwarp();
  return true;
}

// acquire (engine_v3.py:398-454) of request r. slots_out[i] receives the
// slot of item i (-1 if exhausted before it was placed). waits: scratch of
// r.n ints. Returns 0 or MS_E_EXHAUSTED (-3).
__device__ __forceinline__ int warp_acquire(const DevTable& T, OpCtx* c, KeyCache* kc, const Req& r,
                            int* slots_out, int* waits, int lane) {
  const int n = r.n;
  int n_wait = 0, n_issue = 0, status = 0;
  for (int i = lane; i < n; i += 32) slots_out[i] = -1;
  __syncwarp();
  const bool resident = warp_acquire_resident(T, c, kc, r, slots_out, lane);
  for (int i = 0; i < (resident ? 0 : n); ++i) {
    const int ci = r.ci[i];
    int pend = 0, slot = -1;
    if (lane == 0) {                         // lane 0 decides, the warp follows
      pend = (kc->flags[ci] & KF_PENDING) != 0;
      slot = kc->slot[ci];
    }
    pend = __shfl_sync(MS_FULL, pend, 0);
    slot = __shfl_sync(MS_FULL, slot, 0);
    bool issued_now = false;
    if (!pend && slot < 0) {
      __syncwarp();                          // lane 0's writes before the collective scan
      slot = kc_alloc(T, c, kc, ci, lane);
      if (slot < 0) { status = -3; break; }
      if (lane == 0) {
        pin0(T, c, kc, ci);
        touch0(T, c, kc, ci);
        add_fill0(T, c, slot, kc->key[ci]);
      }
      ++n_issue;
      issued_now = true;
    } else if (slot >= 0) {
      if (lane == 0) { pin0(T, c, kc, ci); touch0(T, c, kc, ci); }
    }
    if (lane == 0) {
      if (pend) {
        waits[n_wait] = i;
      } else if (slot >= 0 && !issued_now) {
        const bool early = (kc->flags[ci] & KF_FROMPF) != 0;
        if (early) setflags0(T, kc, ci, (uint8_t)(kc->flags[ci] & ~KF_FROMPF));
        c->st[early ? ST_PREFETCH : ST_CACHE] += 1;
        slots_out[i] = slot;
      }
      if (issued_now) slots_out[i] = slot;
    }
    if (pend) ++n_wait;
  }
  __syncwarp();
  if (status == 0) {
    if (lane == 0 && !resident) {
      c->st[ST_EXPOSED] += n_issue;
      c->st[ST_READS] += n_issue;
      for (int w = 0; w < n_wait; ++w) {            // (:438-446)
        const int i = waits[w];
        const int ci = r.ci[i];
        if (kc->flags[ci] & KF_PENDING) c->st[ST_READS] += 1;
        setflags0(T, kc, ci, (uint8_t)(kc->flags[ci] & ~(KF_PENDING | KF_FROMPF)));
        slots_out[i] = kc->slot[ci];
        pin0(T, c, kc, ci);
        touch0(T, c, kc, ci);
        c->st[ST_PREFETCH] += 1;
      }
      c->st[ST_MISS] += n_issue;
    }
    __syncwarp();
    // pinned = set(slots) (:452-453): unpin every slot on the list, then pin
    // the slots of this request's distinct keys
    // the list holds the previous acquire's slots (loaded up front) plus the
    // slots pinned in this call, which all belong to cache entries
    const int np = c->n_pin;
    const int npp = kc->n_prev_pin;
    if (npp <= KC_MAX) {
      for (int i = lane; i < npp; i += 32) T.pinned[kc->prev_pin[i]] = 0;
      for (int i = lane; i < kc->n; i += 32)
        if (kc->pin[i] && kc->slot[i] >= 0) T.pinned[kc->slot[i]] = 0;
    } else {
      for (int i = lane; i < np; i += 32) T.pinned[T.pin_list[i]] = 0;
    }
    __syncwarp();
    for (int i = lane; i < kc->n; i += 32) kc->pin[i] = 0;
    __syncwarp();
    for (int e = lane; e < r.n_uniq; e += 32) {
      const int ci = r.base + e;
      const int s = kc->slot[ci];
      T.pin_list[e] = s;
      T.pinned[s] = 1;
      kc->pin[ci] = 1;
    }
    __syncwarp();
    if (lane == 0) c->n_pin = r.n_uniq;
  } else if (lane == 0) {
    c->status = status;
  }
  __syncwarp();
  warp_drain(T, c, kc, lane);
  return status;
}

}  // namespace ms
