"""Deterministic restatement of ``ExpertPool``'s slot bookkeeping
(engine_v3.py:125-464). Test infrastructure only.

Follows the reference line by line:
  * ``_alloc``   engine_v3.py:313-374 -- free list popped from the END; once
    it is empty, a sampled scan from ``clock % n`` with stride 7919 that skips
    empty, pinned and pending slots, scores lfu=freq / lru=last_use / asis=0
    plus 1<<30 for entries younger than the protect window (24 * depth,
    :310-311), keeps the first-seen strict minimum, and stops once SAMPLE (24)
    candidates were seen and the best is not young. The victim's freq, born,
    last_use and from_prefetch entries are dropped.
  * ``_touch``   engine_v3.py:376-380
  * ``prefetch`` engine_v3.py:383-396 (bails, and stops, on exhaustion)
  * ``acquire``  engine_v3.py:398-454, including the double touch of a key
    that is still pending and the final ``pinned = set(slots)``.
  * ``stats``    engine_v3.py:456-464 (the timing fields are not modelled).

Timing is removed by one rule: a prefetch read stays pending until the end of
the next ``acquire`` call (or until an ``acquire`` waits on it), at which
point it completes -- pending is cleared and the key joins from_prefetch, as
``_read_task``'s finally block does (engine_v3.py:292-301). This is the rule
the golden fixtures were generated under and the rule the device table
implements.
"""

SAMPLE = 24
STRIDE = 7919
YOUNG = 1 << 30


class PoolExhausted(RuntimeError):
    pass


class PoolSim:
    def __init__(self, n_slots, n_experts, evict="lfu", depth=1, blob=1):
        self.n_slots = n_slots
        self.n_experts = n_experts
        self.evict = evict
        self.window = 24 * max(1, depth)
        self.blob = blob
        self.key_of = [None] * n_slots
        self.slot_of = {}
        self.freq = {}
        self.born = {}
        self.last_use = {}
        self.free = list(range(n_slots))
        self.pending = []          # issue order
        self.from_prefetch = set()
        self.pinned = set()
        self.clock = 0
        self.use_clock = 0
        self.n_prefetch_hit = 0
        self.n_cache_hit = 0
        self.n_miss = 0
        self.n_prefetch_bail = 0
        self.n_prefetch_issued = 0
        self.n_reads = 0
        self.n_exposed = 0

    # engine_v3.py:313-374
    def _alloc(self, key):
        self.clock += 1
        if self.free:
            slot = self.free.pop()
        else:
            n = self.n_slots
            start = self.clock % n
            best = victim = None
            seen = 0
            pend = set(self.pending)
            for j in range(n):
                sidx = (start + j * STRIDE) % n
                k = self.key_of[sidx]
                if k is None or sidx in self.pinned or k in pend:
                    continue
                young = self.clock - self.born.get(k, 0) < self.window
                if self.evict == "asis":
                    base = 0
                elif self.evict == "lru":
                    base = self.last_use.get(k, 0)
                else:
                    base = self.freq.get(k, 0)
                f = base + (YOUNG if young else 0)
                if best is None or f < best:
                    best, victim = f, sidx
                seen += 1
                if seen >= SAMPLE and best is not None and best < YOUNG:
                    break
            if victim is None:
                raise PoolExhausted("pool exhausted: every slot pinned or pending")
            vk = self.key_of[victim]
            self.from_prefetch.discard(vk)
            self.born.pop(vk, None)
            self.last_use.pop(vk, None)
            self.freq.pop(vk, None)
            del self.slot_of[vk]
            slot = victim
        self.key_of[slot] = key
        self.slot_of[key] = slot
        self.born[key] = self.clock
        return slot

    # engine_v3.py:376-380
    def _touch(self, key):
        self.use_clock += 1
        self.last_use[key] = self.use_clock
        self.freq[key] = self.freq.get(key, 0) + 1

    def _complete(self, key):
        """_read_task's finally block (engine_v3.py:298-301)."""
        if key in self.pending:
            self.pending.remove(key)
            self.n_reads += 1
        self.from_prefetch.add(key)

    # engine_v3.py:383-396
    def prefetch(self, layer, experts):
        fills = []
        for e in experts:
            key = layer * self.n_experts + int(e)
            if key in self.slot_of or key in self.pending:
                continue
            try:
                slot = self._alloc(key)
            except PoolExhausted:
                self.n_prefetch_bail += 1
                return fills
            self.n_prefetch_issued += 1
            self.pending.append(key)
            fills.append((slot, key))
        return fills

    # engine_v3.py:398-454
    def acquire(self, layer, experts):
        """Returns (slots, fills); raises PoolExhausted like the reference.
        Outstanding prefetch reads complete when the call ends, also when it
        raises."""
        try:
            return self._acquire(layer, experts)
        finally:
            for key in list(self.pending):
                self._complete(key)

    def _acquire(self, layer, experts):
        n = len(experts)
        slots = [None] * n
        waits, issue = [], []
        for i, e in enumerate(experts):
            key = layer * self.n_experts + int(e)
            pend = key in self.pending
            slot = self.slot_of.get(key)
            issued_now = False
            if not pend and slot is None:
                slot = self._alloc(key)
                self.pinned.add(slot)
                self._touch(key)
                issue.append((i, key, slot))
                issued_now = True
            elif slot is not None:
                self.pinned.add(slot)
                self._touch(key)
            if pend:
                waits.append((i, key))
            elif slot is not None and not issued_now:
                early = key in self.from_prefetch
                self.from_prefetch.discard(key)
                self.n_prefetch_hit += 1 if early else 0
                self.n_cache_hit += 0 if early else 1
                slots[i] = slot
            if issued_now:
                slots[i] = slot
        self.n_exposed += len(issue)
        self.n_reads += len(issue)
        for i, key in waits:
            self._complete(key)
            self.from_prefetch.discard(key)
            slots[i] = self.slot_of[key]
            self.pinned.add(slots[i])
            self._touch(key)
            self.n_prefetch_hit += 1
        self.n_miss += len(issue)
        self.pinned = set(s for s in slots if s is not None)
        return slots, [(s, k) for _, k, s in issue]

    def stats(self):
        tot = self.n_prefetch_hit + self.n_cache_hit + self.n_miss
        return dict(total=tot, prefetch=self.n_prefetch_hit, cache=self.n_cache_hit,
                    miss=self.n_miss, bail=self.n_prefetch_bail,
                    issued=self.n_prefetch_issued,
                    gb=self.n_reads * self.blob / 2 ** 30,
                    exposed_gb=self.n_exposed * self.blob / 2 ** 30)

    def table(self):
        """key per slot (layer*n_experts+expert), -1 for an empty slot."""
        return [-1 if k is None else k for k in self.key_of]
