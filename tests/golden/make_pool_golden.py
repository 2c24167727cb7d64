#!/usr/bin/env python3
"""Generate ``pool_golden.json`` by running the reference's own ExpertPool.

The slot pool of moe-stream (engine_v3.py:125-464) is pure Python apart from
where it stores bytes: MLX arrays made by ``mx.zeros`` and the host address
``mlx_zerocopy_ext.data_ptr`` returns. MLX is not installed here, so this
script puts minimal numpy-backed stand-ins for those imports into
``sys.modules`` (nothing of the pool's logic is replaced), builds a tiny
expert store on disk, and drives the UNMODIFIED ``engine_v3.ExpertPool`` --
its ``prefetch``, ``acquire``, ``_alloc``, ``_touch``, ``_read`` and
``_read_task`` -- through seeded engine-like sequences.

The only timing rule: the worker pool is replaced by a deferred executor, so
a read runs when ``acquire`` waits on it, and every other outstanding read
runs when the ``acquire`` call ends. Under that rule the pool's tables are a
pure function of the call sequence, which is what the fixture records: after
every call, the returned slots, the slot -> key table, the hit/miss/bail
counters and the bytes each slot holds.

Run in a container that has the reference checked out:
    python tests/golden/make_pool_golden.py /path/to/reference
It writes tests/golden/pool_golden.json. The GPU tests never read the
reference; they read only that JSON file.
"""
import importlib
import json
import os
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PAGE = 16384


# --------------------------------------------------------------- stand-ins
def _aligned_zeros(shape, dtype):
    n = int(np.prod(shape)) * np.dtype(dtype).itemsize
    raw = np.zeros(n + PAGE, dtype=np.uint8)
    off = (-raw.ctypes.data) % PAGE
    return raw[off:off + n].view(dtype).reshape(shape)


def install_stubs():
    core = types.ModuleType("mlx.core")
    core.uint32 = np.uint32
    core.bfloat16 = np.uint16          # the pool only stores bits
    core.zeros = lambda shape, dtype=np.float32: _aligned_zeros(tuple(shape), dtype)
    core.eval = lambda *a, **k: None
    nn = types.ModuleType("mlx.nn")
    mlx = types.ModuleType("mlx")
    mlx.core, mlx.nn = core, nn
    sys.modules.update({"mlx": mlx, "mlx.core": core, "mlx.nn": nn})

    lm = types.ModuleType("mlx_lm")
    models = types.ModuleType("mlx_lm.models")
    q3 = types.ModuleType("mlx_lm.models.qwen3_moe")
    act = types.ModuleType("mlx_lm.models.activations")
    act.swiglu = None
    cache = types.ModuleType("mlx_lm.models.cache")
    cache.make_prompt_cache = None
    tok = types.ModuleType("mlx_lm.tokenizer_utils")
    tok.load = None
    models.qwen3_moe = q3
    lm.models = models
    sys.modules.update({"mlx_lm": lm, "mlx_lm.models": models,
                        "mlx_lm.models.qwen3_moe": q3,
                        "mlx_lm.models.activations": act,
                        "mlx_lm.models.cache": cache,
                        "mlx_lm.tokenizer_utils": tok})

    zc = types.ModuleType("mlx_zerocopy_ext")
    zc.data_ptr = lambda a: a.ctypes.data
    zc.page_size = lambda: PAGE
    sys.modules["mlx_zerocopy_ext"] = zc


class DeferredFuture:
    def __init__(self, fn, args):
        self.fn, self.args, self.done = fn, args, False

    def result(self):
        if not self.done:
            self.done = True
            self.fn(*self.args)


class DeferredExecutor:
    def __init__(self):
        self.queue = []

    def submit(self, fn, *args):
        f = DeferredFuture(fn, args)
        self.queue.append(f)
        return f

    def drain(self):
        q, self.queue = self.queue, []
        for f in q:
            f.result()


# ------------------------------------------------------------- tiny store
def make_store(root, n_layers, n_experts):
    """A miniature store with the real component order (repack.py:72-82)
    and a page-padded blob, filled with bytes that identify (layer, expert)."""
    comps, off = [], 0
    for proj in ("gate_proj", "up_proj", "down_proj"):
        for part, dt, shape, nb in (("weight", "U32", [4, 2], 32),
                                    ("scales", "BF16", [4, 1], 8),
                                    ("biases", "BF16", [4, 1], 8)):
            comps.append(dict(proj=proj, part=part, dtype=dt, shape=shape,
                              offset=off, nbytes=nb))
            off += nb
    blob = 256                                   # 144 B payload + 112 B pad
    idx = dict(n_layers=n_layers, n_experts=n_experts, top_k=4,
               blob_bytes=blob, payload_bytes=off, page_size=PAGE,
               quantization=dict(group_size=64, bits=4), components=comps)
    with open(os.path.join(root, "experts_index.json"), "w") as f:
        json.dump(idx, f)
    data = np.zeros((n_layers * n_experts, blob), np.uint8)
    for key in range(n_layers * n_experts):
        data[key] = (np.arange(blob) * 7 + key * 13) % 251
    data.tofile(os.path.join(root, "experts.bin"))
    return data


# ---------------------------------------------------------------- driver
def run_scenario(ref, name, evict, depth, n_slots, n_layers, n_experts, steps,
                 k, kp, p_extra, seed):
    os.environ["MOE_EVICT"] = evict
    os.environ["PF_DEPTH"] = str(depth)
    os.environ["MOE_STAGE"] = "1"
    for m in ("engine_v3", "kernels"):
        sys.modules.pop(m, None)
    sys.path.insert(0, ref)
    try:
        E = importlib.import_module("engine_v3")
    finally:
        sys.path.remove(ref)

    root = tempfile.mkdtemp(prefix="poolgold_")
    data = make_store(root, n_layers, n_experts)
    pool = E.ExpertPool(root, n_slots=n_slots, n_workers=1)
    pool.pool.shutdown(wait=True)
    ex = DeferredExecutor()
    pool.pool = ex

    rng = np.random.default_rng(seed)
    # skewed per-layer popularity so that some experts recur
    pop = rng.permutation(n_experts)
    prob = 1.0 / np.arange(1, n_experts + 1) ** 1.1
    prob /= prob.sum()
    weights = np.empty(n_experts)
    weights[pop] = prob

    def draw(n):
        return sorted(int(e) for e in rng.choice(n_experts, size=n, replace=False, p=weights))

    ops = []

    def snapshot(op, layer, experts, result):
        st = pool.stats()
        held = []
        for s in range(n_slots):
            key = pool.key_of[s]
            if key is None:
                held.append(-1)
            else:
                held.append(key[0] * n_experts + key[1])
        # bytes check: every filled, non-pending slot holds its key's blob,
        # except slots an exhausted acquire allocated and never read
        # (engine_v3.py:410-419 raises before submitting its reads)
        stale = []
        for s in range(n_slots):
            key = pool.key_of[s]
            if key is None or key in pool.pending:
                continue
            got = np.concatenate([np.asarray(mv).view(np.uint8).reshape(-1)
                                  for mv in pool.slots_mv[s]])
            want = data[key[0] * n_experts + key[1]]
            if not np.array_equal(got, want):
                stale.append(s)
        assert not stale or name.endswith("exhaust"), (name, stale)
        ops.append(dict(op=op, layer=layer, experts=experts, result=result,
                        table=held, stale=stale,
                        counters=[st["prefetch"], st["cache"], st["miss"],
                                  st["bail"], st["issued"],
                                  int(round(st["gb"] * 2 ** 30 / pool.blob))],
                        clock=pool.clock, use_clock=pool.use_clock))

    for step in range(steps):
        for layer in range(n_layers):
            for d in range(1, depth + 1):
                if layer + d < n_layers:
                    pr = draw(kp)
                    pool.prefetch(layer + d, pr)
                    snapshot("prefetch", layer + d, pr, None)
            if rng.random() < p_extra:
                # a prefetch of THIS layer right before its acquire: the
                # acquire then finds some keys still pending and waits
                pr = draw(kp)
                pool.prefetch(layer, pr)
                snapshot("prefetch", layer, pr, None)
            want = draw(k)
            try:
                res = [int(s) for s in pool.acquire(layer, want)]
            except RuntimeError:
                res = "exhausted"
            ex.drain()
            snapshot("acquire", layer, want, res)
    fin = dict(freq={f"{a * n_experts + b}": v for (a, b), v in pool.freq.items() if v},
               born={f"{a * n_experts + b}": v for (a, b), v in pool.born.items()},
               last_use={f"{a * n_experts + b}": v for (a, b), v in pool.last_use.items()},
               from_prefetch=sorted(a * n_experts + b for a, b in pool.from_prefetch),
               pinned=sorted(int(s) for s in pool.pinned))
    return dict(name=name, evict=evict, depth=depth, n_slots=n_slots,
                n_layers=n_layers, n_experts=n_experts, k=k, kp=kp,
                ops=ops, final=fin)


SCENARIOS = [
    # name, evict, depth, n_slots, n_layers, n_experts, steps, k, kp, p_extra, seed
    ("lfu_d1", "lfu", 1, 40, 6, 16, 14, 4, 4, 0.0, 1),
    ("lru_d1", "lru", 1, 40, 6, 16, 14, 4, 4, 0.0, 2),
    ("asis_d1", "asis", 1, 40, 6, 16, 14, 4, 4, 0.0, 3),
    ("lfu_d2", "lfu", 2, 48, 6, 16, 12, 4, 4, 0.0, 4),
    ("lfu_wide_pending", "lfu", 1, 36, 6, 16, 14, 4, 8, 0.35, 5),
    ("lru_wide_pending", "lru", 1, 36, 6, 16, 12, 4, 8, 0.35, 6),
    ("lfu_exhaust", "lfu", 1, 11, 4, 16, 12, 4, 4, 0.3, 7),
    ("lfu_big_sample", "lfu", 1, 97, 8, 16, 10, 4, 6, 0.1, 8),
]


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOE_STREAM_REF", "")
    if not os.path.exists(os.path.join(ref, "engine_v3.py")):
        sys.exit("usage: make_pool_golden.py <reference checkout>")
    install_stubs()
    out = dict(generator="tests/golden/make_pool_golden.py",
               source="engine_v3.ExpertPool (engine_v3.py:125-464), run unmodified",
               rule="reads complete when acquire waits on them or when acquire returns",
               scenarios=[run_scenario(ref, *s) for s in SCENARIOS])
    path = os.path.join(HERE, "pool_golden.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    n = sum(len(s["ops"]) for s in out["scenarios"])
    print(f"wrote {path}: {len(out['scenarios'])} scenarios, {n} calls")


if __name__ == "__main__":
    main()
