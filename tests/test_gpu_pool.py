"""GPU tests of the slot pool through the C ABI.

* The device slot table replays every golden scenario -- fixtures made by
  running the reference's own ExpertPool -- and must agree call by call:
  returned slots, the whole slot -> key table and every counter.
* verify_pool.py's checks (verify_pool.py:54-92): byte-exact slot contents
  against the store, at both ends of an arena larger than 4 GiB, and live
  views.
"""
import json
import os

import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry
from moe_stream_b200._lib import PoolExhausted

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "pool_golden.json")))

pytestmark = pytest.mark.gpu


class _Raw:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = dict(shape=(n,), typestr="|u1", data=(ptr, False), version=3)


def arena_bytes(pool, slot):
    t = torch.as_tensor(_Raw(pool.arena_ptr + slot * pool.blob, pool.blob), device="cuda")
    return t.cpu().numpy()


def pattern_store(pool):
    store = pool.alloc_store()
    n = pool.geom.n_keys
    v = store.reshape(n, pool.blob)
    base = (np.arange(pool.blob, dtype=np.int64) * 7) % 251
    for key in range(n):
        v[key] = (base + key * 13) % 251
    return v


@pytest.mark.parametrize("sc", GOLDEN["scenarios"], ids=[s["name"] for s in GOLDEN["scenarios"]])
def test_device_table_matches_reference_expertpool(sc, lib, cuda):
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.make("qwen3", 64, 64, sc["n_experts"], sc["n_layers"], sc["k"])
    pool = ExpertPool(geom, sc["n_slots"], evict=sc["evict"], depths=(sc["depth"],), max_tokens=1)
    store = pattern_store(pool)
    try:
        for i, o in enumerate(sc["ops"]):
            if o["op"] == "prefetch":
                pool.prefetch(o["layer"], o["experts"])
                res = None
            else:
                try:
                    res = pool.acquire(o["layer"], o["experts"])
                except PoolExhausted:
                    res = "exhausted"
            assert res == o["result"], f"call {i} ({o['op']})"
            table = pool.table().tolist()
            assert table == o["table"], f"call {i} ({o['op']}) slot table"
            st = pool.stats()
            got = [st["prefetch"], st["cache"], st["miss"], st["bail"], st["issued"], st["reads"]]
            assert got == o["counters"], f"call {i} counters"
            if o["op"] == "acquire" and i % 7 == 0:
                # every resident slot holds its key's blob, byte for byte
                for s, key in enumerate(table):
                    if key >= 0:
                        assert np.array_equal(arena_bytes(pool, s), store[key]), (i, s, key)
    finally:
        pool.close()


def test_pool_bytes_and_liveness_past_4gib(lib, cuda):
    """verify_pool.py:54-92 on an arena where slot offsets exceed 2^32: every
    tested slot matches a direct read of the store, a refilled slot's view
    changes (views are live, not copies), and the views' element counts are
    64-bit safe."""
    from moe_stream_b200 import store as S
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.qwen3(n_layers=2)
    n = 1700                                     # 4.51 GB arena
    pool = ExpertPool(geom, n, max_tokens=1)
    try:
        assert pool.pool_bytes > 2 ** 32
        st = pool.alloc_store().reshape(geom.n_keys, geom.blob_bytes)
        for key in (7, 11, 128 + 9, 128 + 11):
            st[key] = S.make_blob(geom, 0, key // 128, key % 128, device="cuda").cpu().numpy()
        tested = sorted({0, 1, n // 2, n - 2, n - 1})
        for s in tested:
            pool._read(s, 0, 7)
        torch.cuda.synchronize()
        for s in tested:
            assert np.array_equal(arena_bytes(pool, s), st[7]), s
        v = pool.views["gate_proj.scales"]
        first = v[n - 1].clone()
        pool._read(n - 1, 1, 11)
        torch.cuda.synchronize()
        now = v[n - 1]
        c = geom.comp("gate_proj", "scales")
        want = torch.from_numpy(st[128 + 11][c["offset"]:c["offset"] + c["nbytes"]].copy()).view(torch.bfloat16)
        assert torch.equal(now.cpu().reshape(-1), want)
        assert not torch.equal(now, first)
        for name, t in pool.views.items():
            assert t.shape[0] == n
            assert t.data_ptr() >= pool.arena_ptr
    finally:
        pool.close()


def test_exhaustion_is_a_status_not_a_fault(lib, cuda):
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.make("qwen3", 64, 64, 16, 4, 4)
    pool = ExpertPool(geom, 4, max_tokens=1)
    pattern_store(pool)
    try:
        assert sorted(pool.acquire(0, [0, 1, 2, 3])) == [0, 1, 2, 3]
        with pytest.raises(PoolExhausted):
            pool.acquire(1, [4, 5, 6, 7])        # every slot pinned by layer 0
        with pytest.raises(RuntimeError):        # still a RuntimeError, as in the reference
            pool.acquire(1, [8])
    finally:
        pool.close()


def test_bad_arguments_raise(lib, cuda):
    from moe_stream_b200._lib import MoeStreamError
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.make("qwen3", 64, 64, 16, 4, 4)
    pool = ExpertPool(geom, 8, max_tokens=1)
    try:
        with pytest.raises(MoeStreamError):
            pool.acquire(0, [1])                 # no store yet
        pattern_store(pool)
        with pytest.raises(MoeStreamError):
            pool.acquire(9, [1])                 # layer out of range
        with pytest.raises(MoeStreamError):
            pool.prefetch(0, [16])               # expert out of range
        with pytest.raises(MoeStreamError):
            pool._read(8, 0, 0)                  # slot out of range
    finally:
        pool.close()


def test_bounded_wait_reports_timeout_and_pool_recovers(lib, cuda):
    """Failure detection without a GPU fault: a CTA waits, with the bounded
    wait every kernel uses, on an mbarrier that never completes. The wait
    gives up after its limit, ms_pool_status reports MS_E_TIMEOUT once, and
    the pool then serves a block call as before."""
    import ctypes
    import time
    from moe_stream_b200 import _lib, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.qwen3(1)
    pool = ExpertPool(geom, geom.n_experts, depths=(), max_tokens=1)
    try:
        st = pool.alloc_store()
        torch.from_numpy(st).view(geom.n_keys, geom.blob_bytes).copy_(
            S.make_layer_blobs(geom, 2, 0, device="cuda").cpu())
        blk = MoEBlock(pool, 0, *S.router_weights(geom, 2, 0))
        x = S.rms_norm_tokens(1, geom.d_model, seed=3, device="cuda")
        y0 = blk(x).clone()
        pool.status()
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        t0 = time.monotonic()
        assert lib.ms_pool_selftest_wait(pool._h, 50_000_000, stream) == _lib.MS_OK
        with pytest.raises(_lib.MoeStreamError) as err:
            pool.status()
        waited = time.monotonic() - t0
        assert err.value.code == _lib.MS_E_TIMEOUT
        assert 0.04 <= waited < 5.0
        pool.status()                             # reported once, then cleared
        torch.cuda.synchronize()
        # the same call again: same result (the block is deterministic)
        y1 = blk(x)
        pool.status()
        assert torch.equal(y0, y1)
    finally:
        pool.close()


@pytest.mark.parametrize("cold", [False, True])
def test_open_reads_a_store_in_the_reference_format(cold, lib, cuda, tmp_path):
    """ExpertPool.open on experts.bin + experts_index.json as repack.py
    writes them (repack.py:137-146): the store holds the file byte for byte,
    and acquired slots hold their blobs (verify_pool.py:64-76). cold=True
    reads with O_DIRECT."""
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.make("qwen3", 128, 64, 8, 2, 2)
    src = ExpertPool(geom, 2, max_tokens=1)
    try:
        pattern_store(src)
        src.write_store(str(tmp_path))
    finally:
        src.close()
    raw = np.fromfile(tmp_path / "experts.bin", dtype=np.uint8)
    idx = json.load(open(tmp_path / "experts_index.json"))
    assert idx["offset_formula"] == "(layer * n_experts + expert) * blob_bytes"
    try:
        pool = ExpertPool.open(str(tmp_path), "qwen3", geom.d_model, geom.d_ff, 6,
                               cold=cold, max_tokens=1)
    except OSError as e:
        if cold:
            pytest.skip(f"no O_DIRECT on this filesystem: {e}")
        raise
    try:
        assert pool.geom.blob_bytes == geom.blob_bytes and pool.geom.n_keys == geom.n_keys
        assert np.array_equal(pool.store, raw)
        slots = pool.acquire(1, [3, 5, 7])
        torch.cuda.synchronize()
        for e, s in zip((3, 5, 7), slots):
            key = 1 * geom.n_experts + e
            assert np.array_equal(arena_bytes(pool, s), raw[key * pool.blob:(key + 1) * pool.blob])
    finally:
        pool.close()
