"""ExpertPool: the reference's slot pool (engine_v3.py:125-464) on B200.

Same public surface -- ``prefetch(layer, experts)``, ``acquire(layer,
experts) -> [slot]``, ``stats()``, ``views[name]``, ``_read(slot, layer,
expert)``, ``key_of``, ``slot_of``, ``n_slots``, ``blob``, ``group_size``,
``bits``, ``n_layers``, ``n_experts``, ``top_k`` -- over a different
machine:

* the slots are one contiguous HBM arena (slot s at s*blob_bytes, laid out as
  a store blob), not one MLX array per component; offsets are 64-bit, which
  removes by construction the int32 wrap the reference fixed at
  engine_v3.py:144-167;
* the store is pinned, device-mapped host memory; fills are copies issued on
  the GPU (the SMs read the mapped store), so no host thread and no host
  round trip sit between a table decision and its fill;
* the LFU table (freq / born / last_use / pending / from_prefetch / pinned,
  clocks and counters) lives in device memory and is updated by one warp per
  call, in exactly the reference's order;
* the prefetch fills of a block call run on a stream of the pool and are
  joined into the caller's stream by the next call that reads the arena. A
  caller that reads ``views`` itself right after block calls makes its
  stream wait for them first (``join(stream)``, or a device-wide
  synchronisation), as the reference's readers wait on ``pending`` reads.

Everything here is a thin ctypes wrapper over libmoestream.so; there is no
Python or CPU implementation of any of it.
"""
import ctypes
import json
import os

import numpy as np
import torch

from . import _lib
from .geometry import PROJS, PARTS, Geometry, from_index, to_prec_c


def _stream_ptr(stream):
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class _DevArray:
    """__cuda_array_interface__ over arena memory, so torch can view it."""

    def __init__(self, ptr, shape, typestr, strides):
        self.__cuda_array_interface__ = dict(shape=tuple(shape), typestr=typestr,
                                             data=(ptr, False), strides=tuple(strides),
                                             version=3)


_TYPESTR = {"U32": ("<u4", torch.int32, 4), "BF16": ("<u2", torch.bfloat16, 2)}


class ExpertPool:
    """Fixed HBM pool of expert slots with device-side LFU residency."""

    def __init__(self, geom: Geometry, n_slots, evict="lfu", depths=(1,), pf_widen=1,
                 max_tokens=16, device=None, store=None):
        self._lib = _lib.load()
        if device is None:
            device = torch.cuda.current_device()
        self.device = int(device)
        self.geom = geom
        self.blob = geom.blob_bytes
        self.n_experts = geom.n_experts
        self.n_layers = geom.n_layers
        self.top_k = geom.top_k
        self.group_size = geom.group_size
        self.bits = geom.bits
        self.n_slots = int(n_slots)
        self.payload = geom.payload_bytes
        self.pad = self.blob - self.payload
        self.evict = evict
        self.depths = tuple(depths)
        self.pf_widen = pf_widen
        self.max_tokens = max_tokens
        # stream ordering replaces the reference's per-layer barrier
        # (engine_v3.py:228-231, 601-607): a slot is refilled only after the
        # kernels that read it, so no barrier is ever needed
        self.needs_barrier = False
        cfg = _lib.MsPoolConfig()
        cfg.n_slots = self.n_slots
        cfg.evict = _lib.EVICT[evict]
        cfg.n_depths = len(self.depths)
        for i, d in enumerate(self.depths):
            cfg.depths[i] = d
        cfg.pf_widen = pf_widen
        cfg.max_tokens = max_tokens
        self._geom_c = geom.to_c()
        h = ctypes.c_void_p()
        _lib.check(self._lib.ms_pool_create(ctypes.byref(self._geom_c), ctypes.byref(cfg),
                                            self.device, ctypes.byref(h)))
        self._h = h
        base, size = ctypes.c_void_p(), ctypes.c_size_t()
        _lib.check(self._lib.ms_pool_arena(h, ctypes.byref(base), ctypes.byref(size)))
        self.arena_ptr, self.pool_bytes = base.value, size.value
        self.views = self._make_views()
        self.store = None
        if store is not None:
            self.attach_store(store)

    # ------------------------------------------------------------- store
    def alloc_store(self, n_blobs=None):
        """Pinned, device-mapped host store for n_blobs blobs (default: every
        (layer, expert)); returns it as a numpy uint8 array to be filled."""
        n_blobs = self.geom.n_keys if n_blobs is None else n_blobs
        nbytes = n_blobs * self.blob
        p = ctypes.c_void_p()
        _lib.check(self._lib.ms_store_alloc(self._h, nbytes, ctypes.byref(p)))
        buf = (ctypes.c_uint8 * nbytes).from_address(p.value)
        self.store = np.frombuffer(buf, dtype=np.uint8)
        return self.store

    def attach_store(self, arr):
        """Register an existing host array (numpy uint8) as the store."""
        arr = np.ascontiguousarray(arr, dtype=np.uint8)
        _lib.check(self._lib.ms_store_register(self._h, ctypes.c_void_p(arr.ctypes.data), arr.nbytes))
        self.store = arr
        return arr

    @classmethod
    def open(cls, model_dir, model, d_model, d_ff, n_slots, cold=False, **kw):
        """Pool over an on-disk store (experts_index.json + experts.bin,
        repack.py:137-146): the whole file is read once into the pinned,
        device-mapped store with preadv (engine_v3.py:255-290). cold=True
        reads with O_DIRECT, past the OS page cache -- the Linux form of the
        reference's F_NOCACHE cold-cache mode (engine_v3.py:138-142); the
        pinned store is page aligned and blobs are whole 16 KiB pages, as
        O_DIRECT requires. A filesystem without O_DIRECT raises OSError."""
        idx = json.load(open(os.path.join(model_dir, "experts_index.json")))
        geom = from_index(idx, model, d_model, d_ff)
        path = os.path.join(model_dir, "experts.bin")
        size = os.path.getsize(path)
        if size % geom.blob_bytes:
            raise IOError(f"{path}: {size} bytes is not a whole number of {geom.blob_bytes}-byte blobs")
        n_blobs = size // geom.blob_bytes
        flags = os.O_RDONLY | (os.O_DIRECT if cold else 0)
        fd = os.open(path, flags)
        try:
            pool = cls(geom, n_slots, **kw)
            store = pool.alloc_store(n_blobs)
            mv = memoryview(store)
            off, step = 0, 1 << 28
            while off < n_blobs * geom.blob_bytes:
                got = os.preadv(fd, [mv[off:off + step]], off)
                if got <= 0:
                    raise IOError(f"short read at {off} of {path}")
                off += got
        finally:
            os.close(fd)
        return pool

    def write_store(self, model_dir):
        """Write the attached store as experts.bin + experts_index.json in the
        reference's on-disk format (repack.py:137-146), readable by open()."""
        os.makedirs(model_dir, exist_ok=True)
        with open(os.path.join(model_dir, "experts_index.json"), "w") as f:
            json.dump(self.geom.index(), f, indent=2)
        with open(os.path.join(model_dir, "experts.bin"), "wb") as f:
            f.write(memoryview(self.store))

    # ------------------------------------------------------------- views
    def _make_views(self):
        views = {}
        for proj_i, proj in enumerate(PROJS):
            for part_i, part in enumerate(PARTS):
                try:
                    c = self.geom.comp(proj, part)
                except KeyError:
                    continue
                typestr, tdt, isz = _TYPESTR[c["dtype"]]
                shape = [self.n_slots, *c["shape"]]
                inner = []
                acc = isz
                for s in reversed(c["shape"]):
                    inner.insert(0, acc)
                    acc *= s
                strides = [self.blob, *inner]
                arr = _DevArray(self.arena_ptr + c["offset"], shape, typestr, strides)
                t = torch.as_tensor(arr, device=f"cuda:{self.device}")
                views[f"{proj}.{part}"] = t.view(tdt) if tdt == torch.bfloat16 else t.view(torch.int32)
        return views

    # ------------------------------------------------------- reference API
    def prefetch(self, layer, experts, stream=None):
        """Non-blocking (engine_v3.py:383-396)."""
        e = np.ascontiguousarray(np.asarray(experts, dtype=np.int32).reshape(-1))
        _lib.check(self._lib.ms_pool_prefetch(
            self._h, int(layer), e.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), e.size,
            _stream_ptr(stream)))

    def acquire(self, layer, experts, stream=None):
        """Blocking: the slot of each expert (engine_v3.py:398-454). Raises
        PoolExhausted (a RuntimeError) like the reference."""
        e = np.ascontiguousarray(np.asarray(experts, dtype=np.int32).reshape(-1))
        out = np.empty(e.size, dtype=np.int32)
        _lib.check(self._lib.ms_pool_acquire(
            self._h, int(layer), e.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), e.size,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _stream_ptr(stream)))
        return [int(s) for s in out]

    def _read(self, slot, layer, expert, stream=None):
        """Copy blob (layer, expert) into slot, bypassing the table
        (engine_v3.py:255-290)."""
        _lib.check(self._lib.ms_pool_read(self._h, int(slot), int(layer), int(expert),
                                          _stream_ptr(stream)))

    def stats(self):
        """engine_v3.py:456-464; blocked/busy_s/depth are host timings of the
        reference's I/O threads and have no counterpart (reported as 0)."""
        s = _lib.MsStats()
        _lib.check(self._lib.ms_pool_stats(self._h, ctypes.byref(s)))
        return dict(total=s.total, prefetch=s.prefetch, cache=s.cache, miss=s.miss,
                    blocked=0.0, gb=s.bytes_read / 2 ** 30, busy_s=0.0, depth=0.0,
                    bail=s.bail, issued=s.issued, exposed_gb=s.bytes_exposed / 2 ** 30,
                    reads=s.reads)

    def table(self):
        """Slot -> key (layer*n_experts+expert, -1 empty) as an int32 array."""
        out = np.empty(self.n_slots, dtype=np.int32)
        _lib.check(self._lib.ms_pool_slot_table(self._h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out

    @property
    def key_of(self):
        """engine_v3.py:216: (layer, expert) per slot, None when empty."""
        return [None if k < 0 else (int(k) // self.n_experts, int(k) % self.n_experts)
                for k in self.table()]

    @property
    def slot_of(self):
        """engine_v3.py:215: {(layer, expert): slot}."""
        return {(int(k) // self.n_experts, int(k) % self.n_experts): s
                for s, k in enumerate(self.table()) if k >= 0}

    def set_precision(self, classes, class_of_key):
        """Per-expert precision: blob (layer, expert) is stored as precision
        class classes[class_of_key[layer * n_experts + expert]] (geometries
        from geometry.precision of this pool's geometry; the pool's blob
        stride must hold the largest, see geometry.slot_geometry). Call
        before the first slot fill. Store blobs keep the pool's stride; each
        holds its class's payload from its start."""
        classes = list(classes)
        arr = (_lib.MsPrec * len(classes))(*[to_prec_c(c) for c in classes])
        cok = np.ascontiguousarray(class_of_key, dtype=np.uint8)
        if cok.size != self.geom.n_keys:
            raise ValueError(f"class_of_key has {cok.size} entries, the pool {self.geom.n_keys} keys")
        _lib.check(self._lib.ms_pool_set_precision(self._h, len(classes), ctypes.byref(arr),
                                                   ctypes.c_void_p(cok.ctypes.data)))
        self.classes = classes
        self.class_of_key = cok.copy()

    def status(self, stream=None):
        """Raise the first device-side error of earlier asynchronous calls."""
        _lib.check(self._lib.ms_pool_status(self._h, _stream_ptr(stream)))

    def join(self, stream=None):
        """Make `stream` wait for the prefetch fills still running on the
        pool's side stream (needed before ending a graph capture)."""
        _lib.check(self._lib.ms_pool_join(self._h, _stream_ptr(stream)))

    # ------------------------------------------------------- checkpoints
    def save_state(self, with_arena=True, stream=None):
        """Snapshot of the pool (slot table, clocks, counters and, with_arena,
        the slot contents) as a device uint8 tensor; ``load_state`` puts it
        back, after which the pool continues exactly as it did from here."""
        n = ctypes.c_size_t()
        _lib.check(self._lib.ms_pool_state_bytes(self._h, int(with_arena), ctypes.byref(n)))
        buf = torch.empty(n.value, dtype=torch.uint8, device=f"cuda:{self.device}")
        _lib.check(self._lib.ms_pool_save_state(self._h, ctypes.c_void_p(buf.data_ptr()),
                                                int(with_arena), _stream_ptr(stream)))
        return buf

    def load_state(self, buf, with_arena=True, stream=None):
        _lib.check(self._lib.ms_pool_load_state(self._h, ctypes.c_void_p(buf.data_ptr()),
                                                int(with_arena), _stream_ptr(stream)))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self.views = {}
            self._lib.ms_pool_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
