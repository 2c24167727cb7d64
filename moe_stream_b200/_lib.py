"""ctypes binding of libmoestream.so (include/moestream.h).

There is no fallback: if the shared library is missing or fails to load,
importing the package's GPU entry points raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoestream.so")

MS_OK = 0
MS_E_INVALID = -1
MS_E_CUDA = -2
MS_E_EXHAUSTED = -3
MS_E_TIMEOUT = -4
MS_E_NOMEM = -5
MS_E_STATE = -6
MS_E_IO = -7
MS_E_RANGE = -8

MODEL_QWEN3, MODEL_GPTOSS = 0, 1
SCALE_BF16, SCALE_FP8 = 0, 1
MAX_CLASSES = 8
EVICT = {"lfu": 0, "lru": 1, "asis": 2}
MAX_DEPTHS = 4


class MsGeom(ctypes.Structure):
    _fields_ = [("model", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("d_ff", ctypes.c_int32), ("n_experts", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("group_size", ctypes.c_int32), ("bits", ctypes.c_int32),
                ("norm_topk_prob", ctypes.c_int32), ("proj_bias", ctypes.c_int32),
                ("blob_bytes", ctypes.c_int64),
                ("comp_offset", (ctypes.c_int64 * 4) * 3)]


class MsPrec(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("scale_fmt", ctypes.c_int32),
                ("payload_bytes", ctypes.c_int64),
                ("comp_offset", (ctypes.c_int64 * 6) * 3)]


class MsPoolConfig(ctypes.Structure):
    _fields_ = [("n_slots", ctypes.c_int32), ("evict", ctypes.c_int32),
                ("n_depths", ctypes.c_int32), ("depths", ctypes.c_int32 * MAX_DEPTHS),
                ("pf_widen", ctypes.c_int32), ("max_tokens", ctypes.c_int32)]


class MsStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in
                ("total", "prefetch", "cache", "miss", "bail", "issued", "reads",
                 "exposed", "bytes_read", "bytes_exposed")]


EXPORTS = {
    "ms_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "ms_pool_create": [ctypes.POINTER(MsGeom), ctypes.POINTER(MsPoolConfig), ctypes.c_int,
                       ctypes.POINTER(ctypes.c_void_p)],
    "ms_pool_destroy": [ctypes.c_void_p],
    "ms_store_register": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t],
    "ms_store_alloc": [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)],
    "ms_set_router": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    "ms_pool_prefetch": [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                         ctypes.c_int, ctypes.c_void_p],
    "ms_pool_acquire": [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                        ctypes.c_int, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p],
    "ms_pool_read": [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p],
    "ms_pool_stats": [ctypes.c_void_p, ctypes.POINTER(MsStats)],
    "ms_pool_slot_table": [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)],
    "ms_pool_component_ptr": [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                              ctypes.POINTER(ctypes.c_void_p)],
    "ms_pool_arena": [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                      ctypes.POINTER(ctypes.c_size_t)],
    "ms_route": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    "ms_moe_block": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                     ctypes.c_void_p, ctypes.c_void_p],
    "ms_pool_status": [ctypes.c_void_p, ctypes.c_void_p],
    "ms_pool_join": [ctypes.c_void_p, ctypes.c_void_p],
    "ms_expert_mlp": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    "ms_pool_profile": [ctypes.c_void_p, ctypes.c_int],
    "ms_pool_timing": [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)],
    "ms_expert_mlp_static": [ctypes.POINTER(MsGeom), ctypes.c_void_p, ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                             ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    "ms_expert_mlp_static_status": [ctypes.c_void_p],
    "ms_pool_state_bytes": [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t)],
    "ms_pool_save_state": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p],
    "ms_pool_load_state": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p],
    "ms_pool_selftest_wait": [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p],
    "ms_pool_set_precision": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    "ms_moe_block_fused": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                           ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    "ms_kernel_arch": [ctypes.c_int, ctypes.POINTER(ctypes.c_int)],
    "ms_block_debug": [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                       ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)],
    "ms_ep_pack": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p],
    "ms_ep_combine": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                      ctypes.c_void_p, ctypes.c_void_p],
    "ms_ep_unique_id": [ctypes.c_void_p],
    "ms_ep_init": [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int],
    "ms_ep_moe_block": [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                        ctypes.c_void_p, ctypes.c_void_p],
    "ms_ep_finalize": [ctypes.c_void_p],
}

_LIB = None


class MoeStreamError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{msg} (status {code})")
        self.code = code


class PoolExhausted(MoeStreamError):
    """The reference raises RuntimeError('pool exhausted: ...') here
    (engine_v3.py:355-356)."""


def load(path=LIB_PATH):
    """Load the shared library (once) and declare every exported symbol."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m moe_stream_b200.build`")
    lib = ctypes.CDLL(path)
    for name, argtypes in EXPORTS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    _LIB = lib
    return lib


def last_error():
    buf = ctypes.create_string_buffer(1024)
    load().ms_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc):
    if rc != MS_OK:
        msg = last_error()
        if rc == MS_E_EXHAUSTED:
            raise PoolExhausted(rc, msg)
        if rc == MS_E_IO:
            raise MoeStreamError(rc, "IOError: " + msg)
        raise MoeStreamError(rc, msg)
    return rc
