"""CPU tests of the C-ABI boundary: the library builds for sm_100a, loads,
and exports exactly what include/moestream.h declares. No compute calls."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"^\s*int\s+(ms_\w+)\s*\(", src, flags=re.M))
    return names


def test_header_declares_the_boundary():
    d = declared()
    for need in ("ms_pool_create", "ms_pool_destroy", "ms_store_register", "ms_pool_prefetch",
                 "ms_pool_acquire", "ms_pool_stats", "ms_pool_slot_table",
                 "ms_pool_component_ptr", "ms_route", "ms_moe_block", "ms_last_error"):
        assert need in d


def test_library_loads_and_exports_every_declared_symbol(lib):
    from moe_stream_b200 import _lib
    for name in declared():
        assert hasattr(lib, name), name
        assert name in _lib.EXPORTS, f"{name} has no ctypes declaration"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T (ms_\w+)", out))
    assert declared() <= exported


@pytest.mark.gpu
def test_library_is_sm100a_code(lib, cuda):
    """The kernels the library loads on the device are sm_100 code
    (cudaFuncGetAttributes binaryVersion of the route step)."""
    from moe_stream_b200 import _lib
    v = ctypes.c_int(0)
    assert lib.ms_kernel_arch(0, ctypes.byref(v)) == _lib.MS_OK, _lib.last_error()
    assert v.value == 100


def test_errors_are_status_codes_not_exceptions(lib):
    """Argument errors come back as MS_E_INVALID with a message, without a
    GPU being touched."""
    from moe_stream_b200 import _lib, geometry
    h = ctypes.c_void_p()
    cfg = _lib.MsPoolConfig()
    cfg.n_slots = 0
    g = geometry.qwen3().to_c()
    rc = lib.ms_pool_create(ctypes.byref(g), ctypes.byref(cfg), 0, ctypes.byref(h))
    assert rc == _lib.MS_E_INVALID
    assert "n_slots" in _lib.last_error()
    g.bits = 3
    cfg.n_slots = 4
    rc = lib.ms_pool_create(ctypes.byref(g), ctypes.byref(cfg), 0, ctypes.byref(h))
    assert rc == _lib.MS_E_INVALID and "4-bit" in _lib.last_error()
    assert lib.ms_pool_destroy(None) == _lib.MS_OK


def test_every_entry_point_rejects_a_null_handle(lib):
    """Each exported call given a NULL pool (and NULL pointers) returns
    MS_E_INVALID with a message, on a machine without a GPU."""
    from moe_stream_b200 import _lib
    ints = (ctypes.c_int, ctypes.c_int32, ctypes.c_long, ctypes.c_longlong, ctypes.c_size_t)
    # ms_expert_mlp_static_status takes only a stream (NULL is the default
    # stream), so it has no NULL handle to reject
    skip = {"ms_last_error", "ms_pool_create", "ms_pool_destroy", "ms_expert_mlp_static_status"}
    checked = 0
    for name, argtypes in _lib.EXPORTS.items():
        if name in skip:
            continue
        args = [0 if a in ints else (0.0 if a in (ctypes.c_float, ctypes.c_double) else None)
                for a in argtypes]
        rc = getattr(lib, name)(*args)
        assert rc == _lib.MS_E_INVALID, (name, rc)
        assert "NULL" in _lib.last_error(), (name, _lib.last_error())
        checked += 1
    assert checked >= 20
