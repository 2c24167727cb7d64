"""Errors that the device reports instead of passing on silently.

* fp16 range guard: the expert kernels take x and the SwiGLU output h as
  fp16 tensor-core operands. A value beyond the fp16 range (|v| > 65504)
  would enter them as inf; the writer of the fp16 copy records MS_E_RANGE in
  the pool status instead (ms_pool_status raises it once and clears it). The
  cases reach each writer: x in the decode frag layout and in the prefill
  scatter, h in the decode k_up epilogue and in the prefill GEMM epilogue.
* bounded host waits: with MS_HOST_WAIT_S shorter than a device-side wait
  that is running (the bounded self-test wait), the host call gives up with
  MS_E_TIMEOUT instead of blocking; the device wait then ends by itself.

No case faults or hangs the GPU: every overflow is an ordinary float value,
and the only long wait is the self-test's, bounded on the device.
"""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from moe_stream_b200 import _lib, geometry, store as S

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def layer_pool():
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.pool import ExpertPool
    geom = geometry.qwen3(n_layers=1)
    pool = ExpertPool(geom, geom.n_experts, depths=(), max_tokens=256)
    st = pool.alloc_store()
    torch.from_numpy(st).view(geom.n_keys, geom.blob_bytes).copy_(
        S.make_layer_blobs(geom, 5, 0, device="cuda").cpu())
    blk = MoEBlock(pool, 0, *S.router_weights(geom, 5, 0))
    yield pool, blk, geom
    pool.close()


def _status_code(pool):
    try:
        pool.status()
        return _lib.MS_OK
    except _lib.MoeStreamError as e:
        return e.code


# T = 2: decode kernels (frag layout, k_up); T = 256: 2048 pairs, the
# grouped-GEMM path (scatter, GEMM epilogue)
@pytest.mark.parametrize("T", [2, 256])
@pytest.mark.parametrize("where", ["x", "h"])
def test_fp16_range_is_reported(where, T, layer_pool):
    pool, blk, geom = layer_pool
    x = S.rms_norm_tokens(T, geom.d_model, seed=7, device="cuda")
    blk(x)
    assert _status_code(pool) == _lib.MS_OK
    if where == "x":
        bad = x.clone()
        bad[T - 1, 17] = 1.0e5                # one input beyond fp16
    else:
        # |x| stays far inside fp16 (<= ~1.5e3), but gate and up grow to
        # ~1e2..1e3 and their SwiGLU product past 65504
        bad = (x.float() * 300.0).to(torch.bfloat16)
        assert bad.abs().max().item() < 6e4
    blk(bad)
    assert _status_code(pool) == _lib.MS_E_RANGE
    assert "fp16 range" in _lib.last_error()
    assert _status_code(pool) == _lib.MS_OK       # reported once
    y = blk(x)                                    # a normal call is clean again
    assert _status_code(pool) == _lib.MS_OK
    assert torch.isfinite(y.float()).all()


def test_host_wait_gives_up_before_a_long_device_wait():
    """MS_HOST_WAIT_S=0.2 while the self-test kernel waits 1.5 s on the
    device: ms_pool_status returns MS_E_TIMEOUT after ~0.2 s; once the device
    wait has ended by itself the pool reports its own MS_E_TIMEOUT and then
    runs clean. Runs in a child process: the limit is read once."""
    code = textwrap.dedent(f"""
        import ctypes, sys, time
        sys.path.insert(0, {ROOT!r})
        import torch
        from moe_stream_b200 import _lib, geometry
        from moe_stream_b200.pool import ExpertPool
        geom = geometry.make("qwen3", 256, 128, 16, 1, 4)
        pool = ExpertPool(geom, 16, depths=(), max_tokens=1)
        lib = _lib.load()
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        pool.status()
        t0 = time.monotonic()
        assert lib.ms_pool_selftest_wait(pool._h, 1_500_000_000, s) == _lib.MS_OK
        rc = lib.ms_pool_status(pool._h, s)
        host = time.monotonic() - t0
        msg = _lib.last_error()
        torch.cuda.synchronize()
        dev = time.monotonic() - t0
        rc2 = lib.ms_pool_status(pool._h, s)
        rc3 = lib.ms_pool_status(pool._h, s)
        pool.close()
        print("RESULT", rc, round(host, 3), round(dev, 3), rc2, rc3, "|", msg)
    """)
    env = dict(os.environ, MS_HOST_WAIT_S="0.2")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    line = [l for l in out.stdout.splitlines() if l.startswith("RESULT")][-1]
    head, msg = line.split("|", 1)
    _, rc, host, dev, rc2, rc3 = head.split()
    assert int(rc) == _lib.MS_E_TIMEOUT and "did not finish" in msg, line
    assert 0.15 <= float(host) < 1.0, line
    assert float(dev) >= 1.4, line
    assert int(rc2) == _lib.MS_E_TIMEOUT      # the device wait's own record
    assert int(rc3) == _lib.MS_OK
