"""GPU test of ms_expert_mlp_static, the expert MLP for callers that may not
allocate device memory when they run it (runtimes that reserve all memory up
front and lend plugins only planned buffers, enqueue steps that must not
allocate). It takes the expert weights and the inputs from the caller and
keeps its intermediates in a fixed array inside the library.

The test calls it through the C ABI twice in a row -- different tokens,
experts and token counts, so the second call starts from the first call's
leftovers in the shared array -- and checks each output against the pool
entry point ms_expert_mlp on the same inputs, within the parity tolerance the
other GPU tests use. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry, store as S

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-2


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("model", ["qwen3", "gptoss"])
def test_static_scratch_matches_pool_entry_point(model, lib, cuda):
    from moe_stream_b200 import _lib
    from moe_stream_b200.block import expert_mlp
    from moe_stream_b200.pool import ExpertPool

    geom = geometry.qwen3(n_layers=1) if model == "qwen3" else geometry.gptoss(n_layers=1)
    k = geom.top_k
    n_exp = 10
    pool = ExpertPool(geom, n_exp, max_tokens=8)
    try:
        st = pool.alloc_store(n_exp).reshape(n_exp, geom.blob_bytes)
        for e in range(n_exp):
            st[e] = S.make_blob(geom, 21, 0, e, device="cuda").cpu().numpy()
            pool._read(e, 0, e)                  # slot e holds expert e
        torch.cuda.synchronize()
        g = geom.to_c()
        rng = np.random.default_rng(3)
        for call, T in enumerate((1, 5) if model == "qwen3" else (2, 3)):
            inds = np.stack([rng.choice(n_exp, size=k, replace=False) for _ in range(T)])
            slots = torch.from_numpy(inds.astype(np.int32)).cuda()
            raw = rng.random((T, k)).astype(np.float32) + 0.1
            scores = torch.from_numpy(raw / raw.sum(-1, keepdims=True)).cuda()
            x = S.rms_norm_tokens(T, geom.d_model, seed=40 + call, device="cuda")
            want = expert_mlp(pool, slots, x, scores)
            got = torch.full_like(x, float("nan"))
            rc = lib.ms_expert_mlp_static(ctypes.byref(g), ctypes.c_void_p(pool.arena_ptr),
                                          n_exp, _ptr(slots), _ptr(scores), _ptr(x), T, k,
                                          _ptr(got),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert rc == _lib.MS_OK, _lib.last_error()
            torch.cuda.synchronize()
            a = got.float().cpu().numpy()
            b = want.float().cpu().numpy()
            assert np.isfinite(a).all(), f"call {call}"
            assert np.abs(a - b).max() <= MAX_ABS, f"call {call}"
            assert np.abs(a - b).mean() / (np.abs(b).mean() + 1e-30) <= MEAN_REL, f"call {call}"
    finally:
        pool.close()


def test_static_scratch_rejects_oversized_calls(lib, cuda):
    from moe_stream_b200 import _lib
    geom = geometry.qwen3(n_layers=1)
    g = geom.to_c()
    T = 17                                       # above the 16-token limit
    x = torch.zeros(T, geom.d_model, dtype=torch.bfloat16, device="cuda")
    y = torch.empty_like(x)
    slots = torch.zeros(T, geom.top_k, dtype=torch.int32, device="cuda")
    scores = torch.zeros(T, geom.top_k, dtype=torch.float32, device="cuda")
    rc = lib.ms_expert_mlp_static(ctypes.byref(g), _ptr(x), 4, _ptr(slots), _ptr(scores), _ptr(x),
                                  T, geom.top_k, _ptr(y), None)
    assert rc == _lib.MS_E_INVALID
    assert "MS_STATIC_MAX_TOKENS" in _lib.last_error()
