"""Tests of ms_expert_mlp_static, the expert MLP for callers that may not
allocate device memory when they run it (runtimes that reserve all memory up
front and lend plugins only planned buffers, enqueue steps that must not
allocate). It takes the expert weights and the inputs from the caller and
keeps its intermediates in a fixed array inside the library.

The GPU tests call it through the C ABI twice in a row -- different tokens,
experts and token counts, so the second call starts from the first call's
leftovers in the shared array -- and check each output against the pool
entry point ms_expert_mlp on the same inputs, and one batch-1 call against
the CPU oracle, within the parity tolerance the other GPU tests use; a slot
index out of range must come back as zero rows plus MS_E_INVALID from
ms_expert_mlp_static_status. The CPU tests check that every limit is refused
with MS_E_INVALID before anything touches a GPU. This file is collected last
on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from moe_stream_b200 import geometry, store as S

MAX_ABS = 2e-2
MEAN_REL = 1e-2


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _pool_with_experts(geom, n_exp, seed):
    from moe_stream_b200.pool import ExpertPool
    pool = ExpertPool(geom, n_exp, max_tokens=8)
    st = pool.alloc_store(n_exp).reshape(n_exp, geom.blob_bytes)
    for e in range(n_exp):
        st[e] = S.make_blob(geom, seed, 0, e, device="cuda").cpu().numpy()
        pool._read(e, 0, e)                      # slot e holds expert e
    torch.cuda.synchronize()
    return pool, st


def _call_static(lib, g, arena_ptr, n_slots, slots, scores, x, T, k, y):
    return lib.ms_expert_mlp_static(ctypes.byref(g), ctypes.c_void_p(arena_ptr), n_slots,
                                    _ptr(slots), _ptr(scores), _ptr(x), T, k, _ptr(y), _stream())


@pytest.mark.gpu
@pytest.mark.parametrize("model", ["qwen3", "gptoss"])
def test_static_scratch_matches_pool_entry_point(model, lib, cuda):
    from moe_stream_b200 import _lib
    from moe_stream_b200.block import expert_mlp

    geom = geometry.qwen3(n_layers=1) if model == "qwen3" else geometry.gptoss(n_layers=1)
    if model == "gptoss":
        # the decode kernels take gpt-oss shapes up to 3072 wide
        assert geom.d_model <= 3072
    k = geom.top_k
    n_exp = 10
    pool, _ = _pool_with_experts(geom, n_exp, 21)
    try:
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
            rc = _call_static(lib, g, pool.arena_ptr, n_exp, slots, scores, x, T, k, got)
            assert rc == _lib.MS_OK, _lib.last_error()
            assert lib.ms_expert_mlp_static_status(_stream()) == _lib.MS_OK, _lib.last_error()
            a = got.float().cpu().numpy()
            b = want.float().cpu().numpy()
            assert np.isfinite(a).all(), f"call {call}"
            assert np.abs(a - b).max() <= MAX_ABS, f"call {call}"
            assert np.abs(a - b).mean() / (np.abs(b).mean() + 1e-30) <= MEAN_REL, f"call {call}"
    finally:
        pool.close()


@pytest.mark.gpu
def test_static_scratch_matches_oracle_and_reports_bad_slots(lib, cuda):
    """One batch-1 Qwen3 call against the CPU oracle's MLX-path block, then a
    call with one slot out of range: that token's expert contributes zeros,
    the other experts still count, and the status call reports MS_E_INVALID
    once (it clears the status)."""
    from moe_stream_b200 import _lib
    from oracle import bf16 as OB
    from oracle import moe as OM
    geom = geometry.qwen3(n_layers=1)
    k, n_exp = geom.top_k, 9
    pool, st = _pool_with_experts(geom, n_exp, 33)
    try:
        g = geom.to_c()
        comps = [dict(c) for c in geom.components]
        rng = np.random.default_rng(8)
        inds = rng.choice(n_exp, size=(1, k), replace=False).astype(np.int32)
        raw = rng.random((1, k)).astype(np.float32) + 0.1
        sc = OB.r(raw / raw.sum(-1, keepdims=True))
        x = S.rms_norm_tokens(1, geom.d_model, seed=91, device="cuda")
        xn = x.float().cpu().numpy()
        blobs = {e: st[e] for e in range(n_exp)}
        slots = torch.from_numpy(inds).cuda()
        scores = torch.from_numpy(sc).cuda()
        y = torch.empty_like(x)
        assert _call_static(lib, g, pool.arena_ptr, n_exp, slots, scores, x, 1, k, y) == _lib.MS_OK
        assert lib.ms_expert_mlp_static_status(_stream()) == _lib.MS_OK, _lib.last_error()
        want = OM.expert_block(xn, inds, sc, blobs, comps, "qwen3")
        got = y.float().cpu().numpy()
        assert np.abs(got - want).max() <= MAX_ABS
        assert np.abs(got - want).mean() / (np.abs(want).mean() + 1e-30) <= MEAN_REL
        # slot n_exp does not exist: expert j = 3 must drop out of the sum
        bad = inds.copy()
        bad[0, 3] = n_exp
        slots_bad = torch.from_numpy(bad).cuda()
        y2 = torch.empty_like(x)
        assert _call_static(lib, g, pool.arena_ptr, n_exp, slots_bad, scores, x, 1, k, y2) == _lib.MS_OK
        assert lib.ms_expert_mlp_static_status(_stream()) == _lib.MS_E_INVALID
        assert "outside" in _lib.last_error()
        assert lib.ms_expert_mlp_static_status(_stream()) == _lib.MS_OK    # cleared
        keep = [j for j in range(k) if j != 3]
        want2 = OM.expert_block(xn, inds[:, keep], sc[:, keep], blobs, comps, "qwen3")
        got2 = y2.float().cpu().numpy()
        assert np.abs(got2 - want2).max() <= MAX_ABS
    finally:
        pool.close()


# ------------------------------------------------------------------ limits
# Argument checks run before any CUDA call, so these need no GPU: the
# pointers are stand-in addresses that are never dereferenced.
ALIGNED, MISALIGNED = 0x10000, 0x10008


def _reject(lib, g, *, arena=ALIGNED, n_slots=4, T=1, k=None, x=ALIGNED, y=ALIGNED):
    from moe_stream_b200 import _lib
    k = g.top_k if k is None else k
    rc = lib.ms_expert_mlp_static(ctypes.byref(g), ctypes.c_void_p(arena), n_slots,
                                  ctypes.c_void_p(ALIGNED), ctypes.c_void_p(ALIGNED),
                                  ctypes.c_void_p(x), T, k, ctypes.c_void_p(y), None)
    return rc, _lib.last_error()


def _overlong_component(g):
    # the down-projection weights start one page before the end of the blob
    g.comp_offset[2][0] = g.blob_bytes - 16384
    return g


@pytest.mark.parametrize("case,edit,want", [
    ("tokens", dict(T=17), "MS_STATIC_MAX_TOKENS"),
    ("pairs", dict(T=9), "MS_STATIC_MAX_PAIRS"),
    ("slots", dict(n_slots=65537), "MS_STATIC_MAX_SLOTS"),
    ("no_slots", dict(n_slots=0), "MS_STATIC_MAX_SLOTS"),
    ("k", dict(k=4), "top_k"),
    ("x_align", dict(x=MISALIGNED), "aligned"),
    ("y_align", dict(y=MISALIGNED), "aligned"),
    ("arena_align", dict(arena=MISALIGNED), "aligned"),
])
def test_static_rejects_limits(case, edit, want, lib):
    from moe_stream_b200 import _lib
    g = geometry.qwen3(n_layers=1).to_c()
    rc, msg = _reject(lib, g, **edit)
    assert rc == _lib.MS_E_INVALID, (case, msg)
    assert want in msg, (case, msg)


@pytest.mark.parametrize("case", ["overlong", "misaligned", "missing", "gptoss_wide", "bits"])
def test_static_rejects_bad_geometry(case, lib):
    from moe_stream_b200 import _lib
    if case == "gptoss_wide":
        g = geometry.make("gptoss", 3136, 2880, 128, 1, 4, False).to_c()
    else:
        g = geometry.qwen3(n_layers=1).to_c()
    if case == "overlong":
        _overlong_component(g)
    elif case == "misaligned":
        g.comp_offset[1][1] += 8
    elif case == "missing":
        g.comp_offset[0][2] = -1
    elif case == "bits":
        g.bits = 8
    rc, msg = _reject(lib, g)
    assert rc == _lib.MS_E_INVALID, (case, msg)
    assert msg.startswith("ms_expert_mlp_static:"), msg
