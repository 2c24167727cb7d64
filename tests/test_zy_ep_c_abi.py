"""The expert-parallel block through the C ABI alone (ms_ep_init /
ms_ep_moe_block, ep.EpGroup): the library's own NCCL group, no
torch.distributed on the data path. Two ranks hold half of a gpt-oss-shaped
layer's experts each (plain sharding, and a placement with replicas) and
unequal shares of the tokens; the gathered output must equal one GPU running
the whole layer through ms_moe_block bit for bit, for a first call and a
larger second one. Needs two GPUs; skipped otherwise. Kept apart from
test_gpu_ep.py (the torch.distributed protocol) and collected late.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SEED = 11
E, T = 16, 512              # 2048 token/expert pairs: the grouped-GEMM path


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main_cabi(rank, world, port, out_dir, replicated):
    """The same layer through the C ABI's own NCCL group (EpGroup:
    ms_ep_init / ms_ep_moe_block); torch.distributed (gloo, CPU) only hands
    the NCCL id around and gathers the outputs. The ranks hold unequal
    token counts, and a second call at a larger size grows the scratch."""
    import datetime
    import torch.distributed as dist
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.ep import (DeviceOps, EpGroup, ep_unique_id, load_local_experts,
                                    plan_placement)
    from moe_stream_b200.pool import ExpertPool
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120))
    try:
        geom = geometry.make("gptoss", 2880, 2880, E, 1, 4, False)
        w, b = S.router_weights(geom, SEED, 0, zipf_s=1.1)
        x = S.rms_norm_tokens(T, geom.d_model, seed=SEED + 1, device="cuda")
        blobs = S.make_layer_blobs(geom, SEED, 0).cpu()
        spare = 4 if replicated else 0
        pool = ExpertPool(geom, E // world + spare, depths=(), max_tokens=T)
        st = torch.from_numpy(pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
        st.copy_(blobs)
        block = MoEBlock(pool, 0, w, b)
        cut = [0, T // 2 - 56, T]                   # unequal shares
        xr = x[cut[rank]:cut[rank + 1]].contiguous()
        table = None
        if replicated:
            inds, _ = DeviceOps(block, world).route(xr)
            c = torch.bincount(inds.reshape(-1).long().cpu(), minlength=E)
            dist.all_reduce(c)
            table, slots = plan_placement(c.numpy(), world, E // world + spare)
            load_local_experts(pool, 0, rank, world, slots[rank])
        else:
            load_local_experts(pool, 0, rank, world)
        uid = [ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        grp = EpGroup(block, uid[0], rank, world, placement=table)
        half = xr[: xr.shape[0] // 2].contiguous()
        y_half = grp(half)                          # a smaller call first
        y = grp(xr)                                 # then the full share: scratch grows
        torch.cuda.synchronize()
        pool.status()
        parts = [None] * world
        dist.all_gather_object(parts, (y.cpu(), y_half.cpu()))
        if rank == 0:
            torch.save(torch.cat([p[0] for p in parts]), os.path.join(out_dir, "y_ep.pt"))
            ref_pool = ExpertPool(geom, E, depths=(), max_tokens=T)
            rs = torch.from_numpy(ref_pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
            rs.copy_(blobs)
            ref = MoEBlock(ref_pool, 0, w, b)
            y_ref = ref(x)
            halves = [ref(x[cut[r]:cut[r] + (cut[r + 1] - cut[r]) // 2].contiguous()).cpu()
                      for r in range(world)]
            torch.cuda.synchronize()
            ref_pool.status()
            torch.save(y_ref.cpu(), os.path.join(out_dir, "y_ref.pt"))
            torch.save((torch.cat([p[1] for p in parts]), torch.cat(halves)),
                       os.path.join(out_dir, "halves.pt"))
            ref_pool.close()
        dist.barrier()
        grp.close()
        pool.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("replicated", [False, True])
def test_c_abi_expert_parallel_matches_one_gpu(replicated, lib, cuda, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.start_processes(_rank_main_cabi, args=(world, _free_port(), str(tmp_path), replicated),
                             nprocs=world, start_method="spawn", join=False)
    # the ranks get a deadline: a rank stuck in the library's NCCL calls must
    # fail this test, not stall the run (ending a process ends its GPU work)
    import time
    deadline = time.monotonic() + 900
    while not ctx.join(timeout=5):
        if time.monotonic() > deadline:
            for proc in ctx.processes:
                if proc.is_alive():
                    proc.kill()
            pytest.fail("the expert-parallel ranks did not finish within 900 s")
    y_ep = torch.load(tmp_path / "y_ep.pt")
    y_ref = torch.load(tmp_path / "y_ref.pt")
    assert torch.isfinite(y_ep.float()).all()
    assert torch.equal(y_ep, y_ref)
    got, want = torch.load(tmp_path / "halves.pt")
    assert torch.equal(got, want)
