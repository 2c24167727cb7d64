"""Expert parallelism on real GPUs: two NCCL ranks, each holding half of a
gpt-oss-shaped layer's experts (plain sharding, and a placement that
replicates the hottest experts into spare slots), run the expert-parallel
block on their half of the tokens; the gathered output must equal, bit for
bit, one GPU running the whole layer through ms_moe_block (every row is
computed by the same kernels in the same order either way). Needs two GPUs;
skipped otherwise.
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


def _rank_main(rank, world, port, out_dir, replicated):
    import datetime
    import torch.distributed as dist
    from moe_stream_b200 import geometry, store as S
    from moe_stream_b200.block import MoEBlock
    from moe_stream_b200.ep import (DeviceOps, ep_forward, load_local_experts, plan_placement,
                                    routed_counts)
    from moe_stream_b200.pool import ExpertPool
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
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
        shard = T // world
        xr = x[rank * shard:(rank + 1) * shard].contiguous()
        if replicated:
            table, slots = plan_placement(routed_counts(DeviceOps(block, world), xr), world,
                                          E // world + spare)
            load_local_experts(pool, 0, rank, world, slots[rank])
            ops = DeviceOps(block, world, placement=table)
        else:
            load_local_experts(pool, 0, rank, world)
            ops = DeviceOps(block, world)
        y = ep_forward(xr, ops, world)
        torch.cuda.synchronize()
        pool.status()
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y)
        if rank == 0:
            torch.save(torch.cat(parts).cpu(), os.path.join(out_dir, "y_ep.pt"))
            # the whole layer on one GPU
            ref_pool = ExpertPool(geom, E, depths=(), max_tokens=T)
            rs = torch.from_numpy(ref_pool.alloc_store()).view(geom.n_keys, geom.blob_bytes)
            rs.copy_(blobs)
            y_ref = MoEBlock(ref_pool, 0, w, b)(x)
            torch.cuda.synchronize()
            ref_pool.status()
            torch.save(y_ref.cpu(), os.path.join(out_dir, "y_ref.pt"))
            ref_pool.close()
        dist.barrier()
        pool.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("replicated", [False, True])
def test_expert_parallel_matches_one_gpu(replicated, lib, cuda, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), replicated),
                       nprocs=world, start_method="spawn")
    y_ep = torch.load(tmp_path / "y_ep.pt")
    y_ref = torch.load(tmp_path / "y_ref.pt")
    assert torch.isfinite(y_ep.float()).all()
    assert torch.equal(y_ep, y_ref)
