"""The expert-parallel exchange protocol (moe_stream_b200.ep.ep_forward) on
CPU ranks over gloo, world 2 and 4.

The device operations are replaced by CPU stand-ins with the same contracts
(routing, destination-major packing, k = 1 expert rows, combine), computed
by the oracle. The protocol -- count exchange, split sizes, row and metadata
all-to-alls, the return trip and the combine through pair_pos -- must then
reproduce the single-process oracle block exactly: every row is computed on
its own, so sharding the experts changes no bit of the output.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from moe_stream_b200 import geometry, store as S
from oracle import bf16 as OB
from oracle import moe as OM

SEED = 7


def _geom():
    # gpt-oss arithmetic (top-4 then softmax, biases, clamped SwiGLU) at a
    # size the oracle handles in seconds
    return geometry.make("gptoss", 256, 256, 8, 1, 4, False)


def _inputs(geom, T):
    w, b = S.router_weights(geom, SEED, 0, bias_std=0.5)
    x = S.rms_norm_tokens(T, geom.d_model, seed=SEED + 1)
    blobs = {e: S.make_blob(geom, SEED, 0, e).numpy() for e in range(geom.n_experts)}
    return w, b, x, blobs


class OracleOps:
    """CPU stand-ins for the four device operations of ep_forward, with the
    device pack's dispatch rule: pair p of expert e goes to replica
    p % n_rep(e) of the placement table."""

    def __init__(self, geom, rank, world, w, b, blobs, plan=None):
        from moe_stream_b200.ep import shard_placement
        self.geom, self.rank, self.world = geom, rank, world
        self.table, slots = plan if plan is not None else shard_placement(geom.n_experts, world)
        self.w = w.float().numpy()
        self.b = None if b is None else b.float().numpy()
        self.comps = [dict(c) for c in geom.components]
        self.local = {i: blobs[e] for i, e in enumerate(slots[rank])}

    def route(self, x):
        inds, scores, _ = OM.route_gptoss(x.float().numpy(), self.w, self.geom.top_k, self.b)
        return torch.from_numpy(inds.astype(np.int32)), torch.from_numpy(scores.astype(np.float32))

    def pack(self, x, inds, scores):
        T, k = inds.shape
        flat = inds.reshape(-1).numpy()
        rep = np.arange(T * k) % self.table[flat, 0]
        dest = self.table[flat, 1 + 2 * rep]
        slot = self.table[flat, 2 + 2 * rep]
        order = np.argsort(dest, kind="stable")          # pair index for each send row
        pair_pos = np.empty(T * k, np.int32)
        pair_pos[order] = np.arange(T * k, dtype=np.int32)
        send_x = x[torch.from_numpy(order // k)]
        meta = np.empty((T * k, 2), np.int32)
        meta[:, 0] = slot[order]
        meta[:, 1] = scores.reshape(-1).numpy()[order].view(np.int32)
        counts = np.bincount(dest, minlength=self.world).astype(np.int32)
        return send_x, torch.from_numpy(meta), torch.from_numpy(counts), torch.from_numpy(pair_pos)

    def experts(self, recv_x, recv_meta):
        n = recv_x.shape[0]
        if n == 0:
            return recv_x.new_empty(recv_x.shape)
        meta = recv_meta.numpy()
        slots = meta[:, 0:1].astype(np.int64)
        scores = meta[:, 1:2].copy().view(np.float32)
        y = OM.expert_block(recv_x.float().numpy(), slots, scores, self.local, self.comps, "gptoss")
        return torch.from_numpy(np.asarray(y, np.float32)).to(torch.bfloat16)

    def combine(self, back, pair_pos, T):
        k = self.geom.top_k
        rows = back.float()[pair_pos.long()].reshape(T, k, -1)
        return torch.from_numpy(OB.r(rows.numpy().sum(axis=1, dtype=np.float32))).to(torch.bfloat16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _skewed_plan(geom, world):
    """A placement with replicas: the planner on skewed counts, two spare
    slots per rank."""
    from moe_stream_b200.ep import plan_placement
    counts = np.array([40.0 / (e + 1) for e in range(geom.n_experts)])
    return plan_placement(counts, world, geom.n_experts // world + 2)


def _rank_main(rank, world, port, T, out_dir, replicated):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from moe_stream_b200.ep import ep_forward
        geom = _geom()
        w, b, x, blobs = _inputs(geom, T)
        shard = T // world
        plan = _skewed_plan(geom, world) if replicated else None
        ops = OracleOps(geom, rank, world, w, b, blobs, plan)
        y = ep_forward(x[rank * shard:(rank + 1) * shard], ops, world)
        torch.save(y, os.path.join(out_dir, f"y{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,replicated", [(2, False), (4, False), (4, True)])
def test_ep_protocol_matches_single_process_oracle(world, replicated, tmp_path):
    T = 24
    mp.start_processes(_rank_main, args=(world, _free_port(), T, str(tmp_path), replicated),
                       nprocs=world, start_method="spawn")
    y = torch.cat([torch.load(tmp_path / f"y{r}.pt") for r in range(world)]).float().numpy()
    geom = _geom()
    w, b, x, blobs = _inputs(geom, T)
    inds, scores, _ = OM.route_gptoss(x.float().numpy(), w.float().numpy(), geom.top_k,
                                      b.float().numpy())
    ref = OM.expert_block(x.float().numpy(), inds, scores, blobs,
                          [dict(c) for c in geom.components], "gptoss")
    assert np.array_equal(y, np.asarray(ref, np.float32))


def test_ep_pack_contract():
    """The stand-in's packing obeys the contract the device pack follows:
    rows destination-major, counts per destination, pair_pos the row of each
    pair, metadata (slot on the destination, score bits)."""
    geom = _geom()
    w, b, x, blobs = _inputs(geom, 10)
    plan = _skewed_plan(geom, 4)
    ops = OracleOps(geom, 0, 4, w, b, blobs, plan)
    inds, scores = ops.route(x)
    send_x, meta, counts, pair_pos = ops.pack(x, inds, scores)
    flat = inds.reshape(-1).numpy()
    starts = np.concatenate([[0], np.cumsum(counts.numpy())[:-1]])
    table, slots = plan
    for p in range(flat.size):
        pos = int(pair_pos[p])
        j = p % table[flat[p], 0]
        dest, slot = table[flat[p], 1 + 2 * j], table[flat[p], 2 + 2 * j]
        assert starts[dest] <= pos < starts[dest] + counts[dest]
        assert int(meta[pos, 0]) == slot
        assert slots[dest][slot] == flat[p]
        assert np.int32(meta[pos, 1]).view(np.float32) == scores.reshape(-1)[p].item()
        assert torch.equal(send_x[pos], x[p // geom.top_k])


def test_plan_placement_balances_and_covers():
    from moe_stream_b200.ep import plan_placement
    counts = np.array([1000, 400, 200, 100] + [50] * 12, np.float64)
    table, slots = plan_placement(counts, 4, 6)
    assert all(len(r) <= 6 for r in slots)
    assert (table[:, 0] >= 1).all()
    for e in range(16):                        # replicas on distinct ranks, consistent slots
        ranks = [table[e, 1 + 2 * j] for j in range(table[e, 0])]
        assert len(set(ranks)) == len(ranks)
        for j in range(table[e, 0]):
            assert slots[table[e, 1 + 2 * j]][table[e, 2 + 2 * j]] == e
    load = [sum(counts[e] / table[e, 0] for e in r) for r in slots]
    assert max(load) <= 1.1 * counts.sum() / 4


def _withholding_rank(rank, world, port, out_dir):
    """Rank 1 never sends its pair counts (it stops before the first
    exchange, as a failed rank would); rank 0 must get an error from the
    process group's timeout instead of waiting forever."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    geom = _geom()
    w, b, x, blobs = _inputs(geom, 8)
    result = os.path.join(out_dir, "rank0.txt")
    if rank == 0:
        from moe_stream_b200.ep import ep_forward
        ops = OracleOps(geom, rank, world, w, b, blobs)
        t0 = time.monotonic()
        try:
            ep_forward(x[:4], ops, world)
            msg = "completed"
        except RuntimeError as e:
            msg = f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}: {e}"
        with open(result + ".tmp", "w") as f:
            f.write(msg)
        os.replace(result + ".tmp", result)
    else:
        # the failed rank: no collective at all; it leaves once rank 0 has
        # recorded what it saw (at most 60 s)
        t0 = time.monotonic()
        while not os.path.exists(result) and time.monotonic() - t0 < 60:
            time.sleep(0.1)
    # no destroy_process_group: its barrier would wait on the broken group


def test_ep_rank_that_withholds_its_counts_times_out(tmp_path):
    mp.start_processes(_withholding_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn")
    msg = (tmp_path / "rank0.txt").read_text()
    assert msg.startswith("error after"), msg
    secs = float(msg.split()[2])
    assert 2.0 <= secs <= 30.0, msg


def test_c_abi_group_id_from_run_time_nccl():
    """ms_ep_unique_id reaches NCCL through the library's run-time loader
    (no GPU needed): 128-byte ids, a new one per call. Run in a child process
    so NCCL's bootstrap thread stays out of the test process."""
    import subprocess
    import sys
    code = ("from moe_stream_b200.ep import ep_unique_id\n"
            "a, b = ep_unique_id(), ep_unique_id()\n"
            "assert len(a) == len(b) == 128 and a != b and any(a)\n"
            "print('ok')\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
