"""Expert parallelism for wide batches (the gpt-oss layer on 16384 tokens): the 128 experts
of a layer are sharded over the ranks of one node, expert e living on rank
e // e_local in slot e % e_local of that rank's pool, every rank holding its
experts resident. The reference runs on one device (its MoE block is
engine_120b.py:78-149); this is the multi-GPU form of the same block.

One forward, per rank, on its own T_r tokens:

  1. route the local tokens (ms_route, the tiled tensor-core router);
  2. pack the T_r * top_k token/expert pairs destination-major (ms_ep_pack):
     the token row, the expert's slot on the destination and the score;
  3. exchange the pair counts, then the rows and their metadata, with one
     NCCL all-to-all each (torch.distributed, one process per GPU);
  4. run the received rows through the local experts (ms_expert_mlp with
     k = 1: y = score * expert(x), the grouped tensor-core GEMM);
  5. return the rows with the reverse all-to-all;
  6. combine at the source (ms_ep_combine): y[t] = sum_j rows[pair_pos[t, j]]
     in fp32 in j order, rounded once to bf16, as the single-device block.

Every row is computed on its own by the same kernels as on one device, so
the output equals the single-device block's bit for bit.

Placement. Plain sharding puts expert e on rank e // e_local. Under skewed
routing (config 4's Zipf(1.1) router bias) the hottest expert alone takes
more than a rank's share of the pairs, so `plan_placement` gives each rank a
few spare slots, replicates the experts with the largest load per replica
into them, and assigns every replica, longest first, to the least loaded
rank; pair p of expert e then goes to replica p % n_rep(e). Replicas compute
identical results, so the output stays bit-exact.

`ep_forward` is the exchange protocol alone; the device work comes from an
`ops` object (DeviceOps here), so the same protocol also runs on CPU ranks
with another implementation of the four operations.
"""
import ctypes
import heapq

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .block import expert_mlp, route
from .pool import _stream_ptr


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def ep_forward(x, ops, world, group=None, mark=None):
    """The expert-parallel MoE block on this rank's tokens x [T, d].
    `mark(name)`, if given, is called at every phase boundary (timing)."""
    mark = mark or (lambda name: None)
    T = x.shape[0]
    inds, scores = ops.route(x)
    send_x, send_meta, counts, pair_pos = ops.pack(x, inds, scores)
    mark("routed+packed")
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    # split sizes travel to the host: the one synchronisation of the step
    send_splits = counts.tolist()
    recv_splits = recv_counts.tolist()
    n_recv = sum(recv_splits)
    recv_x = send_x.new_empty((n_recv, send_x.shape[1]))
    recv_meta = send_meta.new_empty((n_recv, 2))
    dist.all_to_all_single(recv_x, send_x, recv_splits, send_splits, group=group)
    dist.all_to_all_single(recv_meta, send_meta, recv_splits, send_splits, group=group)
    mark("dispatched")
    y_recv = ops.experts(recv_x, recv_meta)
    mark("experts")
    back = y_recv.new_empty((send_x.shape[0], y_recv.shape[1]))
    dist.all_to_all_single(back, y_recv, send_splits, recv_splits, group=group)
    mark("returned")
    y = ops.combine(back, pair_pos, T)
    mark("combined")
    return y


def plan_placement(counts, world, slots_per_rank, max_rep=None):
    """Expert placement from per-expert pair counts (e.g. one calibration
    batch, summed over the ranks). Returns (table, slots): table int32
    [E][1 + 2*max_rep] as ms_ep_pack reads it, slots[r] = the expert held in
    each slot of rank r. Deterministic, so every rank computes the same plan."""
    counts = np.asarray(counts, np.float64)
    E = counts.size
    max_rep = min(world, max_rep or world)
    if world * slots_per_rank < E:
        raise ValueError(f"{world} x {slots_per_rank} slots cannot hold {E} experts")
    reps = np.ones(E, np.int64)
    spare = world * slots_per_rank - E
    share = counts.sum() / world
    # replicate while some replica carries more than half a rank's share
    heap = [(-counts[e], e) for e in range(E)]
    heapq.heapify(heap)
    while spare > 0 and heap:
        neg, e = heapq.heappop(heap)
        if -neg <= share / 2:
            break
        if reps[e] >= max_rep:
            continue
        reps[e] += 1
        spare -= 1
        heapq.heappush(heap, (-counts[e] / reps[e], e))
    items = sorted(((counts[e] / reps[e], e) for e in range(E) for _ in range(reps[e])),
                   key=lambda it: (-it[0], it[1]))
    load = np.zeros(world)
    slots = [[] for _ in range(world)]
    for w, e in items:
        cands = [r for r in range(world) if len(slots[r]) < slots_per_rank and e not in slots[r]]
        if not cands:
            continue                            # a replica with nowhere to go is dropped
        r = min(cands, key=lambda r: (load[r], r))
        slots[r].append(e)
        load[r] += w
    table = np.zeros((E, 1 + 2 * max_rep), np.int32)
    for r in range(world):
        for i, e in enumerate(slots[r]):
            n = table[e, 0]
            table[e, 1 + 2 * n] = r
            table[e, 2 + 2 * n] = i
            table[e, 0] = n + 1
    if (table[:, 0] == 0).any():
        raise RuntimeError("placement left an expert without a slot")
    return table, slots


def shard_placement(E, world):
    """Plain sharding as a plan: expert e on rank e // (E / world)."""
    e_local = E // world
    table = np.zeros((E, 3), np.int32)
    for e in range(E):
        table[e] = (1, e // e_local, e % e_local)
    return table, [list(range(r * e_local, (r + 1) * e_local)) for r in range(world)]


class DeviceOps:
    """The four operations of ep_forward on this rank's GPU, through the
    library: block is the rank's MoEBlock (router set on its pool). Without
    a placement table the pool holds experts [rank * e_local, (rank + 1) *
    e_local) in slots 0..; with one (plan_placement) it holds slots[rank]."""

    def __init__(self, block, world, placement=None):
        self.block = block
        self.pool = block.pool
        self.world = world
        E = self.pool.geom.n_experts
        if placement is None and E % world:
            raise ValueError(f"{E} experts do not shard over {world} ranks")
        self.e_local = E // world
        self.placement = None
        self.max_rep = 0
        if placement is not None:
            table = torch.as_tensor(np.ascontiguousarray(placement, np.int32))
            self.max_rep = (table.shape[1] - 1) // 2
            self.placement = table.to(f"cuda:{self.pool.device}")
        self.stream = None

    def route(self, x):
        return route(self.block, x, stream=self.stream)

    def pack(self, x, inds, scores):
        pool = self.pool
        T, k = inds.shape
        dev = x.device
        send_x = torch.empty(T * k, x.shape[1], dtype=x.dtype, device=dev)
        send_meta = torch.empty(T * k, 2, dtype=torch.int32, device=dev)
        counts = torch.empty(self.world, dtype=torch.int32, device=dev)
        pair_pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        table = _ptr(self.placement) if self.placement is not None else None
        _lib.check(pool._lib.ms_ep_pack(pool._h, _ptr(x), T, _ptr(inds), _ptr(scores), self.world,
                                        self.e_local, table, self.max_rep, _ptr(send_x),
                                        _ptr(send_meta), _ptr(counts), _ptr(pair_pos),
                                        _stream_ptr(self.stream)))
        return send_x, send_meta, counts, pair_pos

    def experts(self, recv_x, recv_meta):
        if recv_x.shape[0] == 0:
            return recv_x.new_empty(recv_x.shape)
        slots = recv_meta[:, 0].contiguous()
        scores = recv_meta[:, 1].contiguous().view(torch.float32)
        return expert_mlp(self.pool, slots.view(-1, 1), recv_x, scores.view(-1, 1),
                          stream=self.stream)

    def combine(self, back, pair_pos, T):
        pool = self.pool
        y = back.new_empty((T, back.shape[1]))
        _lib.check(pool._lib.ms_ep_combine(pool._h, _ptr(back), _ptr(pair_pos), T, _ptr(y),
                                           _stream_ptr(self.stream)))
        return y


def ep_unique_id():
    """A new NCCL unique id (bytes) for EpGroup; one rank makes it and hands it to the
    others. The calling process hosts NCCL's bootstrap root until every rank has
    joined."""
    lib = _lib.load()
    buf = (ctypes.c_uint8 * 128)()
    _lib.check(lib.ms_ep_unique_id(buf))
    return bytes(buf)


class EpGroup:
    """The expert-parallel block through the C ABI alone (ms_ep_init /
    ms_ep_moe_block): NCCL send/recv inside the library, no torch.distributed.
    block: this rank's MoEBlock (router set on its pool, the rank's experts
    resident, e.g. load_local_experts); placement: a plan_placement table or
    None for plain sharding. __call__(x) is ep_forward(x, DeviceOps(...)) in one
    library call."""

    def __init__(self, block, unique_id, rank, world, placement=None):
        self.block = block
        self.pool = block.pool
        table, max_rep = None, 0
        if placement is not None:
            self._table = np.ascontiguousarray(placement, np.int32)
            max_rep = (self._table.shape[1] - 1) // 2
            table = self._table.ctypes.data_as(ctypes.c_void_p)
        idb = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        _lib.check(self.pool._lib.ms_ep_init(self.pool._h, idb, rank, world, table, max_rep))

    def __call__(self, x, stream=None):
        y = torch.empty_like(x)
        _lib.check(self.pool._lib.ms_ep_moe_block(self.pool._h, self.block._layer, _ptr(x),
                                                  x.shape[0], _ptr(y), _stream_ptr(stream)))
        return y

    def close(self):
        _lib.check(self.pool._lib.ms_ep_finalize(self.pool._h))


def load_local_experts(pool, layer, rank, world, slots=None):
    """Fill this rank's slots from the attached store (ExpertPool._read),
    once: slot i <- expert slots[i] of `layer` (a plan_placement row), or
    expert rank * e_local + i without a plan."""
    if slots is None:
        e_local = pool.geom.n_experts // world
        slots = [rank * e_local + i for i in range(e_local)]
    for i, e in enumerate(slots):
        pool._read(i, layer, int(e))
    torch.cuda.synchronize(pool.device)


def routed_counts(ops, x, group=None):
    """Pairs per expert of x's routing summed over the ranks (a calibration
    input for plan_placement); host int64 array."""
    inds, _ = ops.route(x)
    c = torch.bincount(inds.reshape(-1).long(), minlength=ops.pool.geom.n_experts)
    if dist.is_initialized():
        dist.all_reduce(c, group=group)
    return c.cpu().numpy()
