"""Expert parallelism for wide batches: the 128 experts
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

`ep_forward` is the exchange protocol alone; the device work comes from an
`ops` object (DeviceOps here), so the same protocol also runs on CPU ranks
with another implementation of the four operations.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .block import expert_mlp, route
from .pool import _stream_ptr


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def ep_forward(x, ops, world, group=None):
    """The expert-parallel MoE block on this rank's tokens x [T, d]."""
    T = x.shape[0]
    inds, scores = ops.route(x)
    send_x, send_meta, counts, pair_pos = ops.pack(x, inds, scores)
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
    y_recv = ops.experts(recv_x, recv_meta)
    back = y_recv.new_empty((send_x.shape[0], y_recv.shape[1]))
    dist.all_to_all_single(back, y_recv, send_splits, recv_splits, group=group)
    return ops.combine(back, pair_pos, T)


class DeviceOps:
    """The four operations of ep_forward on this rank's GPU, through the
    library: block is the rank's MoEBlock (router set on its pool, the pool
    holding experts [rank * e_local, (rank + 1) * e_local) in slots 0..)."""

    def __init__(self, block, world):
        self.block = block
        self.pool = block.pool
        self.world = world
        E = self.pool.geom.n_experts
        if E % world:
            raise ValueError(f"{E} experts do not shard over {world} ranks")
        self.e_local = E // world
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
        _lib.check(pool._lib.ms_ep_pack(pool._h, _ptr(x), T, _ptr(inds), _ptr(scores), self.world,
                                        self.e_local, _ptr(send_x), _ptr(send_meta), _ptr(counts),
                                        _ptr(pair_pos), _stream_ptr(self.stream)))
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


def load_local_experts(pool, layer, rank, world):
    """Fill slot i of this rank's pool with expert rank * e_local + i of
    `layer` from the attached store (ExpertPool._read), once."""
    e_local = pool.geom.n_experts // world
    for i in range(e_local):
        pool._read(i, layer, rank * e_local + i)
    torch.cuda.synchronize(pool.device)
