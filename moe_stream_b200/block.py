"""The MoE block: ``streaming_call`` (engine_v3.py:493-609,
engine_120b.py:78-149) as one asynchronous library call per layer.

The reference routes, evaluates (one host sync per layer), prefetches,
acquires (blocking on reads), then runs three gather_qmm calls, the SwiGLU
and the weighted sum. Here ``ms_moe_block`` enqueues all of it on the
caller's stream -- router, device slot-table step, fills, expert kernels --
and returns without synchronising, so a whole token (every layer) can be
captured into a CUDA graph.

Mirrors of the reference's module-level machinery:
  * ``MoEBlock``          -- a patched block: owns its layer index and router
  * ``streaming_call``    -- the function the reference monkey-patches onto
                             the block class (engine_v3.py:630,
                             engine_120b.py:180)
  * ``expert_mlp``        -- kernels.moe_expert_mlp (kernels.py:231-252)
"""
import ctypes

import torch

from . import _lib
from .pool import ExpertPool, _stream_ptr


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _check_tokens(pool, x):
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise TypeError("x must be a bf16 CUDA tensor")
    if x.shape[-1] != pool.geom.d_model:
        raise ValueError(f"x has {x.shape[-1]} features, the pool's model has {pool.geom.d_model}")
    return x.reshape(-1, x.shape[-1]).contiguous()


class MoEBlock:
    """One layer's MoE block bound to a shared pool (the reference keeps the
    pool in the module global _POOL and the blocks in _BLOCKS,
    engine_v3.py:489-495)."""

    def __init__(self, pool: ExpertPool, layer, gate_weight, gate_bias=None, norm_weight=None,
                 norm_eps=1e-6):
        self.pool = pool
        self._layer = int(layer)
        self.top_k = pool.top_k
        self.num_experts_per_tok = pool.top_k
        self.norm_topk_prob = pool.geom.norm_topk_prob
        self.gate_weight = gate_weight.to(device=f"cuda:{pool.device}", dtype=torch.bfloat16).contiguous()
        self.gate_bias = (None if gate_bias is None else
                          gate_bias.to(device=f"cuda:{pool.device}", dtype=torch.bfloat16).contiguous())
        _lib.check(pool._lib.ms_set_router(pool._h, self._layer, _ptr(self.gate_weight),
                                           _ptr(self.gate_bias) if self.gate_bias is not None else None))
        # the layer's post-attention RMSNorm weight, for fused()
        self.norm_weight = (None if norm_weight is None else
                            norm_weight.to(device=f"cuda:{pool.device}", dtype=torch.bfloat16).contiguous())
        self.norm_eps = float(norm_eps)

    def __call__(self, x, out=None, stream=None):
        return streaming_call(self, x, out=out, stream=stream)

    def fused(self, h, out=None, stream=None):
        """h + block(rms_norm(h) * norm_weight): the block with the decoder
        layer's post-attention norm and residual add (mlx_lm's layer,
        ``h + mlp(post_attention_layernorm(h))``) in the same library call.
        out may be h (in place)."""
        if self.norm_weight is None:
            raise ValueError("the block has no norm_weight")
        pool = self.pool
        h2 = _check_tokens(pool, h)
        T = h2.shape[0]
        y = out if out is not None else torch.empty_like(h2)
        _lib.check(pool._lib.ms_moe_block_fused(pool._h, self._layer, _ptr(h2), _ptr(self.norm_weight),
                                                self.norm_eps, T, _ptr(y), _stream_ptr(stream)))
        return y.reshape(h.shape)


def streaming_call(self, x, out=None, stream=None):
    """y = MoE(x) for x [..., d_model] bf16 on the pool's device."""
    pool = self.pool
    x2 = _check_tokens(pool, x)
    T = x2.shape[0]
    y = out if out is not None else torch.empty_like(x2)
    _lib.check(pool._lib.ms_moe_block(pool._h, self._layer, _ptr(x2), T, _ptr(y),
                                      _stream_ptr(stream)))
    return y.reshape(x.shape)


def route(block, x, stream=None, with_pred=False):
    """Router only (engine_v3.py:467-483 / engine_120b.py:65-75): returns
    (inds int32 [T,k], scores bf16 [T,k][, pred int32 [T, k*pf_widen]])."""
    pool = block.pool
    x2 = _check_tokens(pool, x)
    T = x2.shape[0]
    k = pool.top_k
    inds = torch.empty(T, k, dtype=torch.int32, device=x2.device)
    scores = torch.empty(T, k, dtype=torch.bfloat16, device=x2.device)
    pred = None
    if with_pred:
        kp = min(k * pool.pf_widen, pool.n_experts)
        pred = torch.empty(T, kp, dtype=torch.int32, device=x2.device)
    _lib.check(pool._lib.ms_route(pool._h, block._layer, _ptr(x2), T, _ptr(inds), _ptr(scores),
                                  _ptr(pred) if pred is not None else None, _stream_ptr(stream)))
    return (inds, scores, pred) if with_pred else (inds, scores)


def expert_mlp(pool, slots, x, scores, out=None, stream=None):
    """kernels.moe_expert_mlp generalised to T tokens: slots int32 [T,k],
    scores float32 [T,k], x bf16 [T,d] -> y bf16 [T,d]."""
    x2 = _check_tokens(pool, x)
    T = x2.shape[0]
    slots = slots.to(device=x2.device, dtype=torch.int32).reshape(T, -1).contiguous()
    scores = scores.to(device=x2.device, dtype=torch.float32).reshape(T, -1).contiguous()
    y = out if out is not None else torch.empty_like(x2)
    _lib.check(pool._lib.ms_expert_mlp(pool._h, _ptr(slots), _ptr(scores), _ptr(x2), T,
                                       slots.shape[1], _ptr(y), _stream_ptr(stream)))
    return y


def block_debug(pool, T):
    """Routing of the most recent block call: (inds, scores, slots) copies."""
    pi, ps, psl = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    _lib.check(pool._lib.ms_block_debug(pool._h, ctypes.byref(pi), ctypes.byref(ps), ctypes.byref(psl)))
    k = pool.top_k
    dev = f"cuda:{pool.device}"

    def grab(ptr, dtype, isz):
        n = T * k
        buf = torch.empty(n, dtype=dtype, device=dev)
        torch.cuda.synchronize(pool.device)
        cudart_copy(buf, ptr, n * isz)
        return buf.reshape(T, k)

    return grab(pi.value, torch.int32, 4), grab(ps.value, torch.bfloat16, 2), grab(psl.value, torch.int32, 4)


def cudart_copy(dst, src_ptr, nbytes):
    """Device-to-device copy from a raw pointer into a torch tensor."""
    src = torch.as_tensor(_RawDev(src_ptr, nbytes), device=dst.device)
    dst.view(torch.uint8).copy_(src)


class _RawDev:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = dict(shape=(nbytes,), typestr="|u1", data=(ptr, False),
                                             version=3)


class DecodeGraph:
    """One decode step over a stack of MoE blocks (one per layer) captured
    into a CUDA graph. Every call inside is an ordinary ``streaming_call``:
    the block API never synchronises or allocates, so a whole token replays
    with a single launch while the slot table keeps evolving on the device.
    Layer l reads x[l] and writes y[l] (the synthetic decode configs feed
    each layer its own hidden state)."""

    def __init__(self, blocks, T=1):
        pool = blocks[0].pool
        dev = f"cuda:{pool.device}"
        self.blocks = blocks
        self.x = torch.zeros(len(blocks), T, pool.geom.d_model, dtype=torch.bfloat16, device=dev)
        self.y = torch.zeros_like(self.x)
        self.pool = pool
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        pool.join(torch.cuda.current_stream(dev))
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.graph(self.graph, stream=s):
            for layer, b in enumerate(blocks):
                b(self.x[layer], out=self.y[layer])
            pool.join(s)        # the last layer's side-stream prefetch fills
        torch.cuda.current_stream(dev).wait_stream(s)

    def step(self, x=None):
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        # eager block calls since the capture may have left fills pending
        self.pool.join(torch.cuda.current_stream(self.y.device))
        self.graph.replay()
        return self.y
