"""moe_stream_b200: moe-stream's MoE expert block and slot pool on B200.

Host side in Python over a C-ABI CUDA library (libmoestream.so, sm_100a).
The public surface mirrors the reference's: ``ExpertPool`` (engine_v3.py
ExpertPool), ``MoEBlock`` / ``streaming_call`` (the patched block call), and
``expert_mlp`` (kernels.moe_expert_mlp).
"""
from . import geometry, store
from .geometry import Geometry, qwen3, gptoss


def __getattr__(name):
    # GPU entry points load the shared library lazily and fail loudly if it
    # is missing; there is no CPU implementation behind them.
    if name in ("ExpertPool",):
        from .pool import ExpertPool
        return ExpertPool
    if name in ("MoEBlock", "streaming_call", "route", "expert_mlp", "block_debug"):
        from . import block
        return getattr(block, name)
    raise AttributeError(name)
