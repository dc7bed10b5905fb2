"""Install the B200 attention path into an unmodified nano-vLLM.

nano-vLLM constructs `Attention` inside Qwen3Attention (nanovllm/models/qwen3.py:61-66),
which imported the class by name (qwen3.py:7).  install() rebinds that name
(and the one in nanovllm.layers.attention) to this package's module, and
points it at the reference's own context (nanovllm/utils/context.py), so that
ModelRunner, BlockManager, the prefix cache, the scheduler and CUDA-graph
capture run unchanged on top of the B200 kernels.  Call it before the engine
builds its model.
"""
import importlib

from . import attention as _attention
from .ops import store_kvcache


def install():
    """Patch the importable `nanovllm` package; returns the patched modules."""
    ctx_mod = importlib.import_module("nanovllm.utils.context")
    attn_mod = importlib.import_module("nanovllm.layers.attention")
    qwen3 = importlib.import_module("nanovllm.models.qwen3")
    _attention.set_context_source(ctx_mod.get_context)
    attn_mod.Attention = _attention.Attention
    attn_mod.store_kvcache = store_kvcache
    qwen3.Attention = _attention.Attention
    return attn_mod, qwen3


def uninstall():
    """Point Attention back at this package's own context mirror."""
    from . import context as _ctx
    _attention.set_context_source(_ctx.get_context)
