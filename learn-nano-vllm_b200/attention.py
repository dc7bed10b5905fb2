"""Drop-in `Attention` module for nano-vLLM on B200.

Keeps the reference module's contract (nanovllm/layers/attention.py:43-75):
the constructor takes (num_heads, head_dim, scale, num_kv_heads); `k_cache`
and `v_cache` start empty and are assigned by ModelRunner.allocate_kv_cache
(model_runner.py:116-120); `forward(q, k, v)` reads the side-channel
context, stores the new keys/values into the paged cache when the cache is
bound, then runs causal varlen prefill (over the cache when the context
carries block tables, i.e. a prefix-cache hit or a chunked-prefill
continuation) or paged decode.  Output shapes match the reference:
[T, Hq, D] for prefill, [B, 1, Hq, D] for decode.
"""
import torch
from torch import nn

from . import context as _ctx
from .ops import flash_attn_varlen_func, flash_attn_with_kvcache, qk_norm_rope_store, store_kvcache

# Where forward() reads the metadata from; integrate.install() rebinds it to
# the reference's nanovllm.utils.context.get_context.
_get_context = _ctx.get_context


def set_context_source(fn):
    global _get_context
    _get_context = fn


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        ctx = _get_context()
        cache_bound = self.k_cache.numel() > 0 and self.v_cache.numel() > 0
        if cache_bound:
            store_kvcache(k, v, self.k_cache, self.v_cache, ctx.slot_mapping)
        return self._attend(ctx, q, k, v)

    def forward_fused(self, qkv: torch.Tensor, positions: torch.Tensor, q_norm, k_norm,
                      rotary_emb) -> torch.Tensor:
        """q/k RMSNorm, RoPE and the cache store in one kernel, then attention.

        Same result as Qwen3Attention.forward's q_norm / k_norm / rotary_emb
        (nanovllm/models/qwen3.py:82-85) followed by forward(q, k, v); qkv is the
        fused projection output [T, (Hq + 2 Hkv) * D].
        """
        ctx = _get_context()
        cache_bound = self.k_cache.numel() > 0 and self.v_cache.numel() > 0
        need_k = ctx.is_prefill and (ctx.block_tables is None or not cache_bound)
        q, k, v = qk_norm_rope_store(qkv, positions, self.num_heads, self.num_kv_heads, q_norm.weight,
                                     k_norm.weight, q_norm.eps, rotary_emb.cos_sin_cache,
                                     self.k_cache if cache_bound else None, self.v_cache if cache_bound else None,
                                     ctx.slot_mapping if cache_bound else None, return_k=need_k)
        return self._attend(ctx, q, k, v)

    def _attend(self, ctx, q, k, v):
        if not ctx.is_prefill:
            return flash_attn_with_kvcache(q.unsqueeze(1), self.k_cache, self.v_cache,
                                           cache_seqlens=ctx.context_lens, block_table=ctx.block_tables,
                                           softmax_scale=self.scale, causal=True)
        paged = ctx.block_tables is not None
        return flash_attn_varlen_func(q, self.k_cache if paged else k, self.v_cache if paged else v,
                                      cu_seqlens_q=ctx.cu_seqlens_q, cu_seqlens_k=ctx.cu_seqlens_k,
                                      max_seqlen_q=ctx.max_seqlen_q, max_seqlen_k=ctx.max_seqlen_k,
                                      softmax_scale=self.scale, causal=True, block_table=ctx.block_tables)
