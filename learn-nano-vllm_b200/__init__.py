"""B200-native (sm_100a) attention hot path for nano-vLLM.

Import name: `learn_nano_vllm_b200` (the directory name carries hyphens; the
repository's `__graft_entry__.load_package()` registers it under this name).

Public API
  Attention                 drop-in for nanovllm.layers.attention.Attention
  store_kvcache             drop-in for nanovllm.layers.attention.store_kvcache
  flash_attn_with_kvcache   paged decode / verify attention (decode call site)
  flash_attn_varlen_func    causal varlen prefill, optionally over the paged cache
  paged_attention           the same decode kernel with explicit arguments
  spec_accept               speculative acceptance sampling
  qk_norm_rope_store        fused q/k RMSNorm + RoPE + KV-cache scatter (Qwen3 layer epilogue)
  sample                    fused temperature + exponential-race sampler
  DecodeMetadata            decode-step metadata built on the device
  OprojAllReduce            tensor-parallel o_proj GEMM fused with its all-reduce over peer memory
  AllReduce                 two-shot bf16 all-reduce over peer memory (the row-parallel all-reduce)
  install                   patch nano-vLLM to use this package's Attention (options: the fused
                            q/k epilogue, sampler, device decode metadata, row-parallel
                            GEMM + all-reduce, tensor-parallel worker processes)
  context                   mirror of nanovllm.utils.context
"""
from . import context, ops
from ._native import B200Error, lib
from .attention import Attention
from .decode_meta import DecodeMetadata
from .oproj import OprojAllReduce
from .allreduce import AllReduce
from .integrate import install
from .ops import (flash_attn_varlen_func, flash_attn_with_kvcache, paged_attention, paged_workspace,
                  qk_norm_rope_store, sample, spec_accept, store_kvcache, workspace_error)

__all__ = ["AllReduce", "Attention", "B200Error", "DecodeMetadata", "OprojAllReduce", "context", "flash_attn_varlen_func",
           "flash_attn_with_kvcache", "install", "lib", "paged_attention", "paged_workspace", "qk_norm_rope_store",
           "sample", "spec_accept", "store_kvcache", "workspace_error"]
