"""Torch-facing ops of the B200 attention path.

Names and argument meanings follow the calls of the reference hot path
(nanovllm/layers/attention.py): `store_kvcache` (:33-40), and the two
flash-attn entry points it uses, `flash_attn_with_kvcache` (:72-74) and
`flash_attn_varlen_func` (:67-70), restricted to the arguments nano-vLLM
passes.  Each op checks its tensors, then calls the C ABI of
libb200attn.so on the current CUDA stream; nothing here synchronises the
host or computes on the CPU, so the ops can be captured in CUDA graphs.
"""
import ctypes
import threading

import torch

from . import _native
from ._native import check, lib

_DTYPES = {torch.bfloat16: _native.B200_BF16, torch.float16: _native.B200_F16}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _row_stride(t: torch.Tensor) -> int:
    """Row stride of a 2-D table; a single-row table may carry any stride on its size-1 dim."""
    return t.stride(0) if t.size(0) > 1 else max(t.size(1), 1)


def _require_cuda(*ts):
    dev = ts[0].device
    for t in ts:
        assert t.is_cuda, "B200 attention ops take CUDA tensors"
        assert t.device == dev, f"tensors on different devices ({t.device} vs {dev})"


# ------------------------------------------------------------------ KV store
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """k_cache.view(-1, Hkv*D)[slot] = key[t] (and value) for slot != -1.

    Same contract and asserts as nanovllm/layers/attention.py:33-40; in
    addition slots outside the cache are skipped instead of written.
    """
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "KV caches must be contiguous"
    assert key.dtype == value.dtype == k_cache.dtype == v_cache.dtype, "key/value/cache dtypes differ"
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous(), "slot_mapping must be contiguous int32"
    num_slots = k_cache.numel() // D
    rc = lib().b200_store_kvcache(key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
                                  k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), N,
                                  num_heads, head_dim, num_slots, key.element_size(), _stream(key))
    check(rc, "store_kvcache")


# --------------------------------------------------------- paged attention
DEFAULT_MAX_ITEMS = 32768
_ws_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}


def paged_workspace(device: torch.device, query_len: int, group: int, min_items: int) -> torch.Tensor:
    """Per-device split-K workspace for paged attention (zero-filled, grown on demand).

    Growing it allocates, which is not allowed while a CUDA graph is being
    captured: the first eager call at the largest batch (nano-vLLM's warm-up
    before capture, model_runner.py:240) sizes it.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    items = max(DEFAULT_MAX_ITEMS, min_items)
    need = lib().b200_paged_attention_workspace_size(items, query_len, group, 128)
    with _ws_lock:
        ws = _workspaces.get(idx)
        if ws is None or ws.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("paged attention workspace must be allocated before CUDA-graph capture")
            if ws is not None:
                torch.cuda.current_stream(device).synchronize()
            ws = torch.zeros(need, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = ws
    return ws


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, context_lens: torch.Tensor,
                    block_tables: torch.Tensor, softmax_scale: float, out: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Causal (bottom-right) attention of q [B, Lq, Hq, D] over the paged cache.

    context_lens [B] counts the cached tokens of each row including its Lq
    queries; rows with context_lens <= 0 return zeros.  Returns
    [B, Lq, Hq, D] in q's dtype.
    """
    B, Lq, Hq, D = q.shape
    NB, bs, Hkv, Dk = k_cache.shape
    assert Dk == D and v_cache.shape == k_cache.shape, "cache shape mismatch"
    assert q.stride(-1) == 1 and q.stride(-2) == D, "q heads must be contiguous"
    if Lq == 1:
        q_tok = q.stride(0)
    else:
        assert q.stride(0) == Lq * q.stride(1), "q rows of one sequence must be evenly strided"
        q_tok = q.stride(1)
    _require_cuda(q, k_cache, v_cache, context_lens, block_tables)
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "KV caches must be contiguous"
    assert q.dtype in _DTYPES and k_cache.dtype == q.dtype == v_cache.dtype, "q/cache dtype must match (bf16/fp16)"
    assert context_lens.dtype == torch.int32 and context_lens.is_contiguous() and context_lens.numel() == B
    assert block_tables.dtype == torch.int32 and block_tables.dim() == 2 and block_tables.stride(1) == 1
    assert block_tables.size(0) >= B, "block_tables has fewer rows than q"
    if out is None:
        out = torch.empty((B, Lq, Hq, D), dtype=q.dtype, device=q.device)
    else:
        assert out.shape == (B, Lq, Hq, D) and out.is_contiguous() and out.dtype == q.dtype
    if workspace is None:
        workspace = paged_workspace(q.device, Lq, Hq // Hkv, B * Hkv)
    rc = lib().b200_paged_attention(out.data_ptr(), q.data_ptr(), q_tok, k_cache.data_ptr(), v_cache.data_ptr(), NB, bs, block_tables.data_ptr(),
                                    _row_stride(block_tables), context_lens.data_ptr(), B, Lq, Hq, Hkv, D,
                                    float(softmax_scale), _DTYPES[q.dtype], workspace.data_ptr(),
                                    workspace.numel(), _stream(q))
    check(rc, "paged_attention")
    return out


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=None, block_table=None, softmax_scale=None,
                            causal=True, out=None):
    """Drop-in for the decode call of nanovllm/layers/attention.py:72-74.

    q [B, Lq, Hq, D], k_cache/v_cache [num_blocks, block_size, Hkv, D],
    cache_seqlens int32 [B], block_table int32 [B, W]; returns [B, Lq, Hq, D].
    """
    assert cache_seqlens is not None and block_table is not None, "the B200 path reads a paged cache"
    if not causal and q.size(1) > 1:
        raise NotImplementedError("non-causal multi-query paged attention")
    scale = q.size(-1) ** -0.5 if softmax_scale is None else softmax_scale
    return paged_attention(q, k_cache, v_cache, cache_seqlens, block_table, scale, out=out)


def prefill_error() -> int:
    """Device error word of the prefill kernels (synchronises the current stream)."""
    flag = ctypes.c_int32(0)
    check(lib().b200_varlen_prefill_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(flag)),
          "varlen_prefill_error")
    return flag.value


def workspace_error(workspace: torch.Tensor) -> int:
    """Device error word of a paged-attention workspace (synchronises)."""
    flag = ctypes.c_int32(0)
    check(lib().b200_workspace_error(workspace.data_ptr(), _stream(workspace), ctypes.byref(flag)),
          "workspace_error")
    return flag.value


# ------------------------------------------------------------ varlen prefill
_prefill_workspaces: dict[int, torch.Tensor] = {}


def prefill_workspace(device: torch.device) -> torch.Tensor:
    """Per-device workspace of the prefill kernel (its work counter; zero-filled once)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _prefill_workspaces.get(idx)
        if ws is None:
            n = max(int(lib().b200_varlen_prefill_workspace_size()), 256)
            ws = torch.zeros(n, dtype=torch.uint8, device=torch.device("cuda", idx))
            _prefill_workspaces[idx] = ws
    return ws


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale=None,
                           causal=True, block_table=None, out=None):
    """Drop-in for the prefill call of nanovllm/layers/attention.py:67-70.

    q [Tq, Hq, D]; k/v packed [Tk, Hkv, D] or, with block_table, the layer's
    caches [num_blocks, block_size, Hkv, D]; returns [Tq, Hq, D].
    """
    if not causal:
        raise NotImplementedError("non-causal prefill")
    Tq, Hq, D = q.shape
    _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k)
    assert q.dtype in _DTYPES and k.dtype == q.dtype == v.dtype, "q/k/v dtype must match (bf16/fp16)"
    assert q.stride(-1) == 1 and q.stride(-2) == D, "q heads must be contiguous"
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    S = cu_seqlens_q.numel() - 1
    assert cu_seqlens_k.numel() == S + 1
    if block_table is not None:
        NB, bs, Hkv, Dk = k.shape
        assert k.is_contiguous() and v.is_contiguous() and v.shape == k.shape
        assert block_table.dtype == torch.int32 and block_table.stride(1) == 1
        k_stride = v_stride = Hkv * D
        total_k_rows = NB * bs
        bt_ptr, bt_stride = block_table.data_ptr(), _row_stride(block_table)
    else:
        Tk, Hkv, Dk = k.shape
        assert k.stride(-1) == 1 and k.stride(-2) == D and v.stride(-1) == 1 and v.stride(-2) == D
        k_stride, v_stride = k.stride(0), v.stride(0)
        total_k_rows, bs = Tk, 0
        bt_ptr, bt_stride = None, 0
    assert Dk == D
    if out is None:
        out = torch.empty((Tq, Hq, D), dtype=q.dtype, device=q.device)
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    if Tq == 0 or S == 0:
        return out
    ws = prefill_workspace(q.device)
    rc = lib().b200_varlen_prefill(out.data_ptr(), q.data_ptr(), q.stride(0), k.data_ptr(), k_stride, v.data_ptr(),
                                   v_stride, cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), S, Tq,
                                   int(max_seqlen_q), int(max_seqlen_k), total_k_rows, bt_ptr, bt_stride, bs,
                                   Hq, Hkv, D, float(scale), _DTYPES[q.dtype], ws.data_ptr(), ws.numel(),
                                   _stream(q))
    check(rc, "varlen_prefill")
    return out


# ------------------------------------------------------ speculative decoding
def spec_accept(target_logits, draft_logits, draft_tokens, uniform_accept, uniform_sample, temperatures=None,
                workspace=None):
    """Rejection-sampling acceptance of k draft tokens per sequence.

    target_logits [B, k+1, V], draft_logits [B, k, V] fp32; draft_tokens,
    uniform_accept [B, k]; uniform_sample [B]; temperatures [B] or None.
    Returns (tokens int32 [B, k+1] padded with -1, num_tokens int32 [B]).
    """
    B, k1, V = target_logits.shape
    k = k1 - 1
    _require_cuda(target_logits, draft_logits, draft_tokens, uniform_accept, uniform_sample)
    for t in (target_logits, draft_logits, uniform_accept, uniform_sample):
        assert t.dtype == torch.float32 and t.is_contiguous()
    assert draft_logits.shape == (B, k, V) and draft_tokens.shape == (B, k) and uniform_accept.shape == (B, k)
    assert draft_tokens.dtype == torch.int32 and draft_tokens.is_contiguous() and uniform_sample.shape == (B,)
    if temperatures is not None:
        assert temperatures.dtype == torch.float32 and temperatures.shape == (B,) and temperatures.is_cuda
    tokens = torch.empty((B, k1), dtype=torch.int32, device=target_logits.device)
    num = torch.empty((B,), dtype=torch.int32, device=target_logits.device)
    need = lib().b200_spec_accept_workspace_size(B, k, V)
    if workspace is None:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=target_logits.device)
    rc = lib().b200_spec_accept(tokens.data_ptr(), num.data_ptr(), target_logits.data_ptr(),
                                draft_logits.data_ptr(), draft_tokens.data_ptr(), uniform_accept.data_ptr(),
                                uniform_sample.data_ptr(), None if temperatures is None else temperatures.data_ptr(),
                                B, k, V, workspace.data_ptr(), workspace.numel(), _stream(target_logits))
    check(rc, "spec_accept")
    return tokens, num


# ------------------------------------------- fused q/k norm + RoPE + KV scatter
def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, num_heads: int, num_kv_heads: int,
                       q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float, cos_sin_cache: torch.Tensor,
                       k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None, return_k: bool = True):
    """One pass over the QKV projection output of a Qwen3 attention layer.

    Equivalent to (nanovllm/models/qwen3.py:79-85 and layers/attention.py:60-63)
        q, k, v = qkv.split([Hq*D, Hkv*D, Hkv*D], -1)
        q = q_norm(q.view(-1, Hq, D)); k = k_norm(k.view(-1, Hkv, D))
        q, k = rotary_emb(positions, q, k)
        store_kvcache(k, v.view(-1, Hkv, D), k_cache, v_cache, slot_mapping)
    Returns (q [T, Hq, D], k [T, Hkv, D] or None, v view [T, Hkv, D]).
    cos_sin_cache is the rotary module's buffer ([max_position, 1, D] or
    [max_position, D], fp32, cos | sin).  Empty caches (numel 0, the
    reference's "no cache yet") skip the store.
    """
    assert qkv.dim() == 2 and qkv.stride(-1) == 1, "qkv must be [T, (Hq+2Hkv)*D] with contiguous rows"
    T = qkv.shape[0]
    D = q_weight.numel()
    assert qkv.shape[1] == (num_heads + 2 * num_kv_heads) * D, "qkv width does not match the head counts"
    assert k_weight.numel() == D and q_weight.is_contiguous() and k_weight.is_contiguous()
    assert q_weight.dtype == k_weight.dtype == qkv.dtype, "norm weights must have the model dtype"
    assert qkv.dtype in _DTYPES, f"unsupported dtype {qkv.dtype}"
    assert positions.dtype == torch.int64 and positions.numel() == T and positions.is_contiguous()
    cs = cos_sin_cache.reshape(cos_sin_cache.shape[0], -1)
    assert cs.dtype == torch.float32 and cs.shape[1] == D and cs.is_contiguous(), "cos_sin_cache must be fp32 [P, D]"
    has_cache = k_cache is not None and v_cache is not None and k_cache.numel() > 0 and v_cache.numel() > 0
    tensors = [qkv, positions, q_weight, k_weight, cs]
    if has_cache:
        assert slot_mapping is not None and slot_mapping.dtype == torch.int32 and slot_mapping.numel() == T
        assert slot_mapping.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()
        assert k_cache.dtype == v_cache.dtype == qkv.dtype, "cache dtype differs from qkv"
        assert k_cache.numel() % (num_kv_heads * D) == 0
        tensors += [k_cache, v_cache, slot_mapping]
    _require_cuda(*tensors)
    q = torch.empty((T, num_heads, D), dtype=qkv.dtype, device=qkv.device)
    k = torch.empty((T, num_kv_heads, D), dtype=qkv.dtype, device=qkv.device) if return_k else None
    num_slots = k_cache.numel() // (num_kv_heads * D) if has_cache else 0
    rc = lib().b200_qk_norm_rope_store(
        q.data_ptr(), q.stride(0), k.data_ptr() if k is not None else None, k.stride(0) if k is not None else 0,
        qkv.data_ptr(), qkv.stride(0), positions.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(), float(eps),
        cs.data_ptr(), cs.shape[0], k_cache.data_ptr() if has_cache else None,
        v_cache.data_ptr() if has_cache else None, slot_mapping.data_ptr() if has_cache else None, num_slots, T,
        num_heads, num_kv_heads, D, _DTYPES[qkv.dtype], _stream(qkv))
    check(rc, "qk_norm_rope_store")
    v = qkv[:, (num_heads + num_kv_heads) * D:].view(T, num_kv_heads, D)
    return q, k, v


# ------------------------------------------------------------------ sampler
_DTYPES_ALL = {torch.bfloat16: _native.B200_BF16, torch.float16: _native.B200_F16, torch.float32: _native.B200_F32}
_sample_ws: dict[int, torch.Tensor] = {}


def sample(logits: torch.Tensor, temperatures: torch.Tensor, seed: int = 0, offset: int = 0,
           noise: torch.Tensor | None = None) -> torch.Tensor:
    """Fused temperature + exponential-race sampling (nanovllm/layers/sampler.py:7-12).

    Returns int64 tokens [B].  With `noise` ([B, V] fp32, Exp(1) draws) the result is
    argmax(softmax(logits / T) / clamp_min(noise, 1e-10)) as in the reference; without it
    the noise comes from the counter-based generator keyed by (seed, offset) — advance
    `offset` every step to draw fresh noise.
    """
    assert logits.dim() == 2 and logits.stride(-1) == 1, "logits must be [B, V] with contiguous rows"
    assert logits.dtype in _DTYPES_ALL, f"unsupported dtype {logits.dtype}"
    B, V = logits.shape
    assert temperatures.dtype == torch.float32 and temperatures.numel() == B and temperatures.is_contiguous()
    tensors = [logits, temperatures]
    if noise is not None:
        assert noise.dtype == torch.float32 and noise.shape == (B, V) and noise.stride(-1) == 1
        tensors.append(noise)
    _require_cuda(*tensors)
    need = lib().b200_sample_workspace_size(B)
    dev = logits.device.index if logits.device.index is not None else torch.cuda.current_device()
    ws = _sample_ws.get(dev)
    if ws is None or ws.numel() < need:
        assert not torch.cuda.is_current_stream_capturing(), "call sample() once eagerly before graph capture"
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=logits.device)
        _sample_ws[dev] = ws
    out = torch.empty(B, dtype=torch.int64, device=logits.device)
    rc = lib().b200_sample(out.data_ptr(), logits.data_ptr(), logits.stride(0), _DTYPES_ALL[logits.dtype],
                           temperatures.data_ptr(), B, V, noise.data_ptr() if noise is not None else None,
                           noise.stride(0) if noise is not None else 0, seed & (2 ** 64 - 1),
                           offset & (2 ** 64 - 1), ws.data_ptr(), ws.numel(), _stream(logits))
    check(rc, "sample")
    return out
