"""Attention oracle (test infrastructure only): fp32 recompute from bf16 inputs.

The reference computes attention through flash-attn 2.8.3 (unpinned
dependency, `pyproject.toml:18`; called at nanovllm/layers/attention.py:64-74).
Its published semantics, restated here:
  * softmax(q . k^T * softmax_scale) . v per query head, with query head h
    reading kv head h // (Hq // Hkv) (GQA);
  * causal=True aligns the mask to the bottom-right corner: query i of a
    sequence with Lq queries and Lk keys sees key positions p <= i + Lk - Lq
    (flash_attn_interface.py docstring of flash_attn_varlen_func);
  * paged KV: key position p of batch row b lives at
    cache[block_table[b, p // block_size], p % block_size]
    (flash_attn_with_kvcache docstring; page size a multiple of 256);
  * flash_attn_with_kvcache's cache_seqlens counts the keys of each row.
A query row that sees no key at all gets a zero output.

All arithmetic is float32 (inputs are bf16 values held in float32 arrays).
"""
import numpy as np


def _softmax_weighted(s, vals, mask):
    """s: [..., T] scores (already scaled), vals: [T, ...] handled by caller."""
    s = np.where(mask, s, -np.inf).astype(np.float32)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, np.float32(0.0)).astype(np.float32)
    p = np.exp(s - m).astype(np.float32)
    p = np.where(mask, p, np.float32(0.0)).astype(np.float32)
    l = p.sum(axis=-1, keepdims=True, dtype=np.float32)
    return p, l


def gather_paged(cache, block_row, n):
    """Rows 0..n-1 of one sequence from a paged cache [NB, bs, Hkv, D]."""
    bs = cache.shape[1]
    pos = np.arange(n)
    return cache[np.asarray(block_row)[pos // bs], pos % bs]


def _attend(qs, K, V, scale, lq, lk):
    """qs [Lq, Hq, D], K/V [Lk, Hkv, D] -> [Lq, Hq, D] float32, bottom-right causal."""
    hq, d = qs.shape[1], qs.shape[2]
    hkv = K.shape[1]
    g = hq // hkv
    q4 = qs.reshape(lq, hkv, g, d).astype(np.float32)
    s = np.einsum("jhgd,thd->hgjt", q4, K.astype(np.float32), optimize=True).astype(np.float32)
    s = (s * np.float32(scale)).astype(np.float32)
    limit = np.arange(lq) + (lk - lq)
    mask = (np.arange(lk)[None, :] <= limit[:, None])[None, None]  # [1,1,Lq,Lk]
    p, l = _softmax_weighted(s, V, mask)
    o = np.einsum("hgjt,thd->jhgd", p, V.astype(np.float32), optimize=True).astype(np.float32)
    lt = np.transpose(l[..., 0], (2, 0, 1))[..., None]  # [Lq, Hkv, G, 1]
    o = np.where(lt > 0, o / np.where(lt > 0, lt, 1), 0).astype(np.float32)
    return o.reshape(lq, hq, d)


def paged_attention_ref(q, k_cache, v_cache, block_tables, context_lens, scale, rows=None):
    """Decode (Lq=1) / speculative-verify (Lq=k+1) attention over the paged cache.

    Follows the decode call nanovllm/layers/attention.py:71-74
    (flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
    cache_seqlens=context_lens, block_table=block_tables, causal=True)).
    q [B, Lq, Hq, D]; caches [NB, bs, Hkv, D]; block_tables [B, W];
    context_lens [B] (includes the Lq new tokens).  Returns float32
    [B, Lq, Hq, D]; rows with context_lens <= 0 are zero.  `rows` restricts
    the computation to a subset of batch rows (others stay zero).
    """
    B, lq, hq, d = q.shape
    out = np.zeros((B, lq, hq, d), np.float32)
    for b in (range(B) if rows is None else rows):
        ctx = int(context_lens[b])
        if ctx <= 0:
            continue
        K = gather_paged(k_cache, block_tables[b], ctx)
        V = gather_paged(v_cache, block_tables[b], ctx)
        out[b] = _attend(q[b], K, V, scale, lq, ctx)
    return out


def varlen_prefill_ref(q, k, v, cu_seqlens_q, cu_seqlens_k, scale, block_tables=None):
    """Causal varlen prefill, optionally over the paged cache (prefix caching).

    Follows nanovllm/layers/attention.py:64-70 (flash_attn_varlen_func with
    causal=True; when the context carries block_tables, k/v are the layer's
    caches, :65-66).  q [Tq, Hq, D]; k/v packed [Tk, Hkv, D] or caches
    [NB, bs, Hkv, D]; cu_seqlens int32 [S+1].  Returns float32 [Tq, Hq, D].
    """
    S = len(cu_seqlens_q) - 1
    out = np.zeros(q.shape, np.float32)
    for s in range(S):
        q0, q1 = int(cu_seqlens_q[s]), int(cu_seqlens_q[s + 1])
        k0, k1 = int(cu_seqlens_k[s]), int(cu_seqlens_k[s + 1])
        lq, lk = q1 - q0, k1 - k0
        if lq == 0:
            continue
        if block_tables is None:
            K, V = k[k0:k1], v[k0:k1]
        else:
            K = gather_paged(k, block_tables[s], lk)
            V = gather_paged(v, block_tables[s], lk)
        out[q0:q1] = _attend(q[q0:q1], K, V, scale, lq, lk)
    return out


def first_error(got, want, atol):
    """First index (in C order) where |got - want| > atol, or None.

    The study guide's first-error localisation (master_nano-vllm-v2.md:4137-4145)
    starts debugging from the first bad (row, head, position).
    """
    bad = np.argwhere(np.abs(got.astype(np.float32) - want.astype(np.float32)) > atol)
    return None if len(bad) == 0 else tuple(int(i) for i in bad[0])
