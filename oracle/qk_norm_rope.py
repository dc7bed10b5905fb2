"""Fused q/k RMSNorm + rotary embedding + KV scatter oracle (test infrastructure only).

Restates, in numpy float32 with the reference's rounding points (eager order):
  * RMSNorm.rms_forward (nanovllm/layers/layernorm.py:16-26):
        x = x.float(); var = mean(x^2); x = x * rsqrt(var + eps)
        x = round_to_dtype(x) * weight, rounded to the dtype;
  * apply_rotary_emb / RotaryEmbedding.forward (nanovllm/layers/rotary_embedding.py:6-14, 37-48):
        x1, x2 = halves of x (float32); y1 = x1*cos - x2*sin; y2 = x2*cos + x1*sin
        (each product rounded, then the sum), rounded to the dtype;
        cos, sin = cos_sin_cache[positions] split in halves;
  * the call sequence of Qwen3Attention.forward (nanovllm/models/qwen3.py:79-85) up
    to the attention, plus its store_kvcache (nanovllm/layers/attention.py:60-63):
        q, k, v = split(qkv); q = rope(q_norm(q)); k = rope(k_norm(k));
        k_cache[slot], v_cache[slot] = k, v for slot != -1.
Values are float32 arrays holding dtype-representable numbers.
"""
import numpy as np

from .cases import round_bf16
from .kv_store import store_kvcache_ref

f32 = np.float32


def round_dt(x, dtype):
    """Round float32 values to the model dtype ("bf16" or "fp16"), kept in float32."""
    x = np.asarray(x, f32)
    if dtype == "bf16":
        return round_bf16(x)
    return x.astype(np.float16).astype(f32)


def rms_norm_ref(x, weight, eps, dtype="bf16"):
    """nanovllm/layers/layernorm.py:16-26 on the last axis."""
    x = np.asarray(x, f32)
    var = (x * x).mean(axis=-1, keepdims=True, dtype=f32).astype(f32)
    inv = (f32(1.0) / np.sqrt((var + f32(eps)).astype(f32))).astype(f32)
    y = round_dt((x * inv).astype(f32), dtype)
    return round_dt((y * np.asarray(weight, f32)).astype(f32), dtype)


def rope_ref(x, cos, sin, dtype="bf16"):
    """nanovllm/layers/rotary_embedding.py:6-14; cos/sin broadcast over heads."""
    x = np.asarray(x, f32)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    y1 = ((x1 * cos).astype(f32) - (x2 * sin).astype(f32)).astype(f32)
    y2 = ((x2 * cos).astype(f32) + (x1 * sin).astype(f32)).astype(f32)
    return round_dt(np.concatenate([y1, y2], axis=-1), dtype)


def qk_norm_rope_store_ref(qkv, positions, num_heads, num_kv_heads, q_weight, k_weight, eps, cos_sin,
                           k_cache=None, v_cache=None, slot_mapping=None, dtype="bf16"):
    """Returns (q [T,Hq,D], k [T,Hkv,D], v [T,Hkv,D]); stores k, v into the caches in place."""
    qkv = np.asarray(qkv, f32)
    T = qkv.shape[0]
    D = np.asarray(q_weight).size
    q = qkv[:, :num_heads * D].reshape(T, num_heads, D)
    k = qkv[:, num_heads * D:(num_heads + num_kv_heads) * D].reshape(T, num_kv_heads, D)
    v = qkv[:, (num_heads + num_kv_heads) * D:].reshape(T, num_kv_heads, D)
    cs = np.asarray(cos_sin, f32).reshape(np.asarray(cos_sin).shape[0], D)
    pos = np.clip(np.asarray(positions, np.int64), 0, cs.shape[0] - 1)
    cos = cs[pos, :D // 2][:, None, :]
    sin = cs[pos, D // 2:][:, None, :]
    q = rope_ref(rms_norm_ref(q, q_weight, eps, dtype), cos, sin, dtype)
    k = rope_ref(rms_norm_ref(k, k_weight, eps, dtype), cos, sin, dtype)
    if k_cache is not None and v_cache is not None and slot_mapping is not None:
        store_kvcache_ref(k, v, k_cache, v_cache, np.asarray(slot_mapping))
    return q, k, v
