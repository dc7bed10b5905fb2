"""Seeded synthetic cases for the benchmark configurations (test infrastructure).

The reference benchmarks on real Qwen3 checkpoints and prompts, which are not
available here; these factories produce seeded synthetic inputs with the
shapes, sizes and value distributions the configurations name.  Tensors are
float32 arrays whose values are exactly representable in bf16 (rounded to
nearest-even), so that a bf16 copy on the GPU holds the same numbers.
"""
from dataclasses import dataclass, field
import numpy as np


def round_bf16(x):
    """float32 -> nearest-even bf16 value, kept in float32 (torch's rounding)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def randn_bf16(rng, shape, scale=1.0):
    return round_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


@dataclass
class PagedCase:
    """Decode / verify attention on a paged cache (one layer)."""
    q: np.ndarray              # [B, Lq, Hq, D]
    k_cache: np.ndarray        # [NB, bs, Hkv, D]
    v_cache: np.ndarray
    block_tables: np.ndarray   # int32 [B, W]
    context_lens: np.ndarray   # int32 [B]
    k_new: np.ndarray          # [B*Lq, Hkv, D] rows stored before attending
    v_new: np.ndarray
    slot_mapping: np.ndarray   # int32 [B*Lq]
    scale: float
    block_size: int


def block_tables_for(rng, ctx, block_size, width=None, pool=None):
    """Distinct physical blocks per sequence drawn from a shuffled pool."""
    need = [(int(c) + block_size - 1) // block_size for c in ctx]
    total = sum(need)
    pool = max(pool or 0, total)
    perm = rng.permutation(pool).astype(np.int32)
    width = max(width or 0, max(need) if need else 1, 1)
    bt = np.full((len(ctx), width), -1, np.int32)
    o = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[o:o + n]
        o += n
    return bt, pool


def slots_for(block_tables, ctx, lq, block_size):
    """Cache slots of the last lq positions of every sequence (model_runner.py:181)."""
    out = []
    for b, c in enumerate(ctx):
        for p in range(int(c) - lq, int(c)):
            out.append(int(block_tables[b, p // block_size]) * block_size + p % block_size)
    return np.asarray(out, np.int32)


def make_paged_case(ctx, hq, hkv, d=128, block_size=256, lq=1, seed=0, width=None,
                    pool=None, fill_cache=True, cache_std=1.0):
    """Generic paged case; q/k/v ~ N(0,1)/sqrt(d) as in the configurations."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    B = len(ctx)
    bt, nb = block_tables_for(rng, ctx, block_size, width, pool)
    sc = 1.0 / np.sqrt(d)
    kc = np.zeros((nb, block_size, hkv, d), np.float32)
    vc = np.zeros((nb, block_size, hkv, d), np.float32)
    if fill_cache:
        kc[:] = randn_bf16(rng, kc.shape, sc * cache_std)
        vc[:] = randn_bf16(rng, vc.shape, sc * cache_std)
    q = randn_bf16(rng, (B, lq, hq, d), sc)
    kn = randn_bf16(rng, (B * lq, hkv, d), sc)
    vn = randn_bf16(rng, (B * lq, hkv, d), sc)
    slots = slots_for(bt, np.maximum(ctx, lq), lq, block_size)
    valid = np.repeat(ctx > 0, lq)
    slots = np.where(valid, slots, -1).astype(np.int32)
    return PagedCase(q, kc, vc, bt, ctx, kn, vn, slots, float(d) ** -0.5, block_size)


def config1_case(seed=0):
    """Config 1: Qwen3-0.6B layer (16/8 heads, D 128), B=8, ctx U[100,1024],
    block tables from a seeded permutation of a 64-block pool."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(100, 1025, size=8).astype(np.int32)
    return make_paged_case(ctx, 16, 8, 128, 256, 1, seed=seed + 1, width=8, pool=64)


def config5_context_lens(batch=512, sigma=0.5, seed=0, cap=32768):
    """Config 5: lognormal(ln 2048, sigma) context lengths capped at 32768.

    The configuration leaves sigma open; 0.5 is used and stated."""
    rng = np.random.default_rng(seed)
    c = np.exp(rng.normal(np.log(2048.0), sigma, size=batch))
    return np.clip(np.rint(c), 1, cap).astype(np.int32)


def config4_context_lens(batch=128, seed=0):
    rng = np.random.default_rng(seed)
    return rng.integers(512, 4097, size=batch).astype(np.int32)


@dataclass
class PrefillCase:
    q: np.ndarray            # [Tq, Hq, D]
    k: np.ndarray            # packed [Tk, Hkv, D] or cache [NB, bs, Hkv, D]
    v: np.ndarray
    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    block_tables: np.ndarray | None
    scale: float
    block_size: int
    k_new: np.ndarray | None = None   # suffix rows stored before attending
    v_new: np.ndarray | None = None
    slot_mapping: np.ndarray | None = None


def make_prefill_case(lq, hq, hkv, d=128, seed=0):
    """Plain varlen prefill (no cache hit): cu_seqlens_k == cu_seqlens_q."""
    rng = np.random.default_rng(seed)
    lq = np.asarray(lq, np.int32)
    cu = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    sc = 1.0 / np.sqrt(d)
    T = int(cu[-1])
    q = randn_bf16(rng, (T, hq, d), sc)
    k = randn_bf16(rng, (T, hkv, d), sc)
    v = randn_bf16(rng, (T, hkv, d), sc)
    return PrefillCase(q, k, v, cu, cu.copy(), None, float(d) ** -0.5, 0)


def make_prefix_prefill_case(suffix, prefix_len, hq, hkv, d=128, block_size=256, seed=0):
    """Prefix-cached prefill: every sequence shares `prefix_len` cached tokens
    (whole blocks), then its own suffix; keys come from the paged cache."""
    rng = np.random.default_rng(seed)
    suffix = np.asarray(suffix, np.int32)
    S = len(suffix)
    assert prefix_len % block_size == 0
    npre = prefix_len // block_size
    lk = suffix + prefix_len
    nblk = [(int(x) + block_size - 1) // block_size for x in lk]
    pool = npre + sum(n - npre for n in nblk)
    perm = rng.permutation(pool).astype(np.int32)
    shared = perm[:npre]
    width = max(nblk)
    bt = np.full((S, width), -1, np.int32)
    o = npre
    for s in range(S):
        bt[s, :npre] = shared
        m = nblk[s] - npre
        bt[s, npre:nblk[s]] = perm[o:o + m]
        o += m
    sc = 1.0 / np.sqrt(d)
    kc = randn_bf16(rng, (pool, block_size, hkv, d), sc)
    vc = randn_bf16(rng, (pool, block_size, hkv, d), sc)
    T = int(suffix.sum())
    q = randn_bf16(rng, (T, hq, d), sc)
    kn = randn_bf16(rng, (T, hkv, d), sc)
    vn = randn_bf16(rng, (T, hkv, d), sc)
    slots = []
    for s in range(S):
        for p in range(prefix_len, int(lk[s])):
            slots.append(int(bt[s, p // block_size]) * block_size + p % block_size)
    cu_q = np.concatenate([[0], np.cumsum(suffix)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    return PrefillCase(q, kc, vc, cu_q, cu_k, bt, float(d) ** -0.5, block_size,
                       kn, vn, np.asarray(slots, np.int32))


def config3_case(seed=0, num_seqs=64):
    """Config 3: 64 sequences share a 768-token prefix (3 blocks of 256), each
    with a unique suffix of U[64, 512] tokens; Qwen3-0.6B attention shape."""
    rng = np.random.default_rng(seed)
    suffix = rng.integers(64, 513, size=num_seqs).astype(np.int32)
    return make_prefix_prefill_case(suffix, 768, 16, 8, 128, 256, seed=seed + 1)


@dataclass
class SpecCase:
    target_logits: np.ndarray   # [B, k+1, V] fp32
    draft_logits: np.ndarray    # [B, k, V]
    draft_tokens: np.ndarray    # [B, k] int32
    u_accept: np.ndarray        # [B, k] fp32
    u_sample: np.ndarray        # [B] fp32
    temperatures: np.ndarray | None = None


def make_spec_case(batch, k, vocab, seed=0, std=2.0, correlated=True, temperatures=False):
    """Logits ~ N(0, std^2) fp32.  With `correlated`, the draft logits are the
    target logits plus noise, so that acceptances are frequent enough to
    exercise every branch; draft tokens are drawn from the draft distribution."""
    rng = np.random.default_rng(seed)
    tl = (rng.standard_normal((batch, k + 1, vocab), dtype=np.float32) * np.float32(std))
    if correlated:
        dl = (tl[:, :k] + rng.standard_normal((batch, k, vocab), dtype=np.float32)
              * np.float32(0.5 * std)).astype(np.float32)
    else:
        dl = rng.standard_normal((batch, k, vocab), dtype=np.float32) * np.float32(std)
    # draft tokens ~ q via the Gumbel-max trick (float64 is fine: only the token matters)
    g = -np.log(-np.log(rng.random((batch, k, vocab))))
    toks = np.argmax(dl.astype(np.float64) + g, axis=-1).astype(np.int32)
    ua = rng.random((batch, k), dtype=np.float32)
    us = rng.random(batch, dtype=np.float32)
    temps = None
    if temperatures:
        temps = rng.uniform(0.5, 1.5, size=batch).astype(np.float32)
    return SpecCase(tl, dl, toks, ua, us, temps)
