"""Self-consistency of the attention oracle (CPU)."""
import numpy as np
import pytest

from oracle import attention as oatt
from oracle import cases


def dense_ref(q, K, V, scale, lq, lk):
    """float64 materialised softmax attention with the bottom-right causal mask."""
    hq, hkv = q.shape[1], K.shape[1]
    g = hq // hkv
    out = np.zeros(q.shape, np.float64)
    for j in range(lq):
        for h in range(hq):
            kh = h // g
            s = K[:, kh].astype(np.float64) @ q[j, h].astype(np.float64) * scale
            vis = np.arange(lk) <= j + lk - lq
            if not vis.any():
                continue
            s = np.where(vis, s, -np.inf)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[j, h] = p @ V[:, kh].astype(np.float64)
    return out


@pytest.mark.parametrize("hq,hkv,lq", [(16, 8, 1), (16, 4, 5), (8, 8, 2), (32, 8, 1)])
def test_paged_matches_dense(hq, hkv, lq):
    case = cases.make_paged_case([1, 77, 256, 300], hq, hkv, d=32, block_size=64, lq=lq, seed=1)
    ctx = np.maximum(case.context_lens, 0)
    got = oatt.paged_attention_ref(case.q, case.k_cache, case.v_cache, case.block_tables, ctx, case.scale)
    for b, c in enumerate(ctx):
        K = oatt.gather_paged(case.k_cache, case.block_tables[b], c)
        V = oatt.gather_paged(case.v_cache, case.block_tables[b], c)
        want = dense_ref(case.q[b], K, V, case.scale, lq, c)
        assert np.abs(got[b] - want).max() < 2e-5


def test_bottom_right_mask_by_hand():
    # Lq=2 queries over Lk=3 keys: query 0 sees keys 0,1 ; query 1 sees 0,1,2.
    d = 4
    q = np.zeros((1, 2, 1, d), np.float32)
    K = np.zeros((1, 4, 1, d), np.float32)
    V = np.zeros((1, 4, 1, d), np.float32)
    V[0, :3, 0, 0] = [1.0, 2.0, 4.0]
    out = oatt.paged_attention_ref(q, K, V, np.zeros((1, 1), np.int32), np.asarray([3], np.int32), 1.0)
    assert np.isclose(out[0, 0, 0, 0], 1.5) and np.isclose(out[0, 1, 0, 0], 7.0 / 3.0)


def test_empty_rows_are_zero():
    case = cases.make_paged_case([0, 5], 4, 2, d=16, block_size=64, seed=2)
    out = oatt.paged_attention_ref(case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens, 0.3)
    assert (out[0] == 0).all() and np.abs(out[1]).sum() > 0


def test_gqa_head_mapping():
    """Query head h reads kv head h // (Hq/Hkv): permuting kv heads permutes head groups."""
    case = cases.make_paged_case([70], 8, 4, d=16, block_size=64, seed=3)
    base = oatt.paged_attention_ref(case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens, 0.25)
    perm = np.array([2, 0, 3, 1])
    q2 = case.q.reshape(1, 1, 4, 2, 16)[:, :, perm].reshape(case.q.shape)
    got = oatt.paged_attention_ref(q2, case.k_cache[:, :, perm], case.v_cache[:, :, perm], case.block_tables,
                                   case.context_lens, 0.25)
    assert np.allclose(got.reshape(1, 1, 4, 2, 16), base.reshape(1, 1, 4, 2, 16)[:, :, perm], atol=1e-6)


def test_prefill_paged_equals_packed():
    """The prefix-cache form (keys from the paged cache) equals the packed form on the same rows."""
    c = cases.make_prefix_prefill_case([5, 70, 130], 128, 4, 2, d=16, block_size=64, seed=4)
    kref, vref = c.k.copy(), c.v.copy()
    from oracle import kv_store
    kv_store.store_kvcache_ref(c.k_new, c.v_new, kref, vref, c.slot_mapping)
    paged = oatt.varlen_prefill_ref(c.q, kref, vref, c.cu_seqlens_q, c.cu_seqlens_k, c.scale, c.block_tables)
    lk = np.diff(c.cu_seqlens_k)
    Kp = np.concatenate([oatt.gather_paged(kref, c.block_tables[s], lk[s]) for s in range(len(lk))])
    Vp = np.concatenate([oatt.gather_paged(vref, c.block_tables[s], lk[s]) for s in range(len(lk))])
    packed = oatt.varlen_prefill_ref(c.q, Kp, Vp, c.cu_seqlens_q, c.cu_seqlens_k, c.scale)
    assert np.abs(paged - packed).max() == 0


def test_prefill_without_cache_is_causal():
    c = cases.make_prefill_case([1, 9], 4, 2, d=16, seed=5)
    out = oatt.varlen_prefill_ref(c.q, c.k, c.v, c.cu_seqlens_q, c.cu_seqlens_k, c.scale)
    # the first query of each sequence sees only its own key: output = that key's value
    assert np.allclose(out[0], np.repeat(c.v[0], 2, axis=0), atol=1e-6)
    assert np.allclose(out[1], np.repeat(c.v[1], 2, axis=0), atol=1e-6)
