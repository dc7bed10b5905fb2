"""Causal varlen prefill (tcgen05) on the GPU vs the fp32 oracle and flash-attn goldens."""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import cases, kv_store
from tests.helpers import assert_attn_close, dev_bf16, dev_i32, host

pytestmark = pytest.mark.gpu


def run_packed(pkg, c, dtype=torch.bfloat16, strided_v=False):
    q, k = dev_bf16(c.q, dtype), dev_bf16(c.k, dtype)
    if strided_v:  # the v view of a fused qkv projection (qwen3.py:79-82)
        T, hkv, d = c.v.shape
        buf = torch.zeros(T, 3 * hkv * d, dtype=dtype, device="cuda")
        buf[:, 2 * hkv * d:] = dev_bf16(c.v, dtype).reshape(T, -1)
        v = buf[:, 2 * hkv * d:].view(T, hkv, d)
    else:
        v = dev_bf16(c.v, dtype)
    lq = np.diff(c.cu_seqlens_q)
    out = pkg.flash_attn_varlen_func(q, k, v, cu_seqlens_q=dev_i32(c.cu_seqlens_q), cu_seqlens_k=dev_i32(c.cu_seqlens_k),
                                     max_seqlen_q=int(lq.max()), max_seqlen_k=int(lq.max()), softmax_scale=c.scale,
                                     causal=True)
    torch.cuda.synchronize()
    assert pkg.ops.prefill_error() == 0
    return host(out)


@pytest.mark.parametrize("lens", [[1], [9], [127], [128], [129], [300, 1, 57], [1000], [64, 512, 257, 2, 130]])
@pytest.mark.parametrize("hq,hkv", [(16, 8), (16, 16), (8, 1), (12, 4), (32, 8)])
def test_packed_against_oracle(pkg, lens, hq, hkv):
    c = cases.make_prefill_case(lens, hq, hkv, seed=sum(lens) + hq)
    got = run_packed(pkg, c)
    want = oatt.varlen_prefill_ref(c.q, c.k, c.v, c.cu_seqlens_q, c.cu_seqlens_k, c.scale)
    assert_attn_close(got, want, f"lens={lens} {hq}/{hkv}")


def test_strided_v_and_fp16(pkg):
    c = cases.make_prefill_case([200, 77], 16, 8, seed=3)
    want = oatt.varlen_prefill_ref(c.q, c.k, c.v, c.cu_seqlens_q, c.cu_seqlens_k, c.scale)
    assert_attn_close(run_packed(pkg, c, strided_v=True), want, "strided v")
    assert_attn_close(run_packed(pkg, c, dtype=torch.float16), want, "fp16")


def run_prefix(pkg, c, seqs=None):
    kc, vc = dev_bf16(c.k), dev_bf16(c.v)
    pkg.store_kvcache(dev_bf16(c.k_new), dev_bf16(c.v_new), kc, vc, dev_i32(c.slot_mapping))
    lq, lk = np.diff(c.cu_seqlens_q), np.diff(c.cu_seqlens_k)
    out = pkg.flash_attn_varlen_func(dev_bf16(c.q), kc, vc, cu_seqlens_q=dev_i32(c.cu_seqlens_q),
                                     cu_seqlens_k=dev_i32(c.cu_seqlens_k), max_seqlen_q=int(lq.max()),
                                     max_seqlen_k=int(lk.max()), softmax_scale=c.scale, causal=True,
                                     block_table=dev_i32(c.block_tables))
    torch.cuda.synchronize()
    assert pkg.ops.prefill_error() == 0
    kref, vref = c.k.copy(), c.v.copy()
    kv_store.store_kvcache_ref(c.k_new, c.v_new, kref, vref, c.slot_mapping)
    return host(out), kref, vref


def test_prefix_cached_small(pkg):
    c = cases.make_prefix_prefill_case([5, 70, 130, 256, 1], 512, 16, 8, seed=7)
    got, kref, vref = run_prefix(pkg, c)
    want = oatt.varlen_prefill_ref(c.q, kref, vref, c.cu_seqlens_q, c.cu_seqlens_k, c.scale, c.block_tables)
    assert_attn_close(got, want, "prefix small")


def test_config3_sampled_sequences(pkg):
    """BASELINE config 3 at full size; the oracle checks a sample of sequences."""
    c = cases.config3_case(seed=0)
    got, kref, vref = run_prefix(pkg, c)
    cq = c.cu_seqlens_q
    for s in [0, 1, 17, 40, 63]:
        sub_q = c.q[cq[s]:cq[s + 1]]
        lk = int(c.cu_seqlens_k[s + 1] - c.cu_seqlens_k[s])
        want = oatt.varlen_prefill_ref(sub_q, kref, vref, np.asarray([0, len(sub_q)], np.int32),
                                       np.asarray([0, lk], np.int32), c.scale, c.block_tables[s:s + 1])
        assert_attn_close(got[cq[s]:cq[s + 1]], want, f"config3 seq {s}")


def test_chunked_prefill_continuation(pkg):
    """A continuation chunk whose start is not block-aligned (scheduler.py:42-46)."""
    rng = np.random.default_rng(9)
    prefix, suffix = 300, [77]
    hq, hkv, d, bs = 16, 8, 128, 256
    lk = prefix + suffix[0]
    nb = (lk + bs - 1) // bs
    bt = rng.permutation(6)[:nb].astype(np.int32)[None]
    kc = cases.randn_bf16(rng, (6, bs, hkv, d), d ** -0.5)
    vc = cases.randn_bf16(rng, (6, bs, hkv, d), d ** -0.5)
    q = cases.randn_bf16(rng, (suffix[0], hq, d), d ** -0.5)
    cu_q = np.asarray([0, suffix[0]], np.int32)
    cu_k = np.asarray([0, lk], np.int32)
    out = pkg.flash_attn_varlen_func(dev_bf16(q), dev_bf16(kc), dev_bf16(vc), cu_seqlens_q=dev_i32(cu_q),
                                     cu_seqlens_k=dev_i32(cu_k), max_seqlen_q=suffix[0], max_seqlen_k=lk,
                                     softmax_scale=d ** -0.5, causal=True, block_table=dev_i32(bt))
    want = oatt.varlen_prefill_ref(q, kc, vc, cu_q, cu_k, d ** -0.5, bt)
    assert_attn_close(host(out), want, "chunked continuation")


@pytest.mark.parametrize("name", ["prefill_packed", "prefill_prefix"])
def test_against_flash_attn_golden(pkg, name):
    from tests.test_oracle_golden import golden_case
    kind, c, q, k, v, want, rows = golden_case(name)
    lq, lk = np.diff(c.cu_seqlens_q), np.diff(c.cu_seqlens_k)
    out = pkg.flash_attn_varlen_func(dev_bf16(q), dev_bf16(k), dev_bf16(v), cu_seqlens_q=dev_i32(c.cu_seqlens_q),
                                     cu_seqlens_k=dev_i32(c.cu_seqlens_k), max_seqlen_q=int(lq.max()),
                                     max_seqlen_k=int(lk.max()), softmax_scale=c.scale, causal=True,
                                     block_table=None if c.block_tables is None else dev_i32(c.block_tables))
    assert_attn_close(host(out)[rows], want.reshape(len(rows), *q.shape[1:]), name)


def test_cache_rows_past_keys_may_hold_nan(pkg):
    c = cases.make_prefix_prefill_case([5, 100], 256, 16, 8, seed=8)
    lk = np.diff(c.cu_seqlens_k)
    for s in range(2):  # poison every cache row past each sequence's keys
        for p in range(int(lk[s]), c.block_tables.shape[1] * 256):
            blk = c.block_tables[s, p // 256]
            if blk >= 0:
                c.k[blk, p % 256] = np.nan
                c.v[blk, p % 256] = np.nan
    got, kref, vref = run_prefix(pkg, c)
    want = oatt.varlen_prefill_ref(c.q, kref, vref, c.cu_seqlens_q, c.cu_seqlens_k, c.scale, c.block_tables)
    assert_attn_close(got, want, "nan tail")
