"""Paged decode / verify attention on the GPU vs the fp32 oracle.

Test matrix after the study guide's decode matrix (master_nano-vllm-v2.md:4117-4131):
context lengths 1, 15, 255, 256, 257, 1024, 4096; head ratios 16/16, 16/8,
16/4 (plus 32/8 and 8/1); batches 1, 3, 17; random and reversed block
tables; CUDA-graph padding rows (context 0).
"""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import cases, kv_store
from tests.helpers import assert_attn_close, dev_bf16, dev_i32, host

pytestmark = pytest.mark.gpu


def run(pkg, case, dtype=torch.bfloat16, reverse_tables=False):
    bt = case.block_tables.copy()
    if reverse_tables:  # same blocks, descending physical order
        for b in range(bt.shape[0]):
            n = (max(int(case.context_lens[b]), 1) + case.block_size - 1) // case.block_size
            bt[b, :n] = np.sort(bt[b, :n])[::-1]
        slots = cases.slots_for(bt, np.maximum(case.context_lens, case.q.shape[1]), case.q.shape[1], case.block_size)
        case.slot_mapping = np.where(np.repeat(case.context_lens > 0, case.q.shape[1]), slots, -1).astype(np.int32)
        case.block_tables = bt
    kc, vc = dev_bf16(case.k_cache, dtype), dev_bf16(case.v_cache, dtype)
    pkg.store_kvcache(dev_bf16(case.k_new, dtype), dev_bf16(case.v_new, dtype), kc, vc, dev_i32(case.slot_mapping))
    out = pkg.paged_attention(dev_bf16(case.q, dtype), kc, vc, dev_i32(case.context_lens), dev_i32(case.block_tables),
                              case.scale)
    kref, vref = case.k_cache.copy(), case.v_cache.copy()
    kv_store.store_kvcache_ref(case.k_new, case.v_new, kref, vref, case.slot_mapping)
    want = oatt.paged_attention_ref(case.q, kref, vref, case.block_tables, case.context_lens, case.scale)
    return host(out), want


def test_config1(pkg):
    """Qwen3-0.6B layer, B=8, ctx U[100,1024], 64-block pool."""
    got, want = run(pkg, cases.config1_case(seed=0))
    assert_attn_close(got, want, "config1")


@pytest.mark.parametrize("ctx", [1, 15, 255, 256, 257, 1024, 4096])
@pytest.mark.parametrize("hq,hkv", [(16, 16), (16, 8), (16, 4)])
def test_context_lengths(pkg, ctx, hq, hkv):
    case = cases.make_paged_case([ctx, max(1, ctx // 3), ctx + 1 if ctx < 4096 else 4000], hq, hkv, seed=ctx + hq)
    got, want = run(pkg, case)
    assert_attn_close(got, want, f"ctx={ctx} {hq}/{hkv}")


@pytest.mark.parametrize("batch", [1, 3, 17])
@pytest.mark.parametrize("reverse", [False, True])
def test_batches_and_tables(pkg, batch, reverse):
    rng = np.random.default_rng(batch)
    ctx = rng.integers(1, 2000, size=batch)
    got, want = run(pkg, cases.make_paged_case(ctx, 16, 8, seed=batch), reverse_tables=reverse)
    assert_attn_close(got, want, f"B={batch} reverse={reverse}")


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 1), (64, 8)])
def test_other_group_sizes(pkg, hq, hkv):
    got, want = run(pkg, cases.make_paged_case([700, 65, 3000], hq, hkv, seed=hq))
    assert_attn_close(got, want, f"{hq}/{hkv}")


@pytest.mark.parametrize("lq,hq,hkv", [(5, 16, 8), (2, 16, 2), (4, 16, 4), (3, 8, 8), (16, 4, 4)])
def test_speculative_verify_queries(pkg, lq, hq, hkv):
    """(k+1)-query verify: causal within the new tokens, bottom-right aligned."""
    case = cases.make_paged_case([512, 4096, 7, 1300, 2], hq, hkv, lq=lq, seed=lq * 10 + hkv)
    got, want = run(pkg, case)
    assert_attn_close(got, want, f"verify lq={lq} {hq}/{hkv}")


def test_fp16(pkg):
    got, want = run(pkg, cases.make_paged_case([1000, 33, 2049], 16, 8, seed=11), dtype=torch.float16)
    assert_attn_close(got, want, "fp16")


def test_padding_rows_are_zero_and_do_not_read(pkg):
    """Graph padding: ctx 0 rows (model_runner.py:208-209) return zeros; their
    block-table rows hold garbage that must never be read."""
    case = cases.make_paged_case([300, 0, 0, 70], 16, 8, seed=5)
    case.block_tables[1:3] = 123456789  # would be far out of range if read
    got, want = run(pkg, case)
    assert (got[1:3] == 0).all()
    assert_attn_close(got, want, "padding")


def test_cache_rows_past_context_are_ignored(pkg):
    """Unwritten cache rows past the context may hold NaN bits."""
    case = cases.make_paged_case([5, 300], 16, 8, seed=6)
    case.k_cache[:] = np.nan
    case.v_cache[:] = np.inf
    for b, c in enumerate(case.context_lens):  # valid rows get finite data
        for p in range(c):
            blk = case.block_tables[b, p // 256]
            case.k_cache[blk, p % 256] = 0.01 * (p % 7)
            case.v_cache[blk, p % 256] = 0.02 * (p % 5)
    got, want = run(pkg, case)
    assert_attn_close(got, want, "nan tail")


def test_graph_capture_and_workspace_reuse(pkg):
    """Capture once at a padded batch, replay with new contexts, tables and q."""
    B, hq, hkv = 16, 16, 8
    nb = 64
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = (torch.randn(nb, 256, hkv, 128, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    vc = (torch.randn(nb, 256, hkv, 128, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    q = torch.zeros(B, 1, hq, 128, dtype=torch.bfloat16, device="cuda")
    ctx = torch.zeros(B, dtype=torch.int32, device="cuda")
    bt = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    out = torch.empty(B, 1, hq, 128, dtype=torch.bfloat16, device="cuda")
    ws = pkg.paged_workspace(q.device, 1, hq // hkv, B * hkv)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pkg.paged_attention(q, kc, vc, ctx, bt, 0.088, out=out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            pkg.paged_attention(q, kc, vc, ctx, bt, 0.088, out=out)
    torch.cuda.current_stream().wait_stream(s)
    rng = np.random.default_rng(1)
    kn, vn = host(kc), host(vc)
    for it in range(4):
        live = int(rng.integers(1, B + 1))
        c = np.zeros(B, np.int32)
        c[:live] = rng.integers(1, 4096, size=live)
        tables = np.stack([rng.permutation(nb)[:16] for _ in range(B)]).astype(np.int32)
        qn = (rng.standard_normal((B, 1, hq, 128)) * 0.1).astype(np.float32)
        q.copy_(torch.from_numpy(qn).to(torch.bfloat16))
        ctx.copy_(torch.from_numpy(c))
        bt.copy_(torch.from_numpy(tables))
        graph.replay()
        torch.cuda.synchronize()
        want = oatt.paged_attention_ref(host(q), kn, vn, tables, c, 0.088)
        assert_attn_close(host(out), want, f"replay {it}")
        assert (host(out)[live:] == 0).all()
    assert pkg.workspace_error(ws) == 0
    assert int(ws[:12].view(torch.int32).abs().sum()) == 0          # scheduler re-armed
    assert int(ws[256:256 + 4 * 65536].view(torch.int32).abs().sum()) == 0  # split counters reset
    del graph


def test_config5_sampled_rows_and_determinism(pkg):
    """BASELINE config 5 at full size (B=512, lognormal ctx <= 32768, 32/8 heads):
    sampled rows against the oracle, and bitwise-identical repeated runs."""
    ctx = cases.config5_context_lens(512, 0.5, seed=0)
    ctx[3] = 32768
    hq, hkv, bs = 32, 8, 256
    nblk = (ctx + bs - 1) // bs
    nb = int(nblk.sum())
    g = torch.Generator(device="cuda").manual_seed(5)
    kc = torch.randn(nb, bs, hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(nb, bs, hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g, device="cuda").to(torch.int32)
    W = int(nblk.max())
    bt = torch.full((512, W), -1, dtype=torch.int32, device="cuda")
    off = np.concatenate([[0], np.cumsum(nblk)])
    for b in range(512):
        bt[b, :nblk[b]] = perm[off[b]:off[b + 1]]
    q = (torch.randn(512, 1, hq, 128, generator=g, device="cuda") / 11.3).to(torch.bfloat16)
    cl = dev_i32(ctx)
    o1 = pkg.paged_attention(q, kc, vc, cl, bt, 128 ** -0.5)
    o2 = pkg.paged_attention(q, kc, vc, cl, bt, 128 ** -0.5)
    assert torch.equal(o1, o2)
    rows = [0, 3, 17, int(np.argmin(ctx)), 511]
    qn, btn = host(q), bt.cpu().numpy()
    for b in rows:
        blocks = btn[b, :nblk[b]]
        K = host(kc[torch.from_numpy(blocks).long().cuda()]).reshape(1, -1, hkv, 128)
        V = host(vc[torch.from_numpy(blocks).long().cuda()]).reshape(1, -1, hkv, 128)
        Kp = K.reshape(len(blocks), bs, hkv, 128)
        Vp = V.reshape(len(blocks), bs, hkv, 128)
        want = oatt.paged_attention_ref(qn[b:b + 1], Kp, Vp, np.arange(len(blocks), dtype=np.int32)[None],
                                        ctx[b:b + 1], 128 ** -0.5)
        assert_attn_close(host(o1[b:b + 1]), want, f"config5 row {b} ctx {ctx[b]}")


@pytest.mark.parametrize("name", ["decode_config1", "decode_16_4", "decode_32_8", "verify_5"])
def test_against_flash_attn_golden(pkg, name):
    """Our kernel vs flash-attn 2.8.3's output on the same inputs (fixture from a B200)."""
    from tests.test_oracle_golden import golden_case
    kind, c, q, k, v, want, _ = golden_case(name)
    out = pkg.paged_attention(dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_i32(c.context_lens),
                              dev_i32(c.block_tables), c.scale)
    assert_attn_close(host(out), want.reshape(q.shape), name)


def test_wait_that_runs_out_is_reported(pkg):
    """A stage that is never filled: with the test hook the producer warp issues no loads and
    every wait is limited to 2 ms.  The call must return with error bit 1 in its workspace
    (no hang, no fault), and the next call on the same workspace must run normally."""
    lib = pkg.lib()
    case = cases.make_paged_case([300, 1100, 5, 2600], 16, 8, lq=1, seed=3)
    q, kc, vc = dev_bf16(case.q), dev_bf16(case.k_cache), dev_bf16(case.v_cache)
    cl, bt = dev_i32(case.context_lens), dev_i32(case.block_tables)
    ws = torch.zeros(lib.b200_paged_attention_workspace_size(4096, 1, 2, 128), dtype=torch.uint8, device="cuda")
    assert lib.b200_testing_idle_producer(1, 2_000_000) == 0
    pkg.paged_attention(q, kc, vc, cl, bt, case.scale, workspace=ws)
    assert pkg.workspace_error(ws) & 1
    ws.zero_()  # the error word is sticky; the rest of the control region is re-armed by the kernel
    out = pkg.paged_attention(q, kc, vc, cl, bt, case.scale, workspace=ws)
    assert pkg.workspace_error(ws) == 0
    want = oatt.paged_attention_ref(host(q), host(kc), host(vc), case.block_tables, case.context_lens, case.scale)
    assert_attn_close(host(out), want, "after the stalled call")
