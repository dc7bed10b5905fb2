"""Tensor-parallel sharding of attention by kv head, checked with 2 gloo ranks (CPU).

Rank r of N owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads
(nanovllm/models/qwen3.py:29-35; QKVParallelLinear, linear.py:106-112).
Attention needs no communication; the only collective on the layer is the
row-parallel all-reduce after o_proj (linear.py:152-156).  Each rank runs the
oracle on its shard; the gathered outputs must equal the unsharded result,
and the all-reduced o_proj partial products must equal the full product.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oatt
from oracle import cases


def shard_heads(case, rank, world):
    hq, hkv = case.q.shape[2], case.k_cache.shape[2]
    kv0, kv1 = rank * hkv // world, (rank + 1) * hkv // world
    g = hq // hkv
    return (case.q[:, :, kv0 * g:kv1 * g], case.k_cache[:, :, kv0:kv1], case.v_cache[:, :, kv0:kv1])


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = cases.make_paged_case([300, 37, 1000], 32, 8, d=32, block_size=64, lq=1, seed=5)
        q, kc, vc = shard_heads(case, rank, world)
        part = oatt.paged_attention_ref(q, kc, vc, case.block_tables, case.context_lens, case.scale)
        parts = [torch.zeros_like(torch.from_numpy(part)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        full = np.concatenate([p.numpy() for p in parts], axis=2)
        want = oatt.paged_attention_ref(case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens,
                                        case.scale)
        ok_attn = np.array_equal(full, want)
        # row-parallel o_proj: each rank multiplies its attention columns by its weight rows
        rng = np.random.default_rng(0)
        w = rng.standard_normal((32 * 32, 64)).astype(np.float32)
        flat = want.reshape(want.shape[0], -1)
        cols = flat.shape[1] // world
        y = torch.from_numpy(flat[:, rank * cols:(rank + 1) * cols] @ w[rank * cols:(rank + 1) * cols])
        dist.all_reduce(y)
        ok_ar = np.allclose(y.numpy(), flat @ w, atol=1e-4)
        ret[rank] = (ok_attn, ok_ar)
    finally:
        dist.destroy_process_group()


def test_kv_head_sharding_two_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = mp.get_context("spawn").Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(2, port, ret), nprocs=2, join=True)
    assert ret[0] == (True, True) and ret[1] == (True, True)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_the_heads(world):
    case = cases.make_paged_case([20], 32, 8, d=16, block_size=64, seed=1)
    qs = [shard_heads(case, r, world)[0] for r in range(world)]
    assert np.array_equal(np.concatenate(qs, axis=2), case.q)
    assert all(q.shape[2] == 32 // world for q in qs)


def _dying_worker(rank, world, port, ret):
    """Rank 1 leaves between steps (raises before its next collective); rank 0 must get an
    error from that collective within the process group's short timeout, not wait forever."""
    from datetime import timedelta
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # step 1: both ranks
    if rank == 1:
        ret[1] = "left"
        os._exit(0)      # gone before step 2, with no collective in flight
    t0 = time.time()
    try:
        dist.all_reduce(t)  # step 2: the peer never joins
        ret[0] = "completed"
    except Exception as e:  # gloo reports the closed peer or the timeout
        ret[0] = ("error", round(time.time() - t0, 1), type(e).__name__)


def test_dead_rank_ends_the_next_collective_with_an_error():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert ret.get(1) == "left"
    status = ret.get(0)
    assert isinstance(status, tuple) and status[0] == "error" and status[1] < 30, status
