"""install(fuse_row_parallel=True) dispatch, checked with 2 gloo ranks on CPU.

The patched RowParallelLinear.forward (nanovllm/layers/linear.py:152-156) must send bias-free
2-D bf16 layers with N % 256 == 0, K % 64 == 0 and M within the buffers to the fused
GEMM + all-reduce, with this rank's activations and weight shard, and everything else to the
stock forward; both ranks take the same branch.  The CUDA kernel itself is tested on GPUs
(tests/test_oproj_gpu.py); here a stand-in computes F.linear + all_reduce so that the results
of both branches can be compared with the stock layer.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


class StandIn:
    """F.linear then all_reduce, recording each call's shapes."""

    def __init__(self):
        self.calls = []

    def __call__(self, x, w):
        self.calls.append((tuple(x.shape), tuple(w.shape)))
        y = torch.nn.functional.linear(x, w)
        dist.all_reduce(y)
        return y


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, REF)
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        from nanovllm.layers import linear
        integrate = pkg.integrate
        stock = linear.RowParallelLinear.forward
        integrate._ORIGINAL_ROW[:] = [stock]
        stand_in = StandIn()
        integrate._RowParallelState.get = classmethod(lambda cls, n, dev: stand_in)
        fused = integrate._fused_row_parallel_forward

        torch.manual_seed(3)  # the same full weight on every rank
        layer = linear.RowParallelLinear(256, 512, bias=False).to(torch.bfloat16)
        layer.weight_loader(layer.weight, torch.randn(512, 256).to(torch.bfloat16))
        assert layer.weight.shape == (512, 256 // world)
        results = []

        def run(x, lay=layer):
            n0 = len(stand_in.calls)
            y = fused(lay, x)
            y_ref = stock(lay, x)
            return len(stand_in.calls) - n0, torch.equal(y, y_ref)

        x_full = torch.randn(40, 256).to(torch.bfloat16)
        x = x_full.chunk(world, dim=1)[rank].contiguous()
        results.append(("bf16 2-D", run(x), (1, True)))
        results.append(("fp32 input", run(x.float().contiguous(), _fp32_copy(layer, linear)), (0, True)))
        results.append(("non-unit inner stride", run(x_full[:, rank::world]), (0, True)))
        wide = torch.randn(40, 256 // world + 4).to(torch.bfloat16)
        results.append(("rows not 16-byte aligned", run(wide[:, :256 // world]), (0, True)))
        results.append(("base not 16-byte aligned", run(wide[:, 1:1 + 256 // world]), (0, True)))
        old = integrate._RowParallelState.max_tokens
        integrate._RowParallelState.max_tokens = 39
        results.append(("M above the buffers", run(x), (0, True)))
        integrate._RowParallelState.max_tokens = old
        with_bias = linear.RowParallelLinear(256, 512, bias=True).to(torch.bfloat16)
        with_bias.weight.data.copy_(layer.weight.data)
        with_bias.bias.data.normal_()
        results.append(("bias", run(x, with_bias), (0, True)))
        odd = linear.RowParallelLinear(256, 320, bias=False).to(torch.bfloat16)
        odd.weight.data.normal_()
        results.append(("N % 256 != 0", run(x, odd), (0, True)))
        layer.tp_size = 1
        results.append(("tp_size 1", run(x), (0, True)))
        layer.tp_size = world
        ok = all(got == want for _, got, want in results)
        assert stand_in.calls == [((40, 256 // world), (512, 256 // world))], stand_in.calls

        # install(row_parallel_allreduce=True): F.linear kept, the all-reduce of decode-sized bf16
        # outputs through the two-shot kernel (a stand-in that all-reduces in place here)
        ar_calls = []

        def ar_stand_in(v):
            ar_calls.append(tuple(v.shape))
            dist.all_reduce(v)
            return v

        integrate._AllReduceState.get = classmethod(lambda cls, n, dev: ar_stand_in)
        ar_fwd = integrate._allreduce_row_parallel_forward

        def run_ar(x, lay=layer):
            n0 = len(ar_calls)
            y = ar_fwd(lay, x)
            y_ref = stock(lay, x)
            return len(ar_calls) - n0, torch.equal(y, y_ref)

        ar_results = [("bf16 decode rows", run_ar(x), (1, True)),
                      ("fp32 output", run_ar(x.float().contiguous(), _fp32_copy(layer, linear)), (0, True)),
                      ("bias", run_ar(x, with_bias), (1, True))]
        old = integrate._AllReduceState.max_tokens
        integrate._AllReduceState.max_tokens = 39
        ar_results.append(("rows above max_tokens", run_ar(x), (0, True)))
        integrate._AllReduceState.max_tokens = old
        layer.tp_size = 1
        ar_results.append(("tp_size 1", run_ar(x), (0, True)))
        layer.tp_size = world
        ok = ok and all(got == want for _, got, want in ar_results)
        assert ar_calls == [(40 * 512,), (40 * 512,)], ar_calls
        results += ar_results
        ret[rank] = ok or [r for r in results if r[1] != r[2]]
    except Exception as e:  # reported to the parent
        ret[rank] = repr(e)
    finally:
        dist.destroy_process_group()


def _fp32_copy(layer, linear):
    lay = linear.RowParallelLinear(256, 512, bias=False)
    lay.weight.data.copy_(layer.weight.data.float())
    return lay


def test_row_parallel_dispatch_two_ranks(nanovllm_ref):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    ret = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
    assert dict(ret) == {0: True, 1: True}, dict(ret)
