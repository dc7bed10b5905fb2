"""Child process of tests/test_oproj_gpu.py: one rank of the fused o_proj + all-reduce.

Usage: python tests/oproj_worker.py RANK WORLD PORT   (GPU = RANK).  Exits non-zero on a
mismatch; prints one JSON line per rank.
"""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def check_row_parallel(pkg, rank, world, dev):
    """install(fuse_row_parallel=True) on the reference's own RowParallelLinear
    (nanovllm/layers/linear.py:130-156): the patched forward against the stock one
    (F.linear + NCCL all-reduce), when the reference is installed in baseline/_ref."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nanovllm")):
        return 0.0
    sys.path.insert(0, ref)
    from nanovllm.layers import linear
    pkg.install(fuse_row_parallel=True)
    fused = linear.RowParallelLinear.forward
    stock = pkg.integrate._ORIGINAL_ROW[0]
    torch.manual_seed(99)  # same weights on every rank
    with torch.device(dev):
        layer = linear.RowParallelLinear(2048, 1024, bias=False).to(torch.bfloat16)
    full = (torch.randn(1024, 2048, device=dev) * 0.03).to(torch.bfloat16)
    layer.weight_loader(layer.weight, full)
    worst = 0.0
    for M in (64, 700, 3):
        x_full = torch.randn(M, 2048, device=dev).to(torch.bfloat16)
        x = x_full.chunk(world, dim=1)[rank].contiguous()
        y = fused(layer, x)
        y_ref = stock(layer, x)
        torch.cuda.synchronize()
        d = (y.float() - y_ref.float()).abs().max().item() / y_ref.float().abs().max().item()
        assert d <= 2 ** -6, ("row-parallel", M, d)
        worst = max(worst, d)
    pkg.install()  # stock RowParallelLinear again
    assert linear.RowParallelLinear.forward is stock
    return worst


def main():
    rank, world, port = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3])
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    worst = 0.0
    calls = 0
    # hidden 1024: at most 16 tiles, K split across the SMs; hidden 4096 up to 2560 tokens:
    # 80..320 tiles, unsplit on persistent CTAs (both accumulators of a CTA in use)
    for hidden, k_total, max_tokens, ms in ((1024, 2048, 512, [512, 100, 1, 300, 512, 257, 64, 512]),
                                            (4096, 1024, 2560, [2560, 600, 1200, 2559, 2560])):
        K = k_total // world
        op = pkg.OprojAllReduce(dist.group.WORLD, max_tokens=max_tokens, hidden=hidden)
        g = torch.Generator(device=dev).manual_seed(1234 + hidden)  # same draws on every rank
        w_full = (torch.randn(hidden, k_total, generator=g, device=dev) * 0.03).to(torch.bfloat16)
        w = w_full[:, rank * K:(rank + 1) * K].contiguous()

        def check(M, a_full, y, where):
            a = a_full[:, rank * K:(rank + 1) * K].contiguous()
            # reference 1: sum over ranks of each rank's bf16 partial, in fp32, rounded once
            parts = [(a_full[:, r * K:(r + 1) * K].float() @ w_full[:, r * K:(r + 1) * K].float().T).bfloat16()
                     for r in range(world)]
            ref = torch.stack([p.float() for p in parts]).sum(0).bfloat16()
            # reference 2: the reference engine's path, F.linear then NCCL all-reduce
            y_nccl = torch.nn.functional.linear(a, w)
            dist.all_reduce(y_nccl)
            torch.cuda.synchronize()
            scale = ref.float().abs().max().item()
            d1 = (y.float() - ref.float()).abs().max().item() / scale
            d2 = (y.float() - y_nccl.float()).abs().max().item() / scale
            assert torch.isfinite(y.float()).all(), where
            assert d1 <= 2 ** -6 and d2 <= 2 ** -6, (where, M, d1, d2)
            # every rank holds the same bits
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            assert all(torch.equal(gathered[0], t) for t in gathered), ("ranks disagree", where)
            return max(d1, d2)

        for step, M in enumerate(ms):
            a_full = torch.randn(M, k_total, generator=g, device=dev).to(torch.bfloat16)
            y = op(a_full[:, rank * K:(rank + 1) * K].contiguous(), w)
            worst = max(worst, check(M, a_full, y, f"hidden {hidden} step {step}"))
        # the same call captured in a CUDA graph and replayed on new inputs
        M = ms[1]
        a_static = torch.zeros(M, K, dtype=torch.bfloat16, device=dev)
        out_static = torch.empty(M, hidden, dtype=torch.bfloat16, device=dev)
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
            op(a_static, w, out=out_static)
        torch.cuda.current_stream(dev).wait_stream(s)
        for rep in range(3):
            a_full = torch.randn(M, k_total, generator=g, device=dev).to(torch.bfloat16)
            a_static.copy_(a_full[:, rank * K:(rank + 1) * K])
            graph.replay()
            worst = max(worst, check(M, a_full, out_static, f"hidden {hidden} graph replay {rep}"))
        del graph
        assert op.error() == 0, "a bounded wait gave up"
        calls += op.calls
    worst = max(worst, check_row_parallel(pkg, rank, world, dev))
    print(json.dumps({"rank": rank, "world": world, "calls": calls, "worst_rel": worst}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
