"""Child process of tests/test_allreduce_gpu.py: one rank of the two-shot all-reduce.

Usage: python tests/allreduce_worker.py RANK WORLD PORT   (GPU = RANK).  Exits non-zero on a
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


def inputs(n, world, step, dev):
    """Every rank's input of one call (the same draws on every rank)."""
    g = torch.Generator(device=dev).manual_seed(4321 + 7 * step + n)
    return [(torch.randn(n, generator=g, device=dev) * (r + 1)).to(torch.bfloat16) for r in range(world)]


def main():
    rank, world, port = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3])
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    max_elems = 512 * 4096
    op = pkg.AllReduce(dist.group.WORLD, max_elems)

    def check(xs, y, where):
        # the definition: fp32 sum in rank order, one rounding to bf16 -- bit for bit
        want = xs[0].float()
        for x in xs[1:]:
            want = want + x.float()
        want = want.bfloat16()
        assert torch.equal(y, want), (where, (y.float() - want.float()).abs().max().item())
        # against the reference engine's path (NCCL all-reduce), within bf16 rounding
        y_nccl = xs[rank].clone()
        dist.all_reduce(y_nccl)
        scale = want.float().abs().max().item()
        d = (y.float() - y_nccl.float()).abs().max().item() / scale
        assert d <= 2 ** -6, (where, d)
        return d

    worst, calls = 0.0, 0
    # sizes: one unit, ragged slices, decode batches of Qwen3-8B's hidden size, the largest
    for step, n in enumerate([8, 8 * 777, 4096, 64 * 4096, 512 * 4096, 8 * 12345, 512 * 4096, 16]):
        xs = inputs(n, world, step, dev)
        if step % 2:
            y = op(xs[rank].clone())  # in place
        else:
            y = torch.empty_like(xs[rank])
            op(xs[rank], out=y)
        calls += 1
        worst = max(worst, check(xs, y, f"step {step} n {n}"))
    # zero-copy: the input built in the symmetric input slot, the result read from the result slot
    for step, n in enumerate([4096 * 8, 512 * 4096, 8 * 999]):
        xs = inputs(n, world, 50 + step, dev)
        op.input_buffer(n).copy_(xs[rank])
        y = op(op.input_buffer(n), out=op.result_buffer(n))
        calls += 1
        worst = max(worst, check(xs, y.clone(), f"zero-copy {step} n {n}"))
    # captured in a CUDA graph and replayed on new inputs
    n = 512 * 4096
    x_static = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    y_static = torch.empty_like(x_static)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        op(x_static, out=y_static)
    torch.cuda.current_stream(dev).wait_stream(s)
    for rep in range(4):
        xs = inputs(n, world, 100 + rep, dev)
        x_static.copy_(xs[rank])
        graph.replay()
        calls += 1
        worst = max(worst, check(xs, y_static, f"graph replay {rep}"))
    del graph
    # many back-to-back calls without a host sync between them (slot parity alternation)
    xs_list = [inputs(4096 * 8, world, 200 + i, dev) for i in range(12)]
    ys = [op(xs[rank].clone()) for xs in xs_list]
    calls += len(ys)
    for i, (xs, y) in enumerate(zip(xs_list, ys)):
        worst = max(worst, check(xs, y, f"back-to-back {i}"))
    assert op.error() == 0, "a bounded wait gave up"
    print(json.dumps({"rank": rank, "world": world, "calls": calls, "worst_rel_vs_nccl": worst}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
