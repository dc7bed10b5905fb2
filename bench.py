"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Workload (the largest single-GPU configuration of the
paged-decode metric): one Qwen3-8B attention layer in decode -- 32 query /
8 kv heads, head_dim 128, bf16, block size 256 -- batch 512 with context
lengths lognormal(median 2048, sigma 0.5) capped at 32768 (seed 0).  The
configuration leaves sigma open; 0.5 is used.  With N GPUs the attention is
tensor-parallel by kv head: rank r owns kv heads [r*8/N, (r+1)*8/N) and
their query heads (nanovllm/models/qwen3.py:29-35), so the total work is
fixed (strong scaling) and ranks exchange nothing on the data path.

A step is one decode step of that layer: the KV-cache scatter of the 512
new tokens followed by paged decode attention over every cached token, and
with N > 1 GPUs the row-parallel all-reduce of the layer's o_proj output
([512, 4096] bf16, nanovllm/layers/linear.py:152-156) -- by default this
package's two-shot all-reduce over peer memory (AllReduce), with
--row-parallel nccl the reference's NCCL call, or (--row-parallel fused) the
o_proj GEMM and the all-reduce in one kernel of this package.  The per-rank cache (4.8 GB / N) is far larger than the
126 MB L2, so no flush is needed between steps.  Inputs are synthetic
(random bf16, seeded).

  value      algorithmic HBM bytes of scatter + attention / device time of
             the whole step (GB/s, all ranks)
  e2e        the same bytes over the time of the user-facing call
             (Attention.forward, plus the all-reduce at N > 1) with
             host-side inputs copied in and the output copied back inside
             the timed region; device-timed, with the wall-clock time beside
  roofline   the paged-attention kernel alone: bytes / CUDA-event duration,
             against MEASURED_PEAKS.json's HBM copy bandwidth
  attention_us / row_parallel_us  each part of the step timed alone per rank
             (max over ranks)
  prefill_config3 / verify_config4  (1 GPU) the prefix-cached prefill and
             the speculative verify configurations, kernels timed alone
  cpu_baseline  the numpy oracle of the same math on the host cores

--impl reference times the reference path's math on the host CPU (the
oracle port; the reference itself is CUDA-only) on the same configuration.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ_TOTAL, HKV_TOTAL, HEAD_DIM, BLOCK = 32, 8, 128, 256
BATCH, SIGMA, CAP = 512, 0.5, 32768
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes (read + write) per paged-attention launch over its algorithmic bytes, from one
# ncu capture of a B = 64 case of the same context draw (ncu --set full --clock-control none
# -k regex:paged_attention -s 2 -c 1 python bench.py --batch 64 --steps 3 --warmup 1
# --no-cpu-baseline --no-extras); the full launch is too large to capture with every metric,
# and its traffic grows in proportion (K/V rows are read once), so traffic is reported scaled.
DRAM_TRAFFIC_RATIO = 1.032


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--workload", choices=["decode", "prefill", "verify", "engine", "qknorm", "sample", "oproj"], default="decode",
                    help="decode = config 5 (the bench line); prefill = config 3; verify = config 4; "
                         "engine = config 2 through nano-vLLM's own engine (1 GPU)")
    ap.add_argument("--engine-attn", choices=["b200", "b200-fused", "b200-fused-all", "b200-full", "b200-full-rp", "b200-full-ar", "flash_attn"], default="b200",
                    help="engine workload: this package's Attention, or the reference's stock flash-attn path")
    ap.add_argument("--engine-model", choices=["qwen3-0.6b", "qwen3-8b"], default="qwen3-0.6b")
    ap.add_argument("--engine-requests", type=int, default=256)
    ap.add_argument("--engine-tp", type=int, default=1, help="engine workload: tensor_parallel_size")
    ap.add_argument("--gpu-mem", type=float, default=0.5, help="engine KV-cache share of GPU memory")
    ap.add_argument("--rank-shape", type=int, default=0,
                    help="decode on one GPU with rank 0's head shard of an N-way tensor-parallel job "
                         "(per-rank kernel efficiency at TP N without N GPUs)")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="sequences in the batch (profiling runs use a smaller batch; the bench line uses 512)")
    ap.add_argument("--row-parallel", choices=["nccl", "b200", "fused", "none"], default="b200",
                    help="decode at N > 1: the row-parallel step inside the timed region -- nccl: dist.all_reduce "
                         "of the o_proj output [B, 4096] bf16; b200: the same all-reduce by this package's "
                         "two-shot kernel over peer memory (AllReduce); fused: o_proj GEMM + all-reduce in one "
                         "kernel of this package (OprojAllReduce); none: attention only")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode: leave out the prefill (config 3) and verify (config 4) keys")
    return ap.parse_args()


def workload(batch=BATCH):
    """Config 5 context lengths: lognormal(ln 2048, SIGMA) capped at CAP, seed 0
    (the same draw as the tests' case factory)."""
    rng = np.random.default_rng(0)
    c = np.exp(rng.normal(np.log(2048.0), SIGMA, size=batch))
    return np.clip(np.rint(c), 1, CAP).astype(np.int32)


def step_bytes(ctx, hq, hkv, width):
    """Algorithmic HBM bytes of one step (per rank): decode + store."""
    d, e = HEAD_DIM, 2
    B = len(ctx)
    decode = int(ctx.sum()) * 2 * hkv * d * e + B * hq * d * e * 2 + 4 * B * (1 + width)
    store = B * 2 * 2 * hkv * d * e + 4 * B
    return decode, store


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _peak_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def _all_host_threads():
    """BLAS thread limit raised to every host core (torchrun sets OMP_NUM_THREADS=1)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=os.cpu_count() or 1)
    except Exception:
        import contextlib
        return contextlib.nullcontext()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(ctx, hq, hkv, seconds, per_step=None):
    """Time the numpy oracle of one decode (+store) over sequences of the batch."""
    from oracle import attention as oatt
    from oracle import kv_store
    from oracle.cases import randn_bf16
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    sample = list(range(24)) if per_step is None else list(range(per_step))
    data = []
    for b in sample:
        c = int(ctx[b])
        nblk = (c + BLOCK - 1) // BLOCK
        kc = randn_bf16(rng, (nblk, BLOCK, hkv, HEAD_DIM), 0.09)
        vc = randn_bf16(rng, (nblk, BLOCK, hkv, HEAD_DIM), 0.09)
        q = randn_bf16(rng, (1, 1, hq, HEAD_DIM), 0.09)
        kn = randn_bf16(rng, (1, hkv, HEAD_DIM), 0.09)
        bt = np.arange(nblk, dtype=np.int32)[None]
        slot = np.asarray([(c - 1) // BLOCK * BLOCK + (c - 1) % BLOCK], np.int32)
        data.append((kc, vc, q, kn, bt, np.asarray([c], np.int32), slot))

    def one(item):
        kc, vc, q, kn, bt, cl, slot = item
        kv_store.store_kvcache_ref(kn, kn, kc, vc, slot)
        oatt.paged_attention_ref(q, kc, vc, bt, cl, HEAD_DIM ** -0.5)
        d, s = step_bytes(cl, hq, hkv, bt.shape[1])
        return d + s

    one(data[0])  # warm
    t0 = time.perf_counter()
    nbytes, n, tokens = 0, 0, 0
    while True:
        for item in data:
            nbytes += one(item)
            n += 1
            tokens += int(item[5][0])
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 4), "unit": "GB/s", "cores": int(cores), "kind": "port",
            "sample": f"{n} sequence-decodes ({tokens} cached tokens) cycling over the first {len(data)} sequences "
                      f"of the batch, {hkv} kv / {hq} q heads, numpy fp32 oracle, {dt:.1f} s"}


def run_reference(args, rank, world):
    """Reference arm: the path's math on the host CPU (rank 0 only)."""
    if rank != 0:
        return
    ctx = workload()
    hq, hkv = HQ_TOTAL // world, HKV_TOTAL // world
    # each step: one sequence-decode of the batch (bounded so that the run takes ~minutes)
    from oracle import attention as oatt
    from oracle import kv_store
    from oracle.cases import randn_bf16
    rng = np.random.default_rng(0)
    items = []
    for b in range(min(32, BATCH)):
        c = int(ctx[b])
        nblk = (c + BLOCK - 1) // BLOCK
        items.append((randn_bf16(rng, (nblk, BLOCK, hkv, HEAD_DIM), 0.09),
                      randn_bf16(rng, (nblk, BLOCK, hkv, HEAD_DIM), 0.09),
                      randn_bf16(rng, (1, 1, hq, HEAD_DIM), 0.09), randn_bf16(rng, (1, hkv, HEAD_DIM), 0.09),
                      np.arange(nblk, dtype=np.int32)[None], np.asarray([c], np.int32),
                      np.asarray([c - 1], np.int32)))

    def step(i):
        kc, vc, q, kn, bt, cl, slot = items[i % len(items)]
        kv_store.store_kvcache_ref(kn, kn, kc, vc, slot)
        oatt.paged_attention_ref(q, kc, vc, bt, cl, HEAD_DIM ** -0.5)
        d, s = step_bytes(cl, hq, hkv, bt.shape[1])
        return d + s

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    nbytes = sum(step(i) for i in range(args.steps))
    dt = time.perf_counter() - t0
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    v = nbytes / dt / 1e9
    line = {"metric": "paged-decode attn HBM GB/s", "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": config_dict(world, ctx),
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": int(cores), "kind": "port",
                             "sample": f"each step one sequence-decode (store + attention) cycling over the first "
                                       f"{len(items)} sequences of the batch; numpy fp32 oracle"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(world, ctx):
    return {"workload": "config5: Qwen3-8B attention layer decode (store_kvcache + paged attention)",
            "batch": len(ctx), "q_heads": HQ_TOTAL, "kv_heads": HKV_TOTAL, "head_dim": HEAD_DIM, "block_size": BLOCK,
            "context_lens": f"lognormal(ln 2048, {SIGMA}) capped {CAP}, seed 0", "sum_ctx": int(ctx.sum()),
            "parallelism": f"tp{world} (kv-head sharded)",
            "l2": "no flush: per-step KV bytes per rank >> 126 MB L2"}


def _time(torch, stream, fn, steps, warmup):
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def measure_prefill(pkg, torch, dev, steps, warmup):
    """Config 3: 64 sequences share a 768-token prefix (3 cached blocks), unique
    suffixes U[64, 512]; Qwen3-0.6B attention shape (16 q / 8 kv heads); scatter
    of the suffix K/V + causal prefill over the paged cache.  Returns the step
    time, the prefill kernel alone (CUDA events) and its roofline."""
    hq, hkv, d, bs, prefix = 16, 8, 128, 256, 768
    rng = np.random.default_rng(0)
    suffix = rng.integers(64, 513, size=64).astype(np.int32)
    lk = suffix + prefix
    nblk = (lk + bs - 1) // bs
    pool = 3 + int((nblk - 3).sum())
    perm = rng.permutation(pool).astype(np.int32)
    bt = np.full((64, int(nblk.max())), -1, np.int32)
    o = 3
    for s_ in range(64):
        bt[s_, :3] = perm[:3]
        bt[s_, 3:nblk[s_]] = perm[o:o + nblk[s_] - 3]
        o += nblk[s_] - 3
    slots = np.concatenate([bt[s_, np.arange(prefix, lk[s_]) // bs] * bs + np.arange(prefix, lk[s_]) % bs
                            for s_ in range(64)]).astype(np.int32)
    T = int(suffix.sum())
    g = torch.Generator(device=dev).manual_seed(3)
    rnd = lambda *shape: (torch.randn(*shape, generator=g, device=dev) * d ** -0.5).to(torch.bfloat16)
    kc, vc = rnd(pool, bs, hkv, d), rnd(pool, bs, hkv, d)
    q, kn, vn = rnd(T, hq, d), rnd(T, hkv, d), rnd(T, hkv, d)
    cu_q = torch.from_numpy(np.concatenate([[0], np.cumsum(suffix)]).astype(np.int32)).to(dev)
    cu_k = torch.from_numpy(np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)).to(dev)
    btd, sl = torch.from_numpy(bt).to(dev), torch.from_numpy(slots).to(dev)
    out = torch.empty_like(q)

    def attn():
        pkg.flash_attn_varlen_func(q, kc, vc, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k, max_seqlen_q=int(suffix.max()),
                                   max_seqlen_k=int(lk.max()), softmax_scale=d ** -0.5, causal=True,
                                   block_table=btd, out=out)

    def step():
        pkg.store_kvcache(kn, vn, kc, vc, sl)
        attn()

    stream = torch.cuda.current_stream(dev)
    flops = 4.0 * hq * d * float((suffix.astype(np.float64) * prefix + suffix * (suffix + 1) / 2.0).sum())
    with ClockSampler(dev.index or 0) as clk:
        ms = _time(torch, stream, step, steps, warmup)
        kms = _time(torch, stream, attn, steps, warmup)
    assert pkg.ops.prefill_error() == 0
    peak = _peak_tflops()
    return {"workload": "config3: 64 seqs, shared 768-token prefix, suffix U[64,512], 16/8 heads, D 128",
            "tokens": T, "ms_per_step": round(ms, 4), "step_TFLOPs": round(flops / (ms / 1e3) / 1e12, 2),
            "roofline": {"bound": "tensor", "kernel": "prefill_kernel", "achieved": round(flops / (kms / 1e3) / 1e12, 1),
                         "peak": peak[0], "peak_kind": peak[1], "unit": "TFLOP/s",
                         "frac": round(flops / (kms / 1e3) / 1e12 / peak[0], 4), "us_per_launch": round(kms * 1e3, 2),
                         "flops_per_launch": flops},
            "clocks": clk.summary()}


def run_prefill(args, pkg, torch, dev):
    r = measure_prefill(pkg, torch, dev, args.steps, args.warmup)
    print(json.dumps({
        "metric": "prefix-cached prefill attn TFLOP/s (useful causal flops)", "value": r["step_TFLOPs"],
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded random bf16)",
        "config": {"workload": r["workload"], "tokens": r["tokens"]},
        "roofline": r["roofline"], "clocks": r["clocks"]}), flush=True)


def measure_verify(pkg, torch, dev, steps, warmup):
    """Config 4: speculative verify on the Qwen3-0.6B attention shape -- B=128,
    k=4 drafts (5 queries each), context U[512, 4096]; scatter of the 5 new
    tokens, (k+1)-query paged attention, then acceptance sampling over
    vocab 151936 (logits N(0, 2^2), drafts correlated with the target).
    Returns the step time and each kernel timed alone (CUDA events)."""
    B, k, V, hq, hkv, d, bs = 128, 4, 151936, 16, 8, 128, 256
    rng = np.random.default_rng(0)
    ctx = rng.integers(512, 4097, size=B).astype(np.int32)
    nblk = (ctx + bs - 1) // bs
    nb = int(nblk.sum())
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((B, int(nblk.max())), -1, np.int32)
    off = np.concatenate([[0], np.cumsum(nblk)])
    for b in range(B):
        bt[b, :nblk[b]] = perm[off[b]:off[b + 1]]
    pos = np.concatenate([np.arange(c - k - 1, c) for c in ctx])
    rows = np.repeat(np.arange(B), k + 1)
    slots = (bt[rows, pos // bs] * bs + pos % bs).astype(np.int32)
    g = torch.Generator(device=dev).manual_seed(4)
    rnd = lambda *shape: (torch.randn(*shape, generator=g, device=dev) * d ** -0.5).to(torch.bfloat16)
    kc, vc = rnd(nb, bs, hkv, d), rnd(nb, bs, hkv, d)
    q, kn, vn = rnd(B, k + 1, hq, d), rnd(B * (k + 1), hkv, d), rnd(B * (k + 1), hkv, d)
    cl, btd, sl = (torch.from_numpy(x).to(dev) for x in (ctx, bt, slots))
    tl = torch.randn(B, k + 1, V, generator=g, device=dev) * 2.0
    dl = (tl[:, :k] + torch.randn(B, k, V, generator=g, device=dev)).contiguous()
    gum = -torch.log(-torch.log(torch.rand(B, k, V, generator=g, device=dev).clamp_min(1e-20)))
    dt = (dl + gum).argmax(-1).to(torch.int32)
    del gum
    ua, us = torch.rand(B, k, generator=g, device=dev), torch.rand(B, generator=g, device=dev)
    out = torch.empty_like(q)
    ws = pkg.paged_workspace(dev, k + 1, hq // hkv, B * hkv)
    sws = torch.empty(max(pkg.lib().b200_spec_accept_workspace_size(B, k, V), 256), dtype=torch.uint8, device=dev)

    def attn():
        pkg.paged_attention(q, kc, vc, cl, btd, d ** -0.5, out=out, workspace=ws)

    def accept():
        pkg.spec_accept(tl, dl, dt, ua, us, workspace=sws)

    def step():
        pkg.store_kvcache(kn, vn, kc, vc, sl)
        attn()
        accept()

    stream = torch.cuda.current_stream(dev)
    attn_bytes = int(ctx.sum()) * 2 * hkv * d * 2 + B * (k + 1) * hq * d * 2 * 2
    acc_bytes = (2 * k + 1) * B * V * 4
    with ClockSampler(dev.index or 0) as clk:
        ms = _time(torch, stream, step, steps, warmup)
        ams = _time(torch, stream, attn, steps, warmup)
        sms = _time(torch, stream, accept, steps, warmup)
    assert pkg.workspace_error(ws) == 0, "device wait timed out"
    flops = 4.0 * float(ctx.sum()) * (k + 1) * hq * d
    hbm = measured_peak()
    tfl = _peak_tflops()
    toks, num = pkg.spec_accept(tl, dl, dt, ua, us, workspace=sws)
    return {"workload": "config4: B=128, k=4, ctx U[512,4096], 16/8 heads, V 151936", "ms_per_step": round(ms, 4),
            "attention": {"us": round(ams * 1e3, 2), "GBps": round(attn_bytes / (ams / 1e3) / 1e9, 1),
                          "frac_hbm": round(attn_bytes / (ams / 1e3) / 1e9 / hbm[0], 4),
                          "TFLOPs": round(flops / (ams / 1e3) / 1e12, 2),
                          "frac_bf16_peak": round(flops / (ams / 1e3) / 1e12 / tfl[0], 4),
                          "bytes_per_launch": attn_bytes, "flops_per_launch": flops},
            "acceptance": {"us": round(sms * 1e3, 2), "GBps": round(acc_bytes / (sms / 1e3) / 1e9, 1),
                           "frac_hbm": round(acc_bytes / (sms / 1e3) / 1e9 / hbm[0], 4),
                           "mean_accepted": round(float(num.float().mean().item()) - 1, 3)},
            "peaks": {"hbm_GBps": hbm[0], "hbm_kind": hbm[1], "bf16_TFLOPs": tfl[0], "bf16_kind": tfl[1]},
            "clocks": clk.summary()}


def run_verify(args, pkg, torch, dev):
    r = measure_verify(pkg, torch, dev, args.steps, args.warmup)
    print(json.dumps({
        "metric": "speculative verify step ms (attention + acceptance)", "value": r["ms_per_step"], "unit": "ms",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "dtype": "bf16/fp32",
        "data": "synthetic (seeded)", "config": {"workload": r["workload"]},
        "attention": r["attention"], "acceptance": r["acceptance"], "clocks": r["clocks"]}), flush=True)


def _time_graph(torch, stream, fn, steps, warmup, calls=20):
    """Device time per call with `calls` calls captured in one CUDA graph (no host launch
    overhead in the timed region, as in nano-vLLM's decode graphs)."""
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    ms = _time(torch, stream, g.replay, max(steps // calls, 5), 3) / calls
    del g
    return ms


def run_qknorm(args, pkg, torch, dev):
    """Fused q/k RMSNorm + RoPE + KV scatter (the Qwen3 attention layer's epilogue of
    the QKV projection) on config 3's prefill tokens (0.6B shape) and on config 5's
    decode batch (8B shape), beside the reference's own unfused modules (RMSNorm and
    RotaryEmbedding under torch.compile, Triton store_kvcache) from baseline/_ref."""
    d, base, max_pos, eps = 128, 1e6, 40960, 1e-6
    inv_freq = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float) / d))
    freqs = torch.einsum("i,j -> ij", torch.arange(max_pos, dtype=torch.float), inv_freq)
    cs = torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(dev)
    ref = None
    try:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from nanovllm.layers.layernorm import RMSNorm
        from nanovllm.layers.rotary_embedding import RotaryEmbedding
        from nanovllm.layers.attention import store_kvcache as ref_store
        ref = (RMSNorm, RotaryEmbedding, ref_store)
    except Exception as e:  # the reference arm is optional here
        ref_err = f"{type(e).__name__}: {e}"
    hbm = measured_peak()
    results = {}
    rng = np.random.default_rng(0)
    for name, T, hq, hkv in (("config3 prefill tokens, Qwen3-0.6B", 18715, 16, 8),
                             ("config5 decode batch, Qwen3-8B", 512, 32, 8)):
        g = torch.Generator(device=dev).manual_seed(5)
        qkv = (torch.randn(T, (hq + 2 * hkv) * d, generator=g, device=dev) * 1.5).to(torch.bfloat16)
        positions = torch.from_numpy(rng.integers(0, 4096, T).astype(np.int64)).to(dev)
        wq = (1 + 0.1 * torch.randn(d, generator=g, device=dev)).to(torch.bfloat16)
        wk = (1 + 0.1 * torch.randn(d, generator=g, device=dev)).to(torch.bfloat16)
        nslots = T + 4096
        kc = torch.zeros(nslots // 256 + 1, 256, hkv, d, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        slots = torch.from_numpy(rng.permutation(nslots)[:T].astype(np.int32)).to(dev)
        fused = lambda: pkg.qk_norm_rope_store(qkv, positions, hq, hkv, wq, wk, eps, cs, kc, vc, slots)
        stream = torch.cuda.current_stream(dev)
        timer = _time if T > 4096 else _time_graph  # small calls: graph replay, as the engine's decode does
        with ClockSampler(dev.index or 0) as clk:
            ms = timer(torch, stream, fused, args.steps, args.warmup)
        nbytes = T * ((hq + 2 * hkv) * d * 2 + hq * d * 2 + hkv * d * 2 + 2 * hkv * d * 2 + d * 4 + 12)
        r = {"tokens": T, "heads": f"{hq}/{hkv}", "us": round(ms * 1e3, 2),
             "timing": "event loop" if T > 4096 else "CUDA graph of 20 calls, per call",
             "GBps": round(nbytes / (ms / 1e3) / 1e9, 1), "frac_hbm": round(nbytes / (ms / 1e3) / 1e9 / hbm[0], 4),
             "bytes_per_call": nbytes, "gpu_launches_per_call": 1, "clocks": clk.summary()}
        if ref is not None:
            RMSNorm, RotaryEmbedding, ref_store = ref
            qn, kn = RMSNorm(d, eps).to(dev, torch.bfloat16), RMSNorm(d, eps).to(dev, torch.bfloat16)
            rope = RotaryEmbedding(d, d, max_pos, base).to(dev)

            def unfused():
                q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
                q = qn(q.view(-1, hq, d))
                k = kn(k.view(-1, hkv, d))
                q, k = rope(positions, q, k)
                ref_store(k, v.view(-1, hkv, d), kc, vc, slots)
            rms = timer(torch, stream, unfused, max(args.steps // 4, 20), max(args.warmup, 5))
            r["reference_unfused_us"] = round(rms * 1e3, 2)
            r["speedup_vs_reference"] = round(rms / ms, 2)
        else:
            r["reference_unfused"] = f"unavailable: {ref_err}"
        results[name] = r
    print(json.dumps({"metric": "fused q/k norm + RoPE + KV scatter GB/s", "unit": "GB/s",
                      "value": results["config3 prefill tokens, Qwen3-0.6B"]["GBps"], "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
                      "data": "synthetic (seeded)", "peak_GBps": hbm[0], "peak_kind": hbm[1],
                      "cases": results}), flush=True)


def run_oproj(args, pkg, torch, dev, world, rank):
    """Qwen3-8B attention output projection, row-parallel over the ranks (K = 4096 / world,
    N = 4096), for a decode batch: the fused GEMM + all-reduce kernel against the reference's
    path, F.linear (cuBLAS) then dist.all_reduce (NCCL).  Device time, max over ranks."""
    import torch.distributed as dist
    from datetime import timedelta
    if not dist.is_initialized():
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29531")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev, rank=rank,
                                world_size=world)
    hidden, k_total = 4096, 4096
    K = k_total // world
    results = {}
    op = pkg.OprojAllReduce(dist.group.WORLD, max_tokens=512, hidden=hidden)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    w = (torch.randn(hidden, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    for M in (512, 64, 8):
        a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)

        def fused():
            op(a, w)

        def reference():
            y = torch.nn.functional.linear(a, w)
            dist.all_reduce(y)
        times = {}

        def device_us(run, calls):
            torch.cuda.synchronize()
            dist.barrier(device_ids=[dev.index])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / calls], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.item() * 1e3

        for name, fn in (("fused", fused), ("reference", reference)):
            for _ in range(max(args.warmup, 3)):
                fn()

            def eager():
                for _ in range(args.steps):
                    fn()
            times[name] = device_us(eager, args.steps)
            # as nano-vLLM's decode runs it: captured in a CUDA graph (20 calls per replay)
            graph, side = torch.cuda.CUDAGraph(), torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
                for _ in range(20):
                    fn()
            stream.wait_stream(side)
            graph.replay()
            reps = max(1, args.steps // 20)

            def replay():
                for _ in range(reps):
                    graph.replay()
            times[name + "_graph"] = device_us(replay, reps * 20)
            del graph
        flops = 2.0 * M * hidden * k_total
        results[f"M={M}"] = {"fused_us": round(times["fused"], 2), "reference_us": round(times["reference"], 2),
                             "speedup": round(times["reference"] / times["fused"], 2),
                             "fused_graph_us": round(times["fused_graph"], 2),
                             "reference_graph_us": round(times["reference_graph"], 2),
                             "graph_speedup": round(times["reference_graph"] / times["fused_graph"], 2),
                             "fused_TFLOPs_total": round(flops / (times["fused_graph"] * 1e-6) / 1e12, 1),
                             "nvlink_bytes_in_per_rank": (world - 1) * M * hidden * 2}
    assert op.error() == 0
    if rank == 0:
        print(json.dumps({"metric": "o_proj GEMM + all-reduce us per call (device, max over ranks)",
                          "unit": "us", "higher_is_better": False, "n_gpus": world, "steps": args.steps,
                          "warmup": args.warmup, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"Qwen3-8B o_proj, hidden 4096, tp{world}"},
                          "value": results["M=512"]["fused_graph_us"], "cases": results}), flush=True)
    dist.destroy_process_group()


def run_sample(args, pkg, torch, dev):
    """Fused sampler on a decode batch's logits (B = 512, Qwen3 vocab 151,936, bf16 as the
    LM head returns them), beside the reference's own Sampler (torch.compile) from baseline/_ref."""
    B, V = 512, 151936
    g = torch.Generator(device=dev).manual_seed(6)
    logits = (torch.randn(B, V, generator=g, device=dev) * 2).to(torch.bfloat16)
    temps = torch.empty(B, device=dev).uniform_(0.5, 1.5, generator=g)
    step = [0]

    def fused():
        step[0] += 1
        return pkg.sample(logits, temps, seed=1, offset=step[0])
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(dev.index or 0) as clk:
        ms = _time(torch, stream, fused, args.steps, args.warmup)
    hbm = measured_peak()
    nbytes = B * V * 2 + B * 12
    line = {"metric": "fused sampler GB/s (logits read once)", "value": round(nbytes / (ms / 1e3) / 1e9, 1),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "bf16 logits, fp32 math", "data": "synthetic logits N(0, 4), T U[0.5, 1.5]",
            "config": {"workload": "decode batch 512 x vocab 151936"}, "us_per_call": round(ms * 1e3, 2),
            "frac_hbm": round(nbytes / (ms / 1e3) / 1e9 / hbm[0], 4), "peak_kind": hbm[1],
            "gpu_launches_per_call": 2, "clocks": clk.summary()}
    try:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from nanovllm.layers.sampler import Sampler
        ref = Sampler()
        rms = _time(torch, stream, lambda: ref(logits, temps), max(args.steps // 4, 20), max(args.warmup, 5))
        line["reference_sampler_us"] = round(rms * 1e3, 2)
        line["speedup_vs_reference"] = round(rms / ms, 2)
    except Exception as e:
        line["reference_sampler"] = f"unavailable: {type(e).__name__}: {e}"
    print(json.dumps(line), flush=True)


QWEN3 = {
    "qwen3-0.6b": dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, tie_word_embeddings=True),
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, tie_word_embeddings=False),
}


def _qwen3_config_dir(name):
    """A Hugging Face config directory for a randomly initialised Qwen3 (no checkpoint here)."""
    import tempfile
    cfg = dict(QWEN3[name], architectures=["Qwen3ForCausalLM"], model_type="qwen3", head_dim=128, vocab_size=151936,
               max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1000000.0, attention_bias=False,
               hidden_act="silu", torch_dtype="bfloat16", dtype="bfloat16", bos_token_id=151643,
               eos_token_id=151645)
    d = tempfile.mkdtemp(prefix="b200_qwen3_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


class _IdTokenizer:
    """Prompts are token ids and generation ignores EOS, so no vocabulary is needed."""
    eos_token_id = -1

    @classmethod
    def from_pretrained(cls, *a, **k):
        return cls()

    def encode(self, text):
        return [ord(c) % 151936 for c in text]

    def decode(self, ids):
        return ""


def _random_init(model, path):
    """Stands in for nanovllm.utils.loader.load_model: N(0, 0.02) weights, unit norms."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    with torch.no_grad():
        for _, prm in model.named_parameters():
            if prm.dim() == 1:
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02, generator=g)


def _engine_worker_setup():
    """Run in every engine process (spawned ranks too): the stand-in weight loader and
    tokenizer, and the reference checkout on sys.path."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import nanovllm.engine.llm_engine as le
    import nanovllm.engine.model_runner as mr
    le.AutoTokenizer = _IdTokenizer
    mr.load_model = _random_init


def engine_watchdog(target, period=0.5):
    """Stop within a second when a tensor-parallel engine worker dies: rank 0 would otherwise
    wait in its next collective until the process group's timeout.  Workers are the child
    processes spawned with `target` (nano-vLLM's llm_engine.ModelRunner, llm_engine.py:24-30);
    other children (compile pools) are ignored.  Kills the remaining workers, prints one JSON
    error line, exits 3.  Returns an event that stops the watch (set it once the measured work
    is done, before shutdown)."""
    import threading
    from multiprocessing import context as mp_context
    workers = []
    stop = threading.Event()
    start = mp_context.SpawnProcess.start

    def start_and_record(proc):
        # the target is only readable before start() (which drops it)
        if getattr(proc, "_target", None) is target:
            workers.append(proc)
        return start(proc)

    mp_context.SpawnProcess.start = start_and_record

    def loop():
        while not stop.is_set():
            for proc in list(workers):
                code = proc.exitcode
                if code is None:
                    continue
                if code != 0:
                    print(json.dumps({"error": f"engine worker pid {proc.pid} exited with code {code}"}),
                          flush=True)
                    for other in workers:
                        if other.exitcode is None:
                            other.kill()
                    os._exit(3)
                workers.remove(proc)
            stop.wait(period)

    threading.Thread(target=loop, name="engine-watchdog", daemon=True).start()
    return stop


def run_engine(args, pkg):
    """Config 2 through nano-vLLM's own LLM engine (scheduler, block manager,
    prefix cache, CUDA-graph decode): 256 requests, prompt and output lengths
    U[100, 1024], prompt ids uniform over the vocabulary, temperature 0.6,
    ignore_eos; output tokens / wall time of generate() as in the reference
    bench.py:21-27.  Weights are random (no checkpoint is available)."""
    import torch
    _engine_worker_setup()
    tp = args.engine_tp
    if args.engine_attn.startswith("b200"):
        a = args.engine_attn
        pkg.install(fuse_qk_epilogue=a != "b200",
                    fuse_sampler=a in ("b200-fused-all", "b200-full", "b200-full-rp", "b200-full-ar"),
                    device_metadata=a in ("b200-full", "b200-full-rp", "b200-full-ar"),
                    fuse_row_parallel=a == "b200-full-rp", row_parallel_allreduce=a == "b200-full-ar",
                    workers=tp > 1, worker_setup=("bench:_engine_worker_setup",))
    elif tp > 1:
        # stock path: the spawned ranks still need the stand-in loader and tokenizer
        import functools
        import nanovllm.engine.llm_engine as le
        import __graft_entry__ as entry
        le.ModelRunner = functools.partial(entry.nanovllm_worker_stock, setup=("bench:_engine_worker_setup",))
    from nanovllm import LLM, SamplingParams
    import nanovllm.engine.llm_engine as le
    watch = engine_watchdog(le.ModelRunner) if tp > 1 else None
    path = _qwen3_config_dir(args.engine_model)
    t_init = time.perf_counter()
    llm = LLM(path, enforce_eager=False, max_model_len=4096, gpu_memory_utilization=args.gpu_mem,
              tensor_parallel_size=tp)
    t_init = time.perf_counter() - t_init
    rng = np.random.default_rng(0)
    n = args.engine_requests
    prompts = [rng.integers(0, 151936, size=int(rng.integers(100, 1025))).tolist() for _ in range(n)]
    sps = [SamplingParams(temperature=0.6, ignore_eos=True, max_tokens=int(rng.integers(100, 1025))) for _ in range(n)]
    # Warm-up with varied prompt lengths and batch sizes, so that torch.compile's
    # shape specialisations of the reference's other layers happen before timing.
    llm.generate([p[:int(k)] for p, k in zip(prompts[:24], np.linspace(100, 1024, 24))],
                 SamplingParams(temperature=0.6, ignore_eos=True, max_tokens=24), use_tqdm=False)
    with ClockSampler(torch.cuda.current_device()) as clk:
        t = time.perf_counter()
        out = llm.generate(prompts, sps, use_tqdm=False)
        t = time.perf_counter() - t
    if watch is not None:
        watch.set()  # measured work done: worker exits during shutdown are not failures of the run
    total = sum(sp.max_tokens for sp in sps)
    assert all(len(o["token_ids"]) == sp.max_tokens for o, sp in zip(out, sps))
    print(json.dumps({
        "metric": "e2e output tokens/s (nano-vLLM engine, config 2)", "value": round(total / t, 1), "unit": "tok/s",
        "n_gpus": tp, "higher_is_better": True, "dtype": "bf16", "data": "synthetic prompts, random-init weights",
        "attention": args.engine_attn, "vs_baseline": round(total / t / 1434.13, 3),
        "config": {"workload": f"config2: {args.engine_model}, {n} requests, in/out U[100,1024], T=0.6, ignore_eos",
                   "output_tokens": total, "seconds": round(t, 3), "engine_init_s": round(t_init, 1),
                   "tensor_parallel_size": tp,
                   "gpu_memory_utilization": args.gpu_mem},
        "clocks": clk.summary()}), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        world = args.gpus if "WORLD_SIZE" not in os.environ else world
    assert HKV_TOTAL % world == 0, f"{world} GPUs do not divide {HKV_TOTAL} kv heads"
    if args.impl == "reference":
        with _all_host_threads():
            run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "engine":
        assert world == 1, "the engine workload runs on one GPU"
        run_engine(args, pkg)
        return
    if args.workload == "oproj":
        run_oproj(args, pkg, torch, dev, world, rank)
        return
    if args.workload != "decode":
        assert world == 1, "the prefill / verify / qknorm workloads run on one GPU"
        {"prefill": run_prefill, "verify": run_verify, "qknorm": run_qknorm,
         "sample": run_sample}[args.workload](args, pkg, torch, dev)
        return
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    ctx = workload(args.batch)
    BATCH = len(ctx)
    shard = args.rank_shape if (args.rank_shape and world == 1) else world
    assert HKV_TOTAL % shard == 0, f"{shard} does not divide {HKV_TOTAL} kv heads"
    hq, hkv = HQ_TOTAL // shard, HKV_TOTAL // shard
    nblk = (ctx + BLOCK - 1) // BLOCK
    nb = int(nblk.sum())
    width = int(nblk.max())
    rng = np.random.default_rng(1)
    perm = rng.permutation(nb).astype(np.int32)
    bt_np = np.full((BATCH, width), -1, np.int32)
    off = np.concatenate([[0], np.cumsum(nblk)])
    for b in range(BATCH):
        bt_np[b, :nblk[b]] = perm[off[b]:off[b + 1]]
    slots_np = np.asarray([bt_np[b, (c - 1) // BLOCK] * BLOCK + (c - 1) % BLOCK for b, c in enumerate(ctx)], np.int32)

    g = torch.Generator(device=dev).manual_seed(100 + rank)
    kc = (torch.randn(nb, BLOCK, hkv, HEAD_DIM, generator=g, device=dev) * 0.09).to(torch.bfloat16)
    vc = (torch.randn(nb, BLOCK, hkv, HEAD_DIM, generator=g, device=dev) * 0.09).to(torch.bfloat16)
    q = (torch.randn(BATCH, hq, HEAD_DIM, generator=g, device=dev) * 0.09).to(torch.bfloat16)
    kn = (torch.randn(BATCH, hkv, HEAD_DIM, generator=g, device=dev) * 0.09).to(torch.bfloat16)
    vn = (torch.randn(BATCH, hkv, HEAD_DIM, generator=g, device=dev) * 0.09).to(torch.bfloat16)
    bt = torch.from_numpy(bt_np).to(dev)
    cl = torch.from_numpy(ctx).to(dev)
    slots = torch.from_numpy(slots_np).to(dev)
    out = torch.empty(BATCH, 1, hq, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    scale = HEAD_DIM ** -0.5
    ws = pkg.paged_workspace(dev, 1, hq // hkv, BATCH * hkv)

    # The row-parallel step that follows attention at N > 1 (linear.py:152-156): the o_proj
    # output y [B, 4096] is all-reduced (NCCL), or o_proj and the all-reduce run as one kernel.
    rp = args.row_parallel if world > 1 else "none"
    hidden = HQ_TOTAL * HEAD_DIM
    y = torch.randn(BATCH, hidden, generator=g, device=dev).to(torch.bfloat16) if rp != "none" else None
    oproj, wo, allreduce = None, None, None
    if rp == "b200":
        allreduce = pkg.AllReduce(dist.group.WORLD, BATCH * hidden)
    if rp == "fused":
        oproj = pkg.OprojAllReduce(dist.group.WORLD, max_tokens=BATCH, hidden=hidden)
        wo = (torch.randn(hidden, hq * HEAD_DIM, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    if rp == "b200":
        # o_proj's output built in the symmetric input slot; the next layer reads the result slot
        y_in, y_out = allreduce.input_buffer(y.numel()), allreduce.result_buffer(y.numel())
        y_in.copy_(y.view(-1))

    def row_parallel():
        if rp == "nccl":
            dist.all_reduce(y)
        elif rp == "b200":
            allreduce(y_in, out=y_out)
        elif rp == "fused":
            oproj(out.view(BATCH, hq * HEAD_DIM), wo, out=y)

    def attention():
        pkg.paged_attention(q.unsqueeze(1), kc, vc, cl, bt, scale, out=out, workspace=ws)

    def step():
        pkg.store_kvcache(kn, vn, kc, vc, slots)
        attention()
        row_parallel()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    # -- timed region: K steps on the device, max over ranks
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    ms = e0.elapsed_time(e1)

    def alone(fn, n):
        """Per-call device time of fn alone, CUDA events on its stream."""
        torch.cuda.synchronize(dev)
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(n):
            fn()
        a1.record(stream)
        torch.cuda.synchronize(dev)
        return a0.elapsed_time(a1) / n

    # -- each part of the step alone: the dominant kernel (paged attention), the row-parallel step
    kern_ms = alone(attention, max(20, min(args.steps, 200)))
    rp_ms = alone(row_parallel, max(20, min(args.steps, 200))) if rp != "none" else 0.0
    assert pkg.workspace_error(ws) == 0, "device wait timed out"
    if oproj is not None:
        assert oproj.error() == 0, "o_proj all-reduce wait timed out"
    if allreduce is not None:
        assert allreduce.error() == 0, "all-reduce wait timed out"

    # -- e2e: the user-facing Attention.forward with host inputs and output read-back
    from learn_nano_vllm_b200 import context as pctx
    attn = pkg.Attention(hq, HEAD_DIM, scale, hkv)
    attn.k_cache, attn.v_cache = kc, vc
    h_q = q.cpu().pin_memory()
    h_k, h_v = kn.cpu().pin_memory(), vn.cpu().pin_memory()
    h_bt, h_cl, h_sl = bt.cpu().pin_memory(), cl.cpu().pin_memory(), slots.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_q, d_k, d_v = torch.empty_like(q), torch.empty_like(kn), torch.empty_like(vn)
    d_bt, d_cl, d_sl = torch.empty_like(bt), torch.empty_like(cl), torch.empty_like(slots)
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_bt, h_cl, h_sl))
    d2h = h_out.numel() * h_out.element_size()
    hosts = (h_q, h_k, h_v, h_bt, h_cl, h_sl)

    def layer(b):
        pctx.set_context(False, slot_mapping=b[5], context_lens=b[4], block_tables=b[3])
        o = attn(b[0], b[1], b[2])
        if rp == "nccl":
            dist.all_reduce(y)
        elif rp == "b200":
            allreduce(y_in, out=y_out)
        elif rp == "fused":
            oproj(o.view(BATCH, hq * HEAD_DIM), wo, out=y)
        return o

    serial_bufs = (d_q, d_k, d_v, d_bt, d_cl, d_sl)

    def e2e_serial(n):
        """Each step copies its inputs up, computes and copies the output back, in order on one stream."""
        for _ in range(n):
            for d, h in zip(serial_bufs, hosts):
                d.copy_(h, non_blocking=True)
            o = layer(serial_bufs)
            h_out.copy_(o, non_blocking=True)

    # As a serving loop runs it: step i+1's inputs are copied up on a second stream while step i
    # computes, and step i's output is copied back on that stream as soon as step i is done.
    cs = torch.cuda.Stream(dev)
    bufs = [serial_bufs, tuple(torch.empty_like(d) for d in serial_bufs)]
    h_outs = [h_out, torch.empty(out.shape, dtype=out.dtype).pin_memory()]

    def e2e_pipelined(n, keep):
        """keep collects the steps' outputs: alive until the caller has synchronised, so the
        allocator never hands a block the copy stream still reads to a later step."""
        ev_up = [torch.cuda.Event(), torch.cuda.Event()]
        ev_done = [torch.cuda.Event(), torch.cuda.Event()]
        cs.wait_stream(stream)
        with torch.cuda.stream(cs):
            for d, h in zip(bufs[0], hosts):
                d.copy_(h, non_blocking=True)
            ev_up[0].record(cs)
        for i in range(n):
            j = i & 1
            stream.wait_event(ev_up[j])
            o = layer(bufs[j])
            keep.append(o)
            ev_done[j].record(stream)
            with torch.cuda.stream(cs):
                if i + 1 < n:
                    if i >= 1:  # the other buffer set was read by step i - 1
                        cs.wait_event(ev_done[j ^ 1])
                    for d, h in zip(bufs[j ^ 1], hosts):
                        d.copy_(h, non_blocking=True)
                    ev_up[j ^ 1].record(cs)
                cs.wait_event(ev_done[j])
                h_outs[j].copy_(o, non_blocking=True)
        stream.wait_stream(cs)

    def timed_e2e(fn, n):
        """Device time (events on the compute stream, which waits for the copy stream at the end)
        and wall-clock time per step."""
        torch.cuda.synchronize(dev)
        barrier()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        x0.record(stream)
        fn(n)
        x1.record(stream)
        torch.cuda.synchronize(dev)
        wall = (time.perf_counter() - w0) * 1e3 / n
        barrier()
        return x0.elapsed_time(x1) / n, wall

    ne = max(10, min(args.steps, 200))
    e2e_serial(3)
    # an untimed pass of the same length fills the allocator's pool with the blocks the kept
    # outputs of the timed pass need (no cudaMalloc inside the timed region)
    warm = []
    e2e_pipelined(ne, warm)
    torch.cuda.synchronize(dev)
    del warm
    serial_ms, serial_wall_ms = timed_e2e(e2e_serial, ne)
    kept = []
    e2e_ms, wall_ms = timed_e2e(lambda n: e2e_pipelined(n, kept), ne)
    del kept
    pctx.reset_context()

    # every rank on its own GPU, every rank in the communicator
    gpus_active, comm_ok = 1, True
    if world > 1:
        uuids = [None] * world
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(dev).uuid))
        gpus_active = len(set(uuids))
        one = torch.ones(1, device=dev)
        dist.all_reduce(one)
        comm_ok = int(one.item()) == world == dist.get_world_size()

    dec_b, store_b = step_bytes(ctx, hq, hkv, width)
    t = torch.tensor([ms, kern_ms, e2e_ms, rp_ms, wall_ms, serial_ms, serial_wall_ms], dtype=torch.float64,
                     device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kern_ms, e2e_ms, rp_ms, wall_ms, serial_ms, serial_wall_ms = t.tolist()
    if oproj is not None or allreduce is not None:
        torch.cuda.synchronize(dev)
        barrier()
        del oproj, allreduce
    total_bytes = (dec_b + store_b) * world
    value = total_bytes * args.steps / (ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    achieved = dec_b / (kern_ms / 1e3) / 1e9

    if rank == 0:
        e2e_gbs = (dec_b + store_b) * world / (e2e_ms / 1e3) / 1e9
        line = {"metric": "paged-decode attn HBM GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random bf16 KV cache, q, new k/v)",
                "config": dict(config_dict(world, ctx), **({"rank_shape": f"one GPU running rank 0's shard of tp{shard}"}
                                                        if shard != world else {}),
                               **({"row_parallel": {"nccl": "NCCL all-reduce of the o_proj output [B, 4096] bf16",
                                                    "b200": "all-reduce of the o_proj output [B, 4096] bf16 by "
                                                            "this package's two-shot kernel (AllReduce, peer "
                                                            "loads and stores, no multicast; the output built in "
                                                            "its symmetric input slot, the result read from its "
                                                            "result slot)",
                                                    "fused": "o_proj GEMM + all-reduce in one kernel "
                                                             "(OprojAllReduce, peer stores, no multicast)"}[rp]}
                                  if rp != "none" else {})),
                "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s",
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                        "ms_per_step": round(e2e_ms, 5), "wall_ms_per_step": round(wall_ms, 5),
                        "wall_value": round((dec_b + store_b) * world / (wall_ms / 1e3) / 1e9, 2),
                        "api": "Attention.forward (decode)" + (" + row-parallel all-reduce" if rp != "none" else "")
                               + ", pinned host buffers; step i+1's inputs copied up on a second stream while "
                                 "step i computes, step i's output copied back behind it",
                        "serial": {"value": round((dec_b + store_b) * world / (serial_ms / 1e3) / 1e9, 2),
                                   "ms_per_step": round(serial_ms, 5), "wall_ms_per_step": round(serial_wall_ms, 5),
                                   "note": "copy up, compute, copy back in order on one stream"}},
                "roofline": {"bound": "hbm", "kernel": "paged_attention_kernel", "achieved": round(achieved, 1),
                             "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                             "traffic": round(DRAM_TRAFFIC_RATIO * dec_b),
                             "traffic_kind": f"scaled: {DRAM_TRAFFIC_RATIO} x algorithmic bytes (ncu, B=64 capture)",
                             "bytes_per_launch": int(dec_b), "us_per_launch": round(kern_ms * 1e3, 2)},
                "attention_us": round(kern_ms * 1e3, 2),
                "gpus_active": gpus_active, "comm_nranks_ok": comm_ok,
                "gpu_launches": (3 if rp == "fused" else 2) * args.steps,
                "clocks": clk.summary()}
        if rp != "none":
            line["row_parallel_us"] = round(rp_ms * 1e3, 2)
            line["row_parallel_bytes"] = BATCH * hidden * 2
    if world == 1 and not args.no_extras:
        # the denser configurations of the path, kernels timed alone (1 GPU)
        n = max(10, min(args.steps, 50))
        extras = {"prefill_config3": measure_prefill(pkg, torch, dev, n, args.warmup),
                  "verify_config4": measure_verify(pkg, torch, dev, n, args.warmup)}
        line.update(extras)
    if rank == 0:
        if not args.no_cpu_baseline:
            with _all_host_threads():
                line["cpu_baseline"] = cpu_baseline(ctx, hq, hkv, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
