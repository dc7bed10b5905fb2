"""Generate tests/golden/store_kvcache.npz from the reference's own KV scatter.

Runs nano-vLLM's Triton `store_kvcache` (nanovllm/layers/attention.py:10-40)
on CPU tensors under TRITON_INTERPRET=1 and records inputs and the caches it
produced.  Needs the reference checkout (its directory as argv[1] or in
NANOVLLM_REF) and triton; it is run once in the development container, and its
output is committed.  The GPU box never runs it.

Usage:  TRITON_INTERPRET=1 python tests/golden/gen_store_golden.py [REF_DIR]
"""
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANOVLLM_REF", "")
if not os.path.isdir(os.path.join(REF, "nanovllm")):
    sys.exit(__doc__)
sys.path.insert(0, REF)
from nanovllm.layers.attention import store_kvcache  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "store_kvcache.npz")


def bits(t):
    """Raw bit pattern of a tensor as an unsigned numpy array."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().view(torch.int32).numpy().view(np.uint32)


def run_case(name, key, value, nb, bs, slots, fill):
    n, hkv, d = key.shape
    kc = torch.full((nb, bs, hkv, d), fill, dtype=key.dtype)
    vc = torch.full((nb, bs, hkv, d), fill, dtype=key.dtype)
    sm = torch.tensor(slots, dtype=torch.int32)
    store_kvcache(key, value, kc, vc, sm)
    return {
        f"{name}__key": bits(key), f"{name}__value": bits(value),
        f"{name}__key_stride": np.int64(key.stride(0)),
        f"{name}__value_stride": np.int64(value.stride(0)),
        f"{name}__shape": np.asarray([n, hkv, d, nb, bs], np.int64),
        f"{name}__dtype": np.asarray(str(key.dtype)),
        f"{name}__slots": sm.numpy(),
        f"{name}__fill": np.float64(fill),
        f"{name}__k_after": bits(kc), f"{name}__v_after": bits(vc),
    }


def main():
    out = {}
    # 1. the study guide's hand-worked store example (master_nano-vllm-v2.md:2845-2852):
    #    N=3, Hkv=1, D=2, block_size=4, slots [5, 0, -1], cache pre-filled with -999
    key = torch.tensor([[[10., 11.]], [[20., 21.]], [[30., 31.]]], dtype=torch.float32)
    out.update(run_case("guide", key, key + 100, 2, 4, [5, 0, -1], -999.0))

    g = torch.Generator().manual_seed(1234)
    # 2. decode step of config 1: 8 new tokens, Qwen3-0.6B KV shape (8 x 128), bf16
    hkv, d, bs, nb = 8, 128, 256, 8
    perm = torch.randperm(nb * bs, generator=g)[:8].tolist()
    k = torch.randn(8, hkv, d, generator=g).to(torch.bfloat16)
    v = torch.randn(8, hkv, d, generator=g).to(torch.bfloat16)
    out.update(run_case("decode_bf16", k, v, nb, bs, perm, 0.0))

    # 3. prefill rows with the strided v view of a fused qkv projection
    #    (qwen3.py:79-82: row stride (Hq + 2*Hkv) * D), ragged count, slot -1 rows
    hq, hkv, d, bs, nb, n = 16, 8, 128, 256, 4, 37
    qkv = torch.randn(n, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    _, kk, vv = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    kk = kk.contiguous().view(n, hkv, d)   # rotary returns a new contiguous k
    vv = vv.view(n, hkv, d)                # v stays a strided view
    slots = torch.randperm(nb * bs, generator=g)[:n]
    slots[[3, 17, 36]] = -1
    out.update(run_case("prefill_strided_v", kk, vv, nb, bs, slots.tolist(), 0.0))

    # 4. fp16, one kv head of head_dim 64 (TP=8 shard of a small model)
    k = torch.randn(5, 1, 64, generator=g).to(torch.float16)
    v = torch.randn(5, 1, 64, generator=g).to(torch.float16)
    out.update(run_case("fp16_h1_d64", k, v, 3, 256, [767, 0, 256, -1, 511], 0.0))

    np.savez_compressed(OUT, **out)
    print("wrote", OUT, sorted({k.split("__")[0] for k in out}))


if __name__ == "__main__":
    main()
