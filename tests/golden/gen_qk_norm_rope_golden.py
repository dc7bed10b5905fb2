"""Generate tests/golden/qk_norm_rope.npz from the reference's own modules.

Runs nano-vLLM's RMSNorm.rms_forward (nanovllm/layers/layernorm.py:16-26) and
RotaryEmbedding.forward (nanovllm/layers/rotary_embedding.py:37-48) eagerly on
CPU (torch.compile disabled) in the order of Qwen3Attention.forward
(nanovllm/models/qwen3.py:79-85): split of the fused QKV output, q_norm /
k_norm, rotary embedding.  Records the inputs (as raw bits), the module's
cos_sin_cache and the q / k it produced.  Needs the reference checkout (its
directory as argv[1] or in NANOVLLM_REF); it is run once in the development
container and its output is committed.  The GPU box never runs it.

Usage:  python tests/golden/gen_qk_norm_rope_golden.py [REF_DIR]
"""
import os
import sys

os.environ.setdefault("TORCH_COMPILE_DISABLE", "1")
import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANOVLLM_REF", "")
if not os.path.isdir(os.path.join(REF, "nanovllm")):
    sys.exit(__doc__)
sys.path.insert(0, REF)
from nanovllm.layers.layernorm import RMSNorm  # noqa: E402
from nanovllm.layers.rotary_embedding import RotaryEmbedding  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qk_norm_rope.npz")


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def run_case(name, T, hq, hkv, max_pos, base, eps, seed):
    d = 128
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(T, (hq + 2 * hkv) * d, generator=g) * 1.5).to(torch.bfloat16)
    positions = torch.randint(0, max_pos, (T,), generator=g, dtype=torch.int64)
    q_norm, k_norm = RMSNorm(d, eps=eps), RMSNorm(d, eps=eps)
    with torch.no_grad():
        q_norm.weight.copy_((1.0 + 0.25 * torch.randn(d, generator=g)))
        k_norm.weight.copy_((1.0 + 0.25 * torch.randn(d, generator=g)))
    q_norm, k_norm = q_norm.to(torch.bfloat16), k_norm.to(torch.bfloat16)
    rope = RotaryEmbedding(d, d, max_pos, base)
    with torch.no_grad():
        q, k, _ = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
        q = q_norm.rms_forward(q.reshape(T, hq, d))
        k = k_norm.rms_forward(k.reshape(T, hkv, d))
        q, k = rope.forward(positions, q, k)
    return {
        f"{name}__qkv": bits(qkv), f"{name}__positions": positions.numpy(),
        f"{name}__q_weight": bits(q_norm.weight.data), f"{name}__k_weight": bits(k_norm.weight.data),
        f"{name}__cos_sin": rope.cos_sin_cache.reshape(max_pos, d).numpy().astype(np.float32),
        f"{name}__q": bits(q), f"{name}__k": bits(k),
        f"{name}__meta": np.array([T, hq, hkv, max_pos], np.int64), f"{name}__eps": np.float32(eps),
    }


def main():
    assert torch.compiler.is_compiling() is False
    data = {}
    data.update(run_case("qwen3_0p6b", 10, 16, 8, 64, 1_000_000.0, 1e-6, 0))
    data.update(run_case("group4", 3, 32, 8, 48, 10_000.0, 1e-5, 1))
    np.savez_compressed(OUT, cases=np.array(["qwen3_0p6b", "group4"]), **data)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
