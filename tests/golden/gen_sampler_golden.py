"""Generate tests/golden/sampler.npz from the reference's own Sampler.

Runs nano-vLLM's Sampler.forward (nanovllm/layers/sampler.py:7-12) eagerly on CPU
(torch.compile disabled) on seeded logits and temperatures.  The sampler draws its
Exp(1) noise with torch's CPU generator right after the seed is set (nothing else in
forward draws), so replaying the seed recovers the exact noise tensor; it is
recorded with the tokens, after checking that the reference formula on it gives
them back.  Needs the reference checkout (its directory as argv[1] or in
NANOVLLM_REF); run once in the development container, output committed.  The GPU
box never runs it.

Usage:  python tests/golden/gen_sampler_golden.py [REF_DIR]
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
from nanovllm.layers.sampler import Sampler  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler.npz")


def run_case(name, B, V, scale, dtype, seed, store):
    g = torch.Generator().manual_seed(1000 + seed)
    logits = (torch.randn(B, V, generator=g) * scale).to(dtype)
    temps = (0.5 + torch.rand(B, generator=g)).float()
    torch.manual_seed(seed)
    tokens = Sampler()(logits.clone(), temps)
    torch.manual_seed(seed)
    noise = torch.empty(B, V, dtype=torch.float32).exponential_(1)
    # the reference formula on the recovered noise gives the same tokens
    probs = torch.softmax(logits.float() / temps.unsqueeze(1), dim=-1)
    again = probs.div_(noise.clamp_min(1e-10)).argmax(dim=-1)
    assert torch.equal(again, tokens), name
    store[name + ".logits"] = logits.float().numpy()
    store[name + ".temperatures"] = temps.numpy()
    store[name + ".noise"] = noise.numpy()
    store[name + ".tokens"] = tokens.numpy().astype(np.int64)


def main():
    store = {}
    run_case("f32_16x1024", 16, 1024, 2.0, torch.float32, 1, store)
    run_case("bf16_8x2048", 8, 2048, 4.0, torch.bfloat16, 2, store)
    run_case("f32_8x1024_wide", 8, 1024, 8.0, torch.float32, 3, store)
    np.savez_compressed(OUT, **store)
    print(OUT, sorted(store))


if __name__ == "__main__":
    main()
