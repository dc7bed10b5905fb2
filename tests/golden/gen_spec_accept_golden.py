"""Generate tests/golden/spec_accept_vllm.npz: acceptance decisions of vLLM's rejection
sampler on seeded cases, to pin oracle/spec_sampling.py's acceptance rule.

The reference has no speculative code; the row follows the standard scheme (accept draft i
if u_i < min(1, p_i(x) / q_i(x)), stop at the first rejection).  vLLM 0.22 (in this image,
vllm/v1/sample/rejection_sampler.py: rejection_sample) implements the same rule; its Triton
kernels run here on CPU tensors under TRITON_INTERPRET=1.  Its uniforms are replaced by the
case's own (generate_uniform_probs returns them), so the decisions are comparable one for
one.  Recorded: logits, temperatures, draft tokens, uniforms, and vLLM's output tokens
(accepted drafts, then its recovered or bonus token, then -1).  vLLM draws its recovered
tokens with its own exponential race, so only the decisions are pinned.  Run once in the
development container (CPU); output committed.

Usage:  TRITON_INTERPRET=1 python tests/golden/gen_spec_accept_golden.py
"""
import os
import types

os.environ.setdefault("TRITON_INTERPRET", "1")
import numpy as np
import torch
import vllm.v1.sample.rejection_sampler as rs

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "spec_accept_vllm.npz")


def run_case(name, B, k, V, spread, closeness, seed, store):
    rng = np.random.default_rng(seed)
    target = (rng.standard_normal((B, k + 1, V)) * spread).astype(np.float32)
    # drafts close to the target, so that acceptance runs of every length occur
    draft = (target[:, :k] + rng.standard_normal((B, k, V)) * closeness * spread).astype(np.float32)
    temps = rng.uniform(0.5, 1.5, B).astype(np.float32)
    tt = torch.from_numpy(target)
    td = torch.from_numpy(draft)
    T = torch.from_numpy(temps)
    q = torch.softmax(td / T[:, None, None], dim=-1)
    tokens = torch.stack([torch.multinomial(q[b], 1, generator=torch.Generator().manual_seed(seed * 1000 + b))[:, 0]
                          for b in range(B)]).to(torch.int32)
    u = rng.random((B, k)).astype(np.float32)
    rs.generate_uniform_probs = lambda num_tokens, num_draft, generators, device: torch.from_numpy(
        u.reshape(-1).astype(np.float64))
    meta = types.SimpleNamespace(all_greedy=False, all_random=True, temperature=T, generators={})
    out = rs.rejection_sample(
        tokens.reshape(-1).contiguous(), [k] * B, k, torch.arange(1, B + 1, dtype=torch.int32) * k,
        q.reshape(B * k, V).contiguous(), (tt[:, :k] / T[:, None, None]).reshape(B * k, V).contiguous(),
        torch.full((B, 1), 7, dtype=torch.int32), meta)
    store[name + ".target_logits"] = target
    store[name + ".draft_logits"] = draft
    store[name + ".temperatures"] = temps
    store[name + ".draft_tokens"] = tokens.numpy()
    store[name + ".u_accept"] = u
    store[name + ".vllm_tokens"] = out.numpy().astype(np.int32)


def main():
    store = {}
    run_case("b32_k4_v128", 32, 4, 128, 2.0, 0.6, 1, store)
    run_case("b32_k7_v64_close", 32, 7, 64, 3.0, 0.2, 2, store)
    np.savez_compressed(OUT, **store)
    print(OUT, sorted(store))


if __name__ == "__main__":
    main()
