"""Generate tests/golden/spec_config4.npz: the acceptance oracle's output at the full size of
the speculative-verify configuration (batch 128, k = 4 drafts, vocabulary 151,936, logits
N(0, 2^2) fp32, seeded uniforms).

Two seeded cases from oracle.cases.make_spec_case: "independent" (target and draft logits
drawn independently, as the configuration states them; nearly every draft is rejected, so
the residual sampling runs on every row) and "correlated" (draft logits = target logits +
N(0, 1) noise, so that acceptance runs of every length occur).  Their inputs (700 MB each)
are regenerated from the seed by the test; stored here are the oracle's tokens and counts
and a checksum of the inputs that shows the regenerated inputs are the same.  CPU only,
about 45 s per case; run once, output committed.

Usage:  python tests/golden/gen_spec_config4_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import cases  # noqa: E402
from oracle import spec_sampling as ss  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "spec_config4.npz")
B, K, V = 128, 4, 151936
CASES = {"independent": dict(seed=40, correlated=False), "correlated": dict(seed=41, correlated=True)}


def input_checksum(c):
    """float64 sums of the logits and uniforms plus the draft tokens' sum (order-independent enough
    to notice a different draw, cheap to recompute)."""
    return np.array([c.target_logits.sum(dtype=np.float64), c.draft_logits.sum(dtype=np.float64),
                     float(c.draft_tokens.astype(np.int64).sum()), c.u_accept.sum(dtype=np.float64),
                     c.u_sample.sum(dtype=np.float64)])


def main():
    out = {}
    for name, kw in CASES.items():
        c = cases.make_spec_case(B, K, V, **kw)
        toks, num = ss.spec_accept_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept, c.u_sample,
                                       c.temperatures)
        out[f"{name}_tokens"] = toks
        out[f"{name}_num"] = num
        out[f"{name}_checksum"] = input_checksum(c)
        print(name, "accepted-count histogram", np.bincount(num - 1, minlength=K + 1))
    np.savez_compressed(OUT, **out)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
