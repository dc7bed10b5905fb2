"""Speculative acceptance sampling on the GPU vs the oracle: decisions and
sampled tokens bit-exact given identical uniforms."""
import numpy as np
import pytest
import torch

from oracle import cases
from oracle import spec_sampling as ss

pytestmark = pytest.mark.gpu


def run(pkg, c):
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    temps = None if c.temperatures is None else t(c.temperatures)
    toks, num = pkg.spec_accept(t(c.target_logits), t(c.draft_logits), t(c.draft_tokens), t(c.u_accept),
                                t(c.u_sample), temps)
    want_t, want_n = ss.spec_accept_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept, c.u_sample,
                                        c.temperatures)
    return toks.cpu().numpy(), num.cpu().numpy(), want_t, want_n


@pytest.mark.parametrize("B,k,V,seed", [(16, 4, 1000, 0), (8, 4, 4096, 1), (8, 2, 4097, 2), (4, 4, 151936, 3),
                                        (32, 1, 777, 4), (3, 6, 20000, 5)])
def test_bit_exact_against_oracle(pkg, B, k, V, seed):
    c = cases.make_spec_case(B, k, V, seed=seed)
    toks, num, wt, wn = run(pkg, c)
    assert np.array_equal(num, wn) and np.array_equal(toks, wt)


def test_temperatures_and_invalid_drafts(pkg):
    c = cases.make_spec_case(8, 3, 3000, seed=9, temperatures=True)
    c.draft_tokens[2, 1] = -5
    c.draft_tokens[5, 0] = 3000
    toks, num, wt, wn = run(pkg, c)
    assert np.array_equal(num, wn) and np.array_equal(toks, wt)
    assert num[5] == 1


def test_uncorrelated_drafts_mostly_rejected(pkg):
    c = cases.make_spec_case(16, 4, 2000, seed=10, correlated=False)
    toks, num, wt, wn = run(pkg, c)
    assert np.array_equal(num, wn) and np.array_equal(toks, wt)
    assert num.mean() < 2


@pytest.mark.parametrize("name", ["independent", "correlated"])
def test_config4_full_size_bit_exact(pkg, name):
    """The speculative-verify configuration at full size (B = 128, k = 4, V = 151,936, logits
    N(0, 2^2), seeded uniforms): every count and token equal to the oracle's, recorded in
    tests/golden/spec_config4.npz by its generator (the inputs are regenerated from the seed and
    checked against the recorded checksum), and to the live oracle on 16 sampled sequences."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import gen_spec_config4_golden as gen
    fx = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "spec_config4.npz"))
    c = cases.make_spec_case(gen.B, gen.K, gen.V, **gen.CASES[name])
    assert np.array_equal(gen.input_checksum(c), fx[f"{name}_checksum"]), "regenerated inputs differ"
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    toks, num = pkg.spec_accept(t(c.target_logits), t(c.draft_logits), t(c.draft_tokens), t(c.u_accept),
                                t(c.u_sample), None)
    toks, num = toks.cpu().numpy(), num.cpu().numpy()
    assert np.array_equal(num, fx[f"{name}_num"])
    assert np.array_equal(toks, fx[f"{name}_tokens"])
    rows = np.random.default_rng(7).choice(gen.B, 16, replace=False)
    wt, wn = ss.spec_accept_ref(c.target_logits[rows], c.draft_logits[rows], c.draft_tokens[rows], c.u_accept[rows],
                                c.u_sample[rows], None)
    assert np.array_equal(num[rows], wn) and np.array_equal(toks[rows], wt)


def test_non_finite_logits_weigh_zero(pkg):
    """NaN and -inf logits (masked vocabulary entries) weigh 0 on both sides, bit for bit."""
    c = cases.make_spec_case(8, 3, 5000, seed=12)
    rng = np.random.default_rng(3)
    for arr in (c.target_logits, c.draft_logits):
        flat = arr.reshape(-1)
        idx = rng.choice(flat.size, 400, replace=False)
        flat[idx[:200]] = -np.inf
        flat[idx[200:]] = np.nan
    toks, num, wt, wn = run(pkg, c)
    assert np.array_equal(num, wn) and np.array_equal(toks, wt)
