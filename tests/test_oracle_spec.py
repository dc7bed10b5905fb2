"""Speculative acceptance oracle: fixed-order arithmetic and scheme sanity (CPU)."""
import numpy as np
import pytest

from oracle import cases
from oracle import spec_sampling as ss


def test_exp_c_accuracy():
    x = np.linspace(-80, 0, 200001).astype(np.float32)
    rel = np.abs(ss.exp_c(x) - np.exp(x.astype(np.float64))) / np.exp(x.astype(np.float64))
    assert rel.max() < 1e-5
    assert ss.exp_c(np.float32(-100.0)) == 0 and ss.exp_c(np.float32(0.0)) == 1.0


def test_fma32_single_rounding():
    """The oracle's fused multiply-add rounds a*b + c once, as the GPU's fma does."""
    from fractions import Fraction
    rng = np.random.default_rng(5)
    n = 3000
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    c = (rng.standard_normal(n) * np.exp2(rng.integers(-40, 10, n))).astype(np.float32)
    r = ss.fma32(a, b, c)
    for i in range(n):
        exact = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        got = Fraction(float(r[i]))
        for nb in (np.nextafter(r[i], np.float32(-np.inf)), np.nextafter(r[i], np.float32(np.inf))):
            d_nb, d_got = abs(Fraction(float(nb)) - exact), abs(got - exact)
            assert d_nb > d_got or (d_nb == d_got and not int(r[i].view(np.int32)) & 1), (a[i], b[i], c[i])


def test_canonical_sum_close_to_exact():
    rng = np.random.default_rng(0)
    for V in (1, 4095, 4096, 4097, 151936):
        w = rng.random(V, dtype=np.float32)
        _, S, R = ss.canon_partials(w)
        assert len(S) == (V + 4095) // 4096
        assert abs(float(R) - w.astype(np.float64).sum()) <= 1e-5 * w.sum()


def test_canonical_pick_follows_the_cdf():
    w = np.zeros(9000, np.float32)
    w[[3, 4100, 8999]] = [1.0, 2.0, 1.0]
    picks = [ss.canon_pick(w, u) for u in (0.0, 0.2, 0.26, 0.6, 0.74, 0.76, 0.999)]
    assert picks == [3, 3, 4100, 4100, 4100, 8999, 8999]
    assert ss.canon_pick(np.zeros(10, np.float32), 0.5) == -1


def test_canonical_pick_distribution():
    rng = np.random.default_rng(1)
    w = rng.random(300, dtype=np.float32) ** 4
    us = rng.random(20000, dtype=np.float32)
    counts = np.bincount([ss.canon_pick(w, u) for u in us], minlength=300)
    p = w / w.sum()
    assert np.abs(counts / len(us) - p).max() < 0.01


def test_acceptance_counts_match_float64_scheme():
    c = cases.make_spec_case(64, 4, 1000, seed=3)
    toks, num = ss.spec_accept_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept, c.u_sample)
    ref = ss.spec_accept_float_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept)
    assert (num - 1 == ref).mean() > 0.98          # only near-ties may differ
    assert 0 < (num - 1).mean() < 4                # both branches are exercised
    for b in range(64):
        n = num[b]
        assert (toks[b, :n - 1] == c.draft_tokens[b, :n - 1]).all()
        assert 0 <= toks[b, n - 1] < 1000 and (toks[b, n:] == -1).all()


def test_rejected_position_never_resamples_the_rejected_mass():
    """After a rejection at i the new token has p_i(x) > q_i(x) (residual support)."""
    c = cases.make_spec_case(32, 3, 500, seed=4)
    toks, num = ss.spec_accept_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept, c.u_sample)
    for b in range(32):
        i = num[b] - 1
        if i < 3:
            xt, xd = c.target_logits[b, i], c.draft_logits[b, i]
            p = ss.probs(xt, *ss.row_stats(xt))
            q = ss.probs(xd, *ss.row_stats(xd))
            assert p[toks[b, i]] > q[toks[b, i]]


def test_temperature_and_invalid_draft():
    c = cases.make_spec_case(4, 2, 300, seed=5, temperatures=True)
    c.draft_tokens[1, 0] = 300  # out of range -> rejected at position 0
    toks, num = ss.spec_accept_ref(c.target_logits, c.draft_logits, c.draft_tokens, c.u_accept, c.u_sample,
                                   c.temperatures)
    assert num[1] == 1 and 0 <= toks[1, 0] < 300


def test_acceptance_matches_vllm_rejection_sampler():
    """Pinned to vLLM 0.22's rejection sampler (an independent implementation of the same
    standard scheme) run on CPU with the same uniforms (tests/golden/spec_accept_vllm.npz,
    generator beside it): every sequence's number of accepted drafts and accepted prefix."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "spec_accept_vllm.npz"))
    names = sorted({k.split(".")[0] for k in g.files})
    assert len(names) == 2
    lengths_seen = set()
    for name in names:
        tl, dl, T, dt, u, vt = (g[name + s] for s in (".target_logits", ".draft_logits", ".temperatures",
                                                       ".draft_tokens", ".u_accept", ".vllm_tokens"))
        B = tl.shape[0]
        accepted_vllm = (vt >= 0).sum(axis=1) - 1  # accepted drafts, then one recovered/bonus token
        tokens, num = ss.spec_accept_ref(tl, dl, dt, u, np.full(B, 0.5, np.float32), T)
        assert np.array_equal(num - 1, accepted_vllm), name
        for b in range(B):
            n = accepted_vllm[b]
            assert np.array_equal(tokens[b, :n], vt[b, :n]) and np.array_equal(vt[b, :n], dt[b, :n])
            lengths_seen.add((name, int(n)))
    assert len({n for name, n in lengths_seen if name.startswith("b32_k7")}) == 8  # 0..7 accepted all occur


def test_exp2_coefficients_come_from_their_generator():
    """exp_c's polynomial: the oracle's coefficients and the CUDA kernel's literals are
    exactly what learn-nano-vllm_b200/csrc/gen_exp2_coef.py produces (minimax fit of the
    relative error by linear programming, rounded to float32)."""
    import importlib.util
    import os
    import re
    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "learn-nano-vllm_b200", "csrc")
    spec = importlib.util.spec_from_file_location("gen_exp2_coef", os.path.join(csrc, "gen_exp2_coef.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    want = gen.coefficients_f32()
    assert [float(c) for c in ss.EXP2_COEF] == [float(c) for c in want]
    src = open(os.path.join(csrc, "spec_accept.cu")).read()
    body = re.search(r"kExpCoef\[kExpDeg \+ 1\]\s*=\s*\{([^}]*)\}", src).group(1)
    lits = [float.fromhex(t.strip().rstrip("f")) for t in body.split(",")]
    assert lits == [float(c) for c in want]
    _, t = gen.fit()
    assert t < 1e-7


def test_exp_c_special_values():
    """exp_c is 0 for NaN, -inf and anything below 2^-125, exactly 1 at 0, and within the fit's
    error elsewhere on its domain (x <= 0)."""
    x = np.asarray([np.nan, -np.inf, -200.0, -86.7, 0.0, -0.0, -1e-30, -0.5, -10.0], np.float32)
    e = ss.exp_c(x)
    assert e[0] == 0 and e[1] == 0 and e[2] == 0 and e[3] == 0
    assert e[4] == 1 and e[5] == 1 and e[6] == 1
    xs = -np.random.default_rng(0).exponential(8.0, 20000).astype(np.float32)
    xs = xs[xs > -80]
    rel = np.abs(ss.exp_c(xs).astype(np.float64) / np.exp(xs.astype(np.float64)) - 1)
    # fit error plus the float32 rounding of y = x * log2(e), whose absolute error grows with |x|
    assert (rel <= 3e-7 + np.abs(xs) * 1.2e-7).all()
