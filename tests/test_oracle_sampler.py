"""Sampler oracle: Philox pinned to its published known-answer vectors; scheme checks (CPU)."""
import numpy as np

from oracle import sampler as so

# Philox-4x32-10 known-answer vectors (Random123 distribution, kat_vectors: philox4x32_10)
KAT = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
       ((0xffffffff,) * 4, (0xffffffff, 0xffffffff), (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
       ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
        (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]


def test_philox_known_answers():
    for ctr, key, want in KAT:
        got = so.philox4x32_10(*[np.array([c], np.uint32) for c in ctr], *key)
        assert tuple(int(g[0]) for g in got) == want


def test_uniforms_open_interval_and_mean():
    u = so.uniforms(so.philox_bits(4, 50000, seed=7, offset=3))
    assert u.min() > 0 and u.max() < 1
    assert abs(u.mean() - 0.5) < 0.005


def test_fused_score_equals_reference_formula():
    rng = np.random.default_rng(0)
    B, V = 64, 3000
    x = (rng.standard_normal((B, V)) * 2).astype(np.float32)
    t = rng.uniform(0.5, 1.5, B).astype(np.float32)
    e = rng.exponential(size=(B, V)).astype(np.float32)
    a = np.argmax(so.fused_scores(x, t, e), axis=1)
    b = so.reference_formula(x, t, e)
    assert (a == b).mean() > 0.98


def test_generator_path_distribution():
    # 8 live tokens with known probabilities, the rest -inf; many rows = many draws
    p = np.array([0.3, 0.2, 0.15, 0.1, 0.1, 0.08, 0.05, 0.02])
    rows, V = 4000, 64
    x = np.full((rows, V), -np.inf, np.float32)
    x[:, :8] = np.log(p).astype(np.float32)
    toks = so.sample_ref(x, np.ones(rows, np.float32), seed=11, offset=0)
    freq = np.bincount(toks, minlength=V)[:8] / rows
    assert np.abs(freq - p).max() < 0.03


def test_reference_formula_matches_reference_sampler():
    """Pinned to the reference Sampler's own tokens on its own Exp(1) draw
    (tests/golden/sampler.npz, generator beside it)."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler.npz"))
    names = sorted({k.split(".")[0] for k in g.files})
    assert len(names) == 3
    for name in names:
        x, t, e, want = (g[name + s] for s in (".logits", ".temperatures", ".noise", ".tokens"))
        got = so.reference_formula(x, t, e)
        assert np.array_equal(got, want), (name, np.flatnonzero(got != want))
        # the one-pass score (x/T - ln E) is the same argmax up to float near-ties
        fused = np.argmax(so.fused_scores(x, t, e), axis=1)
        assert (fused == want).mean() >= 0.95, name
