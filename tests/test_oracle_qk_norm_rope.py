"""Fused q/k norm + RoPE + scatter oracle against the reference's own modules (CPU)."""
import os

import numpy as np
import pytest

from oracle import cases
from oracle import qk_norm_rope as qr

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "qk_norm_rope.npz")


def _f32(bits16):
    return (bits16.astype(np.uint32) << 16).view(np.float32)


def load_case(z, name):
    T, hq, hkv, max_pos = (int(x) for x in z[f"{name}__meta"])
    return dict(qkv=_f32(z[f"{name}__qkv"]), positions=z[f"{name}__positions"], hq=hq, hkv=hkv,
                q_weight=_f32(z[f"{name}__q_weight"]), k_weight=_f32(z[f"{name}__k_weight"]),
                eps=float(z[f"{name}__eps"]), cos_sin=z[f"{name}__cos_sin"], q=_f32(z[f"{name}__q"]),
                k=_f32(z[f"{name}__k"]))


def close_bf16(got, want):
    """Equal, or one bf16 step apart (summation order of the mean, rsqrt rounding)."""
    d = np.abs(got - want)
    step = np.abs(want) * 2.0 ** -7 + 1e-30
    return (d <= step).all() and (d > 0).mean() < 0.02


@pytest.mark.parametrize("name", ["qwen3_0p6b", "group4"])
def test_oracle_matches_reference_modules(name):
    z = np.load(GOLDEN)
    c = load_case(z, name)
    q, k, _ = qr.qk_norm_rope_store_ref(c["qkv"], c["positions"], c["hq"], c["hkv"], c["q_weight"],
                                        c["k_weight"], c["eps"], c["cos_sin"])
    assert q.shape == c["q"].shape and k.shape == c["k"].shape
    # same rounding points as the reference's eager modules: bit-exact on these fixtures
    assert (q == c["q"]).all() and (k == c["k"]).all()


def test_oracle_store_and_padding():
    rng = np.random.default_rng(0)
    T, hq, hkv, d = 6, 4, 2, 128
    qkv = cases.randn_bf16(rng, (T, (hq + 2 * hkv) * d))
    cs = rng.standard_normal((32, d)).astype(np.float32)
    w = cases.randn_bf16(rng, (d,))
    kc = np.full((2, 4, hkv, d), 7.0, np.float32)
    vc = np.full((2, 4, hkv, d), 7.0, np.float32)
    slots = np.array([3, -1, 0, 7, 5, -1], np.int32)
    q, k, v = qr.qk_norm_rope_store_ref(qkv, np.arange(T) * 5, hq, hkv, w, w, 1e-6, cs, kc, vc, slots)
    flat_k, flat_v = kc.reshape(-1, hkv, d), vc.reshape(-1, hkv, d)
    for t, s in enumerate(slots):
        if s >= 0:
            assert (flat_k[s] == k[t]).all() and (flat_v[s] == v[t]).all()
    assert (flat_k[[1, 2, 4, 6]] == 7.0).all()


def test_rope_rotates_pairs():
    """With cos = 1, sin = 0 the rotation is the identity; with cos = 0, sin = 1 it swaps halves."""
    x = cases.round_bf16(np.arange(128, dtype=np.float32)[None, None, :] / 64)
    ident = qr.rope_ref(x, np.ones((1, 1, 64), np.float32), np.zeros((1, 1, 64), np.float32))
    assert (ident == x).all()
    swap = qr.rope_ref(x, np.zeros((1, 1, 64), np.float32), np.ones((1, 1, 64), np.float32))
    assert (swap[..., :64] == -x[..., 64:]).all() and (swap[..., 64:] == x[..., :64]).all()
