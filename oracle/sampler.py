"""Fused sampler oracle (test infrastructure only).

The reference sampler (nanovllm/layers/sampler.py:7-12) draws
    token = argmax_j softmax(logits / T)_j / clamp_min(E_j, 1e-10),  E ~ Exp(1)
which equals argmax_j (logits_j / T - log E_j): softmax rescales a row by a
positive constant.  This module restates
  * the reference formula itself (float32, as torch computes it), given E;
  * the noise generator of the fused kernel: Philox-4x32-10 (Salmon, Moraes,
    Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11), counter
    (j // 4, row, offset_lo, offset_hi), key (seed_lo, seed_hi), word j % 4,
    U = ((bits >> 8) + 0.5) * 2^-24, E = -log(U);
  * the fused score argmax in float64 (for comparisons that allow near-ties).
Pinned: Philox to the published known-answer vectors; the reference formula to the
reference Sampler's own tokens on its own Exp(1) draw (tests/golden/sampler.npz).
"""
import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox-4x32-10 over uint32 arrays; returns the four output words."""
    c0, c1, c2, c3 = (np.asarray(c, np.uint32) for c in (c0, c1, c2, c3))
    k0 = np.uint32(k0)
    k1 = np.uint32(k1)
    for _ in range(10):
        p0 = M0 * c0.astype(np.uint64)
        p1 = M1 * c2.astype(np.uint64)
        hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & MASK32).astype(np.uint32)
        hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & MASK32).astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = np.uint32((int(k0) + int(W0)) & 0xFFFFFFFF)
        k1 = np.uint32((int(k1) + int(W1)) & 0xFFFFFFFF)
    return c0, c1, c2, c3


def philox_bits(rows, V, seed, offset):
    """uint32 words [rows, V]: element j of row b is word j % 4 of counter (j//4, b, offset)."""
    g = np.arange((V + 3) // 4, dtype=np.uint64)
    out = np.empty((rows, ((V + 3) // 4) * 4), np.uint32)
    for b in range(rows):
        w = philox4x32_10(g.astype(np.uint32), np.full(g.shape, b, np.uint32),
                          np.full(g.shape, offset & 0xFFFFFFFF, np.uint32),
                          np.full(g.shape, (offset >> 32) & 0xFFFFFFFF, np.uint32),
                          seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
        out[b] = np.stack(w, axis=1).reshape(-1)
    return out[:, :V]


def uniforms(bits):
    """U in (0, 1) from the top 24 bits, exactly as the kernel forms it."""
    return ((bits >> np.uint32(8)).astype(np.float64) + 0.5) * 2.0 ** -24


def fused_scores(logits, temperatures, noise):
    """float64 logits / T - log(clamp_min(E, 1e-10))."""
    x = np.asarray(logits, np.float64) / np.asarray(temperatures, np.float64)[:, None]
    return x - np.log(np.maximum(np.asarray(noise, np.float64), 1e-10))


def sample_ref(logits, temperatures, seed, offset):
    """Tokens of the fused kernel's generator path (float64 scores)."""
    B, V = np.asarray(logits).shape
    e = -np.log(uniforms(philox_bits(B, V, seed, offset)))
    return np.argmax(fused_scores(logits, temperatures, e), axis=1)


def reference_formula(logits, temperatures, noise):
    """nanovllm/layers/sampler.py:9-11 in float32: softmax(x/T) / clamp_min(E, 1e-10), argmax."""
    x = (np.asarray(logits, np.float32) / np.asarray(temperatures, np.float32)[:, None]).astype(np.float32)
    x = x - x.max(axis=1, keepdims=True)
    e = np.exp(x).astype(np.float32)
    p = (e / e.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    r = (p / np.maximum(np.asarray(noise, np.float32), np.float32(1e-10))).astype(np.float32)
    return np.argmax(r, axis=1)
