"""Speculative acceptance-sampling oracle (test infrastructure only).

The reference engine has no speculative path (nothing under nanovllm/ drafts
or verifies tokens); its only sampler is the exponential race of
nanovllm/layers/sampler.py:7-12.  This module restates the standard
rejection scheme for speculative decoding (Leviathan et al. 2023; Chen et
al. 2023):
  for draft position i = 0..k-1 with draft token x_i:
      accept when u_i < min(1, p_i(x_i) / q_i(x_i))
  at the first rejection i: sample from normalise(max(p_i - q_i, 0));
  if all k drafts are accepted: sample a bonus token from p_k,
with p = softmax(target_logits / T) and q = softmax(draft_logits / T).

Pinning: the reference has nothing to pin against.  The acceptance rule is pinned to an
independent implementation of the same scheme, vLLM 0.22's rejection sampler
(vllm/v1/sample/rejection_sampler.py, run on CPU with the same uniforms): decisions equal on
the committed cases (tests/golden/spec_accept_vllm.npz).  vLLM draws the residual token with an
exponential race rather than an inverse CDF, so that step is pinned in distribution only.

Every floating-point operation is defined in a fixed order with float32
rounding, so that the CUDA kernel reproduces the decisions and the sampled
tokens bit for bit given identical uniforms:
  * exp_c (for x <= 0): y = x*log2(e); n = rint(y) by the magic
    constant 1.5*2^23 (t = y + c, n = t - c, round to nearest even);
    f = y - n; P(f) = a degree-5 polynomial for 2^f on [-1/2, 1/2] (the
    minimax fit of the relative error with P(0) = 1, by linear programming,
    1.6e-7 at most in float32; coefficients EXP2_COEF) by Horner with fused
    multiply-add (one rounding per step);
    exp_c = P * 2^n (exponent field add), 0 unless y >= -125 (so 0 for
    NaN and -inf as well);
  * probabilities: p_j = exp_c(x_j - M) * r with r = 1 / S rounded once;
  * sums: the vocabulary is cut into tiles of 4096; in a tile, "thread" i
    (0..255) adds its 16 elements k*1024 + 4*i + c (k = 0..3 outer,
    c = 0..3 inner) left to right; the 32 thread sums of each warp are
    combined by an xor butterfly (16, 8, 4, 2, 1); the 8 warp sums are
    added left to right; tile sums are added left to right;
  * softmax normaliser of a row: per tile t, M_t = max of the tile (NaN
    values ignored, as fmaxf does) and
    S_t = the tile sum of exp_c(x - M_t); then M = max_t M_t and
    S = sum_t S_t * exp_c(M_t - M) (left to right), so that a row is read
    once;
  * sampling: inverse CDF over the same hierarchy (tile sums, then thread
    sums, then the thread's 16 elements), each level scanned left to right
    with float32 running sums; a level where rounding leaves the target
    above the running sum falls back to its last positive entry.
"""
import numpy as np

f32 = np.float32
TILE = 4096
THREADS = 256
LOG2E = f32(1.4426950408889634)
# 2^f ~ sum_k c_k f^k on [-1/2, 1/2] with c_0 = 1: discrete minimax of the relative error by
# linear programming, rounded to float32 (learn-nano-vllm_b200/csrc/gen_exp2_coef.py; the CUDA
# kernel holds the same literals, tests/test_oracle_spec.py checks all three agree)
EXP2_COEF = [f32(float.fromhex(h)) for h in ("0x1.0p+0", "0x1.62e42ap-1", "0x1.ebf9aep-3", "0x1.c6b64ep-5",
                                               "0x1.3cee66p-7", "0x1.5c10d4p-10")]


def fma32(a, b, c):
    """float32 a*b + c with a single rounding (round to nearest even), exactly.

    a*b is exact in float64 (48-bit product).  hi = fl64(a*b + c) and the
    TwoSum error lo give a*b + c = hi + lo exactly.  Rounding hi to float32
    is correct unless hi sits exactly on a float32 midpoint (midpoints are
    float64 numbers, so hi cannot straddle one); there the sign of lo breaks
    the tie.
    """
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    c = np.asarray(c, f32)
    with np.errstate(invalid="ignore", over="ignore"):
        s_ = a.astype(np.float64) * b.astype(np.float64)
        c64 = c.astype(np.float64)
        hi = s_ + c64
        bb = hi - s_
        lo = (s_ - (hi - bb)) + (c64 - bb)
        r = hi.astype(f32)
        r64 = r.astype(np.float64)
        toward = np.where(hi > r64, np.float32(np.inf), np.float32(-np.inf)).astype(f32)
        other = np.nextafter(r, toward)
        mid = (r64 + other.astype(np.float64)) * 0.5
        fix = (hi == mid) & (lo != 0) & np.isfinite(hi)
        up = np.maximum(r, other)
        down = np.minimum(r, other)
        out = np.where(fix, np.where(lo > 0, up, down), r)
    return out.astype(f32)


MAGIC = f32(12582912.0)  # 1.5 * 2^23


def exp_c(x):
    """exp(x) for float32 x <= 0 with the fixed operation order above."""
    x = np.asarray(x, dtype=f32)
    with np.errstate(invalid="ignore"):
        y = (x * LOG2E).astype(f32)
        t = (y + MAGIC).astype(f32)
        n = (t - MAGIC).astype(f32)
        fr = (y - n).astype(f32)
        p = np.full_like(fr, EXP2_COEF[-1])
        for c in EXP2_COEF[-2::-1]:
            p = fma32(p, fr, c)
        keep = y >= f32(-125.0)  # False for NaN and -inf too: those give 0
        ni = np.where(keep, n, f32(0.0)).astype(np.int32)
        bits = (p.view(np.int32) + (ni << np.int32(23))).astype(np.int32)
        r = bits.view(f32)
        return np.where(keep, r, f32(0.0)).astype(f32)


def exp2_coef_hex():
    """The float32 coefficients as C hex literals (the CUDA kernel's constants)."""
    return [float(c).hex() for c in EXP2_COEF]


def canon_partials(w):
    """Thread sums P[..., T, 256], tile sums S[..., T] and total R[...] of w[..., V]."""
    w = np.asarray(w, dtype=f32)
    V = w.shape[-1]
    T = (V + TILE - 1) // TILE
    pad = np.zeros(w.shape[:-1] + (T * TILE,), f32)
    pad[..., :V] = w
    X = pad.reshape(w.shape[:-1] + (T, 4, THREADS, 4))
    P = np.zeros(w.shape[:-1] + (T, THREADS), f32)
    for k in range(4):
        for c in range(4):
            P = (P + X[..., k, :, c]).astype(f32)
    B2 = P.reshape(w.shape[:-1] + (T, THREADS // 32, 32))
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        B2 = (B2 + B2[..., lanes ^ off]).astype(f32)
    W = B2[..., 0]
    S = np.zeros(w.shape[:-1] + (T,), f32)
    for wi in range(THREADS // 32):
        S = (S + W[..., wi]).astype(f32)
    R = np.zeros(w.shape[:-1], f32)
    for t in range(T):
        R = (R + S[..., t]).astype(f32)
    return P, S, R


def _scan_pick(vals, target, acc0):
    """Left-to-right running sum from acc0; first index with target < acc + v.

    Returns (index, running sum before it) or the last positive entry when
    rounding leaves the target above every running sum; (-1, acc0) if no
    entry is positive.
    """
    acc = f32(acc0)
    for i, v in enumerate(vals):
        nxt = f32(acc + f32(v))
        if target < nxt and v > 0:
            return i, acc
        acc = nxt
    acc = f32(acc0)
    last, acc_last = -1, f32(acc0)
    for i, v in enumerate(vals):
        if v > 0:
            last, acc_last = i, acc
        acc = f32(acc + f32(v))
    return last, acc_last


def canon_pick(w, u):
    """Index sampled from weights w[V] >= 0 with uniform u, or -1 if w has no mass."""
    w = np.asarray(w, dtype=f32)
    V = w.shape[-1]
    P, S, R = canon_partials(w)
    target = f32(f32(u) * R)
    t, acc = _scan_pick(S, target, f32(0.0))
    if t < 0:
        return -1
    i, acc = _scan_pick(P[t], target, acc)
    if i < 0:
        return -1
    idx = [t * TILE + k * 1024 + 4 * i + c for k in range(4) for c in range(4)]
    vals = [w[j] if j < V else f32(0.0) for j in idx]
    e, _ = _scan_pick(vals, target, acc)
    return -1 if e < 0 else idx[e]


def scaled_logits(logits, temperature):
    x = np.asarray(logits, dtype=f32)
    if temperature is None:
        return x
    return (x / f32(temperature)).astype(f32)


def row_stats(x):
    """(max M, normaliser S) of one logits row (already / T), tile by tile."""
    x = np.asarray(x, dtype=f32)
    V = x.shape[-1]
    T = (V + TILE - 1) // TILE
    pad = np.full(T * TILE, -np.inf, f32)
    pad[:V] = x
    tiles = pad.reshape(T, TILE)
    Mt = np.fmax.reduce(tiles, axis=1).astype(f32)
    with np.errstate(invalid="ignore"):
        e = exp_c((tiles - Mt[:, None]).astype(f32))
    e = np.where(np.isfinite(tiles), e, f32(0.0)).astype(f32)
    _, St, _ = canon_partials(e.reshape(T * TILE)[:V])
    M = f32(Mt.max())
    S = f32(0.0)
    for t in range(T):
        S = f32(S + f32(St[t] * exp_c(f32(Mt[t] - M))))
    return M, S


def recip(S):
    return (f32(1.0) / f32(S)).astype(f32) if np.ndim(S) else f32(f32(1.0) / f32(S))


def probs(x, M, S):
    return (exp_c((x - M).astype(f32)) * recip(S)).astype(f32)


def spec_accept_ref(target_logits, draft_logits, draft_tokens, u_accept, u_sample,
                    temperatures=None):
    """Returns (tokens [B, k+1] int32 padded with -1, num_tokens [B] int32)."""
    tl = np.asarray(target_logits, f32)
    dl = np.asarray(draft_logits, f32)
    B, k1, V = tl.shape
    k = k1 - 1
    tokens = np.full((B, k1), -1, np.int32)
    num = np.zeros(B, np.int32)
    for b in range(B):
        T = None if temperatures is None else temperatures[b]
        rej = k
        for i in range(k):
            x = int(draft_tokens[b, i])
            if not (0 <= x < V):
                rej = i
                break
            xt = scaled_logits(tl[b, i], T)
            xd = scaled_logits(dl[b, i], T)
            Mt, St = row_stats(xt)
            Md, Sd = row_stats(xd)
            p = f32(exp_c(f32(xt[x] - Mt)) * recip(St))
            q = f32(exp_c(f32(xd[x] - Md)) * recip(Sd))
            if q > 0:
                acc = f32(u_accept[b, i]) < min(f32(1.0), f32(p / q))
            else:
                acc = p > 0
            if not acc:
                rej = i
                break
        xt = scaled_logits(tl[b, rej], T)
        Mt, St = row_stats(xt)
        p_row = probs(xt, Mt, St)
        if rej < k:
            xd = scaled_logits(dl[b, rej], T)
            Md, Sd = row_stats(xd)
            q_row = probs(xd, Md, Sd)
            w = np.maximum((p_row - q_row).astype(f32), f32(0.0))
            tok = canon_pick(w, u_sample[b])
            if tok < 0:
                tok = canon_pick(p_row, u_sample[b])
        else:
            tok = canon_pick(p_row, u_sample[b])
        if tok < 0:
            tok = 0
        tokens[b, :rej] = draft_tokens[b, :rej]
        tokens[b, rej] = tok
        num[b] = rej + 1
    return tokens, num


def spec_accept_float_ref(target_logits, draft_logits, draft_tokens, u_accept):
    """Acceptance count from float64 softmax: a sanity check of the scheme itself."""
    tl = np.asarray(target_logits, np.float64)
    dl = np.asarray(draft_logits, np.float64)
    p = np.exp(tl - tl.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    q = np.exp(dl - dl.max(-1, keepdims=True))
    q /= q.sum(-1, keepdims=True)
    B, k = draft_tokens.shape
    out = np.zeros(B, np.int32)
    for b in range(B):
        n = 0
        for i in range(k):
            x = draft_tokens[b, i]
            if u_accept[b, i] < min(1.0, p[b, i, x] / q[b, i, x]):
                n += 1
            else:
                break
        out[b] = n
    return out
