"""Fused q/k RMSNorm + RoPE + KV scatter on the GPU vs the oracle and the reference's modules."""
import numpy as np
import pytest
import torch

from oracle import qk_norm_rope as qr
from tests.test_oracle_qk_norm_rope import GOLDEN, load_case

pytestmark = pytest.mark.gpu

D = 128


def rope_cache(max_pos, base):
    """cos_sin_cache built as nanovllm/layers/rotary_embedding.py:27-33 does (fp32, [P, D])."""
    inv_freq = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float) / D))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def to_np(t):
    return t.float().cpu().numpy()


def close_dt(got, want, dtype):
    """Within two rounding steps of the rotated pair's magnitude, and equal for most values.

    The GPU sums the squares lane-wise then by butterfly and uses the hardware
    rsqrt; the oracle uses numpy's order.  A one-step difference in a
    normalised value before the rotation moves y_i = x1*cos -/+ x2*sin by a
    step of |(x1, x2)| = sqrt(y_i^2 + y_{i+-64}^2) (the rotation keeps the
    pair's norm), which can be far above a step of |y_i| itself.
    """
    step = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    if np.size(want) == 0:
        return
    got = np.asarray(got, np.float64).reshape(-1, D)
    want = np.asarray(want, np.float64).reshape(-1, D)
    pair = np.sqrt(want ** 2 + np.roll(want, D // 2, axis=-1) ** 2)
    d = np.abs(got - want)
    assert (d <= 2 * step * pair + 1e-6).all(), f"max diff {d.max()} (pair scale {pair[d == d.max()][0]})"
    assert (d > 0).mean() < 0.05, f"{(d > 0).mean():.4f} of values differ"


def run_case(pkg, T, hq, hkv, dtype=torch.bfloat16, max_pos=4096, base=1e6, eps=1e-6, seed=0, nslots=None,
             stride_pad=0, return_k=True, with_cache=True):
    rng = np.random.default_rng(seed)
    tdt = dtype
    dname = "bf16" if dtype == torch.bfloat16 else "fp16"
    width = (hq + 2 * hkv) * D
    buf = np.zeros((T, width + stride_pad), np.float32)
    buf[:, :width] = qr.round_dt(rng.standard_normal((T, width)).astype(np.float32) * 1.5, dname)
    qkv_full = torch.from_numpy(buf).to(tdt).cuda()
    qkv = qkv_full[:, :width]
    positions = torch.from_numpy(rng.integers(0, max_pos, T).astype(np.int64)).cuda()
    wq = qr.round_dt(1 + 0.25 * rng.standard_normal(D).astype(np.float32), dname)
    wk = qr.round_dt(1 + 0.25 * rng.standard_normal(D).astype(np.float32), dname)
    cs = rope_cache(max_pos, base)
    nslots = nslots or (T + 5)
    if with_cache:
        slots = rng.permutation(nslots)[:T].astype(np.int32)
        slots[:: 7] = -1
        kc = torch.full((nslots, hkv, D), 3.0, dtype=tdt, device="cuda")
        vc = torch.full((nslots, hkv, D), 3.0, dtype=tdt, device="cuda")
        sl = torch.from_numpy(slots).cuda()
    else:
        slots, kc, vc, sl = None, None, None, None
    q, k, v = pkg.qk_norm_rope_store(qkv, positions, hq, hkv, torch.from_numpy(wq).to(tdt).cuda(),
                                     torch.from_numpy(wk).to(tdt).cuda(), eps, cs.cuda(), kc, vc, sl,
                                     return_k=return_k)
    torch.cuda.synchronize()
    kc_ref = np.full((nslots, hkv, D), 3.0, np.float32) if with_cache else None
    vc_ref = np.full((nslots, hkv, D), 3.0, np.float32) if with_cache else None
    qo, ko, vo = qr.qk_norm_rope_store_ref(buf[:, :width], positions.cpu().numpy(), hq, hkv, wq, wk, eps,
                                           cs.numpy(), kc_ref.reshape(nslots, 1, hkv, D) if with_cache else None,
                                           vc_ref.reshape(nslots, 1, hkv, D) if with_cache else None, slots,
                                           dtype=dname)
    close_dt(to_np(q), qo, dname)
    if return_k:
        close_dt(to_np(k), ko, dname)
    assert (to_np(v) == vo).all()
    if with_cache:
        got_k, got_v = to_np(kc), to_np(vc)
        for t, s in enumerate(slots):
            if s >= 0:
                if return_k:
                    assert (got_k[s] == to_np(k[t])).all(), "cached k differs from returned k"
                assert (got_v[s] == vo[t]).all(), "cached v is not a bitwise copy"
        untouched = np.setdiff1d(np.arange(nslots), slots[slots >= 0])
        assert (got_k[untouched] == 3.0).all() and (got_v[untouched] == 3.0).all()
        close_dt(got_k[slots[slots >= 0]], kc_ref[slots[slots >= 0]], dname)


@pytest.mark.parametrize("T,hq,hkv", [(1, 16, 8), (37, 16, 8), (300, 32, 8), (64, 40, 8), (9, 8, 8), (5, 8, 1)])
def test_against_oracle(pkg, T, hq, hkv):
    run_case(pkg, T, hq, hkv, seed=T + hq)


def test_fp16_strided_no_k_out(pkg):
    run_case(pkg, 50, 16, 8, dtype=torch.float16, stride_pad=256, return_k=False, base=1e4, eps=1e-5)


def test_without_cache(pkg):
    run_case(pkg, 20, 16, 8, with_cache=False)


@pytest.mark.parametrize("name", ["qwen3_0p6b", "group4"])
def test_against_reference_modules(pkg, name):
    c = load_case(np.load(GOLDEN), name)
    qkv = torch.from_numpy(c["qkv"]).to(torch.bfloat16).cuda()
    q, k, _ = pkg.qk_norm_rope_store(qkv, torch.from_numpy(c["positions"]).cuda(), c["hq"], c["hkv"],
                                     torch.from_numpy(c["q_weight"]).to(torch.bfloat16).cuda(),
                                     torch.from_numpy(c["k_weight"]).to(torch.bfloat16).cuda(), c["eps"],
                                     torch.from_numpy(c["cos_sin"]).cuda())
    close_dt(to_np(q), c["q"], "bf16")
    close_dt(to_np(k), c["k"], "bf16")


def test_prefill_sized_batch_matches_oracle_rows(pkg):
    """Config 3's token count in one call; rows sampled against the oracle."""
    rng = np.random.default_rng(3)
    T, hq, hkv = 18715, 16, 8
    width = (hq + 2 * hkv) * D
    qkv = (torch.randn(T, width, device="cuda") * 1.5).to(torch.bfloat16)
    positions = torch.from_numpy(rng.integers(0, 4096, T).astype(np.int64)).cuda()
    w = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    cs = rope_cache(4096, 1e6)
    q, k, _ = pkg.qk_norm_rope_store(qkv, positions, hq, hkv, w, w, 1e-6, cs.cuda())
    rows = rng.choice(T, 64, replace=False)
    qo, ko, _ = qr.qk_norm_rope_store_ref(to_np(qkv[rows]), positions.cpu().numpy()[rows], hq, hkv, np.ones(D),
                                          np.ones(D), 1e-6, cs.numpy())
    close_dt(to_np(q[rows]), qo, "bf16")
    close_dt(to_np(k[rows]), ko, "bf16")


def test_argument_errors(pkg):
    qkv = torch.zeros(4, 48 * D, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(4, dtype=torch.int64, device="cuda")
    w = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    cs = rope_cache(16, 1e6).cuda()
    with pytest.raises(AssertionError):
        pkg.qk_norm_rope_store(qkv, pos, 16, 8, w, w, 1e-6, cs)  # width 48*D != (16+16)*D
    with pytest.raises(AssertionError):
        pkg.qk_norm_rope_store(qkv[:, :32 * D], pos.int(), 16, 8, w, w, 1e-6, cs)  # int32 positions
