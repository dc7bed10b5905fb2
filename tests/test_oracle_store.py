"""KV-scatter oracle pinned to the reference's own Triton kernel (CPU)."""
import os

import numpy as np
import pytest

from oracle import kv_store

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "store_kvcache.npz")
CASES = ["guide", "decode_bf16", "prefill_strided_v", "fp16_h1_d64"]


def load_case(z, name):
    """Golden case as raw-bit numpy arrays; caches start at the fill value."""
    n, hkv, d, nb, bs = (int(x) for x in z[f"{name}__shape"])
    key = z[f"{name}__key"].reshape(n, hkv, d)
    value = z[f"{name}__value"].reshape(n, hkv, d)
    dt = str(z[f"{name}__dtype"])
    fill = float(z[f"{name}__fill"])
    if dt == "torch.float32":
        fill_bits = np.asarray(fill, np.float32).view(np.uint32)
    else:
        import torch
        t = torch.tensor([fill], dtype=getattr(torch, dt.split(".")[1]))
        fill_bits = t.view(torch.int16).numpy().view(np.uint16)[0]
    kc = np.full((nb, bs, hkv, d), fill_bits, dtype=key.dtype)
    vc = kc.copy()
    return dict(key=key, value=value, slots=z[f"{name}__slots"], kc=kc, vc=vc,
                k_after=z[f"{name}__k_after"].reshape(kc.shape), v_after=z[f"{name}__v_after"].reshape(kc.shape),
                bs=bs, dtype=dt, value_stride=int(z[f"{name}__value_stride"]))


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", CASES)
def test_vectorised_oracle_matches_reference_triton(golden, name):
    c = load_case(golden, name)
    kv_store.store_kvcache_ref(c["key"], c["value"], c["kc"], c["vc"], c["slots"])
    assert np.array_equal(c["kc"], c["k_after"]) and np.array_equal(c["vc"], c["v_after"])


@pytest.mark.parametrize("name", CASES)
def test_loop_oracle_matches_reference_triton(golden, name):
    c = load_case(golden, name)
    kv_store.store_kvcache_loop_ref(c["key"], c["value"], c["kc"], c["vc"], c["slots"], c["bs"])
    assert np.array_equal(c["kc"], c["k_after"]) and np.array_equal(c["vc"], c["v_after"])


def test_guide_example_by_hand(golden):
    """master_nano-vllm-v2.md:2845-2852: token0 -> [block1, off1], token1 -> [block0, off0], token2 skipped."""
    c = load_case(golden, "guide")
    k = c["k_after"].view(np.float32)
    assert k[1, 1, 0].tolist() == [10.0, 11.0]
    assert k[0, 0, 0].tolist() == [20.0, 21.0]
    untouched = np.ones(k.shape[:2], bool)
    untouched[1, 1] = untouched[0, 0] = False
    assert (k[untouched] == -999.0).all()


def test_out_of_range_slots_are_skipped():
    key = np.arange(2 * 1 * 4, dtype=np.float32).reshape(2, 1, 4)
    kc = np.zeros((1, 4, 1, 4), np.float32)
    vc = np.zeros_like(kc)
    kv_store.store_kvcache_ref(key, key, kc, vc, np.asarray([4, 2], np.int32))
    assert (kc[0, 2, 0] == key[1, 0]).all() and kc.sum() == key[1].sum()


def test_reference_asserts_restated():
    key = np.zeros((3, 2, 4), np.float32)[:, :, ::2]  # stride(-1) != 1
    with pytest.raises(AssertionError):
        kv_store.check_store_args(key, key, np.zeros((1, 4, 2, 2), np.float32), np.zeros((1, 4, 2, 2), np.float32),
                                  np.zeros(3, np.int32))
