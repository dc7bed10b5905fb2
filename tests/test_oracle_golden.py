"""Attention oracle pinned to flash-attn 2.8.3 outputs (CPU).

tests/golden/attention_flash_attn.npz holds flash-attn's outputs on seeded
cases, produced on a B200 by tests/golden/gen_attention_golden.py with the
exact calls of nanovllm/layers/attention.py:67-74.  The inputs are rebuilt
here from the same seeds (checked by checksum) and the numpy oracle must
agree within the attention tolerance.
"""
import json
import os
import sys

import numpy as np
import pytest

from oracle import attention as oatt
from tests.helpers import ATOL_MAX, ATOL_MEAN

HERE = os.path.join(os.path.dirname(__file__), "golden")
sys.path.insert(0, HERE)
import gen_attention_golden as gen  # noqa: E402

GOLDEN = os.path.join(HERE, "attention_flash_attn.npz")


def bf16_bits_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def golden_case(name):
    z = np.load(GOLDEN)
    p = json.loads(str(z[f"{name}__params"]))
    kind = p.pop("kind")
    c = gen.build_case(kind, p)
    q, k, v = gen.stored_inputs(kind, c)
    assert np.isclose(gen.checksum(q, k, v), float(z[f"{name}__checksum"]), rtol=0, atol=1e-6), "inputs drifted"
    want = bf16_bits_to_f32(z[f"{name}__out"])
    rows = z[f"{name}__rows"] if f"{name}__rows" in z.files else None
    return kind, c, q, k, v, want, rows


@pytest.mark.parametrize("name", [n for n, _, _ in gen.CASES])
def test_oracle_matches_flash_attn(name):
    kind, c, q, k, v, want, rows = golden_case(name)
    if kind == "decode":
        got = oatt.paged_attention_ref(q, k, v, c.block_tables, c.context_lens, c.scale)
    else:
        got = oatt.varlen_prefill_ref(q, k, v, c.cu_seqlens_q, c.cu_seqlens_k, c.scale, c.block_tables)
        got = got[rows]
    err = np.abs(got - want.reshape(got.shape))
    assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (name, err.max(), err.mean())
    # bf16 rounding of flash-attn's output bounds the agreement from below
    assert err.max() <= 2 ** -8 * max(1.0, np.abs(want).max()) * 2


def test_fixture_metadata():
    meta = json.loads(str(np.load(GOLDEN)["__meta"]))
    assert meta["flash_attn"] == "2.8.3" and "B200" in meta["gpu"]
