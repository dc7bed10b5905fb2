"""Device decode metadata against the reference's own prepare_decode / prepare_sample."""
import numpy as np
import pytest
import torch

from oracle.decode_meta import decode_metadata_ref

pytestmark = pytest.mark.gpu


class _Seq:
    """The attributes prepare_decode / prepare_sample read (nanovllm/engine/sequence.py)."""

    def __init__(self, n, tok, temp, table, bs):
        self.n, self.last_token, self.temperature, self.block_table, self.bs = n, tok, temp, table, bs

    def __len__(self):
        return self.n

    @property
    def last_block_num_tokens(self):
        return self.n - (len(self.block_table) - 1) * self.bs


def make_batch(B, bs=256, seed=0):
    rng = np.random.default_rng(seed)
    seqs = []
    for _ in range(B):
        n = int(rng.integers(1, 5000))
        nb = (n + bs - 1) // bs
        seqs.append(_Seq(n, int(rng.integers(0, 151936)), float(rng.uniform(0.1, 2.0)),
                         [int(x) for x in rng.integers(0, 100000, nb)], bs))
    return seqs


@pytest.mark.parametrize("B", [1, 7, 256, 512])
def test_matches_oracle(pkg, B):
    seqs = make_batch(B, seed=B)
    meta = pkg.DecodeMetadata()
    outs = [t.cpu().numpy() for t in meta.build(seqs, 256)]
    want = decode_metadata_ref([(len(s), s.last_token, s.temperature, s.block_table) for s in seqs], 256)
    for got, ref in zip(outs, want):
        assert got.shape == ref.shape and (got == ref).all()


def test_staging_reuse_across_steps(pkg):
    """Successive builds reuse two pinned buffers; every step's tensors stay intact."""
    meta = pkg.DecodeMetadata()
    results = []
    for step in range(6):
        seqs = make_batch(64 + step, seed=100 + step)
        results.append((seqs, meta.build(seqs, 256)))
    torch.cuda.synchronize()
    for seqs, outs in results:
        want = decode_metadata_ref([(len(s), s.last_token, s.temperature, s.block_table) for s in seqs], 256)
        for got, ref in zip(outs, want):
            assert (got.cpu().numpy() == ref).all()


def test_matches_reference_prepare_decode(pkg, nanovllm_ref):
    from nanovllm.engine.model_runner import ModelRunner
    from nanovllm.utils import context as ref_ctx

    class _Runner:  # the two attributes prepare_decode uses
        block_size = 256
        prepare_block_tables = ModelRunner.prepare_block_tables

    seqs = make_batch(300, seed=5)
    runner = _Runner()
    ids, pos = ModelRunner.prepare_decode(runner, seqs)
    c = ref_ctx.get_context()
    temps = ModelRunner.prepare_sample(runner, seqs)
    ref = [ids, pos, c.slot_mapping, c.context_lens, c.block_tables, temps]
    ref_ctx.reset_context()
    got = pkg.DecodeMetadata().build(seqs, 256)
    for g, r in zip(got, ref):
        assert g.dtype == r.dtype and g.shape == r.shape and torch.equal(g, r)
