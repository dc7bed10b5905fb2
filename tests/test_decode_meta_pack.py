"""Host side of the device decode metadata (CPU): the packed buffer DecodeMetadata.pack
writes, for full sequences (rank 0) and for the trimmed sequences tensor-parallel worker
ranks receive (nanovllm/engine/sequence.py:72-83 pickles no temperature)."""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def DecodeMetadata():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    return importlib.import_module(pkg.__name__ + ".decode_meta").DecodeMetadata


class FullSeq:
    """What rank 0 holds: length, last token, temperature, block table."""

    def __init__(self, n, last, temp, table):
        self.n, self.last_token, self.temperature, self.block_table = n, last, temp, table

    def __len__(self):
        return self.n


class WorkerSeq:
    """What a worker rank unpickles (the state tuple of Sequence.__getstate__): no temperature."""

    def __init__(self, full):
        self.n, self.last_token, self.block_table = full.n, full.last_token, full.block_table

    def __len__(self):
        return self.n


SEQS = [FullSeq(1, 11, 0.6, [7]), FullSeq(256, 12, 1.0, [3]), FullSeq(257, 13, 0.5, [3, 9]),
        FullSeq(600, 14, 1.2, [1, 2, 5])]


def test_pack_layout(DecodeMetadata):
    n, W = DecodeMetadata.packed_size(SEQS)
    assert (n, W) == (4 * 4 + 1 + 7, 3)
    h = np.zeros(n, np.int32)
    assert DecodeMetadata.pack(SEQS, h) == n
    B = 4
    assert h[:B].tolist() == [1, 256, 257, 600]
    assert h[B:2 * B].tolist() == [11, 12, 13, 14]
    assert np.allclose(h[2 * B:3 * B].view(np.float32), [0.6, 1.0, 0.5, 1.2])
    assert h[3 * B:4 * B + 1].tolist() == [0, 1, 2, 4, 7]
    assert h[4 * B + 1:].tolist() == [7, 3, 3, 9, 1, 2, 5]


def test_pack_worker_sequences(DecodeMetadata):
    workers = [WorkerSeq(s) for s in SEQS]
    n, _ = DecodeMetadata.packed_size(workers)
    h = np.zeros(n, np.int32)
    with pytest.raises(AttributeError):
        DecodeMetadata.pack(workers, h)  # a worker cannot read temperatures ...
    DecodeMetadata.pack(workers, h, temperatures=False)  # ... and does not need them
    full = np.zeros(n, np.int32)
    DecodeMetadata.pack(SEQS, full)
    B = len(SEQS)
    assert np.array_equal(np.delete(h, range(2 * B, 3 * B)), np.delete(full, range(2 * B, 3 * B)))
    assert np.all(h[2 * B:3 * B].view(np.float32) == 1.0)


def test_pack_then_kernel_expansion_equals_reference_builders(DecodeMetadata):
    """Random batches: DecodeMetadata.pack followed by the kernel's expansion (restated in
    numpy) gives the reference builders' tensors (oracle pinned to them), on rank 0 and, apart
    from temperatures, on worker ranks."""
    from oracle.decode_meta import decode_metadata_ref, expand_packed_ref
    rng = np.random.default_rng(5)
    for trial in range(60):
        B = int(rng.integers(1, 40))
        ids = rng.permutation(4096)
        seqs, used = [], 0
        for _ in range(B):
            n = int(rng.integers(1, 3000))
            nb = (n + 255) // 256
            seqs.append(FullSeq(n, int(rng.integers(0, 151936)), float(rng.uniform(0.1, 2.0)),
                                [int(x) for x in ids[used:used + nb]]))
            used += nb
        size, W = DecodeMetadata.packed_size(seqs)
        h = np.zeros(size, np.int32)
        DecodeMetadata.pack(seqs, h)
        got = expand_packed_ref(h, B, W, 256)
        want = decode_metadata_ref([(len(s), s.last_token, s.temperature, s.block_table) for s in seqs], 256)
        for g, w in zip(got, want):
            assert g.dtype == w.dtype and np.array_equal(g, w)
        hw = np.zeros(size, np.int32)
        DecodeMetadata.pack([WorkerSeq(s) for s in seqs], hw, temperatures=False)
        gw = expand_packed_ref(hw, B, W, 256)
        for g, w in zip(gw[:5], want[:5]):
            assert np.array_equal(g, w)
