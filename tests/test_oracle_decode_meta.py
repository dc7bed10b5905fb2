"""Decode metadata oracle (CPU): the reference's formulas on hand-made sequences."""
import numpy as np

from oracle.decode_meta import decode_metadata_ref


def test_slots_positions_and_padding():
    bs = 256
    seqs = [(1, 11, 0.6, [7]), (256, 12, 1.0, [3]), (257, 13, 0.5, [3, 9]), (600, 14, 1.2, [1, 2, 5])]
    ids, pos, slots, lens, bt, temps = decode_metadata_ref(seqs, bs)
    assert ids.tolist() == [11, 12, 13, 14] and pos.tolist() == [0, 255, 256, 599]
    # last token sits at offset len-1 of the sequence: block (len-1)//bs, row (len-1)%bs
    assert slots.tolist() == [7 * bs + 0, 3 * bs + 255, 9 * bs + 0, 5 * bs + 87]
    assert lens.tolist() == [1, 256, 257, 600]
    assert bt.shape == (4, 3) and bt[0].tolist() == [7, -1, -1] and bt[3].tolist() == [1, 2, 5]
    assert np.allclose(temps, [0.6, 1.0, 0.5, 1.2])


def _golden():
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_meta.npz")
    return np.load(path)


def _cases(g):
    return sorted({k.split(".")[0] for k in g.files})


def test_oracle_matches_reference_builders():
    """Pinned to the reference's own prepare_decode / prepare_sample outputs
    (tests/golden/decode_meta.npz, generator beside it): every tensor equal."""
    g = _golden()
    names = _cases(g)
    assert names == ["b1", "b17_short", "b256_long", "b64_mixed"]
    for name in names:
        off = g[name + ".table_offsets"]
        flat = g[name + ".tables_flat"]
        seqs = [(int(n), int(t), float(tp), flat[off[i]:off[i + 1]].tolist())
                for i, (n, t, tp) in enumerate(zip(g[name + ".lengths"], g[name + ".last_tokens"],
                                                   g[name + ".temperatures_in"]))]
        ids, pos, slots, lens, bt, temps = decode_metadata_ref(seqs, 256)
        assert np.array_equal(ids, g[name + ".input_ids"]), name
        assert np.array_equal(pos, g[name + ".positions"]), name
        assert np.array_equal(slots, g[name + ".slot_mapping"]) and slots.dtype == g[name + ".slot_mapping"].dtype
        assert np.array_equal(lens, g[name + ".context_lens"]), name
        assert np.array_equal(bt, g[name + ".block_tables"]), name
        assert np.array_equal(temps, g[name + ".temperatures"]) and temps.dtype == np.float32, name
