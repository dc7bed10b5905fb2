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
