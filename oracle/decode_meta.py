"""Decode-step metadata oracle (test infrastructure only).

Restates nanovllm/engine/model_runner.py:123-127 (prepare_block_tables), :167-187
(prepare_decode) and :189-193 (prepare_sample) for sequences given as
(length, last_token, temperature, block_table list):
  input_ids = last tokens; positions = len - 1; context_lens = len;
  slot_mapping = block_table[-1] * block_size + last_block_num_tokens - 1 with
  last_block_num_tokens = len - (len(block_table) - 1) * block_size
  (nanovllm/engine/sequence.py); block_tables padded with -1 to the longest table.
Pinned to the reference builders' own output on reference Sequence objects
(tests/golden/decode_meta.npz).
"""
import numpy as np


def decode_metadata_ref(seqs, block_size):
    """seqs: list of (length, last_token, temperature, block_table)."""
    lens = np.array([s[0] for s in seqs], np.int64)
    toks = np.array([s[1] for s in seqs], np.int64)
    temps = np.array([s[2] for s in seqs], np.float32)
    tables = [list(s[3]) for s in seqs]
    W = max(len(t) for t in tables)
    bt = np.full((len(seqs), W), -1, np.int32)
    slots = np.empty(len(seqs), np.int32)
    for b, t in enumerate(tables):
        bt[b, :len(t)] = t
        last_n = lens[b] - (len(t) - 1) * block_size
        slots[b] = t[-1] * block_size + last_n - 1
    return toks, lens - 1, slots, lens.astype(np.int32), bt, temps


def expand_packed_ref(packed, batch, width, block_size):
    """The device kernel's expansion (learn-nano-vllm_b200/csrc/decode_meta.cu) of the packed
    int32 buffer [B lengths | B last tokens | B temperature bits | B + 1 block-list offsets |
    block ids] into (input_ids, positions, slot_mapping, context_lens, block_tables [B, width],
    temperatures)."""
    h = np.asarray(packed, np.int32)
    B = batch
    lens, toks = h[:B], h[B:2 * B]
    temps = h[2 * B:3 * B].view(np.float32)
    offs, flat = h[3 * B:4 * B + 1], h[4 * B + 1:]
    bt = np.full((B, width), -1, np.int32)
    slots = np.full(B, -1, np.int32)
    for b in range(B):
        n = int(offs[b + 1] - offs[b])
        bt[b, :n] = flat[offs[b]:offs[b + 1]]
        if n > 0:
            slots[b] = flat[offs[b] + n - 1] * block_size + (lens[b] - (n - 1) * block_size) - 1
    return (toks.astype(np.int64), (lens - 1).astype(np.int64), slots, lens.astype(np.int32), bt,
            temps.astype(np.float32))
