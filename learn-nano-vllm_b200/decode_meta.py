"""Decode-step metadata built on the device (nanovllm/engine/model_runner.py:167-193).

DecodeMetadata.build(seqs, block_size) gathers, per sequence, its length, last token,
temperature and block-table list into one pinned int32 buffer (a flat concatenation,
no padded nested lists), copies it to the device in one transfer and expands it there
with b200_decode_metadata.  It returns the tensors prepare_decode / prepare_sample
return: input_ids, positions (int64), slot_mapping, context_lens, block_tables
(int32, -1 padded to the batch's longest table) and temperatures (fp32).

Tensor-parallel worker ranks receive trimmed sequences (Sequence.__getstate__,
nanovllm/engine/sequence.py:72-83, carries no temperature) and never sample
(model_runner.py:216 reads temperatures on rank 0 only): they build with
temperatures=False, which writes 1.0 instead of reading them.
"""
import itertools

import numpy as np
import torch

from ._native import check, lib


class DecodeMetadata:

    def __init__(self, device=None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._host = None  # reusable pinned staging buffers (two, alternated)
        self._copied = [None, None]  # event after the last copy out of each buffer
        self._flip = 0

    def _staging(self, n):
        if self._host is None or self._host[0].numel() < n:
            for ev in self._copied:
                if ev is not None:
                    ev.synchronize()
            size = max(n, 1 << 14)
            self._host = [torch.empty(size, dtype=torch.int32, pin_memory=True) for _ in range(2)]
            self._copied = [None, None]
        self._flip ^= 1
        ev = self._copied[self._flip]
        if ev is not None:
            ev.synchronize()  # the copy that last read this buffer has finished
        return self._host[self._flip]

    @staticmethod
    def packed_size(seqs):
        """(int32 words of the packed buffer, block-table width W) for a batch."""
        nblk = sum(len(s.block_table) for s in seqs)
        W = max(max((len(s.block_table) for s in seqs), default=1), 1)
        return 4 * len(seqs) + 1 + nblk, W

    @staticmethod
    def pack(seqs, h, temperatures=True):
        """Write the packed buffer into the int32 numpy array h: [B] lengths, [B] last tokens,
        [B] temperatures (fp32 bits; 1.0 when temperatures is False), [B + 1] block-list
        offsets, then every block id."""
        B = len(seqs)
        tables = [s.block_table for s in seqs]
        nblk = np.fromiter((len(t) for t in tables), np.int32, B)
        n = 4 * B + 1 + int(nblk.sum())
        h[:B] = np.fromiter((len(s) for s in seqs), np.int32, B)
        h[B:2 * B] = np.fromiter((s.last_token for s in seqs), np.int32, B)
        if temperatures:
            h[2 * B:3 * B] = np.fromiter((s.temperature for s in seqs), np.float32, B).view(np.int32)
        else:
            h[2 * B:3 * B] = np.float32(1.0).view(np.int32)
        h[3 * B] = 0
        np.cumsum(nblk, out=h[3 * B + 1:4 * B + 1])
        h[4 * B + 1:n] = np.fromiter(itertools.chain.from_iterable(tables), np.int32, n - 4 * B - 1)
        return n

    def build(self, seqs, block_size, temperatures=True):
        B = len(seqs)
        n, W = self.packed_size(seqs)
        host = self._staging(n)
        self.pack(seqs, host.numpy(), temperatures)
        stream = torch.cuda.current_stream(self.device)
        packed = torch.empty(n, dtype=torch.int32, device=self.device)
        packed.copy_(host[:n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._copied[self._flip] = ev
        out64 = torch.empty(2 * B, dtype=torch.int64, device=self.device)
        out32 = torch.empty(2 * B + B * W, dtype=torch.int32, device=self.device)
        temps = torch.empty(B, dtype=torch.float32, device=self.device)
        input_ids, positions = out64[:B], out64[B:]
        slot_mapping, context_lens = out32[:B], out32[B:2 * B]
        block_tables = out32[2 * B:].view(B, W)
        rc = lib().b200_decode_metadata(packed.data_ptr(), B, W, block_size, input_ids.data_ptr(),
                                        positions.data_ptr(), slot_mapping.data_ptr(), context_lens.data_ptr(),
                                        block_tables.data_ptr(), temps.data_ptr(), stream.cuda_stream)
        check(rc, "decode_metadata")
        return input_ids, positions, slot_mapping, context_lens, block_tables, temps
