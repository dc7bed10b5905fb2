"""All-reduce of a bf16 tensor over the tensor-parallel group (b200_allreduce_bf16).

AllReduce(group, max_elems) allocates, once, every rank's slot and flag buffers
in CUDA symmetric memory (torch.distributed._symmetric_memory; peers are
reached with plain loads and stores, no multicast) and exchanges their
addresses.  Calling it on a contiguous bf16 tensor sums it over the ranks in
place (or into `out`), as the dist.all_reduce that ends RowParallelLinear.forward
(nanovllm/layers/linear.py:155).  Every rank must make the same calls in the
same order; the call counter lives on the device, so calls may be captured in
a CUDA graph.

input_buffer(n) / result_buffer(n) are this rank's symmetric input and result
slots: a producer that writes its output into input_buffer and a consumer that
reads result_buffer save the kernel's copy in and copy out (the result stays
valid until this rank's next call).
"""
import ctypes

import torch
import torch.distributed as dist

from ._native import check, lib


class AllReduce:

    def __init__(self, group, max_elems: int, device=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.max_elems = (int(max_elems) + 7) // 8 * 8
        # [input, result] slots of max_elems values
        self.buf_elems = 2 * self.max_elems
        self.bufs = symm_mem.empty(self.buf_elems, dtype=torch.bfloat16, device=self.device)
        self.flags = symm_mem.empty(int(lib().b200_allreduce_flag_words()), dtype=torch.int32, device=self.device)
        self.flags.zero_()
        h_bufs = symm_mem.rendezvous(self.bufs, group)
        h_flags = symm_mem.rendezvous(self.flags, group)
        # device arrays of every rank's buffer addresses (this tensor's offset inside each mapping)
        db = self.bufs.data_ptr() - h_bufs.buffer_ptrs[self.rank]
        df = self.flags.data_ptr() - h_flags.buffer_ptrs[self.rank]
        self.buf_ptrs = torch.tensor([b + db for b in h_bufs.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.flag_ptrs = torch.tensor([b + df for b in h_flags.buffer_ptrs], dtype=torch.int64, device=self.device)
        self._handles = (h_bufs, h_flags)
        torch.cuda.synchronize(self.device)
        dist.barrier(group)  # every rank's flags are zero before anyone's first call

    def input_buffer(self, n: int) -> torch.Tensor:
        assert 0 <= n <= self.max_elems
        return self.bufs[:n]

    def result_buffer(self, n: int) -> torch.Tensor:
        assert 0 <= n <= self.max_elems
        return self.bufs[self.max_elems:self.max_elems + n]

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.numel() <= self.max_elems
        if out is None:
            out = x
        assert out.dtype == torch.bfloat16 and out.is_contiguous() and out.numel() == x.numel()
        # inside the slot buffer only as the slots themselves (the kernel copies by CTA ranges)
        lo, hi = self.bufs.data_ptr(), self.bufs.data_ptr() + self.bufs.numel() * 2
        for t, ok in ((x, (lo, lo + self.max_elems * 2)), (out, (lo, lo + self.max_elems * 2))):
            p = t.data_ptr()
            assert not (lo <= p < hi or lo < p + t.numel() * 2 <= hi) or p in ok, \
                "tensors inside the slot buffer must start at input_buffer() or result_buffer()"
        rc = lib().b200_allreduce_bf16(out.data_ptr(), x.data_ptr(), x.numel(), self.buf_ptrs.data_ptr(),
                                       self.buf_elems, self.flag_ptrs.data_ptr(), self.rank, self.world,
                                       torch.cuda.current_stream(x.device).cuda_stream)
        check(rc, "allreduce")
        return out

    def error(self) -> int:
        flag = ctypes.c_int32(0)
        check(lib().b200_allreduce_error(torch.cuda.current_stream(self.device).cuda_stream, ctypes.byref(flag)),
              "allreduce_error")
        return flag.value
