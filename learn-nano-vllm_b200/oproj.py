"""Row-parallel output projection fused with its all-reduce (b200_oproj_allreduce).

OprojAllReduce(group, max_tokens, hidden) allocates, once, every rank's slot and
flag buffers in CUDA symmetric memory (torch.distributed._symmetric_memory; peers
are reached with plain stores, no multicast), exchanges their addresses and
allocates this rank's split-K workspace.  Calling it with this rank's attention
output a [M, K] and o_proj weight shard w [N, K] returns y = sum over ranks of
a_r @ w_r^T, as RowParallelLinear.forward followed by its all-reduce
(nanovllm/layers/linear.py:152-156).  Every rank must make the same calls in the
same order; the call counter lives on the device, so calls may be captured in a
CUDA graph.
"""
import ctypes

import torch
import torch.distributed as dist

from ._native import check, lib

_BN = 256


class OprojAllReduce:

    def __init__(self, group, max_tokens: int, hidden: int, device=None, low_latency: bool = True):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        assert hidden % _BN == 0, "hidden size must be a multiple of 256"
        self.N, self.max_tokens = hidden, max_tokens
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        # ready flags per work unit: a 128 x 256 tile, or a K split of one (never more units than SMs)
        self.max_units = max(((max_tokens + 127) // 128) * (hidden // _BN), sms)
        self.slots = symm_mem.empty(2 * self.world * max_tokens * hidden, dtype=torch.bfloat16, device=self.device)
        self.flags = symm_mem.empty(self.max_units * self.world + 2, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        # low-latency slots for decode batches (M <= 128): words of (2 bf16, epoch)
        self.ll_rows = min(128, max_tokens) if low_latency else 0
        self.ll = symm_mem.empty(max(2 * self.world * self.ll_rows * hidden, 4), dtype=torch.int32, device=self.device)
        self.ll.zero_()
        h_slots = symm_mem.rendezvous(self.slots, group)
        h_flags = symm_mem.rendezvous(self.flags, group)
        h_ll = symm_mem.rendezvous(self.ll, group)
        # device arrays of every rank's buffer addresses (this tensor's offset inside each mapping)
        ds = self.slots.data_ptr() - h_slots.buffer_ptrs[self.rank]
        df = self.flags.data_ptr() - h_flags.buffer_ptrs[self.rank]
        self.slot_ptrs = torch.tensor([b + ds for b in h_slots.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.flag_ptrs = torch.tensor([b + df for b in h_flags.buffer_ptrs], dtype=torch.int64, device=self.device)
        dl = self.ll.data_ptr() - h_ll.buffer_ptrs[self.rank]
        self.ll_ptrs = torch.tensor([b + dl for b in h_ll.buffer_ptrs], dtype=torch.int64, device=self.device)
        self._handles = (h_slots, h_flags, h_ll)
        self.workspace = torch.zeros(lib().b200_oproj_allreduce_workspace_size(), dtype=torch.uint8,
                                     device=self.device)
        self.calls = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(group)  # every rank's flags are zero before anyone's first call

    def __call__(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        assert a.dtype == w.dtype == torch.bfloat16 and a.dim() == 2 and w.dim() == 2
        assert a.stride(-1) == 1 and w.stride(-1) == 1
        M, K = a.shape
        N = w.shape[0]
        assert w.shape[1] == K and N == self.N and M <= self.max_tokens
        if out is None:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
        self.calls += 1
        rc = lib().b200_oproj_allreduce(out.data_ptr(), out.stride(0), a.data_ptr(), a.stride(0), w.data_ptr(),
                                        w.stride(0), M, N, K, self.slot_ptrs.data_ptr(), self.max_tokens,
                                        self.ll_ptrs.data_ptr(), self.ll_rows, self.flag_ptrs.data_ptr(), self.max_units, self.workspace.data_ptr(),
                                        self.workspace.numel(), self.rank, self.world,
                                        torch.cuda.current_stream(a.device).cuda_stream)
        check(rc, "oproj_allreduce")
        return out

    def error(self) -> int:
        flag = ctypes.c_int32(0)
        check(lib().b200_oproj_allreduce_error(torch.cuda.current_stream(self.device).cuda_stream,
                                               ctypes.byref(flag)), "oproj_allreduce_error")
        return flag.value
