"""The allocation-free paged-attention entry point, called through the C ABI.

b200_paged_attention_noalloc serves callers that cannot allocate device
memory on their execution path (a runtime whose allocator owns the whole
device heap, a plugin host that forbids cudaMalloc there, code that must not
risk cudaMalloc's implicit synchronisation).  Its split-K scratch is a fixed
32 MiB array inside the library instead of a caller workspace.  This file
checks, on two calls in a row, that it returns what b200_paged_attention
returns with its own workspace, within the attention tolerance of the other
tests, and that it refuses a batch larger than its scratch.  It is named to be
collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import cases
from tests.helpers import ATOL_MAX, ATOL_MEAN, dev_bf16, dev_i32

pytestmark = pytest.mark.gpu

B200_ERR_WORKSPACE = 3


def _args(out, q, kc, vc, bt, cl, lq, hq, hkv, scale):
    B = q.shape[0]
    return [out.data_ptr(), q.data_ptr(), hq * 128, kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
            bt.data_ptr(), bt.stride(0), cl.data_ptr(), B, lq, hq, hkv, 128, scale, 1]


@pytest.mark.parametrize("ctx,hq,hkv,lq,seed", [
    (list(cases.config5_context_lens(64, 0.5, seed=3)), 32, 8, 1, 1),   # decode, 8B heads, split contexts
    ([512, 4096, 7, 1300, 2, 0], 16, 8, 5, 2),                          # verify, 5 queries, a padding row
])
def test_noalloc_matches_workspace_entry_point(pkg, ctx, hq, hkv, lq, seed):
    lib = pkg.lib()
    case = cases.make_paged_case(ctx, hq, hkv, lq=lq, seed=seed)
    q, kc, vc = dev_bf16(case.q), dev_bf16(case.k_cache), dev_bf16(case.v_cache)
    bt, cl = dev_i32(case.block_tables), dev_i32(case.context_lens)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty_like(q)
    ws = torch.zeros(lib.b200_paged_attention_workspace_size(32768, lq, hq // hkv, 128), dtype=torch.uint8,
                     device="cuda")
    rc = lib.b200_paged_attention(*_args(ref, q, kc, vc, bt, cl, lq, hq, hkv, case.scale), ws.data_ptr(),
                                  ws.numel(), stream)
    assert rc == 0, lib.b200_last_error()
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = lib.b200_paged_attention_noalloc(*_args(out, q, kc, vc, bt, cl, lq, hq, hkv, case.scale), stream)
        assert rc == 0, lib.b200_last_error()
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all(), f"call {call}: non-finite output"
        assert err.max().item() <= ATOL_MAX and err.mean().item() <= ATOL_MEAN, \
            f"call {call}: max {err.max().item():.3e} mean {err.mean().item():.3e}"


def test_noalloc_rejects_batches_beyond_its_scratch(pkg):
    lib = pkg.lib()
    dummy = ctypes.c_void_p(256)
    rc = lib.b200_paged_attention_noalloc(dummy, dummy, 4096, dummy, dummy, 8, 256, dummy, 4, dummy, 2048, 1, 32, 8,
                                          128, 0.088, 1, None)
    assert rc == B200_ERR_WORKSPACE
    assert b"exceeds the built-in" in lib.b200_last_error()
