"""The allocation-free paged-attention entry point, called through the C ABI.

b200_paged_attention_noalloc serves callers that cannot allocate device
memory on their execution path (a runtime whose allocator owns the whole
device heap, a plugin host that forbids cudaMalloc there, code that must not
risk cudaMalloc's implicit synchronisation).  Its split-K scratch is a fixed
32 MiB array inside the library instead of a caller workspace.  This file
checks, on two calls in a row, that it returns what the fp32 oracle returns
and what b200_paged_attention returns with its own workspace, within the
attention tolerance of the other tests; that its error word (read back with
b200_paged_attention_noalloc_error) stays clear on those calls and reports a
wait that runs out; and that it refuses a batch larger than its scratch.  It
is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import cases
from tests.helpers import ATOL_MAX, ATOL_MEAN, assert_attn_close, dev_bf16, dev_i32, host

pytestmark = pytest.mark.gpu

B200_ERR_WORKSPACE = 3
ERR_STAGE_NEVER_FILLED = 1


def _args(out, q, kc, vc, bt, cl, lq, hq, hkv, scale):
    B = q.shape[0]
    return [out.data_ptr(), q.data_ptr(), hq * 128, kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
            bt.data_ptr(), bt.stride(0), cl.data_ptr(), B, lq, hq, hkv, 128, scale, 1]


def _error_word(lib, stream):
    flag = ctypes.c_int32(-1)
    assert lib.b200_paged_attention_noalloc_error(stream, ctypes.byref(flag)) == 0, lib.b200_last_error()
    return flag.value


def _case(ctx, hq, hkv, lq, seed):
    case = cases.make_paged_case(ctx, hq, hkv, lq=lq, seed=seed)
    dev = dict(q=dev_bf16(case.q), kc=dev_bf16(case.k_cache), vc=dev_bf16(case.v_cache),
               bt=dev_i32(case.block_tables), cl=dev_i32(case.context_lens))
    # The oracle reads the bf16-rounded inputs the kernel reads.
    want = oatt.paged_attention_ref(host(dev["q"]), host(dev["kc"]), host(dev["vc"]), case.block_tables,
                                    case.context_lens, case.scale)
    return case, dev, want


@pytest.mark.parametrize("ctx,hq,hkv,lq,seed", [
    (list(cases.config5_context_lens(64, 0.5, seed=3)), 32, 8, 1, 1),   # decode, 8B heads, split contexts
    ([512, 4096, 7, 1300, 2, 0], 16, 8, 5, 2),                          # verify, 5 queries, a padding row
])
def test_noalloc_matches_oracle_and_workspace_entry_point(pkg, ctx, hq, hkv, lq, seed):
    lib = pkg.lib()
    case, d, want = _case(ctx, hq, hkv, lq, seed)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty_like(d["q"])
    ws = torch.zeros(lib.b200_paged_attention_workspace_size(32768, lq, hq // hkv, 128), dtype=torch.uint8,
                     device="cuda")
    rc = lib.b200_paged_attention(*_args(ref, d["q"], d["kc"], d["vc"], d["bt"], d["cl"], lq, hq, hkv, case.scale),
                                  ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, lib.b200_last_error()
    for call in range(2):
        out = torch.full_like(d["q"], float("nan"))
        rc = lib.b200_paged_attention_noalloc(
            *_args(out, d["q"], d["kc"], d["vc"], d["bt"], d["cl"], lq, hq, hkv, case.scale), stream)
        assert rc == 0, lib.b200_last_error()
        assert _error_word(lib, stream) == 0, f"call {call}: a bounded wait ran out"
        assert_attn_close(host(out), want, f"call {call} vs oracle")
        err = (out.float() - ref.float()).abs()
        assert err.max().item() <= ATOL_MAX and err.mean().item() <= ATOL_MEAN, \
            f"call {call} vs b200_paged_attention: max {err.max().item():.3e} mean {err.mean().item():.3e}"


def test_noalloc_reports_a_wait_that_runs_out(pkg):
    """With the test hook the producer warp issues no loads and every wait is limited to
    2 ms: the call returns, its error word says a stage was never filled, and the next call
    (which clears the word) runs normally."""
    lib = pkg.lib()
    case, d, want = _case([300, 1100, 5, 2600], 16, 8, 1, 4)
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.empty_like(d["q"])
    args = _args(out, d["q"], d["kc"], d["vc"], d["bt"], d["cl"], 1, 16, 8, case.scale)
    assert lib.b200_testing_idle_producer(1, 2_000_000) == 0, lib.b200_last_error()
    assert lib.b200_paged_attention_noalloc(*args, stream) == 0, lib.b200_last_error()
    assert _error_word(lib, stream) & ERR_STAGE_NEVER_FILLED
    for call in range(2):
        assert lib.b200_paged_attention_noalloc(*args, stream) == 0, lib.b200_last_error()
        assert _error_word(lib, stream) == 0
        assert_attn_close(host(out), want, f"call {call} after the stalled one")


def test_noalloc_rejects_batches_beyond_its_scratch(pkg):
    lib = pkg.lib()
    dummy = ctypes.c_void_p(256)
    rc = lib.b200_paged_attention_noalloc(dummy, dummy, 4096, dummy, dummy, 8, 256, dummy, 4, dummy, 2048, 1, 32, 8,
                                          128, 0.088, 1, None)
    assert rc == B200_ERR_WORKSPACE
    assert b"exceeds the built-in" in lib.b200_last_error()
