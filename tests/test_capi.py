"""C ABI: the library loads, exports every declared symbol, and rejects bad
arguments before touching the GPU (CPU only)."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200_attn.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"B200_API\s+[\w\s\*]*?\b(b200_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_symbols()
    for n in ("b200_store_kvcache", "b200_paged_attention", "b200_varlen_prefill", "b200_spec_accept"):
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    from learn_nano_vllm_b200 import _native
    for n in declared_symbols():
        assert hasattr(lib, n), f"{n} not exported"
        assert n in _native.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.b200_abi_version() == _native.ABI_VERSION


def test_argument_errors_mirror_reference_asserts(pkg):
    lib = pkg.lib()
    rc = lib.b200_store_kvcache(None, 1024, None, 1024, None, None, None, 4, 8, 128, 1024, 2, None)
    assert rc == 1 and b"null" in lib.b200_last_error()
    assert lib.b200_store_kvcache(None, 0, None, 0, None, None, None, 0, 8, 128, 0, 2, None) == 0  # N = 0: no-op
    dummy = ctypes.c_void_p(256)
    rc = lib.b200_paged_attention(dummy, dummy, 2048, dummy, dummy, 4, 256, dummy, 4, dummy, 2, 1, 16, 8, 64,
                                  0.1, 1, dummy, 1 << 20, None)
    assert rc == 2 and b"head_dim" in lib.b200_last_error()
    rc = lib.b200_paged_attention(dummy, dummy, 2048, dummy, dummy, 4, 256, dummy, 4, dummy, 2, 3, 16, 2, 128,
                                  0.1, 1, dummy, 1 << 20, None)
    assert rc == 2 and b"exceeds 16" in lib.b200_last_error()
    rc = lib.b200_paged_attention(dummy, dummy, 2048, dummy, dummy, 4, 100, dummy, 4, dummy, 2, 1, 16, 8, 128,
                                  0.1, 1, dummy, 1 << 20, None)
    assert rc == 1 and b"block_size" in lib.b200_last_error()
    rc = lib.b200_paged_attention(dummy, dummy, 2048, dummy, dummy, 4, 256, dummy, 4, dummy, 2, 1, 16, 8, 128,
                                  0.1, 1, None, 0, None)
    assert rc == 3
    for bad_scale in (0.0, -0.1, float("inf"), float("nan")):
        rc = lib.b200_paged_attention(dummy, dummy, 2048, dummy, dummy, 4, 256, dummy, 4, dummy, 2, 1, 16, 8, 128,
                                      bad_scale, 1, dummy, 1 << 20, None)
        assert rc == 1 and b"softmax_scale" in lib.b200_last_error()
        rc = lib.b200_paged_attention_noalloc(dummy, dummy, 2048, dummy, dummy, 4, 256, dummy, 4, dummy, 2, 1, 16, 8,
                                              128, bad_scale, 1, None)
        assert rc == 1 and b"softmax_scale" in lib.b200_last_error()


def test_allreduce_argument_errors(pkg):
    """b200_allreduce_bf16 rejects bad arguments before it touches memory or launches."""
    lib = pkg.lib()
    d = ctypes.c_void_p(256)
    assert lib.b200_allreduce_bf16(d, d, 0, d, 0, d, 0, 2, None) == 0  # n = 0: no-op
    rc = lib.b200_allreduce_bf16(None, d, 64, d, 128, d, 0, 2, None)
    assert rc == 1 and b"null" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(d, d, 64, d, 128, d, 2, 2, None)
    assert rc == 1 and b"rank" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(d, d, 64, d, 128, d, 0, 9, None)
    assert rc == 1 and b"rank" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(d, d, 60, d, 128, d, 0, 2, None)
    assert rc == 1 and b"multiple of 8" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(ctypes.c_void_p(264), d, 64, d, 128, d, 0, 2, None)
    assert rc == 1 and b"aligned" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(d, d, 64, d, 112, d, 0, 2, None)
    assert rc == 1 and b"symmetric buffer" in lib.b200_last_error()
    rc = lib.b200_allreduce_bf16(d, d, 64, d, 136, d, 0, 2, None)
    assert rc == 1 and b"multiple of 16" in lib.b200_last_error()
    assert lib.b200_allreduce_flag_words() >= 2 * 8 * 148 + 2


def test_workspace_size():
    import __graft_entry__
    lib = __graft_entry__.load_package().lib()
    a = lib.b200_paged_attention_workspace_size(1000, 1, 2, 128)
    b = lib.b200_paged_attention_workspace_size(2000, 1, 2, 128)
    assert a % 256 == 0 and abs((b - a) - 1000 * 2 * 129 * 4) < 256


def test_python_wrapper_asserts_like_reference(pkg):
    """nanovllm/layers/attention.py:36-39 asserts, raised before any CUDA work."""
    key = torch.zeros(4, 8, 256)[:, :, ::2]          # stride(-1) == 2
    cache = torch.zeros(2, 16, 8, 128)
    with pytest.raises(AssertionError):
        pkg.store_kvcache(key, key, cache, cache, torch.zeros(4, dtype=torch.int32))
    key = torch.zeros(4, 8, 128)
    with pytest.raises(AssertionError):
        pkg.store_kvcache(key, key, cache, cache, torch.zeros(3, dtype=torch.int32))   # numel != N
    with pytest.raises(AssertionError):
        pkg.store_kvcache(key, key, cache, cache, torch.zeros(4, dtype=torch.int32))   # CPU tensors


def test_oproj_allreduce_argument_errors(pkg):
    """b200_oproj_allreduce rejects bad shapes, ranks and pointers before any CUDA call."""
    lib = pkg.lib()
    d = ctypes.c_void_p(256)

    def call(M=64, N=1024, K=512, ldo=1024, out=d, rank=0, world=2):
        return lib.b200_oproj_allreduce(out, ldo, d, K, d, K, M, N, K, d, 512, d, 128, d, 148, d, 1 << 20,
                                        rank, world, None)
    assert call(M=0) == 0                                   # nothing to do, no launch
    assert call(M=-1) == 1
    assert call(out=None) == 1 and b"null" in lib.b200_last_error()
    assert call(rank=2) == 1 and b"rank" in lib.b200_last_error()
    assert call(world=9) == 1
    assert call(N=300) == 2 and b"256" in lib.b200_last_error()
    assert call(K=100) == 2
    assert call(ldo=100) == 1 and b"strides" in lib.b200_last_error()
    assert lib.b200_oproj_allreduce_error(None, None) == 1


def test_decode_metadata_argument_errors(pkg):
    lib = pkg.lib()
    d = ctypes.c_void_p(256)
    assert lib.b200_decode_metadata(d, 0, 4, 256, d, d, d, d, d, d, None) == 0   # empty batch
    assert lib.b200_decode_metadata(d, -1, 4, 256, d, d, d, d, d, d, None) == 1
    assert lib.b200_decode_metadata(d, 4, 0, 256, d, d, d, d, d, d, None) == 1
    assert lib.b200_decode_metadata(None, 4, 4, 256, d, d, d, d, d, d, None) == 1
