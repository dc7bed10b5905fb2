"""ctypes binding of libb200attn.so (the C ABI of include/b200_attn.h).

The library is the only compute path: when it is missing, every op raises
instead of falling back to another implementation.
"""
import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libb200attn.so")

B200_OK, B200_ERR_ARG, B200_ERR_UNSUPPORTED, B200_ERR_WORKSPACE, B200_ERR_CUDA = range(5)
B200_F16, B200_BF16, B200_F32 = range(3)

# Exported symbols and their ctypes signatures (restype, argtypes).
_P, _I32, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
SIGNATURES = {
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_abi_version": (_I32, []),
    "b200_store_kvcache": (_I32, [_P, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _P]),
    "b200_paged_attention_workspace_size": (_SZ, [_I32, _I32, _I32, _I32]),
    "b200_paged_attention": (_I32, [_P, _P, _I64, _P, _P, _I32, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32,
                                    _I32, _F, _I32, _P, _SZ, _P]),
    "b200_paged_attention_noalloc": (_I32, [_P, _P, _I64, _P, _P, _I32, _I32, _P, _I32, _P, _I32, _I32, _I32,
                                            _I32, _I32, _F, _I32, _P]),
    "b200_workspace_error": (_I32, [_P, _P, ctypes.POINTER(ctypes.c_int32)]),
    "b200_paged_attention_noalloc_error": (_I32, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "b200_testing_idle_producer": (_I32, [_I32, _I64]),
    "b200_varlen_prefill_workspace_size": (_SZ, []),
    "b200_varlen_prefill": (_I32, [_P, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _P,
                                   _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _SZ, _P]),
    "b200_varlen_prefill_error": (_I32, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "b200_spec_accept_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "b200_spec_accept": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _SZ, _P]),
    "b200_oproj_allreduce": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I32, _P, _I32, _P, _I32,
                                    _P, _I64, _I32, _I32, _P]),
    "b200_oproj_allreduce_workspace_size": (_I64, []),
    "b200_oproj_allreduce_error": (_I32, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "b200_allreduce_bf16": (_I32, [_P, _P, _I64, _P, _I64, _P, _I32, _I32, _P]),
    "b200_allreduce_flag_words": (_I64, []),
    "b200_allreduce_error": (_I32, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "b200_decode_metadata": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "b200_sample_workspace_size": (_SZ, [_I32]),
    "b200_sample": (_I32, [_P, _P, _I64, _I32, _P, _I32, _I32, _P, _I64, ctypes.c_uint64, ctypes.c_uint64, _P, _SZ,
                           _P]),
    "b200_qk_norm_rope_store": (_I32, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _F, _P, _I32, _P, _P, _P, _I64,
                                       _I32, _I32, _I32, _I32, _I32, _P]),
}
ABI_VERSION = 3

_lib = None
_lock = threading.Lock()


class B200Error(RuntimeError):
    """A kernel launch or CUDA call of the B200 library failed."""


def lib():
    """The loaded library (loaded once); raises if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing: build it with learn-nano-vllm_b200/build.py")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    if not hasattr(handle, name):
                        raise ImportError(f"{LIB_PATH} does not export {name}; rebuild it")
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                if handle.b200_abi_version() != ABI_VERSION:
                    raise ImportError(f"{LIB_PATH}: ABI version {handle.b200_abi_version()} != {ABI_VERSION}")
                _lib = handle
    return _lib


def check(rc, what):
    """Raise for a non-zero status: argument errors as AssertionError (the
    reference launcher asserts, nanovllm/layers/attention.py:36-39), the rest
    as B200Error / NotImplementedError."""
    if rc == B200_OK:
        return
    msg = (lib().b200_last_error() or b"").decode(errors="replace")
    if rc == B200_ERR_ARG:
        raise AssertionError(msg)
    if rc == B200_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise B200Error(f"{what} failed (status {rc}): {msg}")
