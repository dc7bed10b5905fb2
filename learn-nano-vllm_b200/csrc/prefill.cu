// Causal varlen prefill attention (replaces nanovllm/layers/attention.py:64-70).
#include "common.cuh"

extern "C" int32_t b200_varlen_prefill(void*, const void*, int64_t, const void*, int64_t, const void*, int64_t,
                                       const int32_t*, const int32_t*, int32_t, int32_t, int32_t, int32_t,
                                       const int32_t*, int32_t, int32_t, int32_t, int32_t, int32_t, float, int32_t,
                                       void*) {
    return b200::fail(B200_ERR_UNSUPPORTED, "varlen_prefill: kernel not built into this library yet");
}
