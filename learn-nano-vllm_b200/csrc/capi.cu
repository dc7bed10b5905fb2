// Host-side plumbing of the C ABI: error text, device queries, tensor maps.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace b200 {

namespace {
thread_local char g_last_error[512] = {0};

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int32_t fail(int32_t code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = 0; }

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (g_sm_count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

void ensure_smem_attr(const void* kernel, int bytes) {
    // Cheap and idempotent; setting it on every call keeps multi-device use simple.
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int32_t make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool bf16,
                     CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    if (!g_encode) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
        return fail(B200_ERR_ARG, "TMA base address %p is not 16-byte aligned", base);
    if (row_stride_bytes % 16 != 0)
        return fail(B200_ERR_ARG, "TMA row stride %llu bytes is not a multiple of 16",
                    (unsigned long long)row_stride_bytes);
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return B200_OK;
}

}  // namespace b200

extern "C" {

const char* b200_last_error(void) { return b200::g_last_error; }

int32_t b200_abi_version(void) { return B200_ABI_VERSION; }

int32_t b200_workspace_error(const void* workspace, void* stream, int32_t* flag) {
    B200_REQUIRE(workspace != nullptr && flag != nullptr, "workspace_error: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The error word is the third int32 of the control header (see paged_attention.cu).
    B200_CUDA_TRY(cudaMemcpyAsync(flag, static_cast<const int32_t*>(workspace) + 2, sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, s));
    B200_CUDA_TRY(cudaStreamSynchronize(s));
    return B200_OK;
}

}  // extern "C"
