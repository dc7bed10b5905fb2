// Slot-mapped KV-cache scatter (replaces nanovllm/layers/attention.py:10-40).
//
// One warp per token row.  Each lane moves 16-byte vectors of the key row
// and of the value row (all loads of a row are issued before its stores),
// so a 2 KiB Qwen3 row (8 kv heads x 128 x bf16) takes 4 + 4 vector loads
// per lane.  Rows with an unaligned base or stride fall back to element
// copies.  Slots equal to -1 (padding rows, model_runner.py:206-207) and
// slots outside the cache are skipped.
#include "common.cuh"

namespace b200 {
namespace {

constexpr int kStoreWarpsPerBlock = 8;

template <typename V>
__device__ __forceinline__ void copy_row(char* __restrict__ dst, const char* __restrict__ src,
                                         int64_t row_bytes, int lane) {
    constexpr int kUnroll = 4;
    const int64_t step = 32 * static_cast<int64_t>(sizeof(V));
    int64_t off = lane * static_cast<int64_t>(sizeof(V));
    for (; off + (kUnroll - 1) * step < row_bytes; off += kUnroll * step) {
        V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = __ldg(reinterpret_cast<const V*>(src + off + u * step));
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) *reinterpret_cast<V*>(dst + off + u * step) = v[u];
    }
    for (; off < row_bytes; off += step) *reinterpret_cast<V*>(dst + off) = __ldg(reinterpret_cast<const V*>(src + off));
}

template <typename V>
__global__ void __launch_bounds__(kStoreWarpsPerBlock * 32)
    store_kv_kernel(const char* __restrict__ key, int64_t key_stride, const char* __restrict__ value,
                    int64_t value_stride, char* __restrict__ k_cache, char* __restrict__ v_cache,
                    const int32_t* __restrict__ slots, int32_t n, int64_t row_bytes, int64_t num_slots) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kStoreWarpsPerBlock;
    for (int64_t t = blockIdx.x * kStoreWarpsPerBlock + (threadIdx.x >> 5); t < n; t += nwarps) {
        const int64_t slot = slots[t];
        if (slot < 0 || slot >= num_slots) continue;
        copy_row<V>(k_cache + slot * row_bytes, key + t * key_stride, row_bytes, lane);
        copy_row<V>(v_cache + slot * row_bytes, value + t * value_stride, row_bytes, lane);
    }
}

}  // namespace
}  // namespace b200

extern "C" int32_t b200_store_kvcache(const void* key, int64_t key_stride, const void* value,
                                      int64_t value_stride, void* k_cache, void* v_cache,
                                      const int32_t* slot_mapping, int32_t num_tokens, int32_t num_kv_heads,
                                      int32_t head_dim, int64_t num_slots, int32_t elem_bytes, void* stream) {
    using namespace b200;
    clear_error();
    B200_REQUIRE(num_tokens >= 0, "store_kvcache: num_tokens %d < 0", num_tokens);
    if (num_tokens == 0) return B200_OK;
    B200_REQUIRE(key && value && k_cache && v_cache && slot_mapping, "store_kvcache: null pointer");
    B200_REQUIRE(elem_bytes == 2 || elem_bytes == 4, "store_kvcache: elem_bytes %d not 2 or 4", elem_bytes);
    B200_REQUIRE(num_kv_heads > 0 && head_dim > 0, "store_kvcache: bad head shape %d x %d", num_kv_heads, head_dim);
    const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;  // D of the reference
    // Reference asserts (attention.py:36-38): rows hold Hkv*D contiguous elements.
    B200_REQUIRE(key_stride >= row && value_stride >= row,
                 "store_kvcache: token stride (%lld, %lld) below Hkv*D = %lld", (long long)key_stride,
                 (long long)value_stride, (long long)row);
    B200_REQUIRE(num_slots >= 0, "store_kvcache: num_slots < 0");
    const int64_t row_bytes = row * elem_bytes;
    const int64_t ks = key_stride * elem_bytes, vs = value_stride * elem_bytes;
    auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = aligned16(key) && aligned16(value) && aligned16(k_cache) && aligned16(v_cache) &&
                     row_bytes % 16 == 0 && ks % 16 == 0 && vs % 16 == 0;
    const int64_t max_blocks = static_cast<int64_t>(device_sm_count()) * 16;
    const int64_t need = (num_tokens + kStoreWarpsPerBlock - 1) / kStoreWarpsPerBlock;
    const dim3 grid(static_cast<unsigned>(need < max_blocks ? need : max_blocks));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const char* kp = static_cast<const char*>(key);
    const char* vp = static_cast<const char*>(value);
    char* kc = static_cast<char*>(k_cache);
    char* vc = static_cast<char*>(v_cache);
    if (vec)
        store_kv_kernel<uint4><<<grid, kStoreWarpsPerBlock * 32, 0, s>>>(kp, ks, vp, vs, kc, vc, slot_mapping,
                                                                         num_tokens, row_bytes, num_slots);
    else if (elem_bytes == 4)
        store_kv_kernel<uint32_t><<<grid, kStoreWarpsPerBlock * 32, 0, s>>>(kp, ks, vp, vs, kc, vc, slot_mapping,
                                                                            num_tokens, row_bytes, num_slots);
    else
        store_kv_kernel<uint16_t><<<grid, kStoreWarpsPerBlock * 32, 0, s>>>(kp, ks, vp, vs, kc, vc, slot_mapping,
                                                                            num_tokens, row_bytes, num_slots);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
