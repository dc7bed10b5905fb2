// Fused q/k RMSNorm + rotary embedding + KV-cache scatter for Qwen3
// attention.  Replaces, in one pass over the QKV projection output,
//   q = q_norm(q); k = k_norm(k)               nanovllm/models/qwen3.py:82-84
//                                              (RMSNorm.rms_forward, layers/layernorm.py:16-26)
//   q, k = rotary_emb(positions, q, k)         qwen3.py:85 (layers/rotary_embedding.py:6-14, 37-48)
//   store_kvcache(k, v, k_cache, v_cache, slot_mapping)   layers/attention.py:60-63
// with the reference's rounding points (eager order):
//   RMSNorm: x in fp32, var = mean(x^2), x *= rsqrt(var + eps), round to the
//            model dtype, multiply by the weight (fp32 product, rounded);
//   RoPE   : x1, x2 = halves of x in fp32; y1 = x1*cos - x2*sin,
//            y2 = x2*cos + x1*sin (each product rounded, then the sum), round;
//            cos / sin are the caller's cos_sin_cache rows [cos | sin] (fp32).
//
// One warp per (token, group of kHeadsPerWarp heads): all the group's rows
// are loaded first (eight 8-byte loads per lane in flight), the token's
// position, slot and cos / sin row once.  Per row of D = 128, lane l holds
// elements 4l..4l+3, the sum of squares is a warp butterfly, and the rotary
// partner of element i (i +/- 64) sits in lane l ^ 16, one shuffle away.
// Rows of v are copied to the value cache unchanged; rows of k go to the key
// cache after normalisation and rotation.  Slots of -1 (padding) or outside
// the cache are skipped, as in store_kvcache.
#include "common.cuh"

namespace b200 {
namespace qkr {

constexpr int kD = 128;
constexpr int kWarps = 8;         // warps per CTA
constexpr int kHeadsPerWarp = 8;  // rows of one token per warp

struct Params {
    uint16_t* q_out;
    int64_t q_out_stride;  // elements between tokens
    uint16_t* k_out;       // may be null
    int64_t k_out_stride;
    const uint16_t* qkv;
    int64_t qkv_stride;
    const int64_t* positions;
    const uint16_t* q_weight;
    const uint16_t* k_weight;
    float eps;
    const float* cos_sin;  // [max_position][kD]: cos (kD/2) | sin (kD/2)
    int32_t max_position;
    uint16_t* k_cache;  // [num_slots][hkv][kD], may be null (no cache yet)
    uint16_t* v_cache;
    const int32_t* slots;
    int64_t num_slots;
    int32_t num_tokens, hq, hkv;
};

template <bool BF16>
__device__ __forceinline__ float to_f(uint16_t b) {
    if constexpr (BF16) return __uint_as_float(uint32_t(b) << 16);
    else return __half2float(__ushort_as_half(b));
}

template <bool BF16>
__device__ __forceinline__ float round_dt(float x) {
    return to_f<BF16>(to_bits16<BF16>(x));
}

// RMSNorm + RoPE of one q or k row held as 4 values per lane; returns the packed output.
template <bool BF16>
__device__ __forceinline__ uint2 norm_rope_row(uint2 raw, const uint16_t* weight, float eps, const float (&cs)[4],
                                               const float (&sn)[4], int lane) {
    float x[4] = {to_f<BF16>(uint16_t(raw.x)), to_f<BF16>(uint16_t(raw.x >> 16)), to_f<BF16>(uint16_t(raw.y)),
                  to_f<BF16>(uint16_t(raw.y >> 16))};
    float ss = __fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])),
                         __fadd_rn(__fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3])));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(kD)), eps));
    const uint2 wraw = *reinterpret_cast<const uint2*>(weight + 4 * lane);
    const float w[4] = {to_f<BF16>(uint16_t(wraw.x)), to_f<BF16>(uint16_t(wraw.x >> 16)),
                        to_f<BF16>(uint16_t(wraw.y)), to_f<BF16>(uint16_t(wraw.y >> 16))};
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = round_dt<BF16>(__fmul_rn(round_dt<BF16>(__fmul_rn(x[e], inv)), w[e]));
    // lanes 0-15 hold x1 (elements 0-63), lanes 16-31 hold x2; the partner is lane ^ 16
    float z[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) z[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
    const bool first = lane < 16;
    uint16_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float r = first ? __fsub_rn(__fmul_rn(y[e], cs[e]), __fmul_rn(z[e], sn[e]))   // y1 = x1 cos - x2 sin
                              : __fadd_rn(__fmul_rn(y[e], cs[e]), __fmul_rn(z[e], sn[e]));  // y2 = x2 cos + x1 sin
        o[e] = to_bits16<BF16>(r);
    }
    return make_uint2(uint32_t(o[0]) | (uint32_t(o[1]) << 16), uint32_t(o[2]) | (uint32_t(o[3]) << 16));
}

template <bool BF16>
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int heads = p.hq + 2 * p.hkv;
    const int groups = (heads + kHeadsPerWarp - 1) / kHeadsPerWarp;
    const int64_t wid = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    if (wid >= int64_t(p.num_tokens) * groups) return;
    const int64_t t = wid / groups;
    const int h0 = int(wid - t * groups) * kHeadsPerWarp;
    const int nh = min(kHeadsPerWarp, heads - h0);
    const uint16_t* src = p.qkv + t * p.qkv_stride + int64_t(h0) * kD + 4 * lane;
    uint2 raw[kHeadsPerWarp];
#pragma unroll
    for (int i = 0; i < kHeadsPerWarp; ++i)
        if (i < nh) raw[i] = *reinterpret_cast<const uint2*>(src + i * kD);
    const int32_t slot = p.k_cache ? p.slots[t] : -1;
    const bool store = slot >= 0 && slot < p.num_slots;
    float cs[4] = {0.f, 0.f, 0.f, 0.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    if (h0 < p.hq + p.hkv) {  // the group holds q or k rows: this token's cos / sin
        int64_t pos = p.positions[t];
        pos = pos < 0 ? 0 : (pos >= p.max_position ? p.max_position - 1 : pos);
        const int i0 = 4 * (lane & 15);
        const float4 c = *reinterpret_cast<const float4*>(p.cos_sin + pos * kD + i0);
        const float4 s = *reinterpret_cast<const float4*>(p.cos_sin + pos * kD + kD / 2 + i0);
        cs[0] = c.x, cs[1] = c.y, cs[2] = c.z, cs[3] = c.w;
        sn[0] = s.x, sn[1] = s.y, sn[2] = s.z, sn[3] = s.w;
    }
#pragma unroll
    for (int i = 0; i < kHeadsPerWarp; ++i) {
        if (i >= nh) break;
        const int h = h0 + i;
        if (h >= p.hq + p.hkv) {  // v row: straight into the value cache
            if (store)
                *reinterpret_cast<uint2*>(p.v_cache + (int64_t(slot) * p.hkv + (h - p.hq - p.hkv)) * kD + 4 * lane) =
                    raw[i];
            continue;
        }
        const bool is_q = h < p.hq;
        const uint2 out = norm_rope_row<BF16>(raw[i], is_q ? p.q_weight : p.k_weight, p.eps, cs, sn, lane);
        if (is_q) {
            *reinterpret_cast<uint2*>(p.q_out + t * p.q_out_stride + int64_t(h) * kD + 4 * lane) = out;
        } else {
            const int hk = h - p.hq;
            if (p.k_out) *reinterpret_cast<uint2*>(p.k_out + t * p.k_out_stride + int64_t(hk) * kD + 4 * lane) = out;
            if (store) *reinterpret_cast<uint2*>(p.k_cache + (int64_t(slot) * p.hkv + hk) * kD + 4 * lane) = out;
        }
    }
}

}  // namespace qkr
}  // namespace b200

extern "C" int32_t b200_qk_norm_rope_store(void* q_out, int64_t q_out_stride, void* k_out, int64_t k_out_stride,
                                           const void* qkv, int64_t qkv_stride, const int64_t* positions,
                                           const void* q_weight, const void* k_weight, float eps,
                                           const float* cos_sin, int32_t max_position, void* k_cache,
                                           void* v_cache, const int32_t* slot_mapping, int64_t num_slots,
                                           int32_t num_tokens, int32_t num_heads, int32_t num_kv_heads,
                                           int32_t head_dim, int32_t dtype, void* stream) {
    using namespace b200;
    using namespace b200::qkr;
    clear_error();
    B200_REQUIRE(num_tokens >= 0, "qk_norm_rope_store: num_tokens %d < 0", num_tokens);
    if (num_tokens == 0) return B200_OK;
    B200_REQUIRE(q_out && qkv && positions && q_weight && k_weight && cos_sin, "qk_norm_rope_store: null pointer");
    B200_REQUIRE(!k_cache == !v_cache, "qk_norm_rope_store: k_cache and v_cache must both be given or both null");
    B200_REQUIRE(!k_cache || (slot_mapping && num_slots >= 0), "qk_norm_rope_store: cache without slot_mapping");
    B200_REQUIRE(num_heads > 0 && num_kv_heads > 0, "qk_norm_rope_store: heads %d / %d", num_heads, num_kv_heads);
    if (head_dim != kD) return fail(B200_ERR_UNSUPPORTED, "qk_norm_rope_store: head_dim %d (only 128)", head_dim);
    if (dtype != B200_BF16 && dtype != B200_F16)
        return fail(B200_ERR_UNSUPPORTED, "qk_norm_rope_store: dtype %d (bf16 or fp16 only)", dtype);
    B200_REQUIRE(max_position > 0, "qk_norm_rope_store: max_position %d", max_position);
    const int64_t width = int64_t(num_heads + 2 * num_kv_heads) * kD;
    B200_REQUIRE(qkv_stride >= width && q_out_stride >= int64_t(num_heads) * kD &&
                     (!k_out || k_out_stride >= int64_t(num_kv_heads) * kD),
                 "qk_norm_rope_store: token strides below the head rows");
    auto al = [](const void* ptr, int n) { return (reinterpret_cast<uintptr_t>(ptr) % n) == 0; };
    B200_REQUIRE(al(qkv, 8) && al(q_out, 8) && (!k_out || al(k_out, 8)) && (!k_cache || (al(k_cache, 8) && al(v_cache, 8))) &&
                     al(q_weight, 8) && al(k_weight, 8) && al(cos_sin, 16) && qkv_stride % 4 == 0 &&
                     q_out_stride % 4 == 0 && (!k_out || k_out_stride % 4 == 0),
                 "qk_norm_rope_store: rows must be 8-byte aligned (cos_sin 16-byte)");
    Params prm;
    prm.q_out = static_cast<uint16_t*>(q_out);
    prm.q_out_stride = q_out_stride;
    prm.k_out = static_cast<uint16_t*>(k_out);
    prm.k_out_stride = k_out_stride;
    prm.qkv = static_cast<const uint16_t*>(qkv);
    prm.qkv_stride = qkv_stride;
    prm.positions = positions;
    prm.q_weight = static_cast<const uint16_t*>(q_weight);
    prm.k_weight = static_cast<const uint16_t*>(k_weight);
    prm.eps = eps;
    prm.cos_sin = cos_sin;
    prm.max_position = max_position;
    prm.k_cache = static_cast<uint16_t*>(k_cache);
    prm.v_cache = static_cast<uint16_t*>(v_cache);
    prm.slots = slot_mapping;
    prm.num_slots = num_slots;
    prm.num_tokens = num_tokens;
    prm.hq = num_heads;
    prm.hkv = num_kv_heads;
    const int64_t groups = (num_heads + 2 * num_kv_heads + kHeadsPerWarp - 1) / kHeadsPerWarp;
    const int64_t warps = int64_t(num_tokens) * groups;
    const int64_t blocks = (warps + kWarps - 1) / kWarps;
    B200_REQUIRE(blocks < (int64_t(1) << 31), "qk_norm_rope_store: too many rows");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == B200_BF16) qk_norm_rope_kernel<true><<<unsigned(blocks), kWarps * 32, 0, st>>>(prm);
    else qk_norm_rope_kernel<false><<<unsigned(blocks), kWarps * 32, 0, st>>>(prm);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
