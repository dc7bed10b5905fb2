// Fused temperature + exponential-race sampler.  Replaces nanovllm/layers/sampler.py:7-12
//     logits = logits.float() / T;  p = softmax(logits)
//     token  = argmax(p / clamp_min(Exp(1) noise, 1e-10))
// in one pass over the logits.  Since softmax only rescales each row by a
// positive constant, argmax_j p_j / E_j = argmax_j (x_j / T - log E_j), which
// needs neither the row max nor the normaliser: each value is read once.
//
// Noise: either the caller's E tensor [B, V] fp32 (the reference's own
// `exponential_` draw, for like-for-like checks) or E = -log(U) with U from
// Philox-4x32-10 (Salmon et al., SC'11: 10 rounds, multipliers 0xD2511F53 /
// 0xCD9E8D57, Weyl key increments 0x9E3779B9 / 0xBB67AE85), counter
// (j / 4, row, offset_lo, offset_hi), key (seed_lo, seed_hi), lane j % 4,
// U = ((bits >> 8) + 0.5) * 2^-24, so every (seed, offset) gives the same
// tokens on any grid.  Ties go to the smallest index, as torch.argmax.
//
// The generator path scores in base 2: argmax_j (x_j / T - ln E_j) =
// argmax_j (x_j log2(e) / T - log2(-log2 U_j)) (a positive scale and a
// constant shift), two lg2 per value; four values share one Philox call and
// one vector load.
// Kernel 1 (grid rows x chunks): per chunk the best (score, index);
// kernel 2 (one warp per row): the best over the row's chunks.
#include "common.cuh"

namespace b200 {
namespace smp {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 32;

struct Params {
    const void* logits;
    int64_t row_stride;  // elements
    const float* temps;
    const float* noise;  // [B, V] fp32 or null
    int64_t noise_stride;
    uint64_t seed, offset;
    int32_t B, V, chunks;
    float2* part;  // [B][chunks]: (score, index as float bits)
    int64_t* out;
};

__device__ __forceinline__ void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
        const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

template <int DT>
__device__ __forceinline__ float load_logit(const void* row, int j) {
    if constexpr (DT == B200_F32) return static_cast<const float*>(row)[j];
    const uint16_t b = static_cast<const uint16_t*>(row)[j];
    if constexpr (DT == B200_BF16) return __uint_as_float(uint32_t(b) << 16);
    return __half2float(__ushort_as_half(b));
}

// Four consecutive logits starting at j (a multiple of 4) with one vector load.
template <int DT>
__device__ __forceinline__ void load4(const void* row, int j, float (&x)[4]) {
    if constexpr (DT == B200_F32) {
        const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(row) + j);
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else {
        const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(row) + j);
        const uint16_t h[4] = {uint16_t(v.x), uint16_t(v.x >> 16), uint16_t(v.y), uint16_t(v.y >> 16)};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            x[q] = DT == B200_BF16 ? __uint_as_float(uint32_t(h[q]) << 16) : __half2float(__ushort_as_half(h[q]));
    }
}

__device__ __forceinline__ void take(float s, int j, float& best, int& bi) {
    if (s > best || (s == best && j < bi)) {
        best = s;
        bi = j;
    }
}

template <int DT>
__global__ void __launch_bounds__(kThreads) sample_chunks_kernel(const Params p, bool vec) {
    const int b = blockIdx.x / p.chunks, c = blockIdx.x - b * p.chunks;
    const int per = (((p.V + p.chunks - 1) / p.chunks) + 3) & ~3;  // chunk length, a multiple of 4
    const int j0 = c * per, j1 = min(p.V, j0 + per);
    const void* row = static_cast<const char*>(p.logits) + int64_t(b) * p.row_stride * (DT == B200_F32 ? 4 : 2);
    float best = -INFINITY;
    int bi = INT32_MAX;
    if (p.noise) {
        const float inv_t = 1.f / p.temps[b];
        const float* e = p.noise + int64_t(b) * p.noise_stride;
        for (int j = j0 + threadIdx.x; j < j1; j += kThreads)
            take(load_logit<DT>(row, j) * inv_t - __logf(fmaxf(e[j], 1e-10f)), j, best, bi);
    } else {
        const float scale = 1.4426950408889634f / p.temps[b];  // log2(e) / T
        const uint32_t k0 = uint32_t(p.seed), k1 = uint32_t(p.seed >> 32);
#pragma unroll 2
        for (int g = j0 / 4 + threadIdx.x; g * 4 < j1; g += kThreads) {
            uint32_t ctr[4] = {uint32_t(g), uint32_t(b), uint32_t(p.offset), uint32_t(p.offset >> 32)};
            philox4x32_10(ctr, k0, k1);
            float x[4];
            const bool full = g * 4 + 3 < j1;
            if (vec && full) {
                load4<DT>(row, g * 4, x);
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) x[q] = g * 4 + q < j1 ? load_logit<DT>(row, g * 4 + q) : 0.f;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = g * 4 + q;
                if (j >= j1) break;
                const uint32_t k24 = ctr[q] >> 8;
                const float u = (float(k24) + 0.5f) * 0x1.0p-24f;
                // E / ln 2 = -log2(U) > 0.  lg2.approx is accurate relative to |log2 U| only
                // away from 1; for U > 1 - 2^-10 use -ln(1 - v) = v (1 + v/2 + v^2/3 + ...)
                // with v = 1 - U, exact in fp32 there.
                const float v = (float(0xFFFFFFu - k24) + 0.5f) * 0x1.0p-24f;
                const float series = v * fmaf(v, fmaf(v, 0.33333334f, 0.5f), 1.f) * 1.4426950408889634f;
                const float l2e = v < 0x1.0p-10f ? series : -fast_log2(u);
                take(fmaf(x[q], scale, -fast_log2(l2e)), j, best, bi);
            }
        }
    }
    // block reduction of (best, index)
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float s = __shfl_xor_sync(0xffffffffu, best, o);
        const int i = __shfl_xor_sync(0xffffffffu, bi, o);
        take(s, i, best, bi);
    }
    __shared__ float ws[kThreads / 32];
    __shared__ int wi[kThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        ws[warp] = best;
        wi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kThreads / 32; ++w) take(ws[w], wi[w], best, bi);
        p.part[int64_t(b) * p.chunks + c] = make_float2(best, __int_as_float(bi));
    }
}

__global__ void sample_combine_kernel(const Params p) {
    const int b = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= p.B) return;
    float best = -INFINITY;
    int bi = INT32_MAX;
    for (int c = lane; c < p.chunks; c += 32) {
        const float2 v = p.part[int64_t(b) * p.chunks + c];
        take(v.x, __float_as_int(v.y), best, bi);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float s = __shfl_xor_sync(0xffffffffu, best, o);
        const int i = __shfl_xor_sync(0xffffffffu, bi, o);
        take(s, i, best, bi);
    }
    // a row whose scores are all NaN or -inf keeps the first index, as argmax does for a
    // row of equal values
    if (lane == 0) p.out[b] = bi == INT32_MAX ? 0 : bi;
}

inline int chunks_for(int B, int V) {
    int c = (8 * device_sm_count() + B - 1) / B;  // enough CTAs to fill every SM several times
    c = c < 1 ? 1 : (c > kMaxChunks ? kMaxChunks : c);
    const int max_by_len = (V + 1023) / 1024;  // at least ~1024 values per chunk
    return c < max_by_len ? c : (max_by_len < 1 ? 1 : max_by_len);
}

}  // namespace smp
}  // namespace b200

extern "C" size_t b200_sample_workspace_size(int32_t batch) {
    if (batch < 0) return 0;
    return ((size_t(batch) * b200::smp::kMaxChunks * sizeof(float2)) + 255) & ~size_t(255);
}

extern "C" int32_t b200_sample(int64_t* out_tokens, const void* logits, int64_t row_stride, int32_t dtype,
                               const float* temperatures, int32_t batch, int32_t vocab_size, const float* noise,
                               int64_t noise_stride, uint64_t seed, uint64_t offset, void* workspace,
                               size_t workspace_bytes, void* stream) {
    using namespace b200;
    using namespace b200::smp;
    clear_error();
    B200_REQUIRE(batch >= 0, "sample: batch %d < 0", batch);
    if (batch == 0) return B200_OK;
    B200_REQUIRE(out_tokens && logits && temperatures, "sample: null pointer");
    B200_REQUIRE(vocab_size > 0 && row_stride >= vocab_size, "sample: vocab %d / row stride %lld", vocab_size,
                 (long long)row_stride);
    B200_REQUIRE(!noise || noise_stride >= vocab_size, "sample: noise stride %lld", (long long)noise_stride);
    if (dtype != B200_BF16 && dtype != B200_F16 && dtype != B200_F32)
        return fail(B200_ERR_UNSUPPORTED, "sample: dtype %d", dtype);
    const size_t need = b200_sample_workspace_size(batch);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
        return fail(B200_ERR_WORKSPACE, "sample: workspace needs %zu bytes (16-byte aligned)", need);
    Params p;
    p.logits = logits;
    p.row_stride = row_stride;
    p.temps = temperatures;
    p.noise = noise;
    p.noise_stride = noise_stride;
    p.seed = seed;
    p.offset = offset;
    p.B = batch;
    p.V = vocab_size;
    p.chunks = chunks_for(batch, vocab_size);
    p.part = static_cast<float2*>(workspace);
    p.out = out_tokens;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t esz = dtype == B200_F32 ? 4 : 2;
    const bool vec = (reinterpret_cast<uintptr_t>(logits) % (4 * esz)) == 0 && (size_t(row_stride) * esz) % (4 * esz) == 0;
    if (dtype == B200_BF16) sample_chunks_kernel<B200_BF16><<<batch * p.chunks, kThreads, 0, s>>>(p, vec);
    else if (dtype == B200_F16) sample_chunks_kernel<B200_F16><<<batch * p.chunks, kThreads, 0, s>>>(p, vec);
    else sample_chunks_kernel<B200_F32><<<batch * p.chunks, kThreads, 0, s>>>(p, vec);
    B200_CUDA_TRY(cudaGetLastError());
    sample_combine_kernel<<<(batch + 7) / 8, 256, 0, s>>>(p);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
