// Speculative-decoding acceptance sampling (standard rejection scheme).
//
// The reference engine has no speculative path; this op is new.  Its
// arithmetic is defined in a fixed order with float32 rounding at every
// step (__fmul_rn/__fadd_rn/__fdiv_rn, no contraction into FMA), so that a
// CPU restatement reproduces accept/reject decisions and sampled tokens bit
// for bit given the same uniforms:
//   exp_c(x) = 2^n * P(f), y = x*log2(e), n = rint(y), f = y - n, P the
//              degree-7 Taylor polynomial of 2^f in Horner form, 0 below y=-125;
//   row sums: tiles of 4096; thread i of 256 adds its elements
//              k*1024 + 4i + c (k outer, c inner), a warp xor-butterfly
//              (16,8,4,2,1) combines 32 threads, 8 warp sums and then the
//              tile sums are added left to right;
//   normaliser: per tile M_t = tile max, S_t = tile sum of exp_c(x - M_t);
//              M = max_t M_t, S = sum_t S_t * exp_c(M_t - M) (left to right);
//              p_j = exp_c(x_j - M) / S; non-finite logits weigh 0;
//   sampling: inverse CDF over tile sums, thread sums of the chosen tile,
//              then the thread's 16 elements, each scanned left to right.
//
// Kernel 1 (one CTA per logits row, one pass over the row): M and S.
// Kernel 2 (one CTA per sequence): decisions from the per-row statistics,
// then one pass over the rejected row (residual) or the bonus row.
#include "common.cuh"

namespace b200 {
namespace spec {

constexpr int kThreads = 256;
constexpr int kTileElems = 4096;
constexpr int kMaxTiles = 48;  // vocab <= 196608
constexpr float kLog2e = 0x1.715476p+0f;
__device__ __constant__ float kExpCoef[8] = {0x1.0p+0f,      0x1.62e430p-1f,  0x1.ebfbe0p-3f, 0x1.c6b08ep-5f,
                                              0x1.3b2ab6p-7f, 0x1.5d87fep-10f, 0x1.430912p-13f, 0x1.ffcbfcp-17f};

__device__ __forceinline__ float exp_c(float x) {
    const float y = __fmul_rn(x, kLog2e);
    const float n = rintf(y);
    const float f = __fsub_rn(y, n);
    float p = kExpCoef[7];
#pragma unroll
    for (int k = 6; k >= 0; --k) p = __fadd_rn(__fmul_rn(p, f), kExpCoef[k]);
    const int ni = int(fminf(fmaxf(n, -126.f), 127.f));
    const float r = __fmul_rn(p, __int_as_float((ni + 127) << 23));
    return y < -125.f ? 0.f : r;
}

struct Rows {
    const float* tl;   // [B, k+1, V]
    const float* dl;   // [B, k, V]
    const float* temps;
    int32_t B, k, V;
};

__device__ __forceinline__ const float* row_ptr(const Rows& R, int r, int* b_out) {
    const int nt = R.B * (R.k + 1);
    if (r < nt) {
        *b_out = r / (R.k + 1);
        return R.tl + int64_t(r) * R.V;
    }
    const int rd = r - nt;
    *b_out = rd / R.k;
    return R.dl + int64_t(rd) * R.V;
}

__device__ __forceinline__ float scaled(float l, float T) { return T > 0.f ? __fdiv_rn(l, T) : l; }

__device__ __forceinline__ float warp_butterfly(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One tile (4096 values) of a row as this thread's 16 values, in the fixed
// order k = 0..3 (stride 1024), c = 0..3; values past V read as -inf.
__device__ __forceinline__ void load_tile(const float* x, int V, int t, float T, bool vec, float (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int base = t * kTileElems + k * 1024 + 4 * int(threadIdx.x);
        if (vec && base + 3 < V) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(x + base));
            v[4 * k] = scaled(f.x, T);
            v[4 * k + 1] = scaled(f.y, T);
            v[4 * k + 2] = scaled(f.z, T);
            v[4 * k + 3] = scaled(f.w, T);
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) v[4 * k + c] = base + c < V ? scaled(__ldg(x + base + c), T) : -INFINITY;
        }
    }
}

// Per row: M_t and S_t = fixed-order tile sum of exp_c(x - M_t) for every
// tile, then M = max M_t and S = sum_t S_t * exp_c(M_t - M).  Each row is read
// once; the next tile's loads are issued before the current tile's reductions.
__global__ void __launch_bounds__(kThreads) row_stats_kernel(Rows R, float2* stats) {
    __shared__ float wred[kThreads / 32];
    __shared__ float tile_m[kMaxTiles], tile_s[kMaxTiles];
    int b;
    const float* x = row_ptr(R, blockIdx.x, &b);
    const float T = R.temps ? R.temps[b] : 0.f;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool vec = (R.V & 3) == 0;
    const int nt = (R.V + kTileElems - 1) / kTileElems;
    float cur[16], nxt[16];
    load_tile(x, R.V, 0, T, vec, cur);
    for (int t = 0; t < nt; ++t) {
        if (t + 1 < nt) load_tile(x, R.V, t + 1, T, vec, nxt);
        float m = -INFINITY;
#pragma unroll
        for (int e = 0; e < 16; ++e) m = fmaxf(m, cur[e]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wred[warp] = m;
        __syncthreads();
        float Mt = wred[0];
#pragma unroll
        for (int w = 1; w < kThreads / 32; ++w) Mt = fmaxf(Mt, wred[w]);
        __syncthreads();
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e)
            if (isfinite(cur[e])) acc = __fadd_rn(acc, exp_c(__fsub_rn(cur[e], Mt)));
        const float ws = warp_butterfly(acc);
        if (lane == 0) wred[warp] = ws;
        __syncthreads();
        if (tid == 0) {
            float st = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) st = __fadd_rn(st, wred[w]);
            tile_m[t] = Mt;
            tile_s[t] = st;
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 16; ++e) cur[e] = nxt[e];
    }
    if (tid == 0) {
        float M = -INFINITY;
        for (int t = 0; t < nt; ++t) M = fmaxf(M, tile_m[t]);
        float S = 0.f;
        for (int t = 0; t < nt; ++t) S = __fadd_rn(S, __fmul_rn(tile_s[t], exp_c(__fsub_rn(tile_m[t], M))));
        stats[blockIdx.x] = make_float2(M, S);
    }
}

// Left-to-right scan of n values (stride `step` in `vals`) starting at acc0;
// first index with target < acc + v and v > 0, else the last positive entry.
__device__ int scan_pick(const float* vals, int n, float target, float acc0, float* acc_out) {
    float acc = acc0;
    for (int i = 0; i < n; ++i) {
        const float v = vals[i];
        const float nxt = __fadd_rn(acc, v);
        if (target < nxt && v > 0.f) {
            *acc_out = acc;
            return i;
        }
        acc = nxt;
    }
    acc = acc0;
    int last = -1;
    float acc_last = acc0;
    for (int i = 0; i < n; ++i) {
        const float v = vals[i];
        if (v > 0.f) {
            last = i;
            acc_last = acc;
        }
        acc = __fadd_rn(acc, v);
    }
    *acc_out = acc_last;
    return last;
}

struct Decide {
    Rows R;
    const float2* stats;
    const int32_t* draft;
    const float* ua;
    const float* us;
    int32_t* out_tokens;
    int32_t* out_num;
};

// Weight of token j for the sampling row: the residual max(p - q, 0) or p.
struct Weight {
    const float *xt, *xd;
    float T, Mt, St, Md, Sd;
    bool residual;
    bool vec;
    __device__ __forceinline__ float from(float lt, float ld) const {
        const float p = __fdiv_rn(exp_c(__fsub_rn(scaled(lt, T), Mt)), St);
        if (!residual) return p;
        const float q = __fdiv_rn(exp_c(__fsub_rn(scaled(ld, T), Md)), Sd);
        return fmaxf(__fsub_rn(p, q), 0.f);
    }
    __device__ __forceinline__ float operator()(int j) const {
        return from(__ldg(xt + j), residual ? __ldg(xd + j) : 0.f);
    }
};

// Fixed-order thread partial of tile t with float4 loads of both rows.
__device__ __forceinline__ float weight_partial(const Weight& w, int t, int V) {
    float lt[16], ld[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int base = t * kTileElems + k * 1024 + 4 * int(threadIdx.x);
        if (w.vec && base + 3 < V) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w.xt + base));
            lt[4 * k] = a.x, lt[4 * k + 1] = a.y, lt[4 * k + 2] = a.z, lt[4 * k + 3] = a.w;
            if (w.residual) {
                const float4 c = __ldg(reinterpret_cast<const float4*>(w.xd + base));
                ld[4 * k] = c.x, ld[4 * k + 1] = c.y, ld[4 * k + 2] = c.z, ld[4 * k + 3] = c.w;
            } else {
                ld[4 * k] = ld[4 * k + 1] = ld[4 * k + 2] = ld[4 * k + 3] = 0.f;
            }
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const bool in = base + c < V;
                lt[4 * k + c] = in ? __ldg(w.xt + base + c) : 0.f;
                ld[4 * k + c] = in && w.residual ? __ldg(w.xd + base + c) : 0.f;
            }
        }
    }
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const int j = t * kTileElems + (e >> 2) * 1024 + 4 * int(threadIdx.x) + (e & 3);
        if (j < V) acc = __fadd_rn(acc, w.from(lt[e], ld[e]));
    }
    return acc;
}

// Canonical inverse-CDF pick over the whole row; -1 if the row has no mass.
__device__ int canon_pick(const Weight& w, int V, float u, float* part, float* wsum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nt = (V + kTileElems - 1) / kTileElems;
    for (int t = 0; t < nt; ++t) {
        const float pt = weight_partial(w, t, V);
        part[t * kThreads + tid] = pt;
        const float ws = warp_butterfly(pt);
        if (lane == 0) wsum[t * (kThreads / 32) + warp] = ws;
    }
    __syncthreads();
    __shared__ int pick;
    if (tid == 0) {
        float tsum[kMaxTiles];
        float R = 0.f;
        for (int t = 0; t < nt; ++t) {
            float st = 0.f;
            for (int x = 0; x < kThreads / 32; ++x) st = __fadd_rn(st, wsum[t * (kThreads / 32) + x]);
            tsum[t] = st;
            R = __fadd_rn(R, st);
        }
        const float target = __fmul_rn(u, R);
        float acc;
        int res = -1;
        const int t = scan_pick(tsum, nt, target, 0.f, &acc);
        if (t >= 0) {
            const int i = scan_pick(part + t * kThreads, kThreads, target, acc, &acc);
            if (i >= 0) {
                float v16[16];
                int idx[16];
                for (int k = 0; k < 4; ++k)
                    for (int c = 0; c < 4; ++c) {
                        const int j = t * kTileElems + k * 1024 + 4 * i + c;
                        idx[k * 4 + c] = j;
                        v16[k * 4 + c] = j < V ? w(j) : 0.f;
                    }
                const int e = scan_pick(v16, 16, target, acc, &acc);
                res = e < 0 ? -1 : idx[e];
            }
        }
        pick = res;
    }
    __syncthreads();
    const int r = pick;
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kThreads) decide_kernel(Decide d) {
    extern __shared__ float dyn[];
    const Rows& R = d.R;
    const int b = blockIdx.x, k = R.k, V = R.V;
    const int nt = (V + kTileElems - 1) / kTileElems;
    float* part = dyn;                      // [nt][256]
    float* wsum = dyn + nt * kThreads;      // [nt][8]
    __shared__ int rej_s;
    const float T = R.temps ? R.temps[b] : 0.f;
    const int rows_t = R.B * (k + 1);
    // Draft position i's decision on lane i (at most 32 drafts), then the
    // first rejection in order.
    __shared__ int accept_s[32];
    if (threadIdx.x < k) {
        const int i = threadIdx.x;
        const int x = d.draft[b * k + i];
        bool acc = false;
        if (x >= 0 && x < V) {
            const float2 st = d.stats[b * (k + 1) + i];
            const float2 sd = d.stats[rows_t + b * k + i];
            const float* xt = R.tl + (int64_t(b) * (k + 1) + i) * V;
            const float* xd = R.dl + (int64_t(b) * k + i) * V;
            const float p = __fdiv_rn(exp_c(__fsub_rn(scaled(xt[x], T), st.x)), st.y);
            const float q = __fdiv_rn(exp_c(__fsub_rn(scaled(xd[x], T), sd.x)), sd.y);
            acc = q > 0.f ? (d.ua[b * k + i] < fminf(1.f, __fdiv_rn(p, q))) : (p > 0.f);
        }
        accept_s[i] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int rej = k;
        for (int i = 0; i < k; ++i)
            if (!accept_s[i]) {
                rej = i;
                break;
            }
        rej_s = rej;
    }
    __syncthreads();
    const int rej = rej_s;
    Weight w;
    w.T = T;
    w.xt = R.tl + (int64_t(b) * (k + 1) + rej) * V;
    const float2 st = d.stats[b * (k + 1) + rej];
    w.Mt = st.x;
    w.St = st.y;
    w.residual = rej < k;
    w.vec = (V & 3) == 0;
    if (rej < k) {
        w.xd = R.dl + (int64_t(b) * k + rej) * V;
        const float2 sd = d.stats[rows_t + b * k + rej];
        w.Md = sd.x;
        w.Sd = sd.y;
    } else {
        w.xd = nullptr;
        w.Md = w.Sd = 0.f;
    }
    const float u = d.us[b];
    int tok = canon_pick(w, V, u, part, wsum);
    if (tok < 0 && w.residual) {
        w.residual = false;
        tok = canon_pick(w, V, u, part, wsum);
    }
    if (tok < 0) tok = 0;
    if (threadIdx.x == 0) {
        for (int i = 0; i <= k; ++i)
            d.out_tokens[b * (k + 1) + i] = i < rej ? d.draft[b * k + i] : (i == rej ? tok : -1);
        d.out_num[b] = rej + 1;
    }
}

}  // namespace spec
}  // namespace b200

extern "C" size_t b200_spec_accept_workspace_size(int32_t batch, int32_t num_draft, int32_t vocab_size) {
    (void)vocab_size;
    if (batch < 0 || num_draft < 0) return 0;
    const size_t rows = size_t(batch) * (2 * size_t(num_draft) + 1);
    return ((rows * sizeof(float2)) + 255) & ~size_t(255);
}

extern "C" int32_t b200_spec_accept(int32_t* out_tokens, int32_t* out_num_tokens, const float* target_logits,
                                    const float* draft_logits, const int32_t* draft_tokens,
                                    const float* uniform_accept, const float* uniform_sample,
                                    const float* temperatures, int32_t batch, int32_t num_draft, int32_t vocab_size,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    using namespace b200;
    using namespace b200::spec;
    clear_error();
    B200_REQUIRE(batch >= 0 && num_draft >= 0, "spec_accept: negative batch or num_draft");
    if (batch == 0) return B200_OK;
    B200_REQUIRE(out_tokens && out_num_tokens && target_logits && uniform_sample, "spec_accept: null pointer");
    B200_REQUIRE(num_draft == 0 || (draft_logits && draft_tokens && uniform_accept), "spec_accept: null draft pointer");
    B200_REQUIRE(vocab_size > 0, "spec_accept: vocab_size %d", vocab_size);
    if (vocab_size > kMaxTiles * kTileElems)
        return fail(B200_ERR_UNSUPPORTED, "spec_accept: vocab_size %d > %d", vocab_size, kMaxTiles * kTileElems);
    if (num_draft > 32) return fail(B200_ERR_UNSUPPORTED, "spec_accept: num_draft %d > 32", num_draft);
    B200_REQUIRE((reinterpret_cast<uintptr_t>(target_logits) & 15) == 0 &&
                     (num_draft == 0 || (reinterpret_cast<uintptr_t>(draft_logits) & 15) == 0),
                 "spec_accept: logits must be 16-byte aligned");
    const size_t need = b200_spec_accept_workspace_size(batch, num_draft, vocab_size);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
        return fail(B200_ERR_WORKSPACE, "spec_accept: workspace needs %zu bytes (16-byte aligned)", need);
    Rows R{target_logits, draft_logits, temperatures, batch, num_draft, vocab_size};
    float2* stats = static_cast<float2*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int nrows = batch * (2 * num_draft + 1);
    row_stats_kernel<<<nrows, kThreads, 0, s>>>(R, stats);
    B200_CUDA_TRY(cudaGetLastError());
    Decide d{R, stats, draft_tokens, uniform_accept, uniform_sample, out_tokens, out_num_tokens};
    const int nt = (vocab_size + kTileElems - 1) / kTileElems;
    const int smem = nt * (kThreads + kThreads / 32) * int(sizeof(float));
    ensure_smem_attr((const void*)decide_kernel, smem);
    decide_kernel<<<batch, kThreads, smem, s>>>(d);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
