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
//   sampling: inverse CDF over tile sums, thread sums of the chosen tile,
//              then the thread's 16 elements, each scanned left to right.
//
// Kernel 1 (one CTA per logits row): max and canonical sum of exp per row.
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

// Canonical thread partial of tile t for thread i: elements k*1024 + 4i + c.
template <typename F>
__device__ __forceinline__ float thread_partial(int t, int i, int V, F&& w) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int j = t * kTileElems + k * 1024 + 4 * i + c;
            if (j < V) acc = __fadd_rn(acc, w(j));
        }
    }
    return acc;
}

__device__ __forceinline__ float warp_butterfly(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void __launch_bounds__(kThreads) row_stats_kernel(Rows R, float2* stats) {
    __shared__ float red[kThreads / 32];
    __shared__ float wsum[kMaxTiles][kThreads / 32];
    int b;
    const float* x = row_ptr(R, blockIdx.x, &b);
    const float T = R.temps ? R.temps[b] : 0.f;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float m = -INFINITY;
    for (int j = tid; j < R.V; j += kThreads) m = fmaxf(m, scaled(__ldg(x + j), T));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) M = fmaxf(M, red[w]);
    const int nt = (R.V + kTileElems - 1) / kTileElems;
    for (int t = 0; t < nt; ++t) {
        const float part = thread_partial(t, tid, R.V, [&](int j) { return exp_c(__fsub_rn(scaled(__ldg(x + j), T), M)); });
        const float ws = warp_butterfly(part);
        if (lane == 0) wsum[t][warp] = ws;
    }
    __syncthreads();
    if (tid == 0) {
        float S = 0.f;
        for (int t = 0; t < nt; ++t) {
            float st = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) st = __fadd_rn(st, wsum[t][w]);
            S = __fadd_rn(S, st);
        }
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
    __device__ __forceinline__ float operator()(int j) const {
        const float p = __fdiv_rn(exp_c(__fsub_rn(scaled(__ldg(xt + j), T), Mt)), St);
        if (!residual) return p;
        const float q = __fdiv_rn(exp_c(__fsub_rn(scaled(__ldg(xd + j), T), Md)), Sd);
        return fmaxf(__fsub_rn(p, q), 0.f);
    }
};

// Canonical inverse-CDF pick over the whole row; -1 if the row has no mass.
__device__ int canon_pick(const Weight& w, int V, float u, float* part, float* wsum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nt = (V + kTileElems - 1) / kTileElems;
    for (int t = 0; t < nt; ++t) {
        const float pt = thread_partial(t, tid, V, w);
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
    if (threadIdx.x == 0) {
        int rej = k;
        for (int i = 0; i < k; ++i) {
            const int x = d.draft[b * k + i];
            if (x < 0 || x >= V) {
                rej = i;
                break;
            }
            const float2 st = d.stats[b * (k + 1) + i];
            const float2 sd = d.stats[rows_t + b * k + i];
            const float* xt = R.tl + (int64_t(b) * (k + 1) + i) * V;
            const float* xd = R.dl + (int64_t(b) * k + i) * V;
            const float p = __fdiv_rn(exp_c(__fsub_rn(scaled(xt[x], T), st.x)), st.y);
            const float q = __fdiv_rn(exp_c(__fsub_rn(scaled(xd[x], T), sd.x)), sd.y);
            const bool acc = q > 0.f ? (d.ua[b * k + i] < fminf(1.f, __fdiv_rn(p, q))) : (p > 0.f);
            if (!acc) {
                rej = i;
                break;
            }
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
