// Speculative-decoding acceptance sampling (standard rejection scheme).
//
// The reference engine has no speculative path; this op is new.  Its
// arithmetic is defined in a fixed order with float32 rounding at every
// step (__fmul_rn/__fadd_rn/__fmaf_rn/__frcp_rn, no implicit contraction),
// so that a CPU restatement reproduces accept/reject decisions and sampled
// tokens bit for bit given the same uniforms:
//   exp_c(x), x <= 0: y = min(x*log2(e), 0), n = rint(y) through the magic
//              constant 1.5*2^23, f = y - n, P(f) a degree-5 fit of 2^f
//              (relative error 1.7e-7, P(0) = 1) by fused multiply-add steps,
//              exp_c = P * 2^n by an exponent-field add, 0 below y = -125;
//   row sums: tiles of 4096; thread i of 256 adds its elements
//              k*1024 + 4i + c (k outer, c inner), a warp xor-butterfly
//              (16,8,4,2,1) combines 32 threads, 8 warp sums and then the
//              tile sums are added left to right;
//   normaliser: per tile M_t = tile max, S_t = tile sum of exp_c(x - M_t);
//              M = max_t M_t, S = sum_t S_t * exp_c(M_t - M) (left to right);
//              p_j = exp_c(x_j - M) * (1/S), the reciprocal rounded once;
//              non-finite logits weigh 0;
//   sampling: inverse CDF over tile sums, thread sums of the chosen tile,
//              then the thread's 16 elements, each scanned left to right.
//
// Four launches, each spread over the whole GPU:
//   1. tile_stats (one CTA per logits row x 4096-value tile): M_t and S_t;
//   2. decide (one CTA per sequence): M and S of the sequence's 2k+1 rows
//      from their tile statistics, the accept/reject decisions and the row
//      to sample from;
//   3. weights (one CTA per sequence x tile): the fixed-order thread partials
//      and tile sums of the sampling weights -- the residual max(p - q, 0)
//      and p itself (the fallback when the residual has no mass);
//   4. pick (one thread per sequence): the inverse-CDF scans.
// Every sum keeps the order stated above, so splitting the work over CTAs
// changes no result.
#include "common.cuh"

namespace b200 {
namespace spec {

constexpr int kThreads = 256;
constexpr int kTileElems = 4096;
constexpr int kMaxTiles = 48;  // vocab <= 196608
constexpr float kLog2e = 0x1.715476p+0f;
// 2^f on [-1/2, 1/2]: degree-5 relative-error fit with P(0) = 1 (max relative error 1.7e-7)
constexpr int kExpDeg = 5;
__device__ __constant__ float kExpCoef[kExpDeg + 1] = {0x1.0p+0f,       0x1.62e42ap-1f, 0x1.ebf9bcp-3f,
                                                       0x1.c6b752p-5f,  0x1.3cea88p-7f, 0x1.5bba14p-10f};

constexpr float kMagic = 12582912.f;  // 1.5 * 2^23: y + kMagic holds rint(y) in its low mantissa bits

__device__ __forceinline__ float exp_c(float x) {
    const float y = fminf(__fmul_rn(x, kLog2e), 0.f);
    const float t = __fadd_rn(y, kMagic);
    const float n = __fsub_rn(t, kMagic);
    const float f = __fsub_rn(y, n);
    float p = kExpCoef[kExpDeg];
#pragma unroll
    for (int k = kExpDeg - 1; k >= 0; --k) p = __fmaf_rn(p, f, kExpCoef[k]);
    // P in [0.7, 1.42] times 2^n, n in [-125, 0]: add n to the exponent field
    const uint32_t n_bits = __float_as_uint(t) - 0x4B400000u;
    const float r = __uint_as_float(__float_as_uint(p) + (n_bits << 23));
    return y < -125.f ? 0.f : r;
}

// exp_c of two values with packed f32x2 arithmetic: each lane of mul / add /
// fma .rn.f32x2 rounds exactly as the scalar instruction, so the results are
// bit-identical to exp_c and the issue slots are about halved.
__device__ __forceinline__ float2 exp_c2(float2 x) {
    float2 y = fmul2(x, make_float2(kLog2e, kLog2e));
    y.x = fminf(y.x, 0.f);
    y.y = fminf(y.y, 0.f);
    const float2 t = fadd2(y, make_float2(kMagic, kMagic));
    const float2 n = fadd2(t, make_float2(-kMagic, -kMagic));
    const float2 f = fadd2(y, make_float2(-n.x, -n.y));
    float2 p = make_float2(kExpCoef[kExpDeg], kExpCoef[kExpDeg]);
#pragma unroll
    for (int k = kExpDeg - 1; k >= 0; --k) p = ffma2(p, f, make_float2(kExpCoef[k], kExpCoef[k]));
    const float rx = __uint_as_float(__float_as_uint(p.x) + ((__float_as_uint(t.x) - 0x4B400000u) << 23));
    const float ry = __uint_as_float(__float_as_uint(p.y) + ((__float_as_uint(t.y) - 0x4B400000u) << 23));
    return make_float2(y.x < -125.f ? 0.f : rx, y.y < -125.f ? 0.f : ry);
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
// SCALED divides by the temperature (chosen once per CTA, not per value).
template <bool SCALED>
__device__ __forceinline__ void load_tile(const float* x, int V, int t, float T, bool vec, float (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int base = t * kTileElems + k * 1024 + 4 * int(threadIdx.x);
        if (vec && base + 3 < V) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(x + base));
            v[4 * k] = SCALED ? __fdiv_rn(f.x, T) : f.x;
            v[4 * k + 1] = SCALED ? __fdiv_rn(f.y, T) : f.y;
            v[4 * k + 2] = SCALED ? __fdiv_rn(f.z, T) : f.z;
            v[4 * k + 3] = SCALED ? __fdiv_rn(f.w, T) : f.w;
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float l = base + c < V ? __ldg(x + base + c) : -INFINITY;
                v[4 * k + c] = SCALED && base + c < V ? __fdiv_rn(l, T) : l;
            }
        }
    }
}

// One tile of one row: M_t = tile max and S_t = the fixed-order tile sum of
// exp_c(x - M_t) over the tile's finite values.
__global__ void __launch_bounds__(kThreads) tile_stats_kernel(Rows R, float2* tstats, int nt) {
    __shared__ float wred[kThreads / 32];
    const int row = blockIdx.x / nt, t = blockIdx.x - row * nt;
    int b;
    const float* x = row_ptr(R, row, &b);
    const float T = R.temps ? R.temps[b] : 0.f;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float v[16];
    if (T > 0.f)
        load_tile<true>(x, R.V, t, T, (R.V & 3) == 0, v);
    else
        load_tile<false>(x, R.V, t, T, (R.V & 3) == 0, v);
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < 16; ++e) m = fmaxf(m, v[e]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wred[warp] = m;
    __syncthreads();
    float Mt = wred[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) Mt = fmaxf(Mt, wred[w]);
    __syncthreads();
    float ex[16];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        const float2 r = exp_c2(fadd2(make_float2(v[e], v[e + 1]), make_float2(-Mt, -Mt)));
        ex[e] = r.x;
        ex[e + 1] = r.y;
    }
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e)
        if (isfinite(v[e])) acc = __fadd_rn(acc, ex[e]);
    const float ws = warp_butterfly(acc);
    if (lane == 0) wred[warp] = ws;
    __syncthreads();
    if (tid == 0) {
        float st = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) st = __fadd_rn(st, wred[w]);
        tstats[blockIdx.x] = make_float2(Mt, st);
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
    const float2* tstats;  // [rows][nt]
    const int32_t* draft;
    const float* ua;
    const float* us;
    int32_t* out_tokens;
    int32_t* out_num;
    int32_t nt;
};

// Per sequence: the row to sample from and its normalisers.
struct PickInfo {
    int32_t rej;
    float Mt, St, Md, Sd;
    int32_t pad[3];
};

// Weight of token j for the sampling row: p, and the residual max(p - q, 0).
// rt / rd are the once-rounded reciprocals of the rows' normalisers.
struct Weight {
    const float *xt, *xd;
    float T, Mt, rt, Md, rd;
    template <bool SCALED = true>
    __device__ __forceinline__ float p(float lt) const {
        return __fmul_rn(exp_c(__fsub_rn(SCALED ? scaled(lt, T) : lt, Mt)), rt);
    }
    template <bool SCALED = true>
    __device__ __forceinline__ float residual(float pv, float ld) const {
        const float q = __fmul_rn(exp_c(__fsub_rn(SCALED ? scaled(ld, T) : ld, Md)), rd);
        return fmaxf(__fsub_rn(pv, q), 0.f);
    }
};

// M and S of row `row` from its tile statistics (tiles left to right).
__device__ __forceinline__ float2 combine_row(const float2* ts, int nt) {
    float M = -INFINITY;
    for (int t = 0; t < nt; ++t) M = fmaxf(M, ts[t].x);
    float S = 0.f;
    for (int t = 0; t < nt; ++t) S = __fadd_rn(S, __fmul_rn(ts[t].y, exp_c(__fsub_rn(ts[t].x, M))));
    return make_float2(M, S);
}

constexpr int kDecideThreads = 128;  // >= 2 * 32 + 1 rows per sequence

__global__ void __launch_bounds__(kDecideThreads) decide_kernel(Decide d, PickInfo* info) {
    const Rows& R = d.R;
    const int b = blockIdx.x, k = R.k, V = R.V;
    const int rows_t = R.B * (k + 1);
    __shared__ float2 ms[2 * 32 + 1];  // target rows 0..k, then draft rows 0..k-1
    __shared__ int accept_s[32];
    const int r = threadIdx.x;
    if (r < 2 * k + 1) {
        const int row = r <= k ? b * (k + 1) + r : rows_t + b * k + (r - k - 1);
        ms[r] = combine_row(d.tstats + int64_t(row) * d.nt, d.nt);
    }
    __syncthreads();
    const float T = R.temps ? R.temps[b] : 0.f;
    // Draft position i's decision on thread i, then the first rejection in order.
    if (r < k) {
        const int x = d.draft[b * k + r];
        bool acc = false;
        if (x >= 0 && x < V) {
            const float2 st = ms[r], sd = ms[k + 1 + r];
            const float* xt = R.tl + (int64_t(b) * (k + 1) + r) * V;
            const float* xd = R.dl + (int64_t(b) * k + r) * V;
            const float p = __fmul_rn(exp_c(__fsub_rn(scaled(xt[x], T), st.x)), __frcp_rn(st.y));
            const float q = __fmul_rn(exp_c(__fsub_rn(scaled(xd[x], T), sd.x)), __frcp_rn(sd.y));
            acc = q > 0.f ? (d.ua[b * k + r] < fminf(1.f, __fdiv_rn(p, q))) : (p > 0.f);
        }
        accept_s[r] = acc;
    }
    __syncthreads();
    if (r == 0) {
        int rej = k;
        for (int i = 0; i < k; ++i)
            if (!accept_s[i]) {
                rej = i;
                break;
            }
        PickInfo pi;
        pi.rej = rej;
        pi.Mt = ms[rej].x;
        pi.St = ms[rej].y;
        pi.Md = rej < k ? ms[k + 1 + rej].x : 0.f;
        pi.Sd = rej < k ? ms[k + 1 + rej].y : 0.f;
        pi.pad[0] = pi.pad[1] = pi.pad[2] = 0;
        info[b] = pi;
        // accepted drafts and the padding; the sampled token at `rej` comes from pick_kernel
        for (int i = 0; i <= k; ++i)
            if (i != rej) d.out_tokens[b * (k + 1) + i] = i < rej ? d.draft[b * k + i] : -1;
        d.out_num[b] = rej + 1;
    }
}

__device__ __forceinline__ Weight make_weight(const Rows& R, const PickInfo& pi, int b) {
    Weight w;
    w.T = R.temps ? R.temps[b] : 0.f;
    w.xt = R.tl + (int64_t(b) * (R.k + 1) + pi.rej) * R.V;
    w.xd = pi.rej < R.k ? R.dl + (int64_t(b) * R.k + pi.rej) * R.V : nullptr;
    w.Mt = pi.Mt;
    w.rt = __frcp_rn(pi.St);
    w.Md = pi.Md;
    w.rd = pi.rej < R.k ? __frcp_rn(pi.Sd) : 0.f;
    return w;
}

// One tile of one sequence's sampling row: thread partials and tile sums of
// the residual (slot 0, when the sequence rejected a draft) and of p (slot 1).
// part [B][nt][2][256], tsum [B][nt][2].
template <bool SCALED>
__device__ __forceinline__ void weights_tile(const Rows& R, const PickInfo& pi, const Weight& w, int b, int t, int nt,
                                             float* part, float* tsum, float (&wred)[2][kThreads / 32]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = R.V;
    const bool res = pi.rej < R.k;
    const bool vec = (V & 3) == 0;
    float lt[16], ld[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int base = t * kTileElems + k * 1024 + 4 * tid;
        if (vec && base + 3 < V) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w.xt + base));
            lt[4 * k] = a.x, lt[4 * k + 1] = a.y, lt[4 * k + 2] = a.z, lt[4 * k + 3] = a.w;
            if (res) {
                const float4 c = __ldg(reinterpret_cast<const float4*>(w.xd + base));
                ld[4 * k] = c.x, ld[4 * k + 1] = c.y, ld[4 * k + 2] = c.z, ld[4 * k + 3] = c.w;
            }
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const bool in = base + c < V;
                lt[4 * k + c] = in ? __ldg(w.xt + base + c) : 0.f;
                if (res) ld[4 * k + c] = in ? __ldg(w.xd + base + c) : 0.f;
            }
        }
    }
    // p and q for pairs of values (packed f32x2, bit-identical to the scalar path), then the
    // fixed-order sums
    float pv[16], rv[16];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        float2 a = make_float2(lt[e], lt[e + 1]);
        if (SCALED) a = make_float2(scaled(a.x, w.T), scaled(a.y, w.T));
        const float2 pp2 = fmul2(exp_c2(fadd2(a, make_float2(-w.Mt, -w.Mt))), make_float2(w.rt, w.rt));
        pv[e] = pp2.x;
        pv[e + 1] = pp2.y;
        if (res) {
            float2 c = make_float2(ld[e], ld[e + 1]);
            if (SCALED) c = make_float2(scaled(c.x, w.T), scaled(c.y, w.T));
            const float2 q2 = fmul2(exp_c2(fadd2(c, make_float2(-w.Md, -w.Md))), make_float2(w.rd, w.rd));
            rv[e] = fmaxf(__fsub_rn(pp2.x, q2.x), 0.f);
            rv[e + 1] = fmaxf(__fsub_rn(pp2.y, q2.y), 0.f);
        }
    }
    float acc_r = 0.f, acc_p = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const int j = t * kTileElems + (e >> 2) * 1024 + 4 * tid + (e & 3);
        if (j < V) {
            acc_p = __fadd_rn(acc_p, pv[e]);
            if (res) acc_r = __fadd_rn(acc_r, rv[e]);
        }
    }
    float* pp = part + (int64_t(b) * nt + t) * 2 * kThreads;
    pp[tid] = acc_r;
    pp[kThreads + tid] = acc_p;
    const float wr = warp_butterfly(acc_r), wp = warp_butterfly(acc_p);
    if (lane == 0) {
        wred[0][warp] = wr;
        wred[1][warp] = wp;
    }
    __syncthreads();
    if (tid < 2) {
        float st = 0.f;
        for (int x = 0; x < kThreads / 32; ++x) st = __fadd_rn(st, wred[tid][x]);
        tsum[(int64_t(b) * nt + t) * 2 + tid] = st;
    }
}

__global__ void __launch_bounds__(kThreads) weights_kernel(Rows R, const PickInfo* info, int nt, float* part,
                                                           float* tsum) {
    __shared__ float wred[2][kThreads / 32];
    const int b = blockIdx.x / nt, t = blockIdx.x - b * nt;
    const PickInfo pi = info[b];
    const Weight w = make_weight(R, pi, b);
    if (w.T > 0.f)
        weights_tile<true>(R, pi, w, b, t, nt, part, tsum, wred);
    else
        weights_tile<false>(R, pi, w, b, t, nt, part, tsum, wred);
}

// Inverse-CDF pick over one slot's partials (one CTA of kThreads per
// sequence); -1 if that weight row has no mass.  The scans are the serial
// left-to-right ones of the definition, run by thread 0 over values staged in
// shared memory.
__device__ int pick_slot(const Weight& w, bool residual, int V, int nt, const float* part, const float* tsum, int slot,
                         float u, float* sh_t, float* sh_p, float* sh_w, int* sh_i) {
    const int tid = threadIdx.x;
    if (tid < nt) sh_t[tid] = tsum[tid * 2 + slot];
    __syncthreads();
    if (tid == 0) {
        float R = 0.f;
        for (int t = 0; t < nt; ++t) R = __fadd_rn(R, sh_t[t]);
        const float target = __fmul_rn(u, R);
        float acc;
        const int t = scan_pick(sh_t, nt, target, 0.f, &acc);
        sh_i[0] = t;
        sh_w[16] = target;
        sh_w[17] = acc;
    }
    __syncthreads();
    const int t = sh_i[0];
    if (t < 0) return -1;  // uniform: every thread read the same value
    sh_p[tid] = part[(t * 2 + slot) * kThreads + tid];
    __syncthreads();
    if (tid == 0) {
        float acc;
        sh_i[1] = scan_pick(sh_p, kThreads, sh_w[16], sh_w[17], &acc);
        sh_w[18] = acc;
    }
    __syncthreads();
    const int i = sh_i[1];
    if (i < 0) return -1;
    if (tid < 16) {
        const int j = t * kTileElems + (tid >> 2) * 1024 + 4 * i + (tid & 3);
        float wv = 0.f;
        if (j < V) {
            wv = w.p(__ldg(w.xt + j));
            if (residual) wv = w.residual(wv, __ldg(w.xd + j));
        }
        sh_w[tid] = wv;
    }
    __syncthreads();
    if (tid == 0) {
        float acc;
        const int e = scan_pick(sh_w, 16, sh_w[16], sh_w[18], &acc);
        sh_i[2] = e < 0 ? -1 : t * kTileElems + (e >> 2) * 1024 + 4 * i + (e & 3);
    }
    __syncthreads();
    const int r = sh_i[2];
    __syncthreads();  // the shared buffers may be reused by the next call
    return r;
}

__global__ void __launch_bounds__(kThreads) pick_kernel(Rows R, const PickInfo* info, int nt, const float* part,
                                                        const float* tsum, const float* us, int32_t* out_tokens) {
    __shared__ float sh_t[kMaxTiles], sh_p[kThreads], sh_w[20];
    __shared__ int sh_i[3];
    const int b = blockIdx.x;
    const PickInfo pi = info[b];
    const Weight w = make_weight(R, pi, b);
    const float* pb = part + int64_t(b) * nt * 2 * kThreads;
    const float* tb = tsum + int64_t(b) * nt * 2;
    const float u = us[b];
    int tok = -1;
    if (pi.rej < R.k) tok = pick_slot(w, true, R.V, nt, pb, tb, 0, u, sh_t, sh_p, sh_w, sh_i);
    if (tok < 0) tok = pick_slot(w, false, R.V, nt, pb, tb, 1, u, sh_t, sh_p, sh_w, sh_i);
    if (tok < 0) tok = 0;
    if (threadIdx.x == 0) out_tokens[b * (R.k + 1) + pi.rej] = tok;
}

// Workspace carve-up (each part 256-byte aligned).
struct Layout {
    size_t tstats, info, part, tsum, total;
};
__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline Layout layout(int32_t batch, int32_t num_draft, int32_t vocab) {
    const size_t nt = (size_t(vocab) + kTileElems - 1) / kTileElems;
    const size_t rows = size_t(batch) * (2 * size_t(num_draft) + 1);
    Layout L;
    L.tstats = 0;
    L.info = L.tstats + align256(rows * nt * sizeof(float2));
    L.part = L.info + align256(size_t(batch) * sizeof(PickInfo));
    L.tsum = L.part + align256(size_t(batch) * nt * 2 * kThreads * sizeof(float));
    L.total = L.tsum + align256(size_t(batch) * nt * 2 * sizeof(float));
    return L;
}

}  // namespace spec
}  // namespace b200

extern "C" size_t b200_spec_accept_workspace_size(int32_t batch, int32_t num_draft, int32_t vocab_size) {
    if (batch < 0 || num_draft < 0 || vocab_size <= 0) return 0;
    return b200::spec::layout(batch, num_draft, vocab_size).total;
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
    const Layout L = layout(batch, num_draft, vocab_size);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float2* tstats = reinterpret_cast<float2*>(ws + L.tstats);
    PickInfo* info = reinterpret_cast<PickInfo*>(ws + L.info);
    float* part = reinterpret_cast<float*>(ws + L.part);
    float* tsum = reinterpret_cast<float*>(ws + L.tsum);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int nt = (vocab_size + kTileElems - 1) / kTileElems;
    const int nrows = batch * (2 * num_draft + 1);
    tile_stats_kernel<<<nrows * nt, kThreads, 0, s>>>(R, tstats, nt);
    B200_CUDA_TRY(cudaGetLastError());
    Decide d{R, tstats, draft_tokens, uniform_accept, uniform_sample, out_tokens, out_num_tokens, nt};
    decide_kernel<<<batch, kDecideThreads, 0, s>>>(d, info);
    B200_CUDA_TRY(cudaGetLastError());
    weights_kernel<<<batch * nt, kThreads, 0, s>>>(R, info, nt, part, tsum);
    B200_CUDA_TRY(cudaGetLastError());
    pick_kernel<<<batch, kThreads, 0, s>>>(R, info, nt, part, tsum, uniform_sample, out_tokens);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
