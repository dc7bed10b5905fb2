// Causal varlen prefill attention on the 5th-generation tensor cores
// (tcgen05 + tensor memory).  Replaces the flash_attn_varlen_func call of
// nanovllm/layers/attention.py:64-70, with or without a block table (prefix
// caching / chunked prefill reads keys from the paged cache).
//
// One CTA computes two 128-query tiles (A = rows 0-127, B = rows 128-255 of
// a 256-row block) of one query head; both share every K/V tile.  Warp roles:
//   warp 0    producer: TMA loads (no multicast) of both Q tiles once and of
//             128-key K and V tiles into a 2-stage ring (64 KiB per stage),
//             all as 64-dim x 128-row boxes with 128-byte swizzle;
//   warp 1    MMA issuer (one thread) and tensor-memory owner;
//   warps 2-5 softmax of tile A, warps 6-9 softmax of tile B: one thread per
//             query row (TMEM lane = row).
// Tensor memory: S_A cols 0-127, S_B 128-255, O_A 256-383, O_B 384-511.  The
// MMA order per key tile j is PV_A(j-1) S_A(j) PV_B(j-1) S_B(j) (ping-pong):
// while one warpgroup turns S(j) into P(j), the tensor core works on the
// other tile.  S = Q K^T is an SS MMA (M = N = 128, K-major operands); the
// softmax writes P as bf16 over its S columns and O += P V reads P from
// tensor memory (TS MMA) with V as an MN-major operand.  The softmax is two
// passes over its TMEM row (max, then exp / pack / store by 32-column chunk)
// and rescales its O row in tensor memory only when the running max grew by
// more than 2^8 (lazy rescaling; the sum uses the same stale max, so the
// result is exact).
#include "common.cuh"
#include "tcgen05.cuh"

namespace b200 {
namespace pf {

constexpr int kBM = 128;  // queries per tile (two tiles per CTA)
constexpr int kBN = 128;  // keys per tile
constexpr int kD = 128;
constexpr int kHalf = kBM * 128;  // one 64-dim half of a 128-row tile: 16 KiB
constexpr int kStages = 2;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;

struct Params {
    uint16_t* out;
    int64_t out_stride;  // elements between query rows of out
    const int32_t* cu_q;
    const int32_t* cu_k;
    const int32_t* block_tables;
    int32_t bt_stride, block_size, num_blocks;
    int32_t num_seqs, hq, hkv, group, q_blocks;
    float scale_log2;
};

struct Smem {
    uint8_t q[2][2][kHalf];         // [tile A/B][dim half]
    uint8_t kv[kStages][4][kHalf];  // K lo, K hi, V lo, V hi
    uint64_t q_full;
    uint64_t kv_full[kStages], kv_empty[kStages];
    uint64_t s_full[2], p_ready[2], o_done[2];  // per tile A/B
    uint64_t drain;
    uint32_t tmem_base;
    int32_t err;
};

__device__ int32_t g_prefill_error;  // bounded waits that gave up (diagnostics)

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, Smem& sm) {
    if (mbar_wait(bar, parity)) return true;
    atomicOr(&g_prefill_error, 1);
    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
    return false;
}

// Number of 128-key tiles that rows [r0, r1) of a sequence (lq queries, lk keys) may see.
__device__ __forceinline__ int key_tiles(int r0, int r1, int lq, int lk) {
    if (r0 >= lq) return 0;
    const int last = min(r1, lq) - 1;
    const int nkeys = max(0, min(lk, last + (lk - lq) + 1));
    return (nkeys + kBN - 1) / kBN;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int h = blockIdx.x;
    const int blk_q = p.q_blocks - 1 - int(blockIdx.y);  // longest (latest) rows first
    const int s = blockIdx.z;
    const int q0 = p.cu_q[s], lq = p.cu_q[s + 1] - q0;
    const int k0 = p.cu_k[s], lk = p.cu_k[s + 1] - k0;
    const int row0 = blk_q * 2 * kBM;
    if (row0 >= lq) return;  // uniform across the CTA
    const int nt[2] = {key_tiles(row0, row0 + kBM, lq, lk), key_tiles(row0 + kBM, row0 + 2 * kBM, lq, lk)};
    const int ntiles = max(nt[0], nt[1]);
    const bool has_b = row0 + kBM < lq;
    const int kvh = h / p.group;

    if (ntiles == 0) {  // no visible key for any row: zero output
        const int rows = min(2 * kBM, lq - row0);
        for (int i = tid; i < rows * (kD / 8); i += kThreads) {
            const int r = row0 + i / (kD / 8), c = i % (kD / 8);
            reinterpret_cast<uint4*>(p.out + int64_t(q0 + r) * p.out_stride + h * kD)[c] = make_uint4(0, 0, 0, 0);
        }
        return;
    }

    if (tid == 0) {
        mbar_init(&sm.q_full, 1);
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&sm.kv_full[i], 1);
            mbar_init(&sm.kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.p_ready[i], 128);
            mbar_init(&sm.o_done[i], 1);
        }
        mbar_init(&sm.drain, 1);
        sm.err = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&sm.tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&tmq);
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
            const uint64_t pol_q = l2_policy_evict_first();
            const uint64_t pol_kv = l2_policy_evict_last();  // K/V tiles are re-read by the group's q heads
            mbar_arrive_expect_tx(&sm.q_full, (has_b ? 4 : 2) * kHalf);
            for (int t = 0; t < (has_b ? 2 : 1); ++t) {
                tma_load_2d(sm.q[t][0], &tmq, h * kD, q0 + row0 + t * kBM, &sm.q_full, pol_q);
                tma_load_2d(sm.q[t][1], &tmq, h * kD + 64, q0 + row0 + t * kBM, &sm.q_full, pol_q);
            }
            const int32_t* bt = p.block_tables ? p.block_tables + int64_t(s) * p.bt_stride : nullptr;
            int filled = 0;
            for (int j = 0; j < ntiles; ++j) {
                const int st = j % kStages;
                if (*reinterpret_cast<volatile int32_t*>(&sm.err) ||
                    !wait_or_flag(&sm.kv_empty[st], ((j / kStages) & 1) ^ 1, sm))
                    break;
                int y;
                if (bt) {
                    const int pos = j * kBN;
                    const int lb = pos / p.block_size;
                    const int blk = lb < p.bt_stride ? bt[lb] : -1;
                    y = (blk >= 0 && blk < p.num_blocks) ? blk * p.block_size + (pos - lb * p.block_size)
                                                         : p.num_blocks * p.block_size;
                } else {
                    y = k0 + j * kBN;
                }
                mbar_arrive_expect_tx(&sm.kv_full[st], 4 * kHalf);
                const int x = kvh * kD;
                tma_load_2d(sm.kv[st][0], &tmk, x, y, &sm.kv_full[st], pol_kv);
                tma_load_2d(sm.kv[st][1], &tmk, x + 64, y, &sm.kv_full[st], pol_kv);
                tma_load_2d(sm.kv[st][2], &tmv, x, y, &sm.kv_full[st], pol_kv);
                tma_load_2d(sm.kv[st][3], &tmv, x + 64, y, &sm.kv_full[st], pol_kv);
                ++filled;
            }
            // Before the CTA exits, every load issued into its shared memory must have
            // landed (always true on the normal path; bounded wait on error paths).
            mbar_wait(&sm.q_full, 0);
            for (int st = 0; st < kStages && st < filled; ++st) {
                const int last = st + ((filled - 1 - st) / kStages) * kStages;
                mbar_wait(&sm.kv_full[st], (last / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_f16<BF16>(kBM, kBN, false, false);
            constexpr uint32_t idPV = tc::idesc_f16<BF16>(kBM, kD, false, true);
            bool ok = wait_or_flag(&sm.q_full, 0, sm);
            tc::fence_after_sync();
            auto issue_s = [&](int t, int j) {
                const uint32_t qa = smem_u32(sm.q[t][0]);
                const uint32_t ka = smem_u32(sm.kv[j % kStages][0]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    // K-major operands: 16 dims = 32 bytes inside a 128-byte swizzled row
                    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
                    tc::mma_ss(tmem + t * 128, tc::smem_desc_sw128(qa + off, 16, 1024),
                               tc::smem_desc_sw128(ka + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
                }
                tc::commit(&sm.s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                if (!wait_or_flag(&sm.p_ready[t], j & 1, sm)) return false;
                tc::fence_after_sync();
                const uint32_t va = smem_u32(sm.kv[j % kStages][2]);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    // V is MN-major: 16 keys = two 8-row swizzle atoms (SBO 1024 B); the
                    // second 64 dims live in the V-hi half (LBO = kHalf).
                    tc::mma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                               tc::smem_desc_sw128(va + kk * 16 * 128, kHalf, 1024), idPV,
                               (j > 0 || kk > 0) ? 1u : 0u);
                }
                tc::commit(&sm.o_done[t]);
                return true;
            };
            for (int j = 0; ok && j < ntiles; ++j) {
                if (!wait_or_flag(&sm.kv_full[j % kStages], (j / kStages) & 1, sm)) { ok = false; break; }
                tc::fence_after_sync();
                // tile A: PV(j-1) frees S_A before S_A(j) overwrites it (in-order tensor pipe)
                if (j < nt[0]) {
                    if (j > 0 && !issue_pv(0, j - 1)) { ok = false; break; }
                    issue_s(0, j);
                } else if (j == nt[0] && j > 0) {
                    if (!issue_pv(0, j - 1)) { ok = false; break; }
                }
                if (j < nt[1]) {
                    if (j > 0 && !issue_pv(1, j - 1)) { ok = false; break; }
                    issue_s(1, j);
                }
                if (j > 0) tc::commit(&sm.kv_empty[(j - 1) % kStages]);  // both PVs of tile j-1 issued
            }
            if (ok) {
                if (nt[0] == ntiles) ok = issue_pv(0, ntiles - 1);
                if (ok && nt[1] == ntiles) ok = issue_pv(1, ntiles - 1);
                tc::commit(&sm.kv_empty[(ntiles - 1) % kStages]);
            }
            // Wait (bounded) for every MMA issued above before the tensor memory is freed.
            tc::commit(&sm.drain);
            mbar_wait(&sm.drain, 0);
        }
    } else {
        // ------------------------------------------------------------ softmax / epilogue
        const int t = warp >= 6 ? 1 : 0;  // query tile of this warpgroup
        const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31 belong to this warp
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
        const uint32_t s_col = tmem + lane_addr + t * 128;
        const uint32_t o_col = tmem + lane_addr + 256 + t * 128;
        const int qrow = row0 + t * kBM + r;
        const int limit = qrow < lq ? qrow + (lk - lq) : -1;  // last visible key of this row
        const float sl2 = p.scale_log2;
        const int my_tiles = nt[t];
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < my_tiles; ++j) {
            if (!wait_or_flag(&sm.s_full[t], j & 1, sm)) { ok = false; break; }
            tc::fence_after_sync();
            const int kbase = j * kBN;
            const bool full_row = kbase + kBN - 1 <= limit;  // no masking needed in this tile
            // pass 1: row max
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                tc::tmem_ld32(s_col + c * 32, v);
                tc::tmem_wait_ld();
                float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float x = (full_row || kbase + c * 32 + e <= limit) ? v[e] : -INFINITY;
                    m4[e & 3] = fmaxf(m4[e & 3], x);
                }
                mx = fmaxf(mx, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
            }
            // Lazy rescale: keep the old max unless the new one exceeds it by 2^8.
            float alpha = 1.f;
            bool rescale = false;
            if (mx != -INFINITY && (m == -INFINITY || (mx - m) * sl2 > kRescaleLog2)) {
                alpha = m == -INFINITY ? 0.f : fast_exp2((m - mx) * sl2);
                rescale = m != -INFINITY;
                m = mx;
            }
            const float msl = m == -INFINITY ? 0.f : m * sl2;
            // pass 2: P = exp2(S*scale - m) as bf16 over the S columns, row sum
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                tc::tmem_ld32(s_col + c * 32, v);
                tc::tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const bool in0 = full_row || kbase + c * 32 + e <= limit;
                    const bool in1 = full_row || kbase + c * 32 + e + 1 <= limit;
                    const float a = in0 ? fast_exp2(fmaf(v[e], sl2, -msl)) : 0.f;
                    const float b = in1 ? fast_exp2(fmaf(v[e + 1], sl2, -msl)) : 0.f;
                    sum4[(e >> 1) & 3] += a + b;
                    pk[e / 2] = pack2<BF16>(a, b);
                }
                // P chunk c (32 keys) occupies 16 TMEM columns at s_col + 16c
                tc::tmem_st16(s_col + c * 16, pk);
            }
            l = fmaf(l, alpha, (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            if (rescale && j > 0) {
                // O must hold PV(j-1) before it is scaled.
                if (!wait_or_flag(&sm.o_done[t], (j - 1) & 1, sm)) { ok = false; break; }
                tc::fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < kD / 32; ++c) {
                    float o[32];
                    tc::tmem_ld32(o_col + c * 32, o);
                    tc::tmem_wait_ld();
                    uint32_t u[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(o[e] * alpha);
                    tc::tmem_st32(o_col + c * 32, u);
                }
            }
            tc::tmem_wait_st();
            // Cache rows past this sequence's keys may hold NaN bits; P is 0 there but
            // 0 * NaN is NaN, so the first tile to use the stage clears those V rows.
            if (kbase + kBN > lk && (t == 0 || j >= nt[0])) {
                if (kbase + r >= lk) {
                    uint4* v0 = reinterpret_cast<uint4*>(sm.kv[j % kStages][2] + r * 128);
                    uint4* v1 = reinterpret_cast<uint4*>(sm.kv[j % kStages][3] + r * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) v0[c] = v1[c] = make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();
            }
            tc::fence_before_sync();
            mbar_arrive(&sm.p_ready[t]);
        }
        // ---- epilogue: O / l -> bf16, one query row per thread ----
        if (ok && my_tiles > 0 && wait_or_flag(&sm.o_done[t], (my_tiles - 1) & 1, sm)) {
            tc::fence_after_sync();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            uint4* dst = reinterpret_cast<uint4*>(p.out + int64_t(q0 + qrow) * p.out_stride + h * kD);
#pragma unroll 1
            for (int c = 0; c < kD / 32; ++c) {
                float o[32];
                tc::tmem_ld32(o_col + c * 32, o);
                tc::tmem_wait_ld();
                if (qrow < lq) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 w;
                        w.x = pack2<BF16>(o[e] * inv, o[e + 1] * inv);
                        w.y = pack2<BF16>(o[e + 2] * inv, o[e + 3] * inv);
                        w.z = pack2<BF16>(o[e + 4] * inv, o[e + 5] * inv);
                        w.w = pack2<BF16>(o[e + 6] * inv, o[e + 7] * inv);
                        dst[(c * 32 + e) / 8] = w;
                    }
                }
            }
        } else if (my_tiles == 0 && qrow < lq) {
            // rows of tile B that see no key (possible only when lk < lq)
            uint4* dst = reinterpret_cast<uint4*>(p.out + int64_t(q0 + qrow) * p.out_stride + h * kD);
            for (int c = 0; c < kD / 8; ++c) dst[c] = make_uint4(0, 0, 0, 0);
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace pf
}  // namespace b200

extern "C" int32_t b200_varlen_prefill(void* out, const void* q, int64_t q_stride_token, const void* k,
                                       int64_t k_stride_token, const void* v, int64_t v_stride_token,
                                       const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs,
                                       int32_t total_q, int32_t max_seqlen_q, int32_t max_seqlen_k,
                                       int32_t total_k_rows,
                                       const int32_t* block_tables, int32_t block_table_stride, int32_t block_size,
                                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                       int32_t dtype, void* stream) {
    using namespace b200;
    using namespace b200::pf;
    clear_error();
    B200_REQUIRE(num_seqs >= 0 && max_seqlen_q >= 0, "varlen_prefill: negative sizes");
    if (num_seqs == 0 || max_seqlen_q == 0) return B200_OK;
    B200_REQUIRE(out && q && k && v && cu_seqlens_q && cu_seqlens_k, "varlen_prefill: null pointer");
    B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
                 "varlen_prefill: num_heads %d not a multiple of num_kv_heads %d", num_heads, num_kv_heads);
    if (head_dim != kD) return fail(B200_ERR_UNSUPPORTED, "varlen_prefill: head_dim %d (only 128)", head_dim);
    if (dtype != B200_BF16 && dtype != B200_F16)
        return fail(B200_ERR_UNSUPPORTED, "varlen_prefill: dtype %d (bf16 or fp16 only)", dtype);
    B200_REQUIRE(total_k_rows > 0 && total_q > 0, "varlen_prefill: total_q %d / total_k_rows %d", total_q,
                 total_k_rows);
    B200_REQUIRE(q_stride_token >= int64_t(num_heads) * kD && k_stride_token >= int64_t(num_kv_heads) * kD &&
                     v_stride_token >= int64_t(num_kv_heads) * kD,
                 "varlen_prefill: token strides below the head rows");
    B200_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, "varlen_prefill: out must be 16-byte aligned");
    if (block_tables) {
        B200_REQUIRE(block_size > 0 && block_size % kBN == 0, "varlen_prefill: block_size %d not a multiple of %d",
                     block_size, kBN);
        B200_REQUIRE(block_table_stride > 0, "varlen_prefill: block_table_stride %d", block_table_stride);
        B200_REQUIRE(total_k_rows % block_size == 0, "varlen_prefill: cache rows %d not whole blocks", total_k_rows);
    }
    const int q_blocks = (max_seqlen_q + 2 * kBM - 1) / (2 * kBM);
    if (q_blocks > 65535 || num_seqs > 65535)
        return fail(B200_ERR_UNSUPPORTED, "varlen_prefill: %d query blocks x %d sequences", q_blocks, num_seqs);
    const bool bf16 = dtype == B200_BF16;
    // The tensor maps span exactly the caller's q / k / v rows, so a tile that
    // runs past the last token reads the TMA fill value (zero), never memory
    // outside the buffers; such rows are masked and never stored.
    CUtensorMap tmq, tmk, tmv;
    const uint64_t q_rows = uint64_t(total_q);
    int32_t rc = make_tmap_2d(&tmq, q, uint64_t(num_heads) * kD, q_rows, uint64_t(q_stride_token) * 2, 64, kBM, bf16,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tmk, k, uint64_t(num_kv_heads) * kD, uint64_t(total_k_rows), uint64_t(k_stride_token) * 2, 64,
                      kBN, bf16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tmv, v, uint64_t(num_kv_heads) * kD, uint64_t(total_k_rows), uint64_t(v_stride_token) * 2, 64,
                      kBN, bf16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;

    Params prm;
    prm.out = static_cast<uint16_t*>(out);
    prm.out_stride = int64_t(num_heads) * kD;
    prm.cu_q = cu_seqlens_q;
    prm.cu_k = cu_seqlens_k;
    prm.block_tables = block_tables;
    prm.bt_stride = block_table_stride;
    prm.block_size = block_tables ? block_size : 0;
    prm.num_blocks = block_tables ? total_k_rows / block_size : 0;
    prm.num_seqs = num_seqs;
    prm.hq = num_heads;
    prm.hkv = num_kv_heads;
    prm.group = num_heads / num_kv_heads;
    prm.q_blocks = q_blocks;
    prm.scale_log2 = softmax_scale * 1.4426950408889634f;

    const int smem = int(sizeof(Smem)) + 1024;
    const void* fn = bf16 ? (const void*)prefill_kernel<true> : (const void*)prefill_kernel<false>;
    ensure_smem_attr(fn, smem);
    const dim3 grid(num_heads, q_blocks, num_seqs);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (bf16) prefill_kernel<true><<<grid, kThreads, smem, st>>>(prm, tmq, tmk, tmv);
    else prefill_kernel<false><<<grid, kThreads, smem, st>>>(prm, tmq, tmk, tmv);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

extern "C" int32_t b200_varlen_prefill_error(void* stream, int32_t* flag) {
    using namespace b200;
    B200_REQUIRE(flag != nullptr, "varlen_prefill_error: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    B200_CUDA_TRY(cudaStreamSynchronize(s));
    B200_CUDA_TRY(cudaMemcpyFromSymbol(flag, b200::pf::g_prefill_error, sizeof(int32_t)));
    return B200_OK;
}
