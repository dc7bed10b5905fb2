// Causal varlen prefill attention on the 5th-generation tensor cores
// (tcgen05 + tensor memory).  Replaces the flash_attn_varlen_func call of
// nanovllm/layers/attention.py:64-70, with or without a block table (prefix
// caching / chunked prefill reads keys from the paged cache).
//
// Persistent CTAs (one per SM) walk work units -- two 128-row query tiles A
// and B that read the same K/V tiles.  When the GQA group is even a unit is
// 128 query positions of a pair of query heads of one kv head, and each tile
// holds 64 positions of both heads (rows 0-63 the first head, 64-127 the
// second): both heads see the same keys, so a sequence's last, partial block
// of positions fills whole rows of both heads and the diagonal tiles are
// narrower, which saves 8 % of the tensor work of a prefix-cached prefill
// batch against one head per tile.  Otherwise a unit is rows r and r + 128
// of one head.
// Units are numbered heaviest first and claimed dynamically: the producer
// takes the next number from an atomic counter in the caller's workspace
// whenever it is ready for a new unit (numbers past a sequence's queries are
// skipped) and hands it to the other roles through a two-slot unit ring in
// shared memory; the last CTA to finish re-arms the counter, so the call is
// CUDA-graph capturable.  Dynamic claiming keeps the SMs evenly loaded where a
// static assignment left a quarter of their time idle.  Tensor memory is
// allocated once; the K/V rings and every barrier phase run on across units.
// Warp roles (three warpgroups):
//   warps 0-3 / 4-7  softmax of tile A / B, one thread per query row (TMEM
//             lane = row), and the epilogue O / l -> out;
//   warp 8    producer: TMA loads (no multicast) of both Q tiles and of
//             128-key K tiles (3-stage ring) and V tiles (2-stage ring), all
//             64-dim x 128-row boxes with 128-byte swizzle; lane 0 Q and K,
//             lane 1 V;
//   warp 9    S issuer (one thread): S = Q K^T, SS MMA, M = N = 128;
//   warp 10   PV issuer (one thread): O += P V, TS MMA with P from tensor
//             memory and V as an MN-major operand.
// Tensor memory: one S buffer (cols 0-127) shared by both tiles, P_A / P_B
// (bf16 pairs, cols 128-191 / 192-255), O_A / O_B (cols 256-383 / 384-511).
// A softmax warpgroup loads its 128 scores per row into registers and frees
// the S buffer at once, so the S MMA of the other tile runs while it computes
// P; it then waits for its previous PV (P and O free), rescales O when the
// running max grew by more than 2^8 (lazy rescaling: the sum uses the same
// stale max, so the result is exact), and writes P.  The S and PV streams
// share no tensor memory, so the two issuers never wait on each other, and
// two issuing threads keep the tensor pipe busy where one cannot.
#include <climits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace b200 {
namespace pf {

constexpr int kBM = 128;  // queries per tile (two tiles per CTA)
constexpr int kBN = 128;  // keys per tile
constexpr int kD = 128;
constexpr int kHalf = kBM * 128;  // one 64-dim half of a 128-row tile: 16 KiB
constexpr int kKStages = 3;  // K tiles are released after S, so they can run further ahead
constexpr int kVStages = 2;  // V tiles are released after PV
// Warpgroups: 0 = softmax of tile A, 1 = softmax of tile B, 2 = control
// (warp 8 producer, warp 9 S issuer, warp 10 PV issuer, warp 11 idle).  setmaxnreg moves
// registers from the control warpgroup to the softmax warpgroups; the split
// must fit the block's launch allocation: 2*128*kRegsSoftmax + 128*kRegsControl
// <= kThreads * 168.
constexpr int kThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kRegsSoftmax = 216;
constexpr uint32_t kRegsControl = 64;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl <= kThreads * 168, "register split exceeds the launch allocation");
constexpr uint32_t kTmemCols = 512;
// Tensor memory columns: one S buffer shared by both tiles (f32, 128 keys),
// P of tile t (bf16 pairs, 64 columns) and O of tile t (f32, 128 dims).
constexpr uint32_t kColS = 0;
constexpr uint32_t kColP = 128;  // + 64 * t
constexpr uint32_t kColO = 256;  // + 128 * t
constexpr float kRescaleLog2 = 8.0f;
constexpr int kUnitRing = 2;  // claimed units in flight between the producer and the other roles
// Readers of each unit-ring slot: the V loader lane, the two MMA issuers, the eight softmax warps.
constexpr int kUnitReaders = 1 + 2 + 8;
constexpr size_t kWorkspaceBytes = 256;  // [0] next unit, [1] finished CTAs

struct Params {
    uint16_t* out;
    int64_t out_stride;  // elements between query rows of out
    const int32_t* cu_q;
    const int32_t* cu_k;
    const int32_t* block_tables;
    int32_t bt_stride, block_size, num_blocks;
    int32_t num_seqs, hq, hkv, group, q_blocks;
    int32_t pair;   // 1: tile A/B = positions 0-63 / 64-127 of a unit's block, each for two query heads of one
                    //    kv head (even group; rows 0-63 the first head, 64-127 the second); 0: rows r / r+128 of one head
    int32_t slots;  // head slots per sequence: hq / 2 when pairing, else hq
    float scale_log2;
    int32_t* sched;  // caller workspace: [0] next unit to claim, [1] CTAs finished
};

struct Smem {
    uint8_t q[2][2][kHalf];          // [tile A/B][dim half]
    uint8_t k[kKStages][2][kHalf];   // [stage][dim half]
    uint8_t v[kVStages][2][kHalf];
    uint64_t q_full, q_empty;
    uint64_t k_full[kKStages], k_empty[kKStages];
    uint64_t v_full[kVStages], v_empty[kVStages];
    uint64_t s_full[2], p_ready[2], o_done[2];  // per tile A/B
    uint64_t s_free;                            // the S buffer has been read (one phase per S tile)
    uint64_t drain;
    uint64_t unit_full[kUnitRing], unit_empty[kUnitRing];
    int32_t unit_ring[kUnitRing];               // claimed unit numbers, -1 = no more units
    uint32_t tmem_base;
    int32_t err;
};

__device__ int32_t g_prefill_error;  // bounded waits that gave up (diagnostics)

template <bool SPIN = false>
__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, Smem& sm) {
    if (SPIN ? mbar_wait_spin(bar, parity) : mbar_wait(bar, parity)) return true;
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

// One work unit: two 128-row query tiles A and B of one sequence that read the
// same K/V tiles -- positions row[t] .. row[t] + 63 of the heads h[t] and
// h[t] + 1 of one kv head when the group is even, else positions row[t] ..
// row[t] + 127 of head h[t].
// Per-tile fields are scalars with select accessors (no arrays), so that a
// runtime tile index never forces the unit into local memory.
struct Unit {
    int s, q0, lq, k0, lk, h0, h1, row0, row1, nt0, nt1, ntiles;
    bool has_b;
    __device__ __forceinline__ int h(int t) const { return t ? h1 : h0; }
    __device__ __forceinline__ int row(int t) const { return t ? row1 : row0; }
    __device__ __forceinline__ int nt(int t) const { return t ? nt1 : nt0; }
};

// Units are numbered heaviest first (later query blocks see more keys), then by
// sequence and head; returns false for blocks past the sequence's queries.
__device__ __forceinline__ bool load_unit(const Params& p, int u, Unit& w) {
    const int per = p.num_seqs * p.slots;
    const int qb = p.q_blocks - 1 - u / per;
    const int rem = u - (u / per) * per;
    w.s = rem / p.slots;
    const int hs = rem - w.s * p.slots;
    int span;  // query positions per tile
    if (p.pair) {
        w.h0 = w.h1 = 2 * hs;  // first head of the pair; rows 64-127 of a tile are head 2 * hs + 1
        w.row0 = qb * kBM;
        w.row1 = w.row0 + kBM / 2;
        span = kBM / 2;
    } else {
        w.h0 = w.h1 = hs;
        w.row0 = qb * 2 * kBM;
        w.row1 = w.row0 + kBM;
        span = kBM;
    }
    w.q0 = p.cu_q[w.s];
    w.lq = p.cu_q[w.s + 1] - w.q0;
    if (w.row0 >= w.lq) return false;
    w.k0 = p.cu_k[w.s];
    w.lk = p.cu_k[w.s + 1] - w.k0;
    w.nt0 = key_tiles(w.row0, w.row0 + span, w.lq, w.lk);
    w.nt1 = key_tiles(w.row1, w.row1 + span, w.lq, w.lk);
    w.ntiles = max(w.nt0, w.nt1);
    w.has_b = w.row1 < w.lq;
    return true;
}

// One row's share of a key tile: its 128 scores are read from the S buffer
// into registers (the buffer is released at once), the max is taken, the
// running max m is updated lazily (only when it grows by > 2^8), and
// P = 2^(S*scale - m) is packed to bf16 pairs in pk for the caller to store.
// `mask` applies the bottom-right causal / sequence-end masking (diagonal and
// tail tiles only).
// The next claimed unit from the ring (n counts the units this role has
// taken); -1 when there are no more, -2 when the wait ran out.  Called by one
// thread of a role, or by a whole warp (then every lane reads and lane 0
// releases the slot after the warp has read it).
__device__ __forceinline__ int take_unit(Smem& sm, int& n, bool warp_reader) {
    const int slot = n % kUnitRing;
    const uint32_t parity = (n / kUnitRing) & 1;
    bool ok = mbar_wait(&sm.unit_full[slot], parity);
    if (warp_reader) ok = __all_sync(0xffffffffu, ok);
    if (!ok) return -2;
    const int u = *reinterpret_cast<volatile int32_t*>(&sm.unit_ring[slot]);
    if (warp_reader) __syncwarp();
    if (!warp_reader || (threadIdx.x & 31) == 0) mbar_arrive(&sm.unit_empty[slot]);
    ++n;
    return u;
}

template <bool BF16>
__device__ __forceinline__ void softmax_tile(bool mask, uint32_t s_col, uint64_t* s_free, int kbase, int limit,
                                             float sl2, float& m, float& alpha, bool& rescale, float& sum,
                                             uint32_t (&pk)[kBN / 2]) {
    // All 128 scores of the row in registers; the S buffer is released at once
    // so that the next S tile (of either query tile) can be computed into it.
    float v[kBN];
#pragma unroll
    for (int c = 0; c < kBN / 32; ++c) tc::tmem_ld32(s_col + c * 32, *reinterpret_cast<float(*)[32]>(&v[c * 32]));
    tc::tmem_wait_ld();
    tc::fence_before_sync();
    mbar_arrive(s_free);
    if (mask) {
#pragma unroll
        for (int e = 0; e < kBN; ++e)
            if (kbase + e > limit) v[e] = -INFINITY;
    }
    // four chains of three-input max over the row
    float m4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
    for (int e = 4; e < kBN - 4; e += 8)
#pragma unroll
        for (int c = 0; c < 4; ++c) m4[c] = max3f(m4[c], v[e + 2 * c], v[e + 2 * c + 1]);
    const float mx =
        max3f(max3f(m4[0], m4[1], v[kBN - 4]), max3f(m4[2], m4[3], v[kBN - 3]), fmaxf(v[kBN - 2], v[kBN - 1]));
    alpha = 1.f;
    rescale = false;
    if (mx != -INFINITY && (m == -INFINITY || (mx - m) * sl2 > kRescaleLog2)) {
        alpha = m == -INFINITY ? 0.f : fast_exp2((m - mx) * sl2);
        rescale = m != -INFINITY;
        m = mx;
    }
    const float msl = m == -INFINITY ? 0.f : m * sl2;
    // pairs of scores through packed fma / add (half the issue slots of scalar code)
    float2 s2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const float2 sl22 = make_float2(sl2, sl2), nmsl = make_float2(-msl, -msl);
#pragma unroll
    for (int e = 0; e < kBN; e += 2) {
        const float2 x = ffma2(make_float2(v[e], v[e + 1]), sl22, nmsl);
        // masked scores are -inf, and ex2 of -inf is +0
        const float2 y = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        s2[(e >> 1) & 3] = fadd2(s2[(e >> 1) & 3], y);
        pk[e / 2] = pack2<BF16>(y.x, y.y);
    }
    const float2 st = fadd2(fadd2(s2[0], s2[1]), fadd2(s2[2], s2[3]));
    sum = st.x + st.y;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int total_units = p.q_blocks * p.num_seqs * p.slots;

    if (tid == 0) {
        for (int i = 0; i < kUnitRing; ++i) {
            mbar_init(&sm.unit_full[i], 1);
            mbar_init(&sm.unit_empty[i], kUnitReaders);
        }
        mbar_init(&sm.q_full, 1);
        mbar_init(&sm.q_empty, 1);
        for (int i = 0; i < kKStages; ++i) {
            mbar_init(&sm.k_full[i], 1);
            mbar_init(&sm.k_empty[i], 1);
        }
        for (int i = 0; i < kVStages; ++i) {
            mbar_init(&sm.v_full[i], 1);
            mbar_init(&sm.v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.p_ready[i], 128);
            mbar_init(&sm.o_done[i], 1);
        }
        mbar_init(&sm.s_free, 128);
        mbar_init(&sm.drain, 2);  // one commit per MMA issuer
        sm.err = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(&sm.tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    auto failed = [&]() { return *reinterpret_cast<volatile int32_t*>(&sm.err) != 0; };

    // setmaxnreg sits at the top of each warpgroup's branch, so that no code
    // after it is shared between warpgroups of different register budgets.
    if (warp >= 8) {
        setmaxnreg_dec<kRegsControl>();
        if (warp == kProducerWarp) {
            // ------------------------------------------------------------ producer
            // lane 0: Q and K tiles; lane 1: V tiles (independent rings).
            if (lane < 2) {
                const bool kq = lane == 0;
                if (kq) {
                    prefetch_tmap(&tmq);
                    prefetch_tmap(&tmk);
                } else {
                    prefetch_tmap(&tmv);
                }
                const uint64_t pol_q = l2_policy_evict_first();
                const uint64_t pol_kv = l2_policy_evict_last();  // K/V tiles are re-read by the group's q heads
                const int NS = kq ? kKStages : kVStages;
                uint64_t* full = kq ? sm.k_full : sm.v_full;
                uint64_t* empty = kq ? sm.k_empty : sm.v_empty;
                const CUtensorMap* tm = kq ? &tmk : &tmv;
                int nq = 0, g = 0;  // units loaded, tiles loaded (across units)
                int nu = 0;         // units pushed into (lane 0) or taken from (lane 1) the ring
                Unit w;
                while (!failed()) {
                    int u;
                    if (kq) {
                        // claim the next unit that has query rows, and hand it to the other roles
                        do {
                            u = atomicAdd(&p.sched[0], 1);
                        } while (u < total_units && !load_unit(p, u, w));
                        if (u >= total_units) u = -1;
                        const int slot = nu % kUnitRing;
                        if (!wait_or_flag(&sm.unit_empty[slot], ((nu / kUnitRing) & 1) ^ 1, sm)) break;
                        sm.unit_ring[slot] = u;
                        mbar_arrive(&sm.unit_full[slot]);
                        ++nu;
                    } else {
                        u = take_unit(sm, nu, false);
                        if (u == -2) {
                            atomicOr(&g_prefill_error, 1);
                            *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                            break;
                        }
                        if (u >= 0) load_unit(p, u, w);
                    }
                    if (u < 0) break;
                    if (w.ntiles == 0) continue;
                    if (kq) {
                        // Q of the previous unit must no longer be read by S MMAs.
                        if (!wait_or_flag(&sm.q_empty, (nq & 1) ^ 1, sm)) break;
                        mbar_arrive_expect_tx(&sm.q_full, (w.has_b ? 4 : 2) * kHalf);
                        for (int t = 0; t < (w.has_b ? 2 : 1); ++t) {
                            if (p.pair) {
                                // two 64-row boxes per 64-dim half: the pair's heads, 8 KiB apart
                                for (int hh = 0; hh < 2; ++hh) {
                                    const int x = (w.h(t) + hh) * kD;
                                    tma_load_2d(sm.q[t][0] + hh * (kHalf / 2), &tmq, x, w.q0 + w.row(t), &sm.q_full,
                                                pol_q);
                                    tma_load_2d(sm.q[t][1] + hh * (kHalf / 2), &tmq, x + 64, w.q0 + w.row(t),
                                                &sm.q_full, pol_q);
                                }
                            } else {
                                tma_load_2d(sm.q[t][0], &tmq, w.h(t) * kD, w.q0 + w.row(t), &sm.q_full, pol_q);
                                tma_load_2d(sm.q[t][1], &tmq, w.h(t) * kD + 64, w.q0 + w.row(t), &sm.q_full, pol_q);
                            }
                        }
                        ++nq;
                    }
                    const int32_t* bt = p.block_tables ? p.block_tables + int64_t(w.s) * p.bt_stride : nullptr;
                    const int x = (w.h0 / p.group) * kD;
                    for (int j = 0; j < w.ntiles; ++j, ++g) {
                        const int st = g % NS;
                        if (failed() || !wait_or_flag(&empty[st], ((g / NS) & 1) ^ 1, sm)) break;
                        int y;
                        if (bt) {
                            const int pos = j * kBN;
                            const int lb = pos / p.block_size;
                            const int blk = lb < p.bt_stride ? bt[lb] : -1;
                            y = (blk >= 0 && blk < p.num_blocks) ? blk * p.block_size + (pos - lb * p.block_size)
                                                                 : p.num_blocks * p.block_size;
                        } else {
                            y = w.k0 + j * kBN;
                        }
                        mbar_arrive_expect_tx(&full[st], 2 * kHalf);
                        uint8_t* dst0 = kq ? sm.k[st][0] : sm.v[st][0];
                        uint8_t* dst1 = kq ? sm.k[st][1] : sm.v[st][1];
                        tma_load_2d(dst0, tm, x, y, &full[st], pol_kv);
                        tma_load_2d(dst1, tm, x + 64, y, &full[st], pol_kv);
                    }
                }
                // Before the CTA exits, every load issued into its shared memory must have
                // landed (always true on the normal path; bounded wait on error paths).
                if (kq && nq > 0) mbar_wait(&sm.q_full, (nq - 1) & 1);
                for (int st = 0; st < NS && st < g; ++st) {
                    const int last = st + ((g - 1 - st) / NS) * NS;
                    mbar_wait(&full[st], (last / NS) & 1);
                }
            }
        } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
            // ------------------------------------------------------------ MMA issuers
            // Lane 0 of warp kMmaWarp issues every S = Q K^T MMA, lane 0 of warp
            // kMmaWarp + 1 every O += P V MMA.  The two streams share no tensor memory
            // (S buffer vs P / O columns), so neither waits on the other; one issuing
            // thread sustains only about one 128x128x16 MMA per ~110 cycles, and two
            // keep the tensor pipe busy.  Both walk the same units and key tiles.
            if (lane == 0) {
                const bool s_issuer = warp == kMmaWarp;
                constexpr uint32_t idS = tc::idesc_f16<BF16>(kBM, kBN, false, false);
                constexpr uint32_t idPV = tc::idesc_f16<BF16>(kBM, kD, false, true);
                int nq = 0, g = 0;
                int n_s = 0;              // S tiles issued (across units): the S buffer's uses
                int npv[2] = {0, 0};      // PV tiles issued per query tile (across units)
                int nu = 0;               // units taken from the ring
                bool ok = true;
                Unit w;
                while (ok && !failed()) {
                    const int u = take_unit(sm, nu, false);
                    if (u == -2) {
                        atomicOr(&g_prefill_error, 1);
                        *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                        break;
                    }
                    if (u < 0) break;
                    load_unit(p, u, w);
                    if (w.ntiles == 0) continue;
                    const int g0 = g;
                    if (s_issuer) {
                        if (!wait_or_flag(&sm.q_full, nq & 1, sm)) { ok = false; break; }
                        ++nq;
                        tc::fence_after_sync();
                        for (int j = 0; j < w.ntiles && ok; ++j) {
                            const int gj = g0 + j, kst = gj % kKStages;
                            if (!wait_or_flag(&sm.k_full[kst], (gj / kKStages) & 1, sm)) { ok = false; break; }
                            tc::fence_after_sync();
                            const uint32_t ka = smem_u32(sm.k[kst][0]);
                            for (int t = 0; t < 2; ++t) {
                                if (j >= w.nt(t)) continue;
                                // the previous S tile must have been read out of the buffer
                                if (n_s > 0 && !wait_or_flag(&sm.s_free, (n_s - 1) & 1, sm)) { ok = false; break; }
                                ++n_s;
                                tc::fence_after_sync();
                                const uint32_t qa = smem_u32(sm.q[t][0]);
#pragma unroll
                                for (int kk = 0; kk < kD / 16; ++kk) {
                                    // K-major operands: 16 dims = 32 bytes inside a 128-byte swizzled row
                                    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
                                    tc::mma_ss(tmem + kColS, tc::smem_desc_sw128(qa + off, 16, 1024),
                                               tc::smem_desc_sw128(ka + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
                                }
                                tc::commit(&sm.s_full[t]);
                            }
                            if (!ok) break;
                            tc::commit(&sm.k_empty[kst]);                  // both S of key tile j done
                            if (j == w.ntiles - 1) tc::commit(&sm.q_empty);  // last S of the unit done
                        }
                    } else {
                        for (int j = 0; j < w.ntiles && ok; ++j) {
                            const int gj = g0 + j, vst = gj % kVStages;
                            if (!wait_or_flag(&sm.v_full[vst], (gj / kVStages) & 1, sm)) { ok = false; break; }
                            const uint32_t va = smem_u32(sm.v[vst][0]);
                            for (int t = 0; t < 2; ++t) {
                                if (j >= w.nt(t)) continue;
                                if (!wait_or_flag(&sm.p_ready[t], npv[t] & 1, sm)) { ok = false; break; }
                                ++npv[t];
                                tc::fence_after_sync();
#pragma unroll
                                for (int kk = 0; kk < kBN / 16; ++kk) {
                                    // P (K-major, 16 keys = 8 columns of bf16 pairs) from tensor memory;
                                    // V is MN-major: 16 keys = two 8-row swizzle atoms (SBO 1024 B), the
                                    // second 64 dims in the V-hi half (LBO = kHalf).
                                    tc::mma_ts(tmem + kColO + t * 128, tmem + kColP + t * 64 + kk * 8,
                                               tc::smem_desc_sw128(va + kk * 16 * 128, kHalf, 1024), idPV,
                                               (j > 0 || kk > 0) ? 1u : 0u);
                                }
                                tc::commit(&sm.o_done[t]);
                            }
                            if (!ok) break;
                            tc::commit(&sm.v_empty[vst]);  // both PV of key tile j done
                        }
                    }
                    g = g0 + w.ntiles;
                }
                // Wait (bounded) for every MMA issued above before the tensor memory is freed.
                tc::commit(&sm.drain);
                mbar_wait(&sm.drain, 0);
            }
        }
    } else {
        setmaxnreg_inc<kRegsSoftmax>();
        // ------------------------------------------------------------ softmax / epilogue
        const int t = warp >> 2;          // query tile of this warpgroup
        const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31 belong to this warp
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
        const uint32_t s_col = tmem + lane_addr + kColS;
        const uint32_t p_col = tmem + lane_addr + kColP + t * 64;
        const uint32_t o_col = tmem + lane_addr + kColO + t * 128;
        const float sl2 = p.scale_log2;
        int ns = 0;  // S tiles of this query tile consumed (across units) = P tiles written
        int g = 0;   // K/V tiles streamed so far (across units), to find a tile's stage
        int nu = 0;  // units taken from the ring
        Unit w;
        while (!failed()) {
            const int u = take_unit(sm, nu, true);
            if (u == -2) {
                if (lane == 0) atomicOr(&g_prefill_error, 1);
                *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                break;
            }
            if (u < 0) break;
            load_unit(p, u, w);
            const int g0 = g;
            g += w.ntiles;
            // this thread's query row: position and head
            const int qrow = p.pair ? w.row(t) + (r & (kBM / 2 - 1)) : w.row(t) + r;
            const int qhead = p.pair ? w.h(t) + (r >> 6) : w.h(t);
            const int my_tiles = w.nt(t);
            uint4* dst = reinterpret_cast<uint4*>(p.out + int64_t(w.q0 + qrow) * p.out_stride + qhead * kD);
            if (my_tiles == 0) {  // rows that see no key at all (only when lk < lq)
                if (qrow < w.lq)
                    for (int c = 0; c < kD / 8; ++c) dst[c] = make_uint4(0, 0, 0, 0);
                continue;
            }
            const int limit = qrow < w.lq ? qrow + (w.lk - w.lq) : -1;  // last visible key of this row
            const int ns0 = ns;
            float m = -INFINITY, l = 0.f;
            bool ok = true;
            for (int j = 0; j < my_tiles; ++j) {
                if (!wait_or_flag(&sm.s_full[t], ns & 1, sm)) { ok = false; break; }
                ++ns;
                tc::fence_after_sync();
                const int kbase = j * kBN;
                // Tiles inside the visible range of all 32 rows of this warp need no mask.
                // tcgen05.ld/st are warp-collective, so the choice must be warp-uniform.
                const bool full_row = __all_sync(0xffffffffu, kbase + kBN - 1 <= limit);
                float alpha, sum;
                bool rescale;
                uint32_t pk[kBN / 2];
                softmax_tile<BF16>(!full_row, s_col, &sm.s_free, kbase, limit, sl2, m, alpha, rescale, sum, pk);
                l = fmaf(l, alpha, sum);
                if (j > 0) {
                    // PV(j-1) must have read P and written O before P is overwritten or O scaled.
                    if (!wait_or_flag(&sm.o_done[t], (ns0 + j - 1) & 1, sm)) { ok = false; break; }
                    tc::fence_after_sync();
                    // Warp-collective O rescale when any row of the warp needs it (alpha = 1 elsewhere).
                    if (__any_sync(0xffffffffu, rescale)) {
                        if (!rescale) alpha = 1.f;
#pragma unroll 1
                        for (int c = 0; c < kD / 32; ++c) {
                            float o[32];
                            tc::tmem_ld32(o_col + c * 32, o);
                            tc::tmem_wait_ld();
                            uint32_t uo[32];
#pragma unroll
                            for (int e = 0; e < 32; ++e) uo[e] = __float_as_uint(o[e] * alpha);
                            tc::tmem_st32(o_col + c * 32, uo);
                        }
                    }
                }
                tc::tmem_st32(p_col, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
                tc::tmem_st32(p_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
                tc::tmem_wait_st();
                // Cache rows past this sequence's keys may hold NaN bits; P is 0 there but
                // 0 * NaN is NaN, so the first tile to use the stage clears those V rows.
                if (kbase + kBN > w.lk && (t == 0 || j >= w.nt0)) {
                    const int gj = g0 + j, st = gj % kVStages;
                    if (!wait_or_flag(&sm.v_full[st], (gj / kVStages) & 1, sm)) { ok = false; break; }
                    if (kbase + r >= w.lk) {
                        uint4* v0 = reinterpret_cast<uint4*>(sm.v[st][0] + r * 128);
                        uint4* v1 = reinterpret_cast<uint4*>(sm.v[st][1] + r * 128);
#pragma unroll
                        for (int c = 0; c < 8; ++c) v0[c] = v1[c] = make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async_smem();
                }
                tc::fence_before_sync();
                mbar_arrive(&sm.p_ready[t]);
            }
            if (!ok) break;
            // ---- epilogue: O / l -> bf16, one query row per thread.  Loading O before
            // this warpgroup's next p_ready arrive orders it before the next unit's
            // first PV overwrites O.
            if (!wait_or_flag(&sm.o_done[t], (ns - 1) & 1, sm)) break;
            tc::fence_after_sync();
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
            for (int c = 0; c < kD / 32; ++c) {
                float o[32];
                tc::tmem_ld32(o_col + c * 32, o);
                tc::tmem_wait_ld();
                if (qrow < w.lq) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 v4;
                        v4.x = pack2<BF16>(o[e] * inv, o[e + 1] * inv);
                        v4.y = pack2<BF16>(o[e + 2] * inv, o[e + 3] * inv);
                        v4.z = pack2<BF16>(o[e + 4] * inv, o[e + 5] * inv);
                        v4.w = pack2<BF16>(o[e + 6] * inv, o[e + 7] * inv);
                        dst[(c * 32 + e) / 8] = v4;
                    }
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
    if (tid == 0) {
        __threadfence();
        const int done = atomicAdd(&p.sched[1], 1);
        if (done == int(gridDim.x) - 1) {
            // Every CTA has stopped claiming units: re-arm the counter for the next call.
            atomicExch(&p.sched[0], 0);
            atomicExch(&p.sched[1], 0);
        }
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
                                       int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
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
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < kWorkspaceBytes)
        return fail(B200_ERR_WORKSPACE, "varlen_prefill: workspace missing, unaligned or smaller than %zu bytes",
                    kWorkspaceBytes);
    if (block_tables) {
        B200_REQUIRE(block_size > 0 && block_size % kBN == 0, "varlen_prefill: block_size %d not a multiple of %d",
                     block_size, kBN);
        B200_REQUIRE(block_table_stride > 0, "varlen_prefill: block_table_stride %d", block_table_stride);
        B200_REQUIRE(total_k_rows % block_size == 0, "varlen_prefill: cache rows %d not whole blocks", total_k_rows);
    }
    // Even GQA groups pair two query heads per unit (128 positions; each tile
    // holds 64 positions of both heads, which see the same keys); otherwise a
    // unit is 256 rows of one head.
    const int group = num_heads / num_kv_heads;
    const bool pair = group % 2 == 0;
    const int slots = pair ? num_heads / 2 : num_heads;
    const int rows_per_unit = pair ? kBM : 2 * kBM;
    const int q_blocks = (max_seqlen_q + rows_per_unit - 1) / rows_per_unit;
    if (int64_t(q_blocks) * num_seqs * slots > INT32_MAX / 2)
        return fail(B200_ERR_UNSUPPORTED, "varlen_prefill: %d query blocks x %d sequences x %d head slots", q_blocks,
                    num_seqs, slots);
    const bool bf16 = dtype == B200_BF16;
    // The tensor maps span exactly the caller's q / k / v rows, so a tile that
    // runs past the last token reads the TMA fill value (zero), never memory
    // outside the buffers; such rows are masked and never stored.
    CUtensorMap tmq, tmk, tmv;
    const uint64_t q_rows = uint64_t(total_q);
    int32_t rc = make_tmap_2d(&tmq, q, uint64_t(num_heads) * kD, q_rows, uint64_t(q_stride_token) * 2, 64,
                              pair ? kBM / 2 : kBM, bf16, CU_TENSOR_MAP_SWIZZLE_128B);
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
    prm.group = group;
    prm.q_blocks = q_blocks;
    prm.pair = pair ? 1 : 0;
    prm.slots = slots;
    prm.scale_log2 = softmax_scale * 1.4426950408889634f;
    prm.sched = static_cast<int32_t*>(workspace);

    const int smem = int(sizeof(Smem)) + 1024;
    const void* fn = bf16 ? (const void*)prefill_kernel<true> : (const void*)prefill_kernel<false>;
    ensure_smem_attr(fn, smem);
    const int64_t units = int64_t(q_blocks) * num_seqs * slots;
    const dim3 grid(unsigned(units < device_sm_count() ? units : device_sm_count()));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (bf16) prefill_kernel<true><<<grid, kThreads, smem, st>>>(prm, tmq, tmk, tmv);
    else prefill_kernel<false><<<grid, kThreads, smem, st>>>(prm, tmq, tmk, tmv);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

extern "C" size_t b200_varlen_prefill_workspace_size(void) { return b200::pf::kWorkspaceBytes; }

extern "C" int32_t b200_varlen_prefill_error(void* stream, int32_t* flag) {
    using namespace b200;
    B200_REQUIRE(flag != nullptr, "varlen_prefill_error: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    B200_CUDA_TRY(cudaStreamSynchronize(s));
    B200_CUDA_TRY(cudaMemcpyFromSymbol(flag, b200::pf::g_prefill_error, sizeof(int32_t)));
    return B200_OK;
}
