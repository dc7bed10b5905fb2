// Paged multi-query attention for decode (query_len 1) and speculative verify
// (query_len k+1).  Replaces the flash_attn_with_kvcache call of
// nanovllm/layers/attention.py:71-74.
//
// Work decomposition.  A work item is (sequence b, kv head h, chunk c): up to
// `chunk` tiles of 128 cached tokens of one kv head.  All Lq*G query rows
// that read kv head h (G = Hq/Hkv query heads times Lq queries, at most 16)
// are processed together, so every K/V byte is read from HBM once.  The
// chunking is planned on the device from context_lens (no host sync, so the
// call is CUDA-graph capturable): every CTA scans context_lens into shared
// memory and picks the chunk length (about kWaves items per CTA, at most
// kChunkMaxTiles tiles, and coarse enough that the items fit the workspace).
// Items are numbered full-length chunks (and remainders of at least half a
// chunk) first, then the shorter remainders, and are claimed dynamically from
// an atomic counter, so that the large items start early and the tail is made
// of small ones.  Items of a
// sequence that was split write normalised partial outputs plus their
// log-sum-exp to the workspace; the CTA that finishes the last chunk of a
// (b, h) merges them (threadfence-reduction pattern) and writes the output.
//
// CTA layout: one persistent CTA per SM, 9 warps.  Warp 8 is the producer:
// one lane issues 2-D TMA loads (no multicast) of 64-dim x 128-token boxes
// with 128-byte swizzle into a ring of 64 KiB stages (K lo/hi dims, V lo/hi
// dims; 3 stages, 2 for more than 8 query rows) guarded by full/empty
// mbarriers, writes a small header per stage describing the tile, and with
// an item's first tile bulk-copies its query rows into shared memory.  After
// issuing an item's last tile it claims the next item and fetches its
// metadata (context length, block ids) while the issued tiles stream: one
// item ahead, never two, so no CTA holds unstarted work while others run dry.
// Warps 0-7 are consumers (two per SM sub-partition, so that one hides the
// other's latency): each takes 16 of the 128 tokens of a stage and computes
// the scores and P V with mma.sync.m16n8k16.  Up to 8 query rows the tile is
// transposed -- tokens are the MMA's M and the query rows its N of 8
// (S^T = K Q^T, O^T += V^T P^T, P^T turned into a B operand by movmatrix) --
// and a row's running maximum is raised only when a score exceeds it by more
// than 2^kLazyMax; more rows use rows as M (S = Q K^T, O += P V, padded to
// 16).  Each warp keeps its own online-softmax state (max, sum, O) in
// registers; the eight partial states are combined through shared memory at
// the end of an item (8 -> 4 in registers, then 4 -> 1).
//
// Every wait in the kernel is bounded (kWaitLimitNs, or the test limit): the
// stage barriers, and the consumer warps' own barrier around the combine,
// which is an mbarrier with one arrival per consumer thread rather than a
// bar.sync, so that a warp whose sibling left the loop on an error gives up
// after the limit instead of waiting for it forever.
#include <cfloat>
#include <climits>
#include <mutex>

#include "common.cuh"

namespace b200 {
namespace pa {

constexpr int kTile = 128;                   // tokens per stage
constexpr int kD = 128;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kHalfBytes = kTile * 128;      // 128 tokens x 64 dims x 2 B
constexpr int kStageBytes = 4 * kHalfBytes;  // K dims 0-63, K 64-127, V 0-63, V 64-127
constexpr int kMaxBatch = 2048;
constexpr int kCounterSlots = 65536;
constexpr int kCtrlWords = 64;               // [0] next item, [1] finished CTAs, [2] error word
constexpr size_t kFixedBytes = kCtrlWords * 4 + size_t(kCounterSlots) * 4;
constexpr int kWaves = 3;
constexpr int kChunkMaxTiles = 32;           // at most 4096 tokens per item
constexpr int kRemBits = 12;                 // packed offsets: full-chunk offset << 12 | remainder offset
constexpr int kClaimAhead = 1;               // tiles before an item's end at which the next one is claimed
constexpr float kLazyMax = 8.f;              // log2 headroom before a row's running maximum is raised

struct Header {
    int32_t item, b, h, tile, flags, ctx, nchunks, slot0;
};
enum : int32_t { kFirst = 1, kLast = 2 };

struct Params {
    const uint16_t* q;
    int64_t q_stride;
    uint16_t* out;
    const int32_t* block_tables;
    int32_t bt_stride;
    const int32_t* context_lens;
    int32_t batch, lq, hq, hkv, group, rows, block_size, num_blocks;
    float scale_log2;
    uint64_t wait_ns;  // limit of every wait (kWaitLimitNs; shorter under the idle-producer test)
    int32_t idle_producer;  // test hook: the producer issues nothing, so the consumers' first wait runs out
    int32_t* ctrl;
    int32_t* counters;
    float* part_o;    // [max_items][rows][kD]
    float* part_lse;  // [max_items][rows]
    int32_t max_items;
};

template <int RC, int NS>
struct Smem {
    uint8_t stages[NS][kStageBytes];
    uint8_t qbuf[NS][RC * kD * 2];  // query rows of an item, filled with its first tile
    float co[kConsumerWarps / 2][RC][kD];
    float cm[kConsumerWarps][RC];
    float cl[kConsumerWarps][RC];
    Header hdr[NS];
    uint64_t full[NS];
    uint64_t empty[NS];
    uint64_t cbar;                  // consumer barrier: kConsumers arrivals per phase
    int32_t off[kMaxBatch + 1];     // (full-chunk offset << kRemBits) | remainder offset
    int32_t red[kThreads / 32 + 1];
    int32_t flag;
    int32_t err;
};

template <bool ROWS_HI>
constexpr int num_stages() {
    return ROWS_HI ? 2 : 3;
}

template <bool ROWS_HI>
constexpr int smem_bytes() {
    return int(sizeof(Smem<ROWS_HI ? 16 : 8, num_stages<ROWS_HI>()>)) + 1024;
}
static_assert(smem_bytes<false>() <= 232448 && smem_bytes<true>() <= 232448, "shared memory over 227 KB");

// Block-wide exclusive scan of one int per thread; returns the exclusive
// prefix and writes the total to *total.  Uses red[] (one slot per warp).
__device__ __forceinline__ int block_exclusive_scan(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) red[warp] = x;
    __syncthreads();
    int base = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
        if (w < warp) base += red[w];
        tot += red[w];
    }
    __syncthreads();
    *total = tot;
    return base + x - v;
}

// Barrier of the consumer threads, bounded: each arrives (release) and polls
// the phase (acquire) for at most limit_ns.  Returns false, for the whole
// warp alike, when the wait of any of its lanes ran out.
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t& phase, uint64_t limit_ns) {
    mbar_arrive(bar);
    const bool ok = mbar_wait_spin(bar, phase, limit_ns);
    phase ^= 1;
    return __all_sync(0xffffffffu, ok);
}

// Chunk layout of one sequence: `full` items in the first region (chunks of
// `chunk` tiles, the last of them possibly a remainder of at least half a
// chunk) and `rem` (0 or 1) short remainder in the second.
struct SeqChunks {
    int nt, full, rem;
};

// A sequence of nt tiles is cut into chunks of `chunk` tiles and a shorter remainder.  Items
// are numbered in two regions: first every sequence's full chunks together with its remainder
// when that is at least half a chunk ("full" count), then the short remainders ("rem"), so that
// the smallest items come last and the end of a launch is made of them.
__device__ __forceinline__ SeqChunks tile_chunks(int nt, int64_t chunk) {
    SeqChunks s;
    s.nt = nt;
    s.full = int(nt / chunk);
    const int64_t rt = nt - int64_t(s.full) * chunk;
    const bool big = rt > 0 && 2 * rt >= chunk;
    s.full += big ? 1 : 0;
    s.rem = (rt > 0 && !big) ? 1 : 0;
    return s;
}

__device__ __forceinline__ SeqChunks seq_chunks(int ctx, int cap, int64_t chunk) {
    ctx = min(ctx, cap);
    return tile_chunks(ctx > 0 ? (ctx + kTile - 1) / kTile : 0, chunk);
}

// Metadata of one claimed work item.  The producer fetches it one item
// ahead, so that its dependent global loads (context length, block ids)
// overlap the TMA traffic of the current item.
constexpr int kPrefetchPages = 4;
struct ItemMeta {
    int item, b, h, c, nchunks, ctx, t0, slot0, page0;
    int blk[kPrefetchPages];
};

// Partial-output slot (chunk index, before the x Hkv + h) of chunk c of
// sequence b: first-region chunks are numbered first, short remainders after them.
__device__ __forceinline__ int chunk_slot(int packed_off, int c, int full, int total_full) {
    return c < full ? (packed_off >> kRemBits) + c : total_full + (packed_off & ((1 << kRemBits) - 1));
}

__device__ __forceinline__ void fetch_meta(ItemMeta& m, int item, const Params& p, const int32_t* off,
                                           int total_full, int64_t chunk, int cap) {
    m.item = item;
    const int cg = item / p.hkv;
    m.h = item - cg * p.hkv;
    int blo = 0, bhi = p.batch;  // largest b whose offset (in the chunk's group) is <= cg
    if (cg < total_full) {
        while (bhi - blo > 1) {
            const int mid = (blo + bhi) >> 1;
            if ((off[mid] >> kRemBits) <= cg) blo = mid; else bhi = mid;
        }
    } else {
        const int r = cg - total_full;
        while (bhi - blo > 1) {
            const int mid = (blo + bhi) >> 1;
            if ((off[mid] & ((1 << kRemBits) - 1)) <= r) blo = mid; else bhi = mid;
        }
    }
    m.b = blo;
    m.ctx = p.context_lens[blo];
    const SeqChunks sc = seq_chunks(m.ctx, cap, chunk);
    m.c = cg < total_full ? cg - (off[blo] >> kRemBits) : sc.full;
    m.nchunks = sc.full + sc.rem;
    m.slot0 = off[blo];
    m.t0 = int(m.c * chunk);
    m.page0 = (m.t0 * kTile) / p.block_size;
    const int32_t* bt = p.block_tables + int64_t(blo) * p.bt_stride;
#pragma unroll
    for (int j = 0; j < kPrefetchPages; ++j) m.blk[j] = bt[min(m.page0 + j, p.bt_stride - 1)];
}

template <bool BF16, bool ROWS_HI>
__global__ void __launch_bounds__(kThreads, 1)
    paged_attention_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv) {
    constexpr int RC = ROWS_HI ? 16 : 8;
    constexpr int NS = num_stages<ROWS_HI>();
    extern __shared__ uint8_t smem_raw[];
    Smem<RC, NS>& sm =
        *reinterpret_cast<Smem<RC, NS>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
        }
        mbar_init(&sm.cbar, kConsumers);
        sm.err = 0;
        fence_mbar_init();
    }
    if (warp == kConsumerWarps && lane == 0) {
        prefetch_tmap(&tmk);
        prefetch_tmap(&tmv);
    }

    // The producer's first claim does not depend on the plan: its latency overlaps the planning.
    const bool producer = warp == kConsumerWarps && lane == 0 && !p.idle_producer;
    const int first_claim = producer ? atomicAdd(&p.ctrl[0], 1) : 0;

    // ---- plan: tiles per sequence, chunk length, chunk offsets ----------------
    const int cap = p.bt_stride * p.block_size;  // tokens addressable through the block table
    const int seg = (p.batch + kThreads - 1) / kThreads;
    const int lo = min(tid * seg, p.batch), hi = min(lo + seg, p.batch);
    int my_tiles = 0;
    for (int b = lo; b < hi; ++b) {
        const int nt = seq_chunks(p.context_lens[b], cap, 1).nt;
        sm.off[b] = nt;  // this thread's sequences only; replaced by their offsets below
        my_tiles += nt;
    }
    int total_tiles = 0;
    block_exclusive_scan(my_tiles, sm.red, &total_tiles);
    int64_t chunk;
    {
        const int64_t want = int64_t(gridDim.x) * kWaves;
        chunk = (int64_t(total_tiles) * p.hkv + want - 1) / want;
        chunk = chunk < 1 ? 1 : (chunk > kChunkMaxTiles ? kChunkMaxTiles : chunk);
        const int64_t budget = p.max_items / p.hkv;
        if (budget > p.batch) {
            const int64_t need = (int64_t(total_tiles) + (budget - p.batch) - 1) / (budget - p.batch);
            if (need > chunk) chunk = need;
        } else {
            chunk = int64_t(1) << 30;
        }
        // First-region offsets are packed into 31 - kRemBits bits (full chunks, plus at most one
        // remainder per sequence).
        const int64_t max_full = (int64_t(1) << (31 - kRemBits)) - 1 - kMaxBatch;
        if (int64_t(total_tiles) / chunk > max_full) chunk = (int64_t(total_tiles) + max_full - 1) / max_full;
    }
    // Both offsets in one scan of the packed count full << kRemBits | rem: the remainder
    // counts sum to at most the batch (< 2^kRemBits), so no carry reaches the full part.
    int my_packed = 0;
    for (int b = lo; b < hi; ++b) {
        const SeqChunks sc = tile_chunks(sm.off[b], chunk);
        my_packed += (sc.full << kRemBits) + sc.rem;
    }
    int total_packed = 0;
    int opacked = block_exclusive_scan(my_packed, sm.red, &total_packed);
    for (int b = lo; b < hi; ++b) {
        const SeqChunks sc = tile_chunks(sm.off[b], chunk);
        sm.off[b] = opacked;
        opacked += (sc.full << kRemBits) + sc.rem;
    }
    const int total_full = total_packed >> kRemBits, total_rem = total_packed & ((1 << kRemBits) - 1);
    if (tid == 0) sm.off[p.batch] = total_packed;
    __syncthreads();
    const int total_items = (total_full + total_rem) * p.hkv;

    // Rows without a cached token (context_lens <= 0: CUDA-graph padding) have no items and get
    // a zero output.
    const int64_t row_vec = int64_t(p.lq) * p.hq * kD / 8;  // uint4 per batch row
    for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
        if (sm.off[b + 1] == sm.off[b]) {
            uint4* o = reinterpret_cast<uint4*>(p.out) + b * row_vec;
            for (int64_t i = tid; i < row_vec; i += kThreads) o[i] = make_uint4(0, 0, 0, 0);
        }
    }

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (producer) {
            const uint64_t pol = l2_policy_evict_first();
            const uint32_t q_bytes = uint32_t(p.group) * kD * 2;  // one query token's rows of this kv head
            int stage = 0;
            uint32_t phase = 0;
            int64_t fills = 0;
            bool ok = true;
            ItemMeta cur, nxt;
            cur.item = total_items;
            if (first_claim < total_items) fetch_meta(cur, first_claim, p, sm.off, total_full, chunk, cap);
            while (ok && cur.item < total_items) {
                const int ctx = min(cur.ctx, cap);
                const int nt = (ctx + kTile - 1) / kTile;
                const int t0 = cur.t0;
                const int t1 = int(min(int64_t(nt), t0 + chunk));
                const int32_t* bt = p.block_tables + int64_t(cur.b) * p.bt_stride;
                // The next item is claimed once the loads of tile t1 - kClaimAhead are issued: its
                // metadata loads overlap the tiles in flight, and no CTA sits on an unstarted item
                // while others run out of work at the end of the launch.
                const int t_claim = max(t0, t1 - kClaimAhead);
                nxt.item = total_items;
                for (int t = t0; t < t1; ++t) {
                    if (!mbar_wait(&sm.empty[stage], phase ^ 1, p.wait_ns)) {
                        atomicOr(&p.ctrl[2], DEV_ERR_WAIT_EMPTY);
                        ok = false;
                        break;
                    }
                    const bool first = t == t0;
                    const int pos = t * kTile;
                    const int lb = pos / p.block_size;
                    int blk;
                    const int j = lb - cur.page0;
                    if (j < kPrefetchPages) {
                        blk = cur.blk[0];
#pragma unroll
                        for (int u = 1; u < kPrefetchPages; ++u)
                            if (j == u) blk = cur.blk[u];
                    } else {
                        blk = bt[lb];
                    }
                    const int y = (blk >= 0 && blk < p.num_blocks) ? blk * p.block_size + (pos - lb * p.block_size)
                                                                   : p.num_blocks * p.block_size;
                    Header& hd = sm.hdr[stage];
                    hd.item = cur.item;
                    hd.b = cur.b;
                    hd.h = cur.h;
                    hd.tile = t;
                    hd.flags = (first ? kFirst : 0) | (t == t1 - 1 ? kLast : 0);
                    hd.ctx = ctx;
                    hd.nchunks = cur.nchunks;
                    hd.slot0 = cur.slot0;
                    mbar_arrive_expect_tx(&sm.full[stage], kStageBytes + (first ? q_bytes * p.lq : 0u));
                    uint8_t* st = sm.stages[stage];
                    const int x = cur.h * kD;
                    tma_load_2d(st, &tmk, x, y, &sm.full[stage], pol);
                    tma_load_2d(st + kHalfBytes, &tmk, x + 64, y, &sm.full[stage], pol);
                    tma_load_2d(st + 2 * kHalfBytes, &tmv, x, y, &sm.full[stage], pol);
                    tma_load_2d(st + 3 * kHalfBytes, &tmv, x + 64, y, &sm.full[stage], pol);
                    if (first) {
                        const uint16_t* qsrc = p.q + int64_t(cur.b) * p.lq * p.q_stride + int64_t(cur.h) * p.group * kD;
                        for (int jq = 0; jq < p.lq; ++jq)
                            bulk_load(sm.qbuf[stage] + jq * q_bytes, qsrc + int64_t(jq) * p.q_stride, q_bytes,
                                      &sm.full[stage]);
                    }
                    ++fills;
                    if (++stage == NS) { stage = 0; phase ^= 1; }
                    // After this tile's loads are issued, so that the claim's dependent loads
                    // overlap them instead of delaying them.
                    if (t == t_claim) {
                        const int claim = atomicAdd(&p.ctrl[0], 1);
                        if (claim < total_items) fetch_meta(nxt, claim, p, sm.off, total_full, chunk, cap);
                    }
                }
                cur = nxt;
            }
            if (ok) {
                if (mbar_wait(&sm.empty[stage], phase ^ 1, p.wait_ns)) {
                    sm.hdr[stage].item = -1;  // sentinel: no more tiles
                    mbar_arrive(&sm.full[stage]);
                } else {
                    atomicOr(&p.ctrl[2], DEV_ERR_WAIT_EMPTY);
                    ok = false;
                }
            }
            if (!ok) {
                // Error path: wait (bounded) for every copy still in flight
                // before the CTA's shared memory is released.
                for (int s = 0; s < NS; ++s) {
                    if (fills <= s) break;
                    const int64_t last = s + ((fills - 1 - s) / NS) * NS;
                    if (!mbar_wait(&sm.full[s], uint32_t((last / NS) & 1), p.wait_ns))
                        atomicOr(&p.ctrl[2], DEV_ERR_WAIT_DRAIN);
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ consumers
        const int g = lane >> 2, t4 = lane & 3;
        const int mi = lane >> 3, rr = lane & 7;
        // ldmatrix rows (token in the tile) and 16-byte column offsets of this lane.  Up to 8 query
        // rows: tokens are the MMA's M dimension (S^T = K Q^T, O^T += V^T P^T) and the rows its N;
        // more rows: rows are M (S = Q K^T, O += P V).
        const int tok_k = ROWS_HI ? warp * 16 + (mi >> 1) * 8 + rr : warp * 16 + (mi & 1) * 8 + rr;
        const int kadd = ROWS_HI ? (mi & 1) : (mi >> 1);
        const int tok_v = ROWS_HI ? warp * 16 + (mi & 1) * 8 + rr : warp * 16 + (mi >> 1) * 8 + rr;
        const int vadd = ROWS_HI ? (mi >> 1) : (mi & 1);
        const float sl2 = p.scale_log2;
        int stage = 0;
        uint32_t phase = 0, cphase = 0;
        // Running maximum (raw score) and sum of the two rows this lane holds: rows g and g + 8
        // (ROWS_HI) or rows 2 t4 and 2 t4 + 1.  msl = m_run * log2(e) * scale (0 while m_run is -inf).
        float m_run[2], l_run[2], msl[2];
        float o[ROWS_HI ? 16 : 8][4];  // O (rows x dims) or O^T (dims x rows) fragments
        uint32_t qa[8][ROWS_HI ? 4 : 2];  // Q as the A operand, or Q^T as the B operand
        int lim[2];
        int lim_min = 0;
        while (true) {
            // Exit decisions are warp-uniform (the lanes' waits can disagree at the limit).
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.full[stage], phase, p.wait_ns))) {
                atomicOr(&p.ctrl[2], DEV_ERR_WAIT_FULL);
                *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                break;
            }
            // A sibling consumer warp that gave up will not reach the consumer
            // barrier below: leave now rather than run into its time limit.
            if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int32_t*>(&sm.err) != 0)) break;
            const Header hd = sm.hdr[stage];
            if (hd.item < 0) break;
            if (hd.flags & kFirst) {
                const uint32_t* qs = reinterpret_cast<const uint32_t*>(sm.qbuf[stage]);
                if constexpr (ROWS_HI) {
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int r = g + 8 * hr;
                        const bool valid = r < p.rows;
                        lim[hr] = valid ? hd.ctx - p.lq + r / p.group : -1;
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            qa[kk][hr] = valid ? qs[r * (kD / 2) + kk * 8 + t4] : 0u;
                            qa[kk][2 + hr] = valid ? qs[r * (kD / 2) + kk * 8 + 4 + t4] : 0u;
                        }
                    }
                } else {
                    // B fragment of Q^T: this lane's column is query row g.
                    const bool valid = g < p.rows;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        qa[kk][0] = valid ? qs[g * (kD / 2) + kk * 8 + t4] : 0u;
                        qa[kk][1] = valid ? qs[g * (kD / 2) + kk * 8 + 4 + t4] : 0u;
                    }
                    // Padding rows (past p.rows) see the whole context: only rows that exist mask.
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int r = 2 * t4 + j;
                        lim[j] = r < p.rows ? hd.ctx - p.lq + r / p.group : hd.ctx - 1;
                    }
                    lim_min = hd.ctx - p.lq;  // row 0's limit, the smallest
                }
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    m_run[hr] = -INFINITY;
                    l_run[hr] = 0.f;
                    msl[hr] = 0.f;
                }
#pragma unroll
                for (int n = 0; n < (ROWS_HI ? 16 : 8); ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
            }
            const int tok_base = hd.tile * kTile + warp * 16;
            const uint32_t st = smem_u32(sm.stages[stage]);
            bool zeroed = false;
            if (tok_base < hd.ctx) {
                if (tok_base + 16 > hd.ctx) {
                    // Cache rows past the context may hold anything (NaN bits);
                    // P is 0 there but 0 * NaN is NaN, so clear those V rows.
                    const int first = hd.ctx - tok_base;
                    uint8_t* vb = sm.stages[stage] + 2 * kHalfBytes;
                    for (int i = lane; i < (16 - first) * 16; i += 32) {
                        const int row = warp * 16 + first + (i >> 4);
                        const int half = (i >> 3) & 1, ch = i & 7;
                        *reinterpret_cast<uint4*>(vb + half * kHalfBytes + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
                    }
                    zeroed = true;
                    __syncwarp();
                }
                if constexpr (ROWS_HI) {
                    // S = Q K^T for this warp's 16 tokens; two accumulator sets halve the dependent chain
                    float s[2][4], s2[2][4];
#pragma unroll
                    for (int n = 0; n < 2; ++n)
#pragma unroll
                        for (int e = 0; e < 4; ++e) s[n][e] = s2[n][e] = 0.f;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int c16 = 2 * kk + kadd;
                        const uint32_t addr = st + (kk >> 2) * kHalfBytes + tok_k * 128 + (((c16 & 7) ^ rr) << 4);
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(b0, b1, b2, b3, addr);
                        if (kk < 4) {
                            mma_16816<BF16>(s[0], qa[kk], b0, b1);
                            mma_16816<BF16>(s[1], qa[kk], b2, b3);
                        } else {
                            mma_16816<BF16>(s2[0], qa[kk], b0, b1);
                            mma_16816<BF16>(s2[1], qa[kk], b2, b3);
                        }
                    }
#pragma unroll
                    for (int n = 0; n < 2; ++n)
#pragma unroll
                        for (int e = 0; e < 4; ++e) s[n][e] += s2[n][e];
                    float pr[2][4];
                    float alpha[2] = {1.f, 1.f};
#pragma unroll
                    for (int hr = 0; hr < (ROWS_HI ? 2 : 1); ++hr) {
                        float v[4] = {s[0][2 * hr], s[0][2 * hr + 1], s[1][2 * hr], s[1][2 * hr + 1]};
                        const int tk[4] = {tok_base + 2 * t4, tok_base + 2 * t4 + 1, tok_base + 8 + 2 * t4,
                                           tok_base + 9 + 2 * t4};
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (tk[e] > lim[hr]) v[e] = -INFINITY;
                        float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                        const float mnew = fmaxf(m_run[hr], mx);
                        const float msl = mnew == -INFINITY ? 0.f : mnew * sl2;
                        alpha[hr] = mnew == m_run[hr] ? 1.f : fast_exp2(fmaf(m_run[hr], sl2, -msl));
                        float sum = 0.f;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            pr[hr][e] = fast_exp2(fmaf(v[e], sl2, -msl));
                            sum += pr[hr][e];
                        }
                        l_run[hr] = fmaf(l_run[hr], alpha[hr], sum);
                        m_run[hr] = mnew;
                    }
                    // Rescale O only when some row's running max moved (rare after the first tiles).
                    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
                        for (int n = 0; n < 16; ++n) {
                            o[n][0] *= alpha[0];
                            o[n][1] *= alpha[0];
                            if constexpr (ROWS_HI) {
                                o[n][2] *= alpha[1];
                                o[n][3] *= alpha[1];
                            }
                        }
                    }
                    uint32_t pa[4];
                    pa[0] = pack2<BF16>(pr[0][0], pr[0][1]);
                    pa[2] = pack2<BF16>(pr[0][2], pr[0][3]);
                    if constexpr (ROWS_HI) {
                        pa[1] = pack2<BF16>(pr[1][0], pr[1][1]);
                        pa[3] = pack2<BF16>(pr[1][2], pr[1][3]);
                    } else {
                        pa[1] = pa[3] = 0u;
                    }
#pragma unroll
                    for (int pp = 0; pp < 8; ++pp) {
                        const int c16 = 2 * pp + vadd;
                        const uint32_t addr =
                            st + 2 * kHalfBytes + (pp >> 2) * kHalfBytes + tok_v * 128 + (((c16 & 7) ^ rr) << 4);
                        uint32_t v0, v1, v2, v3;
                        ldsm_x4_t(v0, v1, v2, v3, addr);
                        mma_16816<BF16>(o[2 * pp], pa, v0, v1);
                        mma_16816<BF16>(o[2 * pp + 1], pa, v2, v3);
                    }
                } else {
                    // S^T = K Q^T: this warp's 16 tokens (M) x 8 query rows (N); two accumulator sets
                    // halve the dependent chain.  c0/c1: token g, rows 2 t4 / 2 t4 + 1; c2/c3: token g + 8.
                    float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int c16 = 2 * kk + kadd;
                        const uint32_t addr = st + (kk >> 2) * kHalfBytes + tok_k * 128 + (((c16 & 7) ^ rr) << 4);
                        uint32_t a[4];
                        ldsm_x4(a[0], a[1], a[2], a[3], addr);
                        if (kk < 4)
                            mma_16816<BF16>(s, a, qa[kk][0], qa[kk][1]);
                        else
                            mma_16816<BF16>(s2, a, qa[kk][0], qa[kk][1]);
                    }
                    float v[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] = s[e] + s2[e];
                    if (tok_base + 15 > lim_min) {  // the tile reaches past some row's last visible token
                        const int ta = tok_base + g, tb = ta + 8;
                        if (ta > lim[0]) v[0] = -INFINITY;
                        if (ta > lim[1]) v[1] = -INFINITY;
                        if (tb > lim[0]) v[2] = -INFINITY;
                        if (tb > lim[1]) v[3] = -INFINITY;
                    }
                    // Exponents relative to the rows' running maxima.  Those are updated (exact tile
                    // maxima over the warp, O^T and sums rescaled) only when a score exceeds its row's
                    // maximum by more than 2^kLazyMax, or the row has none yet; otherwise P <= 2^kLazyMax.
                    float x[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) x[e] = fmaf(v[e], sl2, -msl[e & 1]);
                    const bool grow = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])) > kLazyMax ||
                                      (m_run[0] == -INFINITY && fmaxf(v[0], v[2]) != -INFINITY) ||
                                      (m_run[1] == -INFINITY && fmaxf(v[1], v[3]) != -INFINITY);
                    if (__any_sync(0xffffffffu, grow)) {
                        float tm[2] = {fmaxf(v[0], v[2]), fmaxf(v[1], v[3])};
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
#pragma unroll
                            for (int sh = 4; sh <= 16; sh <<= 1) tm[j] = fmaxf(tm[j], __shfl_xor_sync(0xffffffffu, tm[j], sh));
                            const float mnew = fmaxf(m_run[j], tm[j]);
                            const float mslnew = mnew == -INFINITY ? 0.f : mnew * sl2;
                            const float alpha = m_run[j] == -INFINITY ? 0.f : fast_exp2(msl[j] - mslnew);
                            l_run[j] *= alpha;
#pragma unroll
                            for (int pp = 0; pp < 8; ++pp) {
                                o[pp][j] *= alpha;
                                o[pp][2 + j] *= alpha;
                            }
                            m_run[j] = mnew;
                            msl[j] = mslnew;
                        }
#pragma unroll
                        for (int e = 0; e < 4; ++e) x[e] = fmaf(v[e], sl2, -msl[e & 1]);
                    }
                    float pr[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) pr[e] = fast_exp2(x[e]);
                    l_run[0] += pr[0] + pr[2];
                    l_run[1] += pr[1] + pr[3];
                    // P^T as the B operand (16 tokens x 8 rows): transpose the two 8 x 8 blocks.
                    const uint32_t pb0 = movmatrix_t(pack2<BF16>(pr[0], pr[1]));
                    const uint32_t pb1 = movmatrix_t(pack2<BF16>(pr[2], pr[3]));
                    // O^T += V^T P^T, 16 dims per MMA.
#pragma unroll
                    for (int pp = 0; pp < 8; ++pp) {
                        const int c16 = 2 * pp + vadd;
                        const uint32_t addr =
                            st + 2 * kHalfBytes + (pp >> 2) * kHalfBytes + tok_v * 128 + (((c16 & 7) ^ rr) << 4);
                        uint32_t a[4];
                        ldsm_x4_t(a[0], a[1], a[2], a[3], addr);
                        mma_16816<BF16>(o[pp], a, pb0, pb1);
                    }
                }
            }
            if (zeroed) fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[stage]);
            if (++stage == NS) { stage = 0; phase ^= 1; }

            if (hd.flags & kLast) {
                // ---- combine the eight warps' states of this item ----
                // Row sums over the lanes that hold the same rows (t4 for ROWS_HI, g otherwise).
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    if constexpr (ROWS_HI) {
                        l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
                        l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
                    } else {
#pragma unroll
                        for (int sh = 4; sh <= 16; sh <<= 1) l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], sh);
                    }
                }
                constexpr int kHalf = kConsumerWarps / 2;
                // 8 -> 4: warps 4-7 hand their state to warps 0-3, which merge it in registers.
                if constexpr (!ROWS_HI) {
                  if (warp >= kHalf) {
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int r = 2 * t4 + j;
                        if (g == 0) {
                            sm.cm[warp][r] = m_run[j];
                            sm.cl[warp][r] = l_run[j];
                        }
#pragma unroll
                        for (int pp = 0; pp < 8; ++pp) {
                            sm.co[warp - kHalf][r][16 * pp + g] = o[pp][j];
                            sm.co[warp - kHalf][r][16 * pp + g + 8] = o[pp][2 + j];
                        }
                    }
                  }
                } else {
                  if (warp >= kHalf) {
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int r = g + 8 * hr;
                        if (t4 == 0) {
                            sm.cm[warp][r] = m_run[hr];
                            sm.cl[warp][r] = l_run[hr];
                        }
#pragma unroll
                        for (int n = 0; n < 16; ++n)
                            *reinterpret_cast<float2*>(&sm.co[warp - kHalf][r][8 * n + 2 * t4]) =
                                make_float2(o[n][2 * hr], o[n][2 * hr + 1]);
                    }
                  }
                }
                if (!consumer_sync(&sm.cbar, cphase, p.wait_ns)) {
                    atomicOr(&p.ctrl[2], DEV_ERR_WAIT_PEER);
                    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                    break;
                }
                if constexpr (!ROWS_HI) {
                  if (warp < kHalf) {
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int r = 2 * t4 + j;
                        const float mb = sm.cm[warp + kHalf][r], lb = sm.cl[warp + kHalf][r];
                        const float M = fmaxf(m_run[j], mb);
                        const float sa = M == -INFINITY ? 0.f : fast_exp2((m_run[j] - M) * sl2);
                        const float sb = M == -INFINITY ? 0.f : fast_exp2((mb - M) * sl2);
#pragma unroll
                        for (int pp = 0; pp < 8; ++pp) {
#pragma unroll
                            for (int eh = 0; eh < 2; ++eh) {
                                float* cp = &sm.co[warp][r][16 * pp + g + 8 * eh];
                                *cp = o[pp][j + 2 * eh] * sa + *cp * sb;
                            }
                        }
                        if (g == 0) {
                            sm.cm[warp][r] = M;
                            sm.cl[warp][r] = l_run[j] * sa + lb * sb;
                        }
                    }
                  }
                } else {
                  if (warp < kHalf) {
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int r = g + 8 * hr;
                        const float mb = sm.cm[warp + kHalf][r], lb = sm.cl[warp + kHalf][r];
                        const float M = fmaxf(m_run[hr], mb);
                        const float sa = M == -INFINITY ? 0.f : fast_exp2((m_run[hr] - M) * sl2);
                        const float sb = M == -INFINITY ? 0.f : fast_exp2((mb - M) * sl2);
#pragma unroll
                        for (int n = 0; n < 16; ++n) {
                            float2* cp = reinterpret_cast<float2*>(&sm.co[warp][r][8 * n + 2 * t4]);
                            const float2 ob = *cp;
                            *cp = make_float2(o[n][2 * hr] * sa + ob.x * sb, o[n][2 * hr + 1] * sa + ob.y * sb);
                        }
                        if (t4 == 0) {
                            sm.cm[warp][r] = M;
                            sm.cl[warp][r] = l_run[hr] * sa + lb * sb;
                        }
                    }
                  }
                }
                if (!consumer_sync(&sm.cbar, cphase, p.wait_ns)) {
                    atomicOr(&p.ctrl[2], DEV_ERR_WAIT_PEER);
                    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                    break;
                }
                // 4 -> 1 over shared memory, one output element per thread and round.
                const bool single = hd.nchunks == 1;
                const int nel = p.rows * kD;
                const int cslot = hd.item / p.hkv;  // this chunk's partial slot (before x Hkv + h)
                for (int idx = tid; idx < nel; idx += kConsumers) {
                    const int r = idx >> 7, d = idx & (kD - 1);
                    float M = -INFINITY;
#pragma unroll
                    for (int w = 0; w < kHalf; ++w) M = fmaxf(M, sm.cm[w][r]);
                    float den = 0.f, acc = 0.f;
                    if (M != -INFINITY) {
#pragma unroll
                        for (int w = 0; w < kHalf; ++w) {
                            const float sc = fast_exp2((sm.cm[w][r] - M) * sl2);
                            den = fmaf(sm.cl[w][r], sc, den);
                            acc = fmaf(sm.co[w][r][d], sc, acc);
                        }
                    }
                    const float val = den > 0.f ? acc / den : 0.f;
                    if (single) {
                        const int j = r / p.group, gq = r - j * p.group;
                        p.out[((int64_t(hd.b) * p.lq + j) * p.hq + hd.h * p.group + gq) * kD + d] = to_bits16<BF16>(val);
                    } else {
                        const int64_t it = int64_t(cslot) * p.hkv + hd.h;
                        p.part_o[(it * p.rows + r) * kD + d] = val;
                        if (d == 0) p.part_lse[it * p.rows + r] = den > 0.f ? fmaf(M, sl2, fast_log2(den)) : -INFINITY;
                    }
                }
                if (!single) {
                    // Publish this chunk (one release fence per CTA, cumulative over
                    // the barrier), then count it; the last chunk's CTA merges.
                    if (!consumer_sync(&sm.cbar, cphase, p.wait_ns)) {
                        atomicOr(&p.ctrl[2], DEV_ERR_WAIT_PEER);
                        *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                        break;
                    }
                    if (tid == 0) {
                        __threadfence();
                        const int prev = atomicAdd(&p.counters[hd.b * p.hkv + hd.h], 1);
                        const bool last = prev == hd.nchunks - 1;
                        if (last) __threadfence();
                        sm.flag = last;
                    }
                    if (!consumer_sync(&sm.cbar, cphase, p.wait_ns)) {
                        atomicOr(&p.ctrl[2], DEV_ERR_WAIT_PEER);
                        *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                        break;
                    }
                    if (sm.flag) {
                        const int nch = hd.nchunks;
                        const int full = nch - (seq_chunks(hd.ctx, cap, chunk).rem);
                        // One pass over the chunks, four at a time: every thread merges the
                        // partials of two output elements at once with a running maximum of the
                        // chunks' log-sum-exps (base 2), the sixteen loads of a group in flight.
                        for (int e0 = 2 * tid; e0 < nel; e0 += 2 * kConsumers) {
                            const int r = e0 >> 7, d = e0 & (kD - 1);  // d even: (d, d + 1) in one row
                            float mrun = -INFINITY, den = 0.f, acc0 = 0.f, acc1 = 0.f;
                            for (int c0 = 0; c0 < nch; c0 += 4) {
                                float lse[4];
                                float2 x[4];
#pragma unroll
                                for (int cc = 0; cc < 4; ++cc) {
                                    if (c0 + cc < nch) {
                                        const int64_t it =
                                            int64_t(chunk_slot(hd.slot0, c0 + cc, full, total_full)) * p.hkv + hd.h;
                                        lse[cc] = __ldcg(p.part_lse + it * p.rows + r);
                                        x[cc] = __ldcg(reinterpret_cast<const float2*>(p.part_o + (it * p.rows + r) * kD + d));
                                    } else {
                                        lse[cc] = -INFINITY;
                                        x[cc] = make_float2(0.f, 0.f);
                                    }
                                }
                                const float mx = fmaxf(fmaxf(mrun, fmaxf(lse[0], lse[1])), fmaxf(lse[2], lse[3]));
                                if (mx == -INFINITY) continue;
                                const float sc = mrun == -INFINITY ? 0.f : fast_exp2(mrun - mx);
                                den *= sc;
                                acc0 *= sc;
                                acc1 *= sc;
#pragma unroll
                                for (int cc = 0; cc < 4; ++cc) {
                                    const float w = lse[cc] == -INFINITY ? 0.f : fast_exp2(lse[cc] - mx);
                                    den += w;
                                    acc0 = fmaf(w, x[cc].x, acc0);
                                    acc1 = fmaf(w, x[cc].y, acc1);
                                }
                                mrun = mx;
                            }
                            const float inv = den > 0.f ? 1.f / den : 0.f;
                            const int j = r / p.group, gq = r - j * p.group;
                            *reinterpret_cast<uint32_t*>(p.out + ((int64_t(hd.b) * p.lq + j) * p.hq + hd.h * p.group + gq) * kD +
                                                         d) = pack2<BF16>(acc0 * inv, acc1 * inv);
                        }
                        if (tid == 0) p.counters[hd.b * p.hkv + hd.h] = 0;
                    }
                }
                if (!consumer_sync(&sm.cbar, cphase, p.wait_ns)) {
                    atomicOr(&p.ctrl[2], DEV_ERR_WAIT_PEER);
                    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
                    break;
                }
            }
        }
    }

    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const int done = atomicAdd(&p.ctrl[1], 1);
        if (done == int(gridDim.x) - 1) {
            // Every CTA has stopped claiming items: re-arm the scheduler.
            atomicExch(&p.ctrl[0], 0);
            atomicExch(&p.ctrl[1], 0);
        }
    }
}

// Test hook state of the calling host thread (b200_testing_idle_producer).
thread_local int g_idle_launches = 0;
thread_local uint64_t g_idle_wait_ns = kWaitLimitNs;

// Wait limit and idle-producer flag of the next launch on this host thread.
inline void apply_test_hook(Params& prm) {
    prm.wait_ns = kWaitLimitNs;
    prm.idle_producer = 0;
    if (g_idle_launches > 0) {
        --g_idle_launches;
        prm.wait_ns = g_idle_wait_ns;
        prm.idle_producer = 1;
    }
}

}  // namespace pa
}  // namespace b200

extern "C" int32_t b200_testing_idle_producer(int32_t launches, int64_t wait_limit_ns) {
    using namespace b200;
    clear_error();
    B200_REQUIRE(launches >= 0, "testing_idle_producer: launches %d < 0", launches);
    B200_REQUIRE(wait_limit_ns >= 1000 && wait_limit_ns <= int64_t(kWaitLimitNs),
                 "testing_idle_producer: wait limit %lld ns outside [1 us, 1 s]", (long long)wait_limit_ns);
    pa::g_idle_launches = launches;
    pa::g_idle_wait_ns = uint64_t(wait_limit_ns);
    return B200_OK;
}

extern "C" size_t b200_paged_attention_workspace_size(int32_t max_items, int32_t query_len, int32_t group_size,
                                                      int32_t head_dim) {
    using namespace b200::pa;
    if (max_items < 0 || query_len < 1 || group_size < 1 || head_dim < 1) return 0;
    const size_t rows = size_t(query_len) * group_size;
    const size_t bytes = kFixedBytes + size_t(max_items) * rows * (size_t(head_dim) + 1) * 4;
    return (bytes + 255) & ~size_t(255);
}

extern "C" int32_t b200_paged_attention(void* out, const void* q, int64_t q_stride_token, const void* k_cache,
                                        const void* v_cache, int32_t num_blocks, int32_t block_size,
                                        const int32_t* block_tables, int32_t block_table_stride,
                                        const int32_t* context_lens, int32_t batch, int32_t query_len,
                                        int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                        float softmax_scale, int32_t dtype, void* workspace, size_t workspace_bytes,
                                        void* stream) {
    using namespace b200;
    using namespace b200::pa;
    clear_error();
    B200_REQUIRE(batch >= 0, "paged_attention: batch %d < 0", batch);
    if (batch == 0) return B200_OK;
    B200_REQUIRE(out && q && k_cache && v_cache && block_tables && context_lens, "paged_attention: null pointer");
    B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
                 "paged_attention: num_heads %d not a multiple of num_kv_heads %d", num_heads, num_kv_heads);
    B200_REQUIRE(query_len >= 1, "paged_attention: query_len %d < 1", query_len);
    B200_REQUIRE(softmax_scale > 0.f && softmax_scale <= FLT_MAX, "paged_attention: softmax_scale %g not positive and finite",
                 double(softmax_scale));
    const int group = num_heads / num_kv_heads;
    const int rows = query_len * group;
    if (head_dim != kD) return fail(B200_ERR_UNSUPPORTED, "paged_attention: head_dim %d (only 128)", head_dim);
    if (rows > 16)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention: query_len * Hq/Hkv = %d exceeds 16", rows);
    if (dtype != B200_BF16 && dtype != B200_F16)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention: dtype %d (bf16 or fp16 only)", dtype);
    if (batch > kMaxBatch) return fail(B200_ERR_UNSUPPORTED, "paged_attention: batch %d > %d", batch, kMaxBatch);
    B200_REQUIRE(block_size > 0 && block_size % kTile == 0, "paged_attention: block_size %d not a multiple of %d",
                 block_size, kTile);
    B200_REQUIRE(num_blocks > 0 && int64_t(num_blocks) * block_size < (int64_t(1) << 31),
                 "paged_attention: num_blocks %d out of range", num_blocks);
    B200_REQUIRE(block_table_stride > 0 && int64_t(block_table_stride) * block_size < (int64_t(1) << 31),
                 "paged_attention: block_table_stride %d out of range", block_table_stride);
    B200_REQUIRE(q_stride_token >= int64_t(num_heads) * head_dim && q_stride_token % 2 == 0,
                 "paged_attention: q token stride %lld", (long long)q_stride_token);
    B200_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && q_stride_token % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                 "paged_attention: q and out must be 16-byte aligned, q token stride a multiple of 8");
    if (int64_t(batch) * num_kv_heads > kCounterSlots)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention: batch * num_kv_heads > %d", kCounterSlots);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < kFixedBytes)
        return fail(B200_ERR_WORKSPACE, "paged_attention: workspace missing, unaligned or smaller than %zu bytes",
                    kFixedBytes);
    const int64_t max_items = int64_t(workspace_bytes - kFixedBytes) / (int64_t(rows) * (kD + 1) * 4);
    if (max_items < int64_t(batch) * num_kv_heads)
        return fail(B200_ERR_WORKSPACE, "paged_attention: workspace holds %lld items, batch * Hkv = %lld",
                    (long long)max_items, (long long)batch * num_kv_heads);

    const bool bf16 = dtype == B200_BF16;
    const uint64_t row_elems = uint64_t(num_kv_heads) * kD;
    const uint64_t rows_total = uint64_t(num_blocks) * block_size;
    CUtensorMap tmk, tmv;
    int32_t rc = make_tmap_2d(&tmk, k_cache, row_elems, rows_total, row_elems * 2, 64, kTile, bf16,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tmv, v_cache, row_elems, rows_total, row_elems * 2, 64, kTile, bf16,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;

    Params prm;
    prm.q = static_cast<const uint16_t*>(q);
    prm.q_stride = q_stride_token;
    prm.out = static_cast<uint16_t*>(out);
    prm.block_tables = block_tables;
    prm.bt_stride = block_table_stride;
    prm.context_lens = context_lens;
    prm.batch = batch;
    prm.lq = query_len;
    prm.hq = num_heads;
    prm.hkv = num_kv_heads;
    prm.group = group;
    prm.rows = rows;
    prm.block_size = block_size;
    prm.num_blocks = num_blocks;
    prm.scale_log2 = softmax_scale * 1.4426950408889634f;
    char* ws = static_cast<char*>(workspace);
    prm.ctrl = reinterpret_cast<int32_t*>(ws);
    prm.counters = reinterpret_cast<int32_t*>(ws + kCtrlWords * 4);
    prm.part_o = reinterpret_cast<float*>(ws + kFixedBytes);
    prm.part_lse = prm.part_o + max_items * rows * kD;
    prm.max_items = int32_t(max_items > INT32_MAX / 2 ? INT32_MAX / 2 : max_items);
    apply_test_hook(prm);

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(device_sm_count()), block(kThreads);
    const bool hi = rows > 8;
    const void* fn;
    int smem;
    if (bf16) {
        fn = hi ? (const void*)paged_attention_kernel<true, true> : (const void*)paged_attention_kernel<true, false>;
    } else {
        fn = hi ? (const void*)paged_attention_kernel<false, true> : (const void*)paged_attention_kernel<false, false>;
    }
    smem = hi ? smem_bytes<true>() : smem_bytes<false>();
    ensure_smem_attr(fn, smem);
    if (bf16) {
        if (hi) paged_attention_kernel<true, true><<<grid, block, smem, s>>>(prm, tmk, tmv);
        else paged_attention_kernel<true, false><<<grid, block, smem, s>>>(prm, tmk, tmv);
    } else {
        if (hi) paged_attention_kernel<false, true><<<grid, block, smem, s>>>(prm, tmk, tmv);
        else paged_attention_kernel<false, false><<<grid, block, smem, s>>>(prm, tmk, tmv);
    }
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of b200_paged_attention.
//
// Some callers cannot call cudaMalloc around an attention call: inference
// runtimes whose own allocator owns the whole device heap and hands plugins
// no workspace, plugin hosts that forbid device allocation on the execution
// path, and code that must not risk the implicit device synchronisation of
// cudaMalloc/cudaFree.  For them this entry point keeps the split-K scratch
// (control block, split counters, partial outputs) in a file-scope device
// array of kNoAllocScratchBytes.  Every GPU that loads this library holds
// that array until the process exits.  The array's host-side name is only a
// stand-in for the symbol, so the first call on each device looks up its
// device address with cudaGetSymbolAddress (with that device current) and
// caches it; make that first call before any stream capture.  The cache is
// keyed by the current CUDA context's unique id (cuCtxGetId), so a call made
// in another context on the same device (a driver-API context, or the new
// primary context after cudaDeviceReset) looks the address up again instead
// of reusing one that belongs to a destroyed or different context.  All calls
// share the one array and it keeps the last call's contents: each call
// clears the control words (error word included) and split counters it uses
// before launching, and calls that overlap on the GPU (two streams, two host
// threads) race on it and must be serialised by the caller.
// b200_paged_attention_noalloc_error reads the error word of the latest call.
namespace b200 {
namespace pa {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
constexpr int kNoAllocCounterSlots = 8192;                  // (sequence, kv head) pairs
constexpr size_t kNoAllocFixedBytes = kCtrlWords * 4 + size_t(kNoAllocCounterSlots) * 4;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
struct ScratchAddr {
    unsigned long long ctx_id;  // unique id of the context the address belongs to (0: none yet)
    void* ptr;
};
ScratchAddr g_noalloc_addr[kNoAllocMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
std::once_flag g_ctx_fns_once;

// Unique id of the calling thread's current CUDA context, 0 if there is none
// or the driver does not report it (then nothing is cached).
unsigned long long current_ctx_id() {
    std::call_once(g_ctx_fns_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_id = reinterpret_cast<CtxGetIdFn>(fn);
    });
    if (!g_ctx_current || !g_ctx_id) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of g_noalloc_scratch in the current context of the current
// device: looked up once per (device, context) and cached.
int32_t noalloc_scratch(void** out) {
    int dev = 0;
    B200_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention_noalloc: device %d beyond %d", dev, kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    const unsigned long long id = current_ctx_id();
    if (id != 0 && g_noalloc_addr[dev].ctx_id == id) {
        *out = g_noalloc_addr[dev].ptr;
        return B200_OK;
    }
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
        return fail(B200_ERR_CUDA, "paged_attention_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
    // The lookup makes the runtime's context current if none was: key the cache on it.
    g_noalloc_addr[dev].ctx_id = current_ctx_id();
    g_noalloc_addr[dev].ptr = p;
    *out = p;
    return B200_OK;
}
}  // namespace

}  // namespace pa
}  // namespace b200

extern "C" int32_t b200_paged_attention_noalloc(void* out, const void* q, int64_t q_stride_token,
                                                const void* k_cache, const void* v_cache, int32_t num_blocks,
                                                int32_t block_size, const int32_t* block_tables,
                                                int32_t block_table_stride, const int32_t* context_lens,
                                                int32_t batch, int32_t query_len, int32_t num_heads,
                                                int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                                int32_t dtype, void* stream) {
    using namespace b200;
    using namespace b200::pa;
    clear_error();
    B200_REQUIRE(batch >= 0, "paged_attention_noalloc: batch %d < 0", batch);
    if (batch == 0) return B200_OK;
    B200_REQUIRE(out && q && k_cache && v_cache && block_tables && context_lens,
                 "paged_attention_noalloc: null pointer");
    B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
                 "paged_attention_noalloc: num_heads %d not a multiple of num_kv_heads %d", num_heads, num_kv_heads);
    B200_REQUIRE(query_len >= 1, "paged_attention_noalloc: query_len %d < 1", query_len);
    B200_REQUIRE(softmax_scale > 0.f && softmax_scale <= FLT_MAX,
                 "paged_attention_noalloc: softmax_scale %g not positive and finite", double(softmax_scale));
    const int group = num_heads / num_kv_heads;
    const int rows = query_len * group;
    if (head_dim != kD) return fail(B200_ERR_UNSUPPORTED, "paged_attention_noalloc: head_dim %d (only 128)", head_dim);
    if (rows > 16)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention_noalloc: query_len * Hq/Hkv = %d exceeds 16", rows);
    if (dtype != B200_BF16 && dtype != B200_F16)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention_noalloc: dtype %d (bf16 or fp16 only)", dtype);
    if (batch > kMaxBatch)
        return fail(B200_ERR_UNSUPPORTED, "paged_attention_noalloc: batch %d > %d", batch, kMaxBatch);
    B200_REQUIRE(block_size > 0 && block_size % kTile == 0,
                 "paged_attention_noalloc: block_size %d not a multiple of %d", block_size, kTile);
    B200_REQUIRE(num_blocks > 0 && int64_t(num_blocks) * block_size < (int64_t(1) << 31),
                 "paged_attention_noalloc: num_blocks %d out of range", num_blocks);
    B200_REQUIRE(block_table_stride > 0 && int64_t(block_table_stride) * block_size < (int64_t(1) << 31),
                 "paged_attention_noalloc: block_table_stride %d out of range", block_table_stride);
    B200_REQUIRE(q_stride_token >= int64_t(num_heads) * head_dim && q_stride_token % 2 == 0,
                 "paged_attention_noalloc: q token stride %lld", (long long)q_stride_token);
    B200_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && q_stride_token % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                 "paged_attention_noalloc: q and out must be 16-byte aligned, q token stride a multiple of 8");
    const int64_t pairs = int64_t(batch) * num_kv_heads;
    const int64_t max_items = int64_t(kNoAllocScratchBytes - kNoAllocFixedBytes) / (int64_t(rows) * (kD + 1) * 4);
    if (pairs > kNoAllocCounterSlots || pairs > max_items)
        return fail(B200_ERR_WORKSPACE,
                    "paged_attention_noalloc: batch * num_kv_heads = %lld exceeds the built-in %zu-byte scratch "
                    "(at most %lld pairs for query_len * Hq/Hkv = %d); use b200_paged_attention with a workspace",
                    (long long)pairs, kNoAllocScratchBytes,
                    (long long)(max_items < kNoAllocCounterSlots ? max_items : kNoAllocCounterSlots), rows);

    void* scratch = nullptr;
    int32_t rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Control block (scheduler, finished CTAs, error word) and this call's split counters start at zero.
    B200_CUDA_TRY(cudaMemsetAsync(scratch, 0, kCtrlWords * 4 + size_t(pairs) * 4, s));

    const bool bf16 = dtype == B200_BF16;
    const uint64_t row_elems = uint64_t(num_kv_heads) * kD;
    const uint64_t rows_total = uint64_t(num_blocks) * block_size;
    CUtensorMap tmk, tmv;
    rc = make_tmap_2d(&tmk, k_cache, row_elems, rows_total, row_elems * 2, 64, kTile, bf16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tmv, v_cache, row_elems, rows_total, row_elems * 2, 64, kTile, bf16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;

    Params prm;
    prm.q = static_cast<const uint16_t*>(q);
    prm.q_stride = q_stride_token;
    prm.out = static_cast<uint16_t*>(out);
    prm.block_tables = block_tables;
    prm.bt_stride = block_table_stride;
    prm.context_lens = context_lens;
    prm.batch = batch;
    prm.lq = query_len;
    prm.hq = num_heads;
    prm.hkv = num_kv_heads;
    prm.group = group;
    prm.rows = rows;
    prm.block_size = block_size;
    prm.num_blocks = num_blocks;
    prm.scale_log2 = softmax_scale * 1.4426950408889634f;
    char* ws = static_cast<char*>(scratch);
    prm.ctrl = reinterpret_cast<int32_t*>(ws);
    prm.counters = reinterpret_cast<int32_t*>(ws + kCtrlWords * 4);
    prm.part_o = reinterpret_cast<float*>(ws + kNoAllocFixedBytes);
    prm.part_lse = prm.part_o + max_items * rows * kD;
    prm.max_items = int32_t(max_items);
    apply_test_hook(prm);

    const dim3 grid(device_sm_count()), block(kThreads);
    const bool hi = rows > 8;
    const void* fn;
    if (bf16)
        fn = hi ? (const void*)paged_attention_kernel<true, true> : (const void*)paged_attention_kernel<true, false>;
    else
        fn = hi ? (const void*)paged_attention_kernel<false, true> : (const void*)paged_attention_kernel<false, false>;
    const int smem = hi ? smem_bytes<true>() : smem_bytes<false>();
    ensure_smem_attr(fn, smem);
    if (bf16) {
        if (hi) paged_attention_kernel<true, true><<<grid, block, smem, s>>>(prm, tmk, tmv);
        else paged_attention_kernel<true, false><<<grid, block, smem, s>>>(prm, tmk, tmv);
    } else {
        if (hi) paged_attention_kernel<false, true><<<grid, block, smem, s>>>(prm, tmk, tmv);
        else paged_attention_kernel<false, false><<<grid, block, smem, s>>>(prm, tmk, tmv);
    }
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

extern "C" int32_t b200_paged_attention_noalloc_error(void* stream, int32_t* flag) {
    using namespace b200;
    using namespace b200::pa;
    clear_error();
    B200_REQUIRE(flag != nullptr, "paged_attention_noalloc_error: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The error word is the third int32 of the control block at the start of the scratch.
    B200_CUDA_TRY(cudaMemcpyFromSymbolAsync(flag, g_noalloc_scratch, sizeof(int32_t), 2 * sizeof(int32_t),
                                            cudaMemcpyDeviceToHost, s));
    B200_CUDA_TRY(cudaStreamSynchronize(s));
    return B200_OK;
}
