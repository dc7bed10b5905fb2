// Row-parallel output projection fused with its all-reduce over peer memory.
// Replaces, for the attention output projection of a tensor-parallel Qwen3
// layer (nanovllm/models/qwen3.py:87, RowParallelLinear.forward at
// nanovllm/layers/linear.py:152-156):
//     y = F.linear(x_r, W_r)          (this rank's K shard, rounded to bf16)
//     dist.all_reduce(y)              (sum over ranks)
// in one kernel per rank over buffers every rank can address (CUDA symmetric
// memory; peers are reached with plain stores over NVLink, no multicast).
//
// Work unit = (128 x 256 output tile, K split).  Few tiles (decode batches)
// are split along K so that every SM has a unit; many tiles run unsplit on
// persistent CTAs.
//   phase 1  tcgen05 GEMM: TMA loads (no multicast), SS MMA M=128 N=256 into
//            one of two fp32 accumulators in tensor memory.  Unsplit tiles are
//            rounded to bf16 and PUSHED into every rank's slot buffer (this
//            rank's source region), then published with a system-scope release
//            of a ready flag on every rank (after a CTA barrier: the release is
//            cumulative, so no per-thread system fence is needed).  Split tiles
//            stage their fp32 partial in shared memory and write it to a local
//            workspace with one bulk copy, then release a local arrival flag.
//   phase 1b (split tiles) each of a tile's `splits` CTAs sums the tile's fp32
//            partials for its share of the rows, in split order (deterministic),
//            rounds to bf16 and pushes / publishes as above.
//   phase 2  for its rows, each CTA waits (bounded) for every rank's ready flag,
//            sums the ranks' bf16 partials from LOCAL memory in fp32 in rank
//            order (every rank gets the same bits) and writes bf16 y.
// Low-latency slots (split calls with M <= ll_rows, i.e. decode batches): each
// 8-byte word holds two bf16 values and the epoch, written with single 16-byte
// stores (8-byte halves are single-copy atomic), and readers poll the words
// themselves: no ready flags, no system-scope release or acquire on the path,
// at twice the bytes over NVLink.
// Phases 1 and 1b wait only on CTAs of this grid on this GPU (all resident: the
// grid never exceeds the SM count and a CTA fills an SM), so phase 2's waits end.
//
// Epochs: the call's epoch is read from this rank's flag words (the grid's last
// CTA of the previous call left it there), so a launch captured in a CUDA graph
// stays correct.  Slot buffers [2][world][slot_rows][N] alternate by epoch
// parity.  Rewriting a slot needs no extra handshake: a rank pushes epoch e+2
// only after its own call e+1 ended, which waited for every rank's e+1 ready
// flags; a rank publishes those only after its call e (its last read of that
// parity) ended.  Unit 0 always has rows, so every call carries such a flag.
// Epoch 0 is skipped when the counter wraps (zeroed words never look current).
// A peer may already have published the NEXT epoch into a ready flag (it ran
// ahead by one call), never the one after.  Waits poll with one lane per flag,
// give up after kWaitLimitNs and set the error word.  Flag words per rank (uint32,
// zeroed once): [max_units][world] ready epochs, a finished-CTA counter, the
// last epoch.
#include "common.cuh"
#include "peer_sync.cuh"
#include "tcgen05.cuh"

namespace b200 {
namespace oar {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue; all: 1b, 2
constexpr int kABytes = kBM * kBK * 2, kBBytes = kBN * kBK * 2;
constexpr uint32_t kTmemCols = 512;  // two 256-column fp32 accumulators
constexpr int kMaxSplits = 16;
constexpr int kArriveWords = 256;  // workspace head: per-unit split arrival epochs (units <= SM count)

struct Params {
    uint16_t* out;
    int64_t ldo;
    int32_t M, N, K, rank, world, tiles_n, splits, num_units, kb_count;
    uint16_t* const* slots;   // [world] -> each rank's slots: [2][world][slot_rows][N] bf16
    uint32_t* const* ll;      // [world] -> each rank's low-latency slots [2][world][ll_rows][N/2] x (2 bf16, epoch)
    uint32_t* const* flags;   // [world] -> each rank's flag words
    int32_t max_units, slot_rows, ll_rows, use_ll;
    uint32_t* arrive;  // local [kArriveWords] split arrival epochs
    float* part;       // local [units][kBM][kBN] fp32 split partials
};

struct Smem {
    uint8_t a[kStages][kABytes];  // a and b are contiguous: phase 1b stages partials here
    uint8_t b[kStages][kBBytes];
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2], drain, fix;
    uint32_t tmem_base;
    int32_t err, ok;
};

__device__ int32_t g_oar_error;

// Bulk copy shared -> global (no multicast): start, then wait until the writes are performed.
// Every thread that wrote the source executed fence_proxy_async_smem() before the barrier
// that precedes this call.
__device__ __forceinline__ void bulk_store_wait(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_volatile_v4(uint32_t* p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// Named barrier that returns, to every participating thread, the OR of `pred`:
// loop exits decided with it are uniform, so no thread is left at a later barrier.
__device__ __forceinline__ bool named_bar_any(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, %2, %3, p;\nselp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(uint32_t(pred)), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void flag_error(Smem& sm, int code) {
    atomicOr(&g_oar_error, code);
    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
}

// Rows [r0, r1) of unit u's tile that unit u reduces (phase 1b) and all-reduces (phase 2).
struct UnitRows {
    int t, s, m0, n0, r0, r1;
};
__device__ __forceinline__ UnitRows unit_rows(const Params& p, int u) {
    UnitRows r;
    r.t = u / p.splits;
    r.s = u - r.t * p.splits;
    r.m0 = (r.t / p.tiles_n) * kBM;
    r.n0 = (r.t % p.tiles_n) * kBN;
    const int valid = min(kBM, p.M - r.m0);
    const int per = (valid + p.splits - 1) / p.splits;
    r.r0 = min(valid, r.s * per);
    r.r1 = min(valid, r.r0 + per);
    return r;
}

__device__ __forceinline__ uint4 pack8(const float* v) {
    uint4 o;
    o.x = pack2<true>(v[0], v[1]);
    o.y = pack2<true>(v[2], v[3]);
    o.z = pack2<true>(v[4], v[5]);
    o.w = pack2<true>(v[6], v[7]);
    return o;
}

__global__ void __launch_bounds__(kThreads, 1)
    oproj_allreduce_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tma,
                           const __grid_constant__ CUtensorMap tmb) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* my_flags = p.flags[p.rank];
    const int fl_count = p.max_units * p.world;  // finished-CTA counter, then the last epoch
    const uint32_t epoch = next_epoch(__ldcg(my_flags + fl_count + 1));
    const int parity = epoch & 1;
    const size_t slot_half = size_t(p.world) * p.slot_rows * p.N;
    // this rank's source region inside every rank's slot buffer
    const size_t push_off = size_t(parity) * slot_half + size_t(p.rank) * p.slot_rows * p.N;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.acc_full[b], 1);
            mbar_init(&sm.acc_empty[b], 128);
        }
        mbar_init(&sm.drain, 1);
        mbar_init(&sm.fix, 1);
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
    auto failed = [&]() { return *reinterpret_cast<volatile int32_t*>(&sm.err) != 0; };

    // ------------------------------------------------------------------ phase 1
    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tma);
            prefetch_tmap(&tmb);
            const uint64_t pol_a = l2_policy_evict_last(), pol_w = l2_policy_evict_first();
            int g = 0;
            for (int u = blockIdx.x; u < p.num_units && !failed(); u += gridDim.x) {
                const UnitRows ur = unit_rows(p, u);
                const int kb0 = ur.s * p.kb_count / p.splits, kb1 = (ur.s + 1) * p.kb_count / p.splits;
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int st = g % kStages;
                    if (!mbar_wait(&sm.empty[st], ((g / kStages) & 1) ^ 1)) { flag_error(sm, 1); break; }
                    mbar_arrive_expect_tx(&sm.full[st], kABytes + kBBytes);
                    tma_load_2d(sm.a[st], &tma, kb * kBK, ur.m0, &sm.full[st], pol_a);
                    tma_load_2d(sm.b[st], &tmb, kb * kBK, ur.n0, &sm.full[st], pol_w);
                }
            }
            // every load issued above has landed before the stages are reused or the CTA exits (bounded)
            for (int st = 0; st < kStages && st < g; ++st) {
                const int last = st + ((g - 1 - st) / kStages) * kStages;
                mbar_wait(&sm.full[st], (last / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16<true>(kBM, kBN, false, false);
            int g = 0, n_acc = 0;
            for (int u = blockIdx.x; u < p.num_units && !failed(); u += gridDim.x, ++n_acc) {
                const UnitRows ur = unit_rows(p, u);
                const int kb0 = ur.s * p.kb_count / p.splits, kb1 = (ur.s + 1) * p.kb_count / p.splits;
                const int buf = n_acc & 1;
                // the epilogue has read this accumulator's previous unit
                if (n_acc >= 2 && !mbar_wait(&sm.acc_empty[buf], ((n_acc >> 1) - 1) & 1)) {
                    flag_error(sm, 2);
                    break;
                }
                tc::fence_after_sync();
                const uint32_t acc = tmem + uint32_t(buf * kBN);
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int st = g % kStages;
                    if (!mbar_wait(&sm.full[st], (g / kStages) & 1)) { flag_error(sm, 2); break; }
                    tc::fence_after_sync();
                    const uint32_t aa = smem_u32(sm.a[st]), ba = smem_u32(sm.b[st]);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        tc::mma_ss(acc, tc::smem_desc_sw128(aa + kk * 32, 16, 1024),
                                   tc::smem_desc_sw128(ba + kk * 32, 16, 1024), idesc,
                                   (kb > kb0 || kk > 0) ? 1u : 0u);
                    tc::commit(&sm.empty[st]);
                }
                tc::commit(&sm.acc_full[buf]);
            }
            tc::commit(&sm.drain);  // every MMA issued above has completed before TMEM is freed
            mbar_wait(&sm.drain, 0);
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4).., one output row per thread
        const int q = warp & 3, row_in = q * 32 + lane;
        int n_acc = 0;
        for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++n_acc) {
            const UnitRows ur = unit_rows(p, u);
            const int buf = n_acc & 1;
            const bool got = mbar_wait(&sm.acc_full[buf], (n_acc >> 1) & 1);
            if (!got) flag_error(sm, 4);
            if (named_bar_any(1, 128, !got || failed())) break;
            tc::fence_after_sync();
            const uint32_t taddr = tmem + uint32_t(buf * kBN) + (uint32_t(q * 32) << 16);
            const bool live = row_in < ur.r1;  // unsplit: r0 = 0, r1 = valid rows
            if (p.splits == 1) {
                const size_t row_off = push_off + size_t(ur.m0 + row_in) * p.N + ur.n0;
#pragma unroll 1
                for (int c = 0; c < kBN / 32; ++c) {
                    float v[32];
                    tc::tmem_ld32(taddr + c * 32, v);
                    tc::tmem_wait_ld();
                    if (live) {
                        const uint4 o0 = pack8(v), o1 = pack8(v + 8), o2 = pack8(v + 16), o3 = pack8(v + 24);
                        for (int r = 0; r < p.world; ++r) {
                            uint4* dst = reinterpret_cast<uint4*>(p.slots[r] + row_off + c * 32);
                            dst[0] = o0;
                            dst[1] = o1;
                            dst[2] = o2;
                            dst[3] = o3;
                        }
                    }
                }
                tc::fence_before_sync();
                mbar_arrive(&sm.acc_empty[buf]);
                // publish: every epilogue thread's stores, then one system-scope release per rank
                named_bar_sync(1, 128);
                if (row_in < p.world) st_release_sys(p.flags[row_in] + u * p.world + p.rank, epoch);
            } else {
                // One unit per CTA: every MMA has completed, so the operand stages are free.
                // Row r's 16-byte chunk j goes to chunk j ^ (r & 7) of its 1 KB row (conflict-free
                // stores); the summing side undoes the swizzle.
                float* srow = reinterpret_cast<float*>(&sm.a[0][0]) + row_in * kBN;
                const int valid = min(kBM, p.M - ur.m0);
#pragma unroll 1
                for (int c = 0; c < kBN / 32; ++c) {
                    float v[32];
                    tc::tmem_ld32(taddr + c * 32, v);
                    tc::tmem_wait_ld();
                    if (row_in < valid) {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            *reinterpret_cast<float4*>(srow + (((c * 8 + e) ^ (row_in & 7)) * 4)) =
                                make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
                    }
                }
                fence_proxy_async_smem();
                tc::fence_before_sync();
                mbar_arrive(&sm.acc_empty[buf]);
                named_bar_sync(1, 128);
                if (row_in == 0) {
                    bulk_store_wait(p.part + size_t(u) * kBM * kBN, &sm.a[0][0], uint32_t(valid) * kBN * 4);
                    st_release_gpu(p.arrive + u, epoch);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }

    // ----------------------------------------------------------------- phase 1b
    if (p.splits > 1) {
        const int u = blockIdx.x;  // one unit per CTA when split
        const UnitRows ur = unit_rows(p, u);
        float* stage = reinterpret_cast<float*>(&sm.a[0][0]);
        const uint32_t part_bytes = uint32_t(ur.r1 - ur.r0) * kBN * 4;
        if (warp == 0) {
            // every lane takes part in the warp-collective wait
            const bool arrived = warp_wait_flags<false>(p.arrive + ur.t * p.splits, 1, p.splits, epoch);
            const bool ok = arrived && !failed();
            if (!ok && lane == 0) flag_error(sm, 32);
            if (ok && part_bytes && lane == 0) {
                // the partials were written through the generic proxy; the bulk copies read them
                asm volatile("fence.proxy.async.global;" ::: "memory");
                mbar_arrive_expect_tx(&sm.fix, part_bytes * p.splits);
                for (int s = 0; s < p.splits; ++s)
                    bulk_load(reinterpret_cast<uint8_t*>(stage) + size_t(s) * part_bytes,
                              p.part + (size_t(ur.t * p.splits + s) * kBM + ur.r0) * kBN, part_bytes, &sm.fix);
            }
            if (lane == 0) sm.ok = ok;
        }
        __syncthreads();
        const bool go = sm.ok && part_bytes && !failed();
        if (go) {
            if (!mbar_wait(&sm.fix, 0)) flag_error(sm, 32);
            const int items = (ur.r1 - ur.r0) * (kBN / 8);
            const int part_floats = (ur.r1 - ur.r0) * kBN;
            for (int i = tid; i < items && !failed(); i += kThreads) {
                // item i: physical chunks 2k, 2k+1 of its staged row hold logical chunks
                // (2k, 2k+1) ^ (row & 7): the 8 columns at 8 * (k ^ ((row & 7) >> 1)), swapped
                // halves when row is odd
                float acc[8];
                const float4* s0 = reinterpret_cast<const float4*>(stage + i * 8);
                float4 x = s0[0], y = s0[1];
                acc[0] = x.x, acc[1] = x.y, acc[2] = x.z, acc[3] = x.w;
                acc[4] = y.x, acc[5] = y.y, acc[6] = y.z, acc[7] = y.w;
                for (int s = 1; s < p.splits; ++s) {
                    const float4* sp = reinterpret_cast<const float4*>(stage + size_t(s) * part_floats + i * 8);
                    x = sp[0];
                    y = sp[1];
                    acc[0] += x.x, acc[1] += x.y, acc[2] += x.z, acc[3] += x.w;
                    acc[4] += y.x, acc[5] += y.y, acc[6] += y.z, acc[7] += y.w;
                }
                const int row = ur.r0 + i / (kBN / 8), k = i % (kBN / 8);
                const int sw = row & 7, c8 = k ^ (sw >> 1);
                uint4 o = pack8(acc);
                if (sw & 1) o = make_uint4(o.z, o.w, o.x, o.y);
                if (p.use_ll) {
                    // 4 words (2 bf16 + epoch each) in two 16-byte stores; M <= ll_rows so m0 == 0
                    const size_t w = (size_t(parity) * p.world + p.rank) * p.ll_rows * (p.N / 2) +
                                     (size_t(row) * p.N + ur.n0 + c8 * 8) / 2;
                    const uint4 w0 = make_uint4(o.x, epoch, o.y, epoch), w1 = make_uint4(o.z, epoch, o.w, epoch);
                    for (int r = 0; r < p.world; ++r) {
                        st_volatile_v4(p.ll[r] + 2 * w, w0);
                        st_volatile_v4(p.ll[r] + 2 * w + 4, w1);
                    }
                } else {
                    const size_t off = push_off + size_t(ur.m0 + row) * p.N + ur.n0 + c8 * 8;
                    for (int r = 0; r < p.world; ++r) *reinterpret_cast<uint4*>(p.slots[r] + off) = o;
                }
            }
        }
        __syncthreads();
        if (go && !p.use_ll && !failed() && tid < p.world)
            st_release_sys(p.flags[tid] + u * p.world + p.rank, epoch);
    }

    // ------------------------------------------------------------------ phase 2
    const uint16_t* local = p.slots[p.rank] + size_t(parity) * slot_half;
    const size_t src_stride = size_t(p.slot_rows) * p.N;
    if (p.use_ll) {
        // one unit per CTA (split); poll this CTA's rows' words from every rank, sum in rank order
        const UnitRows ur = unit_rows(p, blockIdx.x);
        const uint32_t* ll_local = p.ll[p.rank] + size_t(parity) * p.world * p.ll_rows * p.N;
        const size_t src_words = size_t(p.ll_rows) * (p.N / 2);
        const int items = (ur.r1 - ur.r0) * (kBN / 8);
        constexpr int kMaxWorld = 8;
        for (int i = tid; i < items && !failed(); i += kThreads) {
            const int row = ur.r0 + i / (kBN / 8), c8 = i % (kBN / 8);
            const size_t w = (size_t(row) * p.N + ur.n0 + c8 * 8) / 2;
            uint4 v0[kMaxWorld], v1[kMaxWorld];
            bool all = true;
#pragma unroll
            for (int r = 0; r < kMaxWorld; ++r)
                if (r < p.world) {
                    v0[r] = ld_volatile_v4(ll_local + 2 * (r * src_words + w));
                    v1[r] = ld_volatile_v4(ll_local + 2 * (r * src_words + w) + 4);
                    all = all && v0[r].y == epoch && v0[r].w == epoch && v1[r].y == epoch && v1[r].w == epoch;
                }
            if (!all) {
                const uint64_t t0 = global_timer_ns();
                while (!all) {
                    all = true;
#pragma unroll
                    for (int r = 0; r < kMaxWorld; ++r)
                        if (r < p.world && !(v0[r].y == epoch && v0[r].w == epoch && v1[r].y == epoch &&
                                             v1[r].w == epoch)) {
                            v0[r] = ld_volatile_v4(ll_local + 2 * (r * src_words + w));
                            v1[r] = ld_volatile_v4(ll_local + 2 * (r * src_words + w) + 4);
                            all = all && v0[r].y == epoch && v0[r].w == epoch && v1[r].y == epoch &&
                                  v1[r].w == epoch;
                        }
                    if (!all && global_timer_ns() - t0 > kWaitLimitNs) {
                        flag_error(sm, 16);
                        break;
                    }
                }
            }
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < kMaxWorld; ++r)
                if (r < p.world) {
                    const uint32_t d[4] = {v0[r].x, v0[r].z, v1[r].x, v1[r].z};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[2 * e] += __uint_as_float(d[e] << 16);
                        acc[2 * e + 1] += __uint_as_float(d[e] & 0xFFFF0000u);
                    }
                }
            *reinterpret_cast<uint4*>(p.out + int64_t(row) * p.ldo + ur.n0 + c8 * 8) = pack8(acc);
        }
    }
    for (int u = blockIdx.x; u < p.num_units && !p.use_ll; u += gridDim.x) {
        const UnitRows ur = unit_rows(p, u);
        if (ur.r0 >= ur.r1) continue;
        if (warp == 0) {
            const bool ready = warp_wait_flags<true>(my_flags + u * p.world, 1, p.world, epoch);
            const bool ok = ready && !failed();
            if (lane == 0) {
                if (!ok) flag_error(sm, 16);
                sm.ok = ok;
            }
        }
        __syncthreads();
        if (!sm.ok) break;
        const int items = (ur.r1 - ur.r0) * (kBN / 8);
        constexpr int kU = 4;
        for (int i0 = tid; i0 < items; i0 += kThreads * kU) {
            float acc[kU][8];
            size_t off[kU];
#pragma unroll
            for (int j = 0; j < kU; ++j) {
                const int i = min(i0 + j * kThreads, items - 1);
                off[j] = size_t(ur.m0 + ur.r0 + i / (kBN / 8)) * p.N + ur.n0 + (i % (kBN / 8)) * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[j][e] = 0.f;
            }
            for (int r = 0; r < p.world; ++r) {
                uint4 v[kU];
#pragma unroll
                for (int j = 0; j < kU; ++j) v[j] = __ldcg(reinterpret_cast<const uint4*>(local + r * src_stride + off[j]));
#pragma unroll
                for (int j = 0; j < kU; ++j) {
                    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[j][2 * e] += __uint_as_float(w[e] << 16);
                        acc[j][2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kU; ++j) {
                const int i = i0 + j * kThreads;
                if (i >= items) break;
                const int row = ur.m0 + ur.r0 + i / (kBN / 8);
                *reinterpret_cast<uint4*>(p.out + int64_t(row) * p.ldo + ur.n0 + (i % (kBN / 8)) * 8) = pack8(acc[j]);
            }
        }
        __syncthreads();
    }
    // The last CTA to finish (every CTA has read the epoch by then) leaves it for the next call.
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(my_flags + fl_count, 1u);
        if (prev == gridDim.x - 1) {
            my_flags[fl_count] = 0;
            my_flags[fl_count + 1] = epoch;
        }
    }
}

}  // namespace oar
}  // namespace b200

extern "C" int64_t b200_oproj_allreduce_workspace_size(void) {
    using namespace b200;
    return int64_t(oar::kArriveWords) * 4 + int64_t(device_sm_count()) * oar::kBM * oar::kBN * 4;
}

extern "C" int32_t b200_oproj_allreduce(void* out, int64_t ldo, const void* a, int64_t lda, const void* w,
                                        int64_t ldw, int32_t M, int32_t N, int32_t K, void* const* slots,
                                        int32_t slot_rows, uint32_t* const* ll_slots, int32_t ll_rows,
                                        uint32_t* const* flags, int32_t max_units,
                                        void* workspace, int64_t workspace_bytes, int32_t rank, int32_t world,
                                        void* stream) {
    using namespace b200;
    using namespace b200::oar;
    clear_error();
    B200_REQUIRE(M >= 0 && N > 0 && K > 0, "oproj_allreduce: M %d N %d K %d", M, N, K);
    if (M == 0) return B200_OK;
    B200_REQUIRE(out && a && w && slots && flags, "oproj_allreduce: null pointer");
    B200_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world, "oproj_allreduce: rank %d of %d", rank,
                 world);
    if (N % kBN != 0 || K % kBK != 0)
        return fail(B200_ERR_UNSUPPORTED, "oproj_allreduce: N %% 256 and K %% 64 must be 0 (N %d, K %d)", N, K);
    B200_REQUIRE(ldo >= N && lda >= K && ldw >= K && ldo % 8 == 0, "oproj_allreduce: strides");
    const int tiles_n = N / kBN, tiles_m = (M + kBM - 1) / kBM;
    const int num_tiles = tiles_m * tiles_n, kb_count = K / kBK;
    const int sms = device_sm_count();
    B200_REQUIRE(num_tiles <= max_units, "oproj_allreduce: %d tiles > flag capacity %d", num_tiles, max_units);
    B200_REQUIRE(M <= slot_rows, "oproj_allreduce: M %d > slot rows %d", M, slot_rows);
    // split K while that gives every SM a unit and the workspace holds the partials
    int splits = 1;
    if (workspace && workspace_bytes >= b200_oproj_allreduce_workspace_size()) {
        splits = sms / num_tiles;
        splits = splits < kMaxSplits ? splits : kMaxSplits;
        splits = splits < kb_count ? splits : kb_count;
        if (num_tiles * splits > max_units) splits = max_units / num_tiles;
        if (num_tiles * splits > kArriveWords) splits = kArriveWords / num_tiles;
        if (splits < 1) splits = 1;
    }
    CUtensorMap tma, tmb;
    int32_t rc = make_tmap_2d(&tma, a, uint64_t(K), uint64_t(M), uint64_t(lda) * 2, kBK, kBM, true,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tmb, w, uint64_t(K), uint64_t(N), uint64_t(ldw) * 2, kBK, kBN, true, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Params p;
    p.out = static_cast<uint16_t*>(out);
    p.ldo = ldo;
    p.M = M;
    p.N = N;
    p.K = K;
    p.rank = rank;
    p.world = world;
    p.tiles_n = tiles_n;
    p.splits = splits;
    p.num_units = num_tiles * splits;
    p.kb_count = kb_count;
    p.slots = reinterpret_cast<uint16_t* const*>(slots);
    p.flags = flags;
    p.max_units = max_units;
    p.slot_rows = slot_rows;
    p.ll = ll_slots;
    p.ll_rows = ll_rows;
    p.use_ll = splits > 1 && ll_slots != nullptr && M <= ll_rows && M <= kBM;
    p.arrive = static_cast<uint32_t*>(workspace);
    p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kArriveWords * 4);
    const int smem = int(sizeof(Smem)) + 1024;
    ensure_smem_attr((const void*)oproj_allreduce_kernel, smem);
    const int grid = p.num_units < sms ? p.num_units : sms;
    oproj_allreduce_kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(p, tma, tmb);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

extern "C" int32_t b200_oproj_allreduce_error(void* stream, int32_t* flag) {
    using namespace b200;
    B200_REQUIRE(flag != nullptr, "oproj_allreduce_error: null pointer");
    B200_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    B200_CUDA_TRY(cudaMemcpyFromSymbol(flag, b200::oar::g_oar_error, sizeof(int32_t)));
    return B200_OK;
}
