// Row-parallel output projection fused with its all-reduce over peer memory.
// Replaces, for the attention output projection of a tensor-parallel Qwen3
// layer (nanovllm/models/qwen3.py:87, RowParallelLinear.forward at
// nanovllm/layers/linear.py:152-156):
//     y = F.linear(x_r, W_r)          (this rank's K shard, rounded to bf16)
//     dist.all_reduce(y)              (sum over ranks)
// in one kernel per rank, over buffers every rank can read (CUDA symmetric
// memory; peers are reached with plain loads over NVLink, no multicast):
//   phase 1: persistent CTAs compute 128 x 256 output tiles of y_r with
//            tcgen05 (TMA loads without multicast, SS MMA M=128 N=256, fp32
//            accumulators in tensor memory), round them to bf16, store them
//            in this rank's slot buffer and publish each tile with a
//            system-scope release of its ready flag (= the call's epoch);
//   phase 2: for the same tiles, each CTA waits (bounded) for every rank's
//            ready flag, sums the ranks' bf16 tiles in fp32 in rank order
//            (so every rank gets the same bits) and writes bf16 y.
// Phase 1 never waits on a peer, so phase 2's waits always end.  Slot buffers
// ([2][slot_rows][N] per rank) alternate by epoch parity; the grid's last CTA
// to finish phase 2 publishes the rank's done epoch, and a call waits for
// every rank's done epoch >= epoch - 2 before rewriting its slot (the one
// read two calls ago).  Waits give up after kWaitLimitNs and set the error
// word.  Flags per rank (uint32, zeroed once): [max_tiles] ready epochs,
// then the done epoch, then a local finished-CTA counter.
#include "common.cuh"
#include "tcgen05.cuh"

namespace b200 {
namespace oar {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue; all reduce
constexpr int kABytes = kBM * kBK * 2, kBBytes = kBN * kBK * 2;
constexpr uint32_t kTmemCols = 256;

struct Params {
    uint16_t* out;
    int64_t ldo;
    int32_t M, N, K, rank, world, tiles_n, num_tiles;
    uint32_t epoch;
    uint16_t* const* slots;  // [world] -> each rank's slot buffers: [2][slot_rows][N] bf16
    uint32_t* const* flags;  // [world] -> each rank's flags: [max_tiles] ready, done epoch, CTA counter
    int32_t max_tiles, slot_rows;
};

struct Smem {
    uint8_t a[kStages][kABytes];
    uint8_t b[kStages][kBBytes];
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full, acc_empty, drain;
    uint32_t tmem_base;
    int32_t err;
};

__device__ int32_t g_oar_error;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag >= epoch (epochs only grow); false on timeout.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t epoch) {
    if (ld_acquire_sys(flag) >= epoch) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (ld_acquire_sys(flag) >= epoch) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
        __nanosleep(64);
    }
}

__device__ __forceinline__ void flag_error(Smem& sm, int code) {
    atomicOr(&g_oar_error, code);
    *reinterpret_cast<volatile int32_t*>(&sm.err) = 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    oproj_allreduce_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tma,
                           const __grid_constant__ CUtensorMap tmb) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kb_count = (p.K + kBK - 1) / kBK;
    const int parity = p.epoch & 1;
    uint32_t* my_flags = p.flags[p.rank];
    uint16_t* my_slot = p.slots[p.rank] + size_t(parity) * p.slot_rows * p.N;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        mbar_init(&sm.acc_full, 1);
        mbar_init(&sm.acc_empty, 128);
        mbar_init(&sm.drain, 1);
        sm.err = 0;
        fence_mbar_init();
        // this call rewrites the slot every rank read two calls ago
        if (p.epoch > 2)
            for (int r = 0; r < p.world; ++r)
                if (!wait_flag(p.flags[r] + p.max_tiles, p.epoch - 2)) {
                    atomicOr(&g_oar_error, 8);
                    sm.err = 1;
                }
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
            const uint64_t pol = l2_policy_evict_first();
            int g = 0;
            for (int t = blockIdx.x; t < p.num_tiles && !failed(); t += gridDim.x) {
                const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * kBN;
                for (int kb = 0; kb < kb_count; ++kb, ++g) {
                    const int st = g % kStages;
                    if (!mbar_wait(&sm.empty[st], ((g / kStages) & 1) ^ 1)) { flag_error(sm, 1); break; }
                    mbar_arrive_expect_tx(&sm.full[st], kABytes + kBBytes);
                    tma_load_2d(sm.a[st], &tma, kb * kBK, m0, &sm.full[st], pol);
                    tma_load_2d(sm.b[st], &tmb, kb * kBK, n0, &sm.full[st], pol);
                }
            }
            // every load issued above has landed before the CTA exits (bounded)
            for (int st = 0; st < kStages && st < g; ++st) {
                const int last = st + ((g - 1 - st) / kStages) * kStages;
                mbar_wait(&sm.full[st], (last / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16<true>(kBM, kBN, false, false);
            int g = 0, n_acc = 0;
            for (int t = blockIdx.x; t < p.num_tiles && !failed(); t += gridDim.x, ++n_acc) {
                // the epilogue must have read the previous tile's accumulator
                if (n_acc > 0 && !mbar_wait(&sm.acc_empty, (n_acc - 1) & 1)) { flag_error(sm, 2); break; }
                tc::fence_after_sync();
                for (int kb = 0; kb < kb_count; ++kb, ++g) {
                    const int st = g % kStages;
                    if (!mbar_wait(&sm.full[st], (g / kStages) & 1)) { flag_error(sm, 2); break; }
                    tc::fence_after_sync();
                    const uint32_t aa = smem_u32(sm.a[st]), ba = smem_u32(sm.b[st]);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        tc::mma_ss(tmem, tc::smem_desc_sw128(aa + kk * 32, 16, 1024),
                                   tc::smem_desc_sw128(ba + kk * 32, 16, 1024), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    tc::commit(&sm.empty[st]);
                }
                tc::commit(&sm.acc_full);
            }
            tc::commit(&sm.drain);  // every MMA issued above has completed before TMEM is freed
            mbar_wait(&sm.drain, 0);
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4).., one output row per thread
        const int q = warp & 3, row_in = q * 32 + lane;
        int n_acc = 0;
        for (int t = blockIdx.x; t < p.num_tiles && !failed(); t += gridDim.x, ++n_acc) {
            const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * kBN;
            if (!mbar_wait(&sm.acc_full, n_acc & 1)) { flag_error(sm, 4); break; }
            tc::fence_after_sync();
            const int row = m0 + row_in;
            const uint32_t lane_addr = uint32_t(q * 32) << 16;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                tc::tmem_ld32(tmem + lane_addr + c * 32, v);
                tc::tmem_wait_ld();
                if (row < p.M) {
                    uint4* dst = reinterpret_cast<uint4*>(my_slot + size_t(row) * p.N + n0 + c * 32);
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 o;
                        o.x = pack2<true>(v[e], v[e + 1]);
                        o.y = pack2<true>(v[e + 2], v[e + 3]);
                        o.z = pack2<true>(v[e + 4], v[e + 5]);
                        o.w = pack2<true>(v[e + 6], v[e + 7]);
                        dst[e / 8] = o;
                    }
                }
            }
            tc::fence_before_sync();
            mbar_arrive(&sm.acc_empty);
            // publish the tile: every epilogue thread's stores, then one system-scope release
            __threadfence_system();
            named_bar_sync(1, 128);
            if (row_in == 0) st_release_sys(my_flags + t, p.epoch);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }

    // ------------------------------------------------------------------ phase 2
    __shared__ int ready_ok;
    const uint16_t* const* slots = p.slots;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * kBN;
        if (tid == 0) {
            int ok = !failed();
            for (int r = 0; r < p.world && ok; ++r)
                if (!wait_flag(p.flags[r] + t, p.epoch)) ok = 0;
            if (!ok) flag_error(sm, 16);
            ready_ok = ok;
        }
        __syncthreads();
        if (!ready_ok) break;
        // 128 x 256 bf16 tile = 4096 16-byte groups; sum the ranks' copies in rank order
        for (int i = tid; i < kBM * kBN / 8; i += kThreads) {
            const int r_in = i / (kBN / 8), c8 = i % (kBN / 8);
            const int row = m0 + r_in;
            if (row >= p.M) continue;
            const size_t off = size_t(parity) * p.slot_rows * p.N + size_t(row) * p.N + n0 + c8 * 8;
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int r = 0; r < p.world; ++r) {
                const uint4 v = __ldcg(reinterpret_cast<const uint4*>(slots[r] + off));
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc[2 * e] += __uint_as_float(w[e] << 16);
                    acc[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
                }
            }
            uint4 o;
            o.x = pack2<true>(acc[0], acc[1]);
            o.y = pack2<true>(acc[2], acc[3]);
            o.z = pack2<true>(acc[4], acc[5]);
            o.w = pack2<true>(acc[6], acc[7]);
            *reinterpret_cast<uint4*>(p.out + int64_t(row) * p.ldo + n0 + c8 * 8) = o;
        }
        __syncthreads();
    }
    // The last CTA to finish publishes that this rank has read every slot of this epoch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(my_flags + p.max_tiles + 1, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            my_flags[p.max_tiles + 1] = 0;
            st_release_sys(my_flags + p.max_tiles, p.epoch);
        }
    }
}

}  // namespace oar
}  // namespace b200

extern "C" int32_t b200_oproj_allreduce(void* out, int64_t ldo, const void* a, int64_t lda, const void* w,
                                        int64_t ldw, int32_t M, int32_t N, int32_t K, void* const* slots,
                                        int32_t slot_rows, uint32_t* const* flags, int32_t max_tiles,
                                        int32_t rank, int32_t world, uint32_t epoch, void* stream) {
    using namespace b200;
    using namespace b200::oar;
    clear_error();
    B200_REQUIRE(M >= 0 && N > 0 && K > 0, "oproj_allreduce: M %d N %d K %d", M, N, K);
    if (M == 0) return B200_OK;
    B200_REQUIRE(out && a && w && slots && flags, "oproj_allreduce: null pointer");
    B200_REQUIRE(world >= 1 && rank >= 0 && rank < world, "oproj_allreduce: rank %d of %d", rank, world);
    B200_REQUIRE(epoch >= 1, "oproj_allreduce: epochs start at 1");
    if (N % kBN != 0 || K % kBK != 0)
        return fail(B200_ERR_UNSUPPORTED, "oproj_allreduce: N %% 256 and K %% 64 must be 0 (N %d, K %d)", N, K);
    B200_REQUIRE(ldo >= N && lda >= K && ldw >= K && ldo % 8 == 0, "oproj_allreduce: strides");
    const int tiles_n = N / kBN, tiles_m = (M + kBM - 1) / kBM;
    const int num_tiles = tiles_m * tiles_n;
    B200_REQUIRE(num_tiles <= max_tiles, "oproj_allreduce: %d tiles > flag capacity %d", num_tiles, max_tiles);
    B200_REQUIRE(M <= slot_rows, "oproj_allreduce: M %d > slot rows %d", M, slot_rows);
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
    p.num_tiles = num_tiles;
    p.epoch = epoch;
    p.slots = reinterpret_cast<uint16_t* const*>(slots);
    p.flags = flags;
    p.max_tiles = max_tiles;
    p.slot_rows = slot_rows;
    const int smem = int(sizeof(Smem)) + 1024;
    ensure_smem_attr((const void*)oproj_allreduce_kernel, smem);
    const int grid = num_tiles < device_sm_count() ? num_tiles : device_sm_count();
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
