// All-reduce (sum) of a bf16 vector over the GPUs of a tensor-parallel group,
// through buffers every rank maps (CUDA symmetric memory; plain loads and
// stores over NVLink, no multicast).  Replaces, for decode-sized tensors, the
// NCCL call that ends a row-parallel layer (nanovllm/layers/linear.py:155,
// dist.all_reduce(y) after o_proj and down_proj).
//
// Two shots, as reduce-scatter + all-gather.  The vector is cut into `world`
// slices (16-byte units) and every slice into one sub-chunk per CTA; CTA c of
// every rank handles sub-chunk c of every slice, so CTAs synchronise only with
// their counterparts on the other GPUs (no grid-wide barrier):
//   1. copy the input's sub-chunks c into this rank's symmetric input slot
//      (nothing to copy when the caller built the input there), then release
//      flag (phase 1, src = rank, c) on every rank;
//   2. wait for every rank's phase-1 flag c, sum sub-chunk c of slice `rank`
//      over the ranks' input slots (peer loads, fp32, rank order), round once
//      to bf16 and store the result into every rank's result slot (peer
//      stores), then release flag (phase 2, rank, c) on every rank;
//   3. wait for every rank's phase-2 flag c and copy the result sub-chunks c
//      of every slice out (nothing to copy when the caller reads the result
//      slot itself).
// Each slice is reduced by one rank and broadcast, so every rank gets the
// same bits.  Per rank that is 2 (world - 1) / world of the vector over
// NVLink each way, against world - 1 times the vector for a one-shot scheme.
// Releases are system-scope stores after a CTA barrier (cumulative over the
// CTA's writes); waits poll with one lane per flag and give up after
// kWaitLimitNs, setting the error word, so a missing peer never hangs a GPU.
// All CTAs of the grid are resident (grid <= SM count, one CTA fits an SM),
// and a CTA waits only for CTAs of the same index on other GPUs.
//
// Epochs and slots: the call's epoch is read from this rank's flag words,
// where the grid's last CTA of the previous call left it (so a launch captured
// in a CUDA graph stays correct).  One input and one result slot per rank
// suffice: every sub-chunk of a rank's input slot is read by one peer CTA,
// whose phase-2 flag the rank's own CTA of that index waits for before the
// call ends, so the next call's input never overwrites data a peer still
// reads; and a peer pushes into a rank's result slot only after it saw that
// rank's phase-1 flag of the same call, i.e. after the rank's previous call
// (and, in stream order, whatever read its result) finished.
#include "common.cuh"
#include "peer_sync.cuh"

namespace b200 {
namespace ar {

constexpr int kThreads = 512;
constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 160;                                // flag words per (phase, source rank)
constexpr int kCtrl = 2 * kMaxWorld * kMaxCtas;              // then: finished-CTA counter, last epoch
constexpr int kFlagWords = kCtrl + 2;
constexpr int64_t kMinUnitsPerCta = 32;                      // 512 bytes of a slice per CTA at least

struct Params {
    const uint4* in;
    uint4* out;
    int64_t units;         // 16-byte units (8 bf16) of the vector
    uint4* const* bufs;    // [world] -> each rank's slots: [input, result][cap]
    uint32_t* const* flags;  // [world] -> each rank's kFlagWords flag words
    int64_t cap;           // units per slot
    int32_t rank, world;
};

__device__ int32_t g_ar_error;

__device__ __forceinline__ int flag_index(int phase, int src, int cta) { return (phase * kMaxWorld + src) * kMaxCtas + cta; }

// Units [lo, hi) of slice s that CTA c handles.
__device__ __forceinline__ void sub_chunk(const Params& p, int s, int c, int64_t& lo, int64_t& hi) {
    const int64_t s0 = p.units * s / p.world, s1 = p.units * (s + 1) / p.world;
    const int64_t len = s1 - s0, g = gridDim.x;
    lo = s0 + len * c / g;
    hi = s0 + len * (c + 1) / g;
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        acc[2 * e] += __uint_as_float(w[e] << 16);
        acc[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ uint4 to_bf16x8(const float (&acc)[8]) {
    return make_uint4(pack2<true>(acc[0], acc[1]), pack2<true>(acc[2], acc[3]), pack2<true>(acc[4], acc[5]),
                      pack2<true>(acc[6], acc[7]));
}

__global__ void __launch_bounds__(kThreads, 1) allreduce_kernel(const __grid_constant__ Params p) {
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, c = blockIdx.x;
    uint32_t* my_flags = p.flags[p.rank];
    const uint32_t epoch = next_epoch(__ldcg(my_flags + kCtrl + 1));
    constexpr int64_t in_off = 0;
    const int64_t res_off = p.cap;
    uint4* mine = p.bufs[p.rank];

    // 1. this CTA's sub-chunks of every slice into the symmetric input slot
    if (p.in != mine) {
        for (int s = 0; s < p.world; ++s) {
            int64_t lo, hi;
            sub_chunk(p, s, c, lo, hi);
            for (int64_t i = lo + tid; i < hi; i += kThreads) mine[in_off + i] = __ldcs(p.in + i);
        }
    }
    __syncthreads();
    if (tid < p.world) st_release_sys(p.flags[tid] + flag_index(0, p.rank, c), epoch);

    // 2. reduce sub-chunk c of this rank's slice over every rank's input, push the result to all
    if (warp == 0) {
        const bool ok = warp_wait_flags<true>(my_flags + flag_index(0, 0, c), kMaxCtas, p.world, epoch);
        if (lane == 0) {
            if (!ok) atomicOr(&g_ar_error, 1);
            s_ok = ok;
        }
    }
    __syncthreads();
    const bool ok1 = s_ok;
    if (ok1) {
        int64_t lo, hi;
        sub_chunk(p, p.rank, c, lo, hi);
        // two units per thread and round: 2 x world loads in flight
        for (int64_t i0 = lo + tid; i0 < hi; i0 += 2 * kThreads) {
            const int64_t i1 = i0 + kThreads < hi ? i0 + kThreads : i0;
            uint4 v0[kMaxWorld], v1[kMaxWorld];
#pragma unroll
            for (int r = 0; r < kMaxWorld; ++r)
                if (r < p.world) {
                    v0[r] = __ldcg(p.bufs[r] + in_off + i0);
                    v1[r] = __ldcg(p.bufs[r] + in_off + i1);
                }
            float a0[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, a1[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < kMaxWorld; ++r)
                if (r < p.world) {
                    add_bf16x8(a0, v0[r]);
                    add_bf16x8(a1, v1[r]);
                }
            const uint4 o0 = to_bf16x8(a0), o1 = to_bf16x8(a1);
#pragma unroll
            for (int r = 0; r < kMaxWorld; ++r)
                if (r < p.world) {
                    p.bufs[r][res_off + i0] = o0;
                    p.bufs[r][res_off + i1] = o1;
                }
        }
    }
    __syncthreads();
    if (ok1 && tid < p.world) st_release_sys(p.flags[tid] + flag_index(1, p.rank, c), epoch);

    // 3. every rank's result sub-chunks c out of this rank's result slot
    if (ok1) {
        if (warp == 0) {
            const bool ok = warp_wait_flags<true>(my_flags + flag_index(1, 0, c), kMaxCtas, p.world, epoch);
            if (lane == 0) {
                if (!ok) atomicOr(&g_ar_error, 2);
                s_ok = ok;
            }
        }
        __syncthreads();
        if (s_ok && p.out != mine + res_off) {
            for (int s = 0; s < p.world; ++s) {
                int64_t lo, hi;
                sub_chunk(p, s, c, lo, hi);
                for (int64_t i = lo + tid; i < hi; i += kThreads) p.out[i] = __ldcg(mine + res_off + i);
            }
        }
    }

    // The last CTA to finish (every CTA has read the epoch by then) leaves it for the next call.
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(my_flags + kCtrl, 1u);
        if (prev == gridDim.x - 1) {
            my_flags[kCtrl] = 0;
            my_flags[kCtrl + 1] = epoch;
        }
    }
}

}  // namespace ar
}  // namespace b200

extern "C" int64_t b200_allreduce_flag_words(void) { return b200::ar::kFlagWords; }

extern "C" int32_t b200_allreduce_bf16(void* out, const void* in, int64_t n, void* const* bufs, int64_t buf_elems,
                                       uint32_t* const* flags, int32_t rank, int32_t world, void* stream) {
    using namespace b200;
    using namespace b200::ar;
    clear_error();
    B200_REQUIRE(n >= 0, "allreduce: n %lld < 0", (long long)n);
    if (n == 0) return B200_OK;
    B200_REQUIRE(out && in && bufs && flags, "allreduce: null pointer");
    B200_REQUIRE(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "allreduce: rank %d of %d", rank,
                 world);
    B200_REQUIRE(n % 8 == 0, "allreduce: n %lld not a multiple of 8", (long long)n);
    B200_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0,
                 "allreduce: in and out must be 16-byte aligned");
    B200_REQUIRE(buf_elems % 16 == 0 && buf_elems >= 2 * n,
                 "allreduce: symmetric buffer of %lld elements not a multiple of 16 or < 2 x n = %lld",
                 (long long)buf_elems, (long long)(2 * n));
    Params p;
    p.in = static_cast<const uint4*>(in);
    p.out = static_cast<uint4*>(out);
    p.units = n / 8;
    p.bufs = reinterpret_cast<uint4* const*>(bufs);
    p.flags = flags;
    p.cap = buf_elems / 2 / 8;
    p.rank = rank;
    p.world = world;
    // Same grid on every rank: it depends only on n, world and the SM count.
    int64_t grid = p.units / world / kMinUnitsPerCta;
    const int64_t most = device_sm_count() < kMaxCtas ? device_sm_count() : kMaxCtas;
    grid = grid < 1 ? 1 : (grid > most ? most : grid);
    allreduce_kernel<<<unsigned(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}

extern "C" int32_t b200_allreduce_error(void* stream, int32_t* flag) {
    using namespace b200;
    B200_REQUIRE(flag != nullptr, "allreduce_error: null pointer");
    B200_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    B200_CUDA_TRY(cudaMemcpyFromSymbol(flag, b200::ar::g_ar_error, sizeof(int32_t)));
    return B200_OK;
}
