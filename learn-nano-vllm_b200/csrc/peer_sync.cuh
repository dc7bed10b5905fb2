// Synchronisation between the GPUs of a tensor-parallel group over memory
// that every rank maps (CUDA symmetric memory): release / acquire flag words
// at system scope, call epochs, and a warp-collective bounded wait.
#pragma once
#include "common.cuh"

namespace b200 {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t next_epoch(uint32_t e) { return e + 1u == 0u ? 2u : e + 1u; }
// A ready flag shows epoch e: it holds e, or already the next epoch (its writer ran ahead by one
// call).  Split arrival flags (this GPU, this grid) can only hold e or older.
template <bool SYS>
__device__ __forceinline__ bool shows(uint32_t v, uint32_t e) { return v == e || (SYS && v == next_epoch(e)); }

// Whole warp: lane l < n waits until flags[l * stride] shows epoch, all lanes in
// parallel; true in every lane once all do, false in every lane on timeout.
template <bool SYS>
__device__ __forceinline__ bool warp_wait_flags(const uint32_t* flags, int stride, int n, uint32_t epoch) {
    const int lane = threadIdx.x & 31;
    auto ok = [&]() {
        if (lane >= n) return true;
        const uint32_t* f = flags + lane * stride;
        return shows<SYS>(SYS ? ld_acquire_sys(f) : ld_acquire_gpu(f), epoch);
    };
    bool done = ok();
    if (__all_sync(0xffffffffu, done)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (!done) done = ok();
        if (__all_sync(0xffffffffu, done)) return true;
        if (__shfl_sync(0xffffffffu, global_timer_ns() - t0 > kWaitLimitNs, 0)) return false;
        __nanosleep(32);
    }
}

}  // namespace b200
