// Device-side primitives shared by the probe and GEMV kernels (sm_100a inline PTX).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace l2d {
namespace dev {

__device__ __forceinline__ uint32_t smid() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t r;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(r));
    return r;
}

__device__ __forceinline__ uint64_t clock64_now() {
    uint64_t r;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(r));
    return r;
}

// L2-only load (bypasses L1), so every probe access is served by the L2 slice that holds it.
__device__ __forceinline__ uint64_t ld_cg_u64(const void *p) {
    uint64_t v;
    asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_u32(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Latency of one L2 access in SM cycles.  The store of the loaded value to shared memory cannot
// issue before the data arrives, and the second clock read issues after that store (in-order
// issue), so the interval covers the whole round trip.
__device__ __forceinline__ uint32_t timed_load(const void *p, volatile uint64_t *sink) {
    uint64_t t0 = clock64_now();
    uint64_t v = ld_cg_u64(p);
    *sink = v;
    uint64_t t1 = clock64_now();
    return static_cast<uint32_t>(t1 - t0);
}

// Waits until *p >= target or the deadline passes; returns false on timeout.  Every device wait
// in this library goes through a bounded loop like this one.
__device__ __forceinline__ bool wait_at_least(const uint32_t *p, uint32_t target, uint64_t deadline_ns) {
    while (ld_acquire_u32(p) < target) {
        if (globaltimer_ns() > deadline_ns) return false;
        __nanosleep(256);
    }
    return true;
}

}  // namespace dev
}  // namespace l2d
