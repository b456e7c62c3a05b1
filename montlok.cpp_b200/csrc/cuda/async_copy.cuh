// Shared-memory streaming helpers of the tree kernels: explicit 32-bit shared
// addresses and loads, mbarrier-counted one-dimensional bulk async copies
// (cp.async.bulk, global -> this CTA's shared memory), time-bounded waits, and
// L2 prefetch of the next rows.
#pragma once

#include <cstddef>
#include <cstdint>

namespace mlk::cuda {

// How long a wait on a copy may take before the kernel gives up (ns of the
// GPU's global timer); kernels receive it as a launch argument.
inline constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__host__ __device__ constexpr int align128(int n) { return (n + 127) & ~127; }

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t arrivals = 1) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals) : "memory");
}

// One arrival on `bar` (release: this thread's earlier writes are seen by the
// threads whose wait on the phase returns).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arms `bar` for `bytes` and starts the copy global -> shared (one thread).
// Both addresses are 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for phase `parity` of `bar` to complete; false once `limit_ns` of the
// global timer have passed (or after 2^30 polls, whichever comes first), or as
// soon as `*abort` (when given) is raised.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns,
                                          const volatile int* abort = nullptr) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (int polls = 0; polls < (1 << 30); ++polls) {
        if (mbar_try(bar, parity)) return true;
        if (abort && *abort) return false;
        if (global_ns() - t0 > limit_ns) return false;
    }
    return false;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ int lds_s32(uint32_t a) {
    int v;
    asm volatile("ld.shared.s32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ int4 lds_v4(uint32_t a) {
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ double lds_leaf(uint32_t a, bool f32) {
    if (f32) {
        float v;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
        return static_cast<double>(v);
    }
    double v;
    asm volatile("ld.shared.f64 %0, [%1];" : "=d"(v) : "r"(a));
    return v;
}

// Starts pulling [p, p + bytes) into L2 (16-byte aligned interior only).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t{15};
    const uintptr_t hi = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t{15};
    for (uintptr_t a = lo; a < hi; a += (1u << 20)) {
        const uint32_t n = static_cast<uint32_t>(min(static_cast<uintptr_t>(1u << 20), hi - a));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

}  // namespace mlk::cuda
