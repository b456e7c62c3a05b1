// Tensor memory (TMEM) of sm_100a used as an on-chip staging area between
// warps: 128 lanes x up to 512 columns of 32 bits per SM, allocated per CTA
// by one warp, written and read with tcgen05.st / tcgen05.ld. A warp reaches
// only its own quarter of the lanes: warp w of the CTA the 32 lanes from
// 32 * (w % 4), each lane its own lane; the column is the same for the whole
// warp. Hand-offs between warps go through an ordinary thread
// synchronisation (here mbarriers) bracketed by tcgen05.fence.
#pragma once

#include <cstdint>

#include "async_copy.cuh"

namespace mlk::cuda {

// One full warp: allocates `cols` columns (a power of two, 32..512) and
// writes the TMEM address to `dst` in shared memory; the CTA then gives up
// its right to allocate more, so other CTAs of the SM are not held back.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// The allocating warp, once every TMEM access of the CTA is done.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tmem_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole warp, warp-uniform `taddr`: lane i's `v` into (lane of taddr + i, column of taddr).
__device__ __forceinline__ void tmem_st1(uint32_t taddr, int v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}

// Waits until this warp's earlier tcgen05.st have landed.
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Whole warp, warp-uniform `taddr`: 16 consecutive columns of this lane's
// TMEM lane into v, complete on return (the load and its wait are one asm
// statement, so no use of v can move above the wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

}  // namespace mlk::cuda
