// Fifth-generation tensor-core helpers (sm_100a): TMEM allocation, loads and
// stores, tcgen05.mma of kind::tf32 with the A operand in TMEM and the B
// operand in shared memory, commit to an mbarrier, and a bounded mbarrier wait.
//
// Layout used by the pass kernels: a K-major operand tile without swizzle,
// 16 tf32 values of K per row (one CRESSO5 carrier row: (a1_k, a2_k) for
// k < 8), stored as 8-row x 16-byte core matrices:
//   byte offset(row, k) = (row / 8) * kTcSBO + (k / 4) * kTcLBO + (row % 8) * 16 + (k % 4) * 4
// so one K step of 8 tf32 values spans two core matrices kTcLBO bytes apart,
// and the next K step starts 2 * kTcLBO bytes further on.
#pragma once

#include <stdint.h>

namespace cresso {

constexpr int kTcLBO = 128;  // bytes between K-adjacent core matrices
constexpr int kTcSBO = 512;  // bytes between 8-row groups (4 core matrices of 16 K values)
constexpr int kTcTileBytes = 1024;  // one 16-row x 16-K float tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Rounds to the nearest tf32 value (ties away from zero); the low 13 mantissa bits are zero.
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ int tc_kmajor_off(int row, int k) {
    return (row >> 3) * kTcSBO + (k >> 2) * kTcLBO + (row & 7) * 16 + (k & 3) * 4;
}

// Shared-memory matrix descriptor: no swizzle, K-major, the offsets above.
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((kTcLBO >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((kTcSBO >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version of sm_100
    return d;                // base offset 0, legacy leading-offset mode, layout "no swizzle"
}

// Instruction descriptor of kind::tf32: D float32, A and B tf32, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[M x N] (+)= A[M x 8] * B[N x 8]^T with A read from TMEM and B from shared memory.
__device__ __forceinline__ void tc_mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %4, p;\n\t"
        "}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(accumulate), "r"(idesc));
}

// Arrives on the mbarrier once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// This warp's 32 lanes, 16 consecutive 32-bit columns.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16};\n" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
        "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]));
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]), "=f"(v[8]),
          "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15])
        : "r"(taddr));
}
// N = 2 or 4 consecutive 32-bit columns of this warp's 32 lanes.
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[N]) {
    static_assert(N == 2 || N == 4, "tc_ld: 2 or 4 columns");
    if constexpr (N == 2) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];\n" : "=f"(v[0]), "=f"(v[1]) : "r"(taddr));
    } else {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                     : "r"(taddr));
    }
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Makes this thread's generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void tc_fence_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// TMEM allocation by one whole warp; the base address is written to *slot.
__device__ __forceinline__ void tc_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tc_dealloc(uint32_t base, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Waits until the mbarrier phase of the given parity has completed; gives up
// (returns false) after limit_ns nanoseconds.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}

}  // namespace cresso
