// tcgen05.cuh -- 5th-generation tensor core plumbing shared by the sm_100a matmul kernels:
// shared-memory matrix descriptors, kind::i8 MMA issue, commit to mbarriers, tensor-memory loads,
// and the stream-K work split.
#pragma once
#include <stdint.h>
#include <stdlib.h>

#include "tma.cuh"

namespace dcg {

// ---- tcgen05 plumbing ----
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: start >> 4, leading (K-direction) byte offset >> 4, stride (8-row
    // group) byte offset >> 4, version 1 (bits 46-47), base offset 0, layout type 0
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}
// K-major, 128-byte swizzle (rows of 128 B, 8-row atoms of 1 KB at 1 KB-aligned addresses, as a
// TMA box with CU_TENSOR_MAP_SWIZZLE_128B lands): leading offset unused (1), stride between 8-row
// groups 1 KB, layout type 2 (bits 61-63).  A k-step further along the row adds its byte offset
// (< 128) to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int M, int N>
__host__ __device__ constexpr uint32_t idesc_i8() {
    // D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1), both K-major,
    // N >> 3 at bits 17-22, M >> 4 at bits 24-28
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// the same MMA with A (M rows x K int8, row r in TMEM lane r, 4 consecutive K elements per 32-bit
// column) read from tensor memory instead of shared memory
__device__ __forceinline__ void mma_i8_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (warp w reaches lanes 32 (w % 4) .. +31)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// exact int -> float for |v| < 2^22 with two full-rate ops (the float magic-number method: v added
// to the mantissa of 1.5 * 2^23, whose unit in the last place is 1, then the bias subtracted); the
// conversion instruction runs at a fraction of that rate
__device__ __forceinline__ float i2f_exact22(int v) { return __int_as_float(0x4B400000 + v) - 12582912.0f; }


// stream-K ranges: CTA c owns units [begin(c), begin(c+1)); owner(u) is the CTA whose range holds u
__host__ __device__ __forceinline__ int64_t sk_begin(int64_t c, int64_t T, int64_t G) { return c * T / G; }
__device__ __forceinline__ int64_t sk_owner(int64_t u, int64_t T, int64_t G) { return ((u + 1) * G - 1) / T; }

// minimum stream-K units per CTA when the matrix has fewer units than SMs (DCG_SK_MIN_UNITS
// overrides it for tuning)
inline int64_t sk_min_units() {
    static const int64_t v = [] {
        const char* e = getenv("DCG_SK_MIN_UNITS");
        const long x = e ? atol(e) : 1;
        return (int64_t)(x > 0 ? x : 1);
    }();
    return v;
}

}  // namespace dcg
