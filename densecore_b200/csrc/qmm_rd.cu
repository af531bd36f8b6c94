// qmm_rd.cu -- tensor-core matmul for Q8_0 and Q6_K weights (batched decode / prefill, any M),
// register-direct: each warp streams the A fragments of its own 16 weight rows from global memory
// into registers (one super-block ahead) and reuses them across NT mma n-tiles of activations,
// whose B fragments come through L1 (every warp of the GPU reads the same small activation).
// Replaces ggml_mul_mat / vec_dot_{q8_0_q8_0,q6_K_q8_K} (core/src/inference.cpp:1063,
// :1794-1797, :1817; simd_ops.cpp:82-93) for these formats.
//
// Q8_0: one m16n8k32 mma per 32-element block; k order permuted so lane (gid, tig) supplies
//       bytes 8*tig..8*tig+7 of its rows' block (a0|a2, a1|a3) and of the activation column
//       (b0|b1).  y += d_w * d_x * C in fp32 per block.
// Q6_K: one m16n8k16 mma per 16-element sub-block (lane: elements 4*tig..+3 of it); the 6-bit
//       value is (ql nibble | qh 2 bits << 4) - 32; isum += scale_s * C (int32) over the
//       super-block, y += d_w * d_x * isum.
// Device weight layout (common.cuh): payload rows + separate fp16 scale array.
// Split-K: when the row x column blocks cannot fill the GPU, grid.z splits K and the splits of a
// tile form one thread-block cluster that reduces through distributed shared memory.
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace dcg {

constexpr int RD_WARPS = 4;  // 64 rows per CTA

__device__ __forceinline__ void mma_k32(int* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_k16(int* c, uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint2 ldg64_stream(const void* p) {
    uint2 r;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg32_stream(const void* p) {
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

constexpr int RD_RS = 68;  // row stride of the split-K reduction tile: conflict-free lane writes

// S splits (one cluster): rank 0 adds the S partial tiles parked in shared memory in rank order
// through distributed shared memory.  Kept out of line: inlined, the cluster barriers changed the
// main loops' schedule (240 -> 168 registers, a 2.5x slower Q8_0 loop).
__device__ __noinline__ void rd_cluster_reduce(const float* red, float* __restrict__ y, int64_t n, int m,
                                               int64_t r0, int c0, int ncols) {
    cluster_sync_all();
    if (cluster_rank() == 0) {
        for (int idx = threadIdx.x; idx < RD_WARPS * 16 * ncols; idx += blockDim.x) {
            const int row = idx % (RD_WARPS * 16), col = idx / (RD_WARPS * 16);
            float sum = 0.0f;
            for (uint32_t r = 0; r < gridDim.z; r++) sum += ld_cluster_f32(red + col * RD_RS + row, r);
            if (c0 + col < m && r0 + row < n) y[(size_t)(c0 + col) * n + r0 + row] = sum;
        }
    }
    cluster_sync_all();   // keeps every CTA's tile alive until rank 0 has read it
}

// Output of a warp's 16 rows x 8*NT columns: stored directly (one split) or parked in shared
// memory for the cluster reduction; the result does not depend on timing either way.
template <int NT>
__device__ __forceinline__ void rd_store(const float (&acc)[NT][4], float* red, float* __restrict__ y,
                                         int64_t n, int m, int64_t r0, int c0, int warp, int gid, int tig,
                                         bool live) {
    if (gridDim.z == 1) {
        if (!live) return;
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int col = c0 + t * 8 + 2 * tig + (i & 1);
                const int64_t row = r0 + warp * 16 + gid + (i < 2 ? 0 : 8);
                if (col < m && row < n) y[(size_t)col * n + row] = acc[t][i];
            }
        return;
    }
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int i = 0; i < 4; i++)
            red[(t * 8 + 2 * tig + (i & 1)) * RD_RS + warp * 16 + gid + (i < 2 ? 0 : 8)] = acc[t][i];
    rd_cluster_reduce(red, y, n, m, r0, c0, 8 * NT);
}

// ------------------------------------------------------------------------------------------
// Q8_0.  A super-block here is 8 blocks (256 elements) so the loop shape matches Q6_K.
// ------------------------------------------------------------------------------------------
struct Q80Frag {
    uint2 a[8], b[8];   // rows gid / gid+8, blocks 0..7: bytes 8*tig..+7
    uint4 dA, dB;       // fp16 scales of the 8 blocks, rows gid / gid+8
};

__device__ __forceinline__ void q80_load(Q80Frag& f, const PackedW& w, int64_t rowA, int64_t rowB,
                                         int64_t n, int sb, int tig) {
    const int64_t ra = rowA < n ? rowA : n - 1, rb = rowB < n ? rowB : n - 1;
    const uint8_t* pa = w.payload + ra * w.row_bytes + (size_t)sb * 256 + 8 * tig;
    const uint8_t* pb = w.payload + rb * w.row_bytes + (size_t)sb * 256 + 8 * tig;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        f.a[j] = ldg64_stream(pa + 32 * j);
        f.b[j] = ldg64_stream(pb + 32 * j);
    }
    f.dA = __ldg((const uint4*)(w.d + ra * w.nb + (size_t)sb * 8));
    f.dB = __ldg((const uint4*)(w.d + rb * w.nb + (size_t)sb * 8));
}

__device__ __forceinline__ float h_at(const uint4& v, int j) {  // fp16 j (0..7) of 8 packed
    const uint32_t w = j < 2 ? v.x : (j < 4 ? v.y : (j < 6 ? v.z : v.w));
    const __half2 h = *reinterpret_cast<const __half2*>(&w);
    return (j & 1) ? __high2float(h) : __low2float(h);
}

template <int NT>
__global__ void __launch_bounds__(RD_WARPS * 32) qmm_q8_0_rd_kernel(PackedW w, int64_t n, int64_t k,
                                                                   ActQ a, int m, float* __restrict__ y,
                                                                   int sps) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int64_t rowA = ((int64_t)blockIdx.x * RD_WARPS + warp) * 16 + gid, rowB = rowA + 8;
    const int c0 = blockIdx.y * 8 * NT;
    // this split's super-blocks [sb0, sb0 + nsb): base pointers move, the loop stays 0-based
    // (a loop from sb0 compiled to a slower schedule)
    const int sb0 = blockIdx.z * sps;
    const int nsb = min((int)(k / 256) - sb0, sps);
    w.payload += (size_t)sb0 * 256;
    w.d += (size_t)sb0 * 8;
    a.qs += (size_t)sb0 * 256;
    a.d = (uint8_t*)a.d + (size_t)sb0 * 8 * sizeof(__half);
    extern __shared__ float red[];  // 8 * NT * RD_RS floats when split
    const int nbx = (int)(k / QK8_0);
    const __half* xd = (const __half*)a.d;
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[t][i] = 0.0f;
    const bool live = rowA - gid < n;

    if (!live) {   // rows past n: no loads, but the warp still takes part in the split reduction
        pdl_wait();
        rd_store<NT>(acc, red, y, n, m, (int64_t)blockIdx.x * RD_WARPS * 16, c0, warp, gid, tig, false);
        pdl_trigger();
        return;
    }
    Q80Frag cur, nxt;
    q80_load(cur, w, rowA, rowB, n, 0, tig);
    pdl_wait();   // the first weight fragments (constant) are already in flight
    for (int sb = 0; sb < nsb; sb++) {
        if (sb + 1 < nsb) q80_load(nxt, w, rowA, rowB, n, sb + 1, tig);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const int colB = c0 + t * 8 + gid;  // B column of this lane
            const int cA = c0 + t * 8 + 2 * tig;  // C columns 2tig, 2tig+1
            const int8_t* xb = a.qs + (size_t)(colB < m ? colB : 0) * k + (size_t)sb * 256 + 8 * tig;
            uint4 dx0 = make_uint4(0, 0, 0, 0), dx1 = make_uint4(0, 0, 0, 0);
            if (cA < m) dx0 = __ldg((const uint4*)(xd + (size_t)cA * nbx + (size_t)sb * 8));
            if (cA + 1 < m) dx1 = __ldg((const uint4*)(xd + (size_t)(cA + 1) * nbx + (size_t)sb * 8));
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint2 xv = make_uint2(0, 0);
                if (colB < m) xv = __ldg((const uint2*)(xb + 32 * j));
                int c[4] = {0, 0, 0, 0};
                mma_k32(c, cur.a[j].x, cur.b[j].x, cur.a[j].y, cur.b[j].y, xv.x, xv.y);
                const float wa = h_at(cur.dA, j), wb = h_at(cur.dB, j);
                const float x0 = h_at(dx0, j), x1 = h_at(dx1, j);
                acc[t][0] += (wa * x0) * (float)c[0];
                acc[t][1] += (wa * x1) * (float)c[1];
                acc[t][2] += (wb * x0) * (float)c[2];
                acc[t][3] += (wb * x1) * (float)c[3];
            }
        }
        if (sb + 1 < nsb) cur = nxt;
    }
    rd_store<NT>(acc, red, y, n, m, (int64_t)blockIdx.x * RD_WARPS * 16, c0, warp, gid, tig, live);
    pdl_trigger();   // after the split reduction: see the Q4_K M = 1 kernel
}

// ------------------------------------------------------------------------------------------
// Q6_K.  Sub-block s (16 elements): half h = s>>3, group grp = (s&7)>>1, l-range 16*(s&1)..+15.
// Lane tig takes elements 4*tig..+3 of it: one ql word (nibble grp>>1) and one qh word (bits 2*grp).
// ------------------------------------------------------------------------------------------
struct Q6Frag {
    uint32_t ql[2][8];  // [row A/B][h*4 + (grp&1)*2 + half]
    uint32_t qh[2][4];  // [row][h*2 + half]
    uint4 sc[2];        // int8 scales of the 16 sub-blocks
    float d[2];
};

__device__ __forceinline__ void q6_load(Q6Frag& f, const PackedW& w, int64_t rowA, int64_t rowB,
                                        int64_t n, int sb, int tig) {
    const int64_t rows[2] = {rowA < n ? rowA : n - 1, rowB < n ? rowB : n - 1};
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint8_t* p = w.payload + rows[r] * w.row_bytes + (size_t)sb * Q6_K_PAYLOAD + 4 * tig;
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int q = 0; q < 2; q++)
#pragma unroll
                for (int half = 0; half < 2; half++)
                    f.ql[r][h * 4 + q * 2 + half] = ldg32_stream(p + h * 64 + q * 32 + half * 16);
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int half = 0; half < 2; half++)
                f.qh[r][h * 2 + half] = ldg32_stream(p + 128 + h * 32 + half * 16);
        f.sc[r] = __ldg((const uint4*)(w.payload + rows[r] * w.row_bytes + (size_t)sb * Q6_K_PAYLOAD + 192));
        f.d[r] = __half2float(w.d[rows[r] * w.nb + sb]);
    }
}

__device__ __forceinline__ uint32_t q6_word(const Q6Frag& f, int r, int s) {
    const int h = s >> 3, grp = (s & 7) >> 1, half = s & 1;
    const uint32_t ql = f.ql[r][h * 4 + (grp & 1) * 2 + half];
    const uint32_t qh = f.qh[r][h * 2 + half];
    const uint32_t q = ((ql >> (4 * (grp >> 1))) & 0x0F0F0F0Fu) | (((qh >> (2 * grp)) & 0x03030303u) << 4);
    return __vsub4(q, 0x20202020u);
}

__device__ __forceinline__ int sc_at(const uint4& v, int s) {  // signed int8 scale s (0..15)
    const uint32_t w = s < 4 ? v.x : (s < 8 ? v.y : (s < 12 ? v.z : v.w));
    return (int)(int8_t)((w >> (8 * (s & 3))) & 0xFF);
}

template <int NT>
__global__ void __launch_bounds__(RD_WARPS * 32) qmm_q6k_rd_kernel(PackedW w, int64_t n, int64_t k,
                                                                  ActQ a, int m, float* __restrict__ y,
                                                                   int sps) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int64_t rowA = ((int64_t)blockIdx.x * RD_WARPS + warp) * 16 + gid, rowB = rowA + 8;
    const int c0 = blockIdx.y * 8 * NT;
    const int sb0 = blockIdx.z * sps;   // base pointers move to the split, the loop stays 0-based
    const int nsb = min((int)(k / QK_K) - sb0, sps);
    const int nsb_all = (int)(k / QK_K);
    w.payload += (size_t)sb0 * Q6_K_PAYLOAD;
    w.d += sb0;
    a.qs += (size_t)sb0 * QK_K;
    a.d = (uint8_t*)a.d + (size_t)sb0 * sizeof(float);
    extern __shared__ float red[];  // 8 * NT * RD_RS floats when split
    const float* xd = (const float*)a.d;
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[t][i] = 0.0f;
    const bool live = rowA - gid < n;

    if (!live) {   // rows past n: no loads, but the warp still takes part in the split reduction
        pdl_wait();
        rd_store<NT>(acc, red, y, n, m, (int64_t)blockIdx.x * RD_WARPS * 16, c0, warp, gid, tig, false);
        pdl_trigger();
        return;
    }
    Q6Frag cur, nxt;
    q6_load(cur, w, rowA, rowB, n, 0, tig);
    pdl_wait();   // the first weight fragments (constant) are already in flight
    for (int sb = 0; sb < nsb; sb++) {
        if (sb + 1 < nsb) q6_load(nxt, w, rowA, rowB, n, sb + 1, tig);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const int colB = c0 + t * 8 + gid;
            const int cA = c0 + t * 8 + 2 * tig;
            const int8_t* xb = a.qs + (size_t)(colB < m ? colB : 0) * k + (size_t)sb * QK_K + 4 * tig;
            int is[4] = {0, 0, 0, 0};
#pragma unroll
            for (int s = 0; s < 16; s++) {
                const uint32_t xv = colB < m ? __ldg((const uint32_t*)(xb + 16 * s)) : 0u;
                int c[4] = {0, 0, 0, 0};
                mma_k16(c, q6_word(cur, 0, s), q6_word(cur, 1, s), xv);
                const int sa = sc_at(cur.sc[0], s), sbb = sc_at(cur.sc[1], s);
                is[0] += sa * c[0];
                is[1] += sa * c[1];
                is[2] += sbb * c[2];
                is[3] += sbb * c[3];
            }
            const float x0 = cA < m ? xd[(size_t)cA * nsb_all + sb] : 0.0f;
            const float x1 = cA + 1 < m ? xd[(size_t)(cA + 1) * nsb_all + sb] : 0.0f;
            acc[t][0] += (cur.d[0] * x0) * (float)is[0];
            acc[t][1] += (cur.d[0] * x1) * (float)is[1];
            acc[t][2] += (cur.d[1] * x0) * (float)is[2];
            acc[t][3] += (cur.d[1] * x1) * (float)is[3];
        }
        if (sb + 1 < nsb) cur = nxt;
    }
    rd_store<NT>(acc, red, y, n, m, (int64_t)blockIdx.x * RD_WARPS * 16, c0, warp, gid, tig, live);
    pdl_trigger();   // after the split reduction: see the Q4_K M = 1 kernel
}

// grid (row blocks, column blocks, splits): split K until one wave of resident CTAs is filled, at
// most 8 splits (one portable cluster), keeping >= 4 super-blocks per split for Q8_0 and >= 2 for
// Q6_K (its super-blocks cost 16 mmas; shorter splits measured slower than fewer).
template <int TYPE, int NT>
static cudaError_t launch_rd_t(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m, float* y,
                               cudaStream_t st) {
    const int rb = (int)((n + RD_WARPS * 16 - 1) / (RD_WARPS * 16)), cb = (m + 8 * NT - 1) / (8 * NT);
    const int nsb = (int)(k / 256);
    auto kern = TYPE == DCG_TYPE_Q8_0 ? qmm_q8_0_rd_kernel<NT> : qmm_q6k_rd_kernel<NT>;
    static int per_sm[MAX_DEVICES] = {};   // CTAs per SM the kernel's registers allow, per device
    static PerDevice pd;
    cudaError_t e = per_device_once(pd, [&] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaError_t r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, RD_WARPS * 32, 0);
        per_sm[dev] = v > 0 ? v : 1;
        return r;
    });
    if (e != cudaSuccess) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    const int resident = per_sm[dev] * num_sms();
    int S = (resident + rb * cb - 1) / (rb * cb);
    S = S < 1 ? 1 : (S > 8 ? 8 : S);
    // below min_sps super-blocks per split a split costs more than it gains (DCG_RD_MIN_SPS
    // overrides it, for tuning)
    static const int min_sps_env = getenv("DCG_RD_MIN_SPS") ? atoi(getenv("DCG_RD_MIN_SPS")) : 0;
    const int min_sps = min_sps_env > 0 ? min_sps_env : (TYPE == DCG_TYPE_Q8_0 ? 4 : 2);
    S = S > nsb / min_sps ? (nsb / min_sps > 0 ? nsb / min_sps : 1) : S;
    const int sps = (nsb + S - 1) / S;
    S = (nsb + sps - 1) / sps;
    const dim3 grid((unsigned)rb, (unsigned)cb, (unsigned)S);
    const size_t smem = S == 1 ? 0 : sizeof(float) * 8 * NT * RD_RS;
    return launch_ex(kern, grid, dim3(RD_WARPS * 32), smem, st, (unsigned)S, w, n, k, a, m, y, sps);
}

bool qmm_rd_supports(int type, int64_t k, int64_t m) {
    return (type == DCG_TYPE_Q8_0 || type == DCG_TYPE_Q6_K) && k % 256 == 0 && m >= 2;
}

cudaError_t launch_qmm_rd(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                          int64_t m, float* y, cudaStream_t st) {
    const PackedW w = packed_view(type, packed_w, n, k);
    const int act_type = type == DCG_TYPE_Q8_0 ? DCG_TYPE_Q8_0 : DCG_TYPE_Q8_K;
    const ActQ a = act_view(act_type, const_cast<void*>(act), m, k);
    // column blocks of 8*NT activation rows run as grid.y: CTAs over the same weight rows share
    // them through L2
    const int mi = (int)m;
    if (type == DCG_TYPE_Q8_0) {
        if (mi <= 8) return launch_rd_t<DCG_TYPE_Q8_0, 1>(w, n, k, a, mi, y, st);
        if (mi <= 16) return launch_rd_t<DCG_TYPE_Q8_0, 2>(w, n, k, a, mi, y, st);
        return launch_rd_t<DCG_TYPE_Q8_0, 4>(w, n, k, a, mi, y, st);
    }
    if (mi <= 8) return launch_rd_t<DCG_TYPE_Q6_K, 1>(w, n, k, a, mi, y, st);
    if (mi <= 16) return launch_rd_t<DCG_TYPE_Q6_K, 2>(w, n, k, a, mi, y, st);
    return launch_rd_t<DCG_TYPE_Q6_K, 4>(w, n, k, a, mi, y, st);
}

}  // namespace dcg
