// qmm_tc.cu -- Q4_K weight x Q8_K activation matmul on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory), for batched decode (column tiles of
// N = 32 activation rows).  Replaces ggml_mul_mat's vec_dot_q4_K_q8_K row loop for these shapes
// (core/src/inference.cpp:1063, :1794-1797; the dot product of simd_ops.cpp:82-93).
//
// One CTA owns 128 weight rows (the MMA's M) x N activation rows (the MMA's N) over a range of K
// super-blocks (split-K across a cluster when the tiles alone cannot fill the GPU).  Per
// super-block (K = 256):
//   producer warp   TMA: the 128 x 144 B Q4_K weight tile, and the N x 256 B Q8_K activation tile
//                   as one 3-D box (16 B x N rows x 16 K chunks: the K-major no-swizzle
//                   core-matrix layout); its lanes stage the columns' dx and pair sums
//   prep warpgroup  (warps 2-5) thread r expands weight row r into two int8 planes, H = q * sh and
//                   L = q * sl with the 6-bit sub-block scale sc = 8 * sh + sl (q <= 15, sh, sl
//                   <= 7: every product fits int8, four at a time in one 32-bit multiply), written
//                   in the core-matrix layout the MMA reads
//   MMA thread      16 x tcgen05.mma.kind::i8 (8 k-steps of 32 for each plane) into two int32
//                   accumulators C_H, C_L in tensor memory; double-buffered across super-blocks
//   epilogue        (warps 6-9, concurrent with the prep of the next super-block) thread r reads row r of C_H, C_L (tcgen05.ld) and the
//                   columns' dx and pair sums (staged in shared memory by the producer warp), forms the
//                   exact integer sum isum = 8 C_H + C_L, the min term sum_j m_j * bsum32_j (dp2a),
//                   and accumulates y += dx * (d * isum - dmin * msum) in fp32, as ggml does
// Every wait is bounded (device error flag), and tensor memory is always freed before exit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace dcg {

__device__ int g_tc_error = 0;

cudaError_t qmm_tc_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_tc_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int TC_ROWS = 128;                     // weight rows per CTA (MMA M)
constexpr int TC_THREADS = 576;                  // warp 0 producer, 1 MMA, 2-9 prep, 10-17 epilogue
constexpr int TC_EPI0 = 10;                      // first epilogue warp
constexpr int TC_WTILE = TC_ROWS * Q4_K_BYTES;   // 18432 B raw weight tile per super-block
constexpr int TC_PLANE = TC_ROWS * QK_K;         // 32 KB: one int8 plane of a super-block
constexpr int TC_PLANE_SBO = 16 * 128;           // plane: 8-row groups 2 KB apart, 16-B K chunks 128 B

template <int N>
struct TcCfg {
    static constexpr int STAGES = N <= 32 ? 3 : 2;
    static constexpr int ATILE = N * QK_K;                       // activation tile per super-block
    static constexpr int OFF_RAW = 1024;                         // after barriers
    static constexpr int OFF_ACT = OFF_RAW + STAGES * TC_WTILE;
    static constexpr int OFF_PL = OFF_ACT + STAGES * ATILE;      // [2 buffers][H, L]
    static constexpr int MSLOTS = STAGES + 2;                    // metadata lives until the epilogue
    static constexpr int META = N * 4 + N * 16;                  // per column: dx, 8 pair sums
    static constexpr int OFF_META = OFF_PL + 4 * TC_PLANE;
    static constexpr int OFF_ROWP = OFF_META + MSLOTS * META;    // [slot][128 rows] d | dmin, mins
    static constexpr int SMEM = OFF_ROWP + MSLOTS * TC_ROWS * 16;
    static constexpr int TMEM_COLS = 4 * N;                      // [2 buffers][C_H, C_L] x N
};

// ---- tcgen05 plumbing ----
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: start >> 4, leading (K-direction) byte offset >> 4, stride (8-row
    // group) byte offset >> 4, version 1 (bits 46-47), base offset 0, layout type 0
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

template <int N>
__host__ __device__ constexpr uint32_t idesc_i8() {
    // D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1), both K-major,
    // N >> 3 at bits 17-22, M >> 4 at bits 24-28
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
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
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- the kernel ----
template <int N>
__global__ void __launch_bounds__(TC_THREADS, 1)
    qmm_q4k_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                      int nb, int64_t n, ActQ a, int m, float* __restrict__ y, int sps) {
    using C = TcCfg<N>;
    constexpr int R = C::STAGES;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;          // [R] weight + activation tiles landed (tx)
    uint64_t* raw_empty = full + R;            // [R] 128 prep threads read the weight tile
    uint64_t* act_empty = raw_empty + R;       // [R] MMAs that read the activation tile done
    uint64_t* pl_full = act_empty + R;         // [2] planes written (128 arrivals)
    uint64_t* pl_empty = pl_full + 2;          // [2] MMAs that read the planes done
    uint64_t* acc_full = pl_empty + 2;         // [2] accumulators complete
    uint64_t* acc_empty = acc_full + 2;        // [2] 128 epilogue threads read them
    uint64_t* meta_empty = acc_empty + 2;      // [MSLOTS] epilogue done with a metadata slot
    uint64_t* mma_done = meta_empty + C::MSLOTS; // [1] every MMA of the CTA retired
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
    uint8_t* raw = smem + C::OFF_RAW;
    uint8_t* act = smem + C::OFF_ACT;
    uint8_t* planes = smem + C::OFF_PL;
    uint8_t* meta = smem + C::OFF_META;        // [MSLOTS][dx: N floats | pair sums: N x 8 int16]
    uint4* rowp = (uint4*)(smem + C::OFF_ROWP);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * TC_ROWS;
    const int c0 = blockIdx.y * N;
    const int sb0 = blockIdx.z * sps, sb1 = min(nb, sb0 + sps);
    const int nsb = sb1 - sb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&raw_empty[s], 256);
            mbar_init(&act_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&pl_full[b], 256);
            mbar_init(&pl_empty[b], 1);
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 256);
        }
        for (int s = 0; s < C::MSLOTS; s++) mbar_init(&meta_empty[s], 256);
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer ----------------
        // lane 0 issues the tile copies; lane c stages column c's dx and pair sums (strided in
        // global memory) into the stage's metadata before lane 0 arrives on the full barrier
        // column c's dx and pair sums for super-block s, loaded one super-block ahead
        auto load_meta = [&](int s, float (&dx)[(N + 31) / 32], uint4 (&bs)[(N + 31) / 32]) {
#pragma unroll
            for (int i = 0; i < (N + 31) / 32; i++) {
                const int c = lane + 32 * i, col = c0 + c;
                dx[i] = 0.0f;
                bs[i] = make_uint4(0, 0, 0, 0);
                if (c < N && col < m && s < nsb) {
                    dx[i] = __ldg(&((const float*)a.d)[(size_t)col * nb + sb0 + s]);
                    bs[i] = __ldg((const uint4*)(a.bs32 + ((size_t)col * nb + sb0 + s) * 8));
                }
            }
        };
        float ndx[(N + 31) / 32];
        uint4 nbs[(N + 31) / 32];
        load_meta(0, ndx, nbs);
        for (int s = 0; s < nsb && ok; s++) {
            const int st = s % R, ms = s % C::MSLOTS;
            float cdx[(N + 31) / 32];
            uint4 cbs[(N + 31) / 32];
#pragma unroll
            for (int i = 0; i < (N + 31) / 32; i++) {
                cdx[i] = ndx[i];
                cbs[i] = nbs[i];
            }
            load_meta(s + 1, ndx, nbs);
            if (s >= R) {
                const uint32_t par = (uint32_t)(((s / R) - 1) & 1);
                ok = mbar_wait(&raw_empty[st], par, &g_tc_error) && mbar_wait(&act_empty[st], par, &g_tc_error);
            }
            if (ok && s >= C::MSLOTS)
                ok = mbar_wait(&meta_empty[ms], (uint32_t)(((s / C::MSLOTS) - 1) & 1), &g_tc_error);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            float* mdx = (float*)(meta + (size_t)ms * C::META);
            uint4* mbs = (uint4*)(mdx + N);
#pragma unroll
            for (int i = 0; i < (N + 31) / 32; i++) {
                const int c = lane + 32 * i;
                if (c < N) {
                    mdx[c] = cdx[i];
                    mbs[c] = cbs[i];
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[st], (uint32_t)(TC_WTILE + C::ATILE));
                tma_load_2d(raw + (size_t)st * TC_WTILE, &wmap, (sb0 + s) * (Q4_K_BYTES / 4), (int)r0, &full[st]);
                // the activation tile in one box: [16-B K chunk][row][16 B], the core-matrix layout
                tma_load_3d(act + (size_t)st * C::ATILE, &amap, 0, c0, (sb0 + s) * 16, &full[st]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8<N>();
            for (int s = 0; s < nsb && ok; s++) {
                const int st = s % R, b = s & 1;
                ok = mbar_wait(&full[st], (uint32_t)((s / R) & 1), &g_tc_error) &&
                     mbar_wait(&pl_full[b], (uint32_t)((s >> 1) & 1), &g_tc_error) &&
                     (s < 2 || mbar_wait(&acc_empty[b], (uint32_t)(((s >> 1) - 1) & 1), &g_tc_error));
                if (!ok) break;
                tc_fence_after();
                const uint32_t pH = smem_u32(planes + (size_t)(2 * b) * TC_PLANE);
                const uint32_t pL = pH + TC_PLANE;
                const uint32_t pa = smem_u32(act + (size_t)st * C::ATILE);
                const uint32_t dH = tmem + (uint32_t)(b * 2 * N), dL = dH + N;
#pragma unroll
                for (int j = 0; j < 8; j++) {   // k-step j: K chunks 2j, 2j+1
                    const uint64_t bd = umma_desc(pa + j * 2 * N * 16, N * 16, 128);
                    mma_i8(dH, umma_desc(pH + j * 256, 128, TC_PLANE_SBO), bd, idesc, j > 0);
                    mma_i8(dL, umma_desc(pL + j * 256, 128, TC_PLANE_SBO), bd, idesc, j > 0);
                }
                tc_commit(&pl_empty[b]);
                tc_commit(&act_empty[st]);
                tc_commit(&acc_full[b]);
            }
            tc_commit(mma_done);
            mbar_wait(mma_done, 0, &g_tc_error);
        }
    }

    // ---- prep (warps 2-9) and epilogue (warps 10-17): thread <-> weight row <-> TMEM lane; two
    // warps per row quarter, splitting the K chunks (prep) or the columns (epilogue) ----
    constexpr int NH = N / 2;                       // columns per epilogue thread
    float yacc[NH];
#pragma unroll
    for (int c = 0; c < NH; c++) yacc[c] = 0.0f;
    const int quarter = warp & 3;                   // TMEM lanes 32*quarter .. +31 for this warp
    const int row = quarter * 32 + lane;
    const int half = warp < TC_EPI0 ? (warp - 2) >> 2 : (warp - TC_EPI0) >> 2;
    if (warp >= 2 && warp < TC_EPI0) {
        for (int s = 0; s < nsb && ok; s++) {
            const int st = s % R, b = s & 1;
            ok = mbar_wait(&full[st], (uint32_t)((s / R) & 1), &g_tc_error) &&
                 (s < 2 || mbar_wait(&pl_empty[b], (uint32_t)(((s >> 1) - 1) & 1), &g_tc_error));
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const uint4* src = (const uint4*)(raw + (size_t)st * TC_WTILE + (size_t)row * Q4_K_BYTES);
            uint4 q[5];   // header + the 64 nibble bytes of this half (sub-blocks 4*half .. +3)
            q[0] = src[0];
#pragma unroll
            for (int i = 1; i < 5; i++) q[i] = src[half * 4 + i];
            mbar_arrive(&raw_empty[st]);
            const Q4kScales sc = q4k_unpack(q[0]);
            // the row's d | dmin, packed mins, for the epilogue of this super-block
            if (half == 0) rowp[(s % C::MSLOTS) * TC_ROWS + row] = make_uint4(q[0].x, sc.mn03, sc.mn47, 0u);
            uint8_t* pH = planes + (size_t)(2 * b) * TC_PLANE + (size_t)(row >> 3) * TC_PLANE_SBO + (row & 7) * 16;
            uint8_t* pL = pH + TC_PLANE;
            const uint32_t* qs = (const uint32_t*)&q[1];   // nibble bytes 64*half .. +63
#pragma unroll
            for (int kh = 0; kh < 8; kh++) {    // elements 16kc .. 16kc+15: sub-block kc/2
                const int kc = half * 8 + kh;
                const int sbk = kc >> 1, g = (kh >> 1) >> 1;
                const uint32_t scs = ((sbk < 4 ? sc.sc03 : sc.sc47) >> (8 * (sbk & 3))) & 0x3Fu;
                const uint32_t sh = scs >> 3, sl = scs & 7u;
                uint4 vh, vl;
                uint32_t* ph = (uint32_t*)&vh;
                uint32_t* pl = (uint32_t*)&vl;
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const uint32_t word = qs[g * 8 + (kc & 1) * 4 + w];
                    const uint32_t nib = (sbk & 1) ? (word >> 4) & 0x0F0F0F0Fu : word & 0x0F0F0F0Fu;
                    ph[w] = nib * sh;
                    pl[w] = nib * sl;
                }
                *(uint4*)(pH + kc * 128) = vh;
                *(uint4*)(pL + kc * 128) = vl;
            }
            fence_proxy_async_smem();
            mbar_arrive(&pl_full[b]);
        }
    } else if (warp >= TC_EPI0) {
        for (int e = 0; e < nsb && ok; e++) {
            const int b = e & 1, ms = e % C::MSLOTS;
            // warp-uniform outcome: the TMEM loads below are .sync.aligned
            ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (uint32_t)((e >> 1) & 1), &g_tc_error));
            if (!ok) break;
            tc_fence_after();
            const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 2 * N + half * NH);
            const uint4 rp = rowp[ms * TC_ROWS + row];
            const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&rp.x));
            // mins as (m0, m1), (m2, m3), ... pairs in the low bytes for dp2a
            const int mp0 = (int)(rp.y & 0xFFu) | (int)((rp.y >> 8) & 0xFFu) << 8;
            const int mp1 = (int)((rp.y >> 16) & 0xFFu) | (int)(rp.y >> 24) << 8;
            const int mp2 = (int)(rp.z & 0xFFu) | (int)((rp.z >> 8) & 0xFFu) << 8;
            const int mp3 = (int)((rp.z >> 16) & 0xFFu) | (int)(rp.z >> 24) << 8;
            const float* mdx = (const float*)(meta + (size_t)ms * C::META) + half * NH;
            const uint4* mbs = (const uint4*)((const float*)(meta + (size_t)ms * C::META) + N) + half * NH;
#pragma unroll
            for (int cc = 0; cc < NH; cc += 16) {
                uint32_t h[16], l[16];
                tmem_ld16(lane_addr + cc, h);
                tmem_ld16(lane_addr + N + cc, l);
                tmem_wait_ld();
                if (cc + 16 == NH) {   // all reads of this buffer issued and complete
                    tc_fence_before();
                    mbar_arrive(&acc_empty[b]);
                }
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float dx = mdx[cc + j];       // 0 for columns past m
                    const uint4 bs = mbs[cc + j];
                    int ms = __dp2a_lo((int)bs.x, mp0, 0);
                    ms = __dp2a_lo((int)bs.y, mp1, ms);
                    ms = __dp2a_lo((int)bs.z, mp2, ms);
                    ms = __dp2a_lo((int)bs.w, mp3, ms);
                    const int isum = 8 * (int)h[j] + (int)l[j];
                    yacc[cc + j] += dx * (dd.x * (float)isum - dd.y * (float)ms);
                }
            }
            mbar_arrive(&meta_empty[ms]);   // row parameters and metadata of super-block e released
        }
    }

    // ---------------- output: direct, or rank-ordered sum over the split cluster ----------------
    tc_fence_before();
    __syncthreads();   // every MMA retired (mma_done) and every TMEM read done
    float* red = (float*)planes;   // [N][128] partial tile, reusing the plane buffers
    if (gridDim.z == 1) {
        if (warp >= TC_EPI0 && r0 + row < n)
#pragma unroll
            for (int c = 0; c < NH; c++)
                if (c0 + half * NH + c < m) y[(size_t)(c0 + half * NH + c) * n + r0 + row] = yacc[c];
    } else {
        if (warp >= TC_EPI0)
#pragma unroll
            for (int c = 0; c < NH; c++) red[(half * NH + c) * TC_ROWS + row] = yacc[c];
        cluster_sync_all();
        if (cluster_rank() == 0)
            for (int idx = threadIdx.x; idx < N * TC_ROWS; idx += TC_THREADS) {
                const int rr = idx % TC_ROWS, c = idx / TC_ROWS;
                float sum = 0.0f;
                for (uint32_t q = 0; q < gridDim.z; q++) sum += ld_cluster_f32(red + idx, q);
                if (c0 + c < m && r0 + rr < n) y[(size_t)(c0 + c) * n + r0 + rr] = sum;
            }
        cluster_sync_all();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
    }
    pdl_trigger();   // dependents are released only after this CTA's tensor memory is free
}

// ---- host side ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();  // qmm.cu

static cudaError_t tc_maps(CUtensorMap* wm, CUtensorMap* am, const void* W, int64_t n, int64_t k, const void* qs,
                           int64_t m, int N) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const size_t row_bytes = (size_t)(k / QK_K) * Q4_K_BYTES;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)n};
        const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
        const cuuint32_t box[2] = {(cuuint32_t)(Q4_K_BYTES / 4), (cuuint32_t)TC_ROWS};
        const cuuint32_t estr[2] = {1, 1};
        if (fn(wm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(W), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {   // Q8_K quants as [k/16 chunks][m rows][16 B]: dims (16 B, rows, chunks), strides (k, 16)
        const cuuint64_t dims[3] = {16u, (cuuint64_t)m, (cuuint64_t)(k / 16)};
        const cuuint64_t strides[2] = {(cuuint64_t)k, 16u};
        const cuuint32_t box[3] = {16u, (cuuint32_t)N, 16u};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (fn(am, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(qs), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

template <int N>
static cudaError_t launch_tc_t(const uint8_t* W, int64_t n, int64_t k, const ActQ& a, int m, float* y,
                               cudaStream_t st) {
    using C = TcCfg<N>;
    cudaError_t e = DCG_SMEM_ATTR((qmm_q4k_tc_kernel<N>), C::SMEM);
    if (e != cudaSuccess) return e;
    CUtensorMap wm, am;
    e = tc_maps(&wm, &am, W, n, k, a.qs, m, N);
    if (e != cudaSuccess) return e;
    const int nb = (int)(k / QK_K);
    const int rt = (int)((n + TC_ROWS - 1) / TC_ROWS), ct = (m + N - 1) / N;
    int S = 148 / (rt * ct);                             // one CTA per SM: at most one wave
    S = S < 1 ? 1 : S;
    S = S > 8 ? 8 : S;
    S = S > nb / 2 ? (nb / 2 > 0 ? nb / 2 : 1) : S;     // >= 2 super-blocks per split
    const int sps = (nb + S - 1) / S;
    S = (nb + sps - 1) / sps;
    return launch_ex(qmm_q4k_tc_kernel<N>, dim3((unsigned)rt, (unsigned)ct, (unsigned)S), dim3(TC_THREADS),
                     (size_t)C::SMEM, st, (unsigned)S, wm, am, nb, n, a, m, y, sps);
}

bool qmm_tc_supports(int type, int64_t n, int64_t k, int64_t m) {
    return type == DCG_TYPE_Q4_K && m >= 2 && k % QK_K == 0 && n > 0;
}

cudaError_t launch_qmm_tc(const void* packed_w, int64_t n, int64_t k, const void* act, int64_t m, float* y,
                          cudaStream_t st) {
    const ActQ a = act_view(DCG_TYPE_Q8_K, const_cast<void*>(act), m, k);
    return launch_tc_t<32>((const uint8_t*)packed_w, n, k, a, (int)m, y, st);
}

}  // namespace dcg
