// qmm_tc.cu -- Q4_K weight x Q8_K activation matmul on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory), for batched decode (column tiles of
// N = 32 activation rows).  Replaces ggml_mul_mat's vec_dot_q4_K_q8_K row loop for these shapes
// (core/src/inference.cpp:1063, :1794-1797; the dot product of simd_ops.cpp:82-93).
//
// One CTA owns 128 weight rows (the MMA's M) x N activation rows (the MMA's N) over a range of K
// super-blocks (split-K across a cluster when the tiles alone cannot fill the GPU).  Per
// super-block (K = 256):
//   producer warp   TMA: the 128 x 144 B Q4_K weight tile, and the N x 256 B Q8_K activation tile
//                   as 16 boxes of 16 B x N rows (the K-major no-swizzle core-matrix layout)
//   prep warpgroup  thread r expands weight row r into two int8 planes, H = q * sh and
//                   L = q * sl with the 6-bit sub-block scale sc = 8 * sh + sl (q <= 15, sh, sl
//                   <= 7: every product fits int8, four at a time in one 32-bit multiply), written
//                   in the core-matrix layout the MMA reads
//   MMA thread      16 x tcgen05.mma.kind::i8 (8 k-steps of 32 for each plane) into two int32
//                   accumulators C_H, C_L in tensor memory; double-buffered across super-blocks
//   epilogue        the same warpgroup: thread r reads row r of C_H, C_L (tcgen05.ld) and the
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
constexpr int TC_THREADS = 192;                  // warp 0 producer, warp 1 MMA, warps 2-5 prep/epilogue
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
    static constexpr int META = N * 4 + N * 16;                  // per column: dx, 8 pair sums
    static constexpr int OFF_META = OFF_PL + 4 * TC_PLANE;
    static constexpr int SMEM = OFF_META + STAGES * META;
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
    uint64_t* raw_empty = full + R;            // [R] 128 threads done with the weight tile and metadata
    uint64_t* act_empty = raw_empty + R;       // [R] MMAs that read the activation tile done
    uint64_t* pl_full = act_empty + R;         // [2] planes written (128 arrivals)
    uint64_t* pl_empty = pl_full + 2;          // [2] MMAs that read the planes done
    uint64_t* acc_full = pl_empty + 2;         // [2] accumulators complete
    uint64_t* acc_empty = acc_full + 2;        // [2] 128 epilogue threads read them
    uint64_t* mma_done = acc_empty + 2;        // [1] every MMA of the CTA retired
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
    uint8_t* raw = smem + C::OFF_RAW;
    uint8_t* act = smem + C::OFF_ACT;
    uint8_t* planes = smem + C::OFF_PL;
    uint8_t* meta = smem + C::OFF_META;        // [R][dx: N floats | pair sums: N x 8 int16]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * TC_ROWS;
    const int c0 = blockIdx.y * N;
    const int sb0 = blockIdx.z * sps, sb1 = min(nb, sb0 + sps);
    const int nsb = sb1 - sb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&raw_empty[s], 128);
            mbar_init(&act_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&pl_full[b], 128);
            mbar_init(&pl_empty[b], 1);
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
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
        for (int s = 0; s < nsb && ok; s++) {
            const int st = s % R;
            if (s >= R) {
                const uint32_t par = (uint32_t)(((s / R) - 1) & 1);
                ok = mbar_wait(&raw_empty[st], par, &g_tc_error) && mbar_wait(&act_empty[st], par, &g_tc_error);
            }
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            float* mdx = (float*)(meta + (size_t)st * C::META);
            uint4* mbs = (uint4*)(mdx + N);
            for (int c = lane; c < N; c += 32) {
                const int col = c0 + c;
                float dx = 0.0f;
                uint4 bs = make_uint4(0, 0, 0, 0);
                if (col < m) {
                    dx = __ldg(&((const float*)a.d)[(size_t)col * nb + sb0 + s]);
                    bs = __ldg((const uint4*)(a.bs32 + ((size_t)col * nb + sb0 + s) * 8));
                }
                mdx[c] = dx;
                mbs[c] = bs;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[st], (uint32_t)(TC_WTILE + C::ATILE));
                tma_load_2d(raw + (size_t)st * TC_WTILE, &wmap, (sb0 + s) * (Q4_K_BYTES / 4), (int)r0, &full[st]);
                uint8_t* dst = act + (size_t)st * C::ATILE;
#pragma unroll 4
                for (int kc = 0; kc < 16; kc++)   // 16-B K chunk kc of N rows -> [kc][row][16 B]
                    tma_load_2d(dst + kc * N * 16, &amap, (sb0 + s) * QK_K + kc * 16, c0, &full[st]);
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

    // ---------------- prep + epilogue: thread r <-> weight row r <-> TMEM lane r ----------------
    float yacc[N];
#pragma unroll
    for (int c = 0; c < N; c++) yacc[c] = 0.0f;
    const int quarter = warp & 3;                   // TMEM lanes 32*quarter .. +31 for this warp
    const int row = quarter * 32 + lane;
    if (warp >= 2) {
        float pd = 0.0f, pdm = 0.0f;                // previous super-block's d, dmin, packed mins
        uint32_t pmn03 = 0, pmn47 = 0;
        auto epilogue = [&](int e, float d, float dmin, uint32_t mn03, uint32_t mn47) -> bool {
            const int b = e & 1;
            // warp-uniform outcome: the TMEM loads below are .sync.aligned
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[b], (uint32_t)((e >> 1) & 1), &g_tc_error))) return false;
            tc_fence_after();
            const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 2 * N);
            // mins as (m0, m1), (m2, m3), ... pairs in the low bytes for dp2a
            const int mp0 = (int)(mn03 & 0xFFu) | (int)((mn03 >> 8) & 0xFFu) << 8;
            const int mp1 = (int)((mn03 >> 16) & 0xFFu) | (int)(mn03 >> 24) << 8;
            const int mp2 = (int)(mn47 & 0xFFu) | (int)((mn47 >> 8) & 0xFFu) << 8;
            const int mp3 = (int)((mn47 >> 16) & 0xFFu) | (int)(mn47 >> 24) << 8;
#pragma unroll
            for (int cc = 0; cc < N; cc += 16) {
                uint32_t h[16], l[16];
                tmem_ld16(lane_addr + cc, h);
                tmem_ld16(lane_addr + N + cc, l);
                tmem_wait_ld();
                if (cc + 16 == N) {   // all reads of this buffer issued and complete
                    tc_fence_before();
                    mbar_arrive(&acc_empty[b]);
                }
                const float* mdx = (const float*)(meta + (size_t)(e % R) * C::META);
                const uint4* mbs = (const uint4*)(mdx + N);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float dx = mdx[cc + j];       // 0 for columns past m
                    const uint4 bs = mbs[cc + j];
                    int ms = __dp2a_lo((int)bs.x, mp0, 0);
                    ms = __dp2a_lo((int)bs.y, mp1, ms);
                    ms = __dp2a_lo((int)bs.z, mp2, ms);
                    ms = __dp2a_lo((int)bs.w, mp3, ms);
                    const int isum = 8 * (int)h[j] + (int)l[j];
                    yacc[cc + j] += dx * (d * (float)isum - dmin * (float)ms);
                }
            }
            mbar_arrive(&raw_empty[e % R]);   // weight tile and metadata of super-block e released
            return true;
        };
        for (int s = 0; s < nsb && ok; s++) {
            const int st = s % R, b = s & 1;
            ok = mbar_wait(&full[st], (uint32_t)((s / R) & 1), &g_tc_error) &&
                 (s < 2 || mbar_wait(&pl_empty[b], (uint32_t)(((s >> 1) - 1) & 1), &g_tc_error));
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const uint4* src = (const uint4*)(raw + (size_t)st * TC_WTILE + (size_t)row * Q4_K_BYTES);
            uint4 q[9];
#pragma unroll
            for (int i = 0; i < 9; i++) q[i] = src[i];
            const Q4kScales sc = q4k_unpack(q[0]);
            const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&q[0].x));
            uint8_t* pH = planes + (size_t)(2 * b) * TC_PLANE + (size_t)(row >> 3) * TC_PLANE_SBO + (row & 7) * 16;
            uint8_t* pL = pH + TC_PLANE;
            const uint32_t* qs = (const uint32_t*)&q[1];   // 128 bytes of nibbles
#pragma unroll
            for (int kc = 0; kc < 16; kc++) {   // elements 16kc .. 16kc+15: sub-block kc/2
                const int sbk = kc >> 1, g = sbk >> 1;
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
            if (s > 0) ok = epilogue(s - 1, pd, pdm, pmn03, pmn47);
            pd = dd.x;
            pdm = dd.y;
            pmn03 = sc.mn03;
            pmn47 = sc.mn47;
        }
        if (ok && nsb > 0) ok = epilogue(nsb - 1, pd, pdm, pmn03, pmn47);
    }

    // ---------------- output: direct, or rank-ordered sum over the split cluster ----------------
    tc_fence_before();
    __syncthreads();   // every MMA retired (mma_done) and every TMEM read done
    float* red = (float*)planes;   // [N][128] partial tile, reusing the plane buffers
    if (gridDim.z == 1) {
        if (warp >= 2 && r0 + row < n)
#pragma unroll
            for (int c = 0; c < N; c++)
                if (c0 + c < m) y[(size_t)(c0 + c) * n + r0 + row] = yacc[c];
    } else {
        if (warp >= 2)
#pragma unroll
            for (int c = 0; c < N; c++) red[c * TC_ROWS + row] = yacc[c];
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
    pdl_trigger();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
    }
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
    {
        const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
        const cuuint64_t strides[1] = {(cuuint64_t)k};
        const cuuint32_t box[2] = {16u, (cuuint32_t)N};
        const cuuint32_t estr[2] = {1, 1};
        if (fn(am, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(qs), dims, strides, box, estr,
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
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(qmm_q4k_tc_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    CUtensorMap wm, am;
    cudaError_t e = tc_maps(&wm, &am, W, n, k, a.qs, m, N);
    if (e != cudaSuccess) return e;
    const int nb = (int)(k / QK_K);
    const int rt = (int)((n + TC_ROWS - 1) / TC_ROWS), ct = (m + N - 1) / N;
    int S = 148 / (rt * ct);                             // one CTA per SM: at most one wave
    S = S < 1 ? 1 : S;
    S = S > 8 ? 8 : S;
    S = S > nb / 2 ? (nb / 2 > 0 ? nb / 2 : 1) : S;     // >= 2 super-blocks per split
    const int sps = (nb + S - 1) / S;
    S = (nb + sps - 1) / sps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)rt, (unsigned)ct, (unsigned)S);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = S;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmm_q4k_tc_kernel<N>, wm, am, nb, n, a, m, y, sps);
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
