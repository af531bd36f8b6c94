// qmm.cu -- quantized weight x quantized activation matmul on the int8 tensor cores
// (mma.sync m16n8k32 s8 -> s32), for every M: the decode GEMV (M < 16) and the batched-decode /
// prefill GEMM.  Replaces cb_gemv_custom's vec_dot row loop and ggml_mul_mat
// (core/src/inference.cpp:840-948, :1063, :1794-1797, :1817).
//
// Tiling.  A CTA (4 warps) owns 64 weight rows (16 per warp: the mma's M dimension) and 8*NT
// activation rows (NT mma n-tiles), over a contiguous range of K super-blocks (split-K when the
// row blocks alone cannot fill the GPU).  K is streamed in chunks of KS super-blocks: each chunk
// is one bulk copy (TMA) per weight row into a padded shared-memory row (stride = 32 mod 128 B,
// so the fragment loads are bank-conflict free), STAGES chunks in flight on mbarriers.
//
// Fragments.  The products of one 32-element sub-block are an m16n8k32 mma.  The mma's k order
// is a permutation of the sub-block's elements chosen so that lane (gid, tig) reads its A
// registers {a0,a2} from 8 consecutive bytes of weight row gid (and {a1,a3} from row gid+8) and
// its B registers from 8 consecutive activation bytes: mma k slots 4*tig..+3 <-> elements
// 8*tig..+3, slots 16+4*tig..+3 <-> elements 8*tig+4..+7.  Q4_K's sub-blocks 2g and 2g+1 share
// their 32 bytes (low / high nibbles), so one 8-byte load per row feeds two mmas.
//
// Scales.  Each mma result (exact int32 dot of one sub-block) is multiplied by its 6-bit
// sub-block scale and summed in int32 over the super-block; the Q4_K min term
// sum_j m_j * bsum32_j uses dp2a on the packed 6-bit mins and the pair-summed Q8_K block sums;
// then y += dx * (d * isum - dmin * msum) in fp32 once per super-block.
//
// Split-K partials (M > 1) go to scratch; the last CTA of a tile (atomic ticket) adds them in split
// order, so results are deterministic.  Tickets must be zero when a launch starts and are left zero
// (dcg_mul_mat clears them inside its activation-quantize launch).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "quant_dev.cuh"
#include "tma.cuh"

#include <algorithm>
#include <mutex>
#include <stdlib.h>

namespace dcg {

__device__ int g_qmm_error = 0;

cudaError_t qmm_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_qmm_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_qmm_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int QMM_ROWS = 64;     // weight rows per CTA
constexpr int QMM_THREADS = 256;
constexpr int QMM_WARPS = 8;     // 4 row groups of 16 x 2 halves of each super-block
constexpr int QMM_KS = 2;        // super-blocks per stage
constexpr int QMM_STAGES = 3;
constexpr int Q4K_SROW = QMM_KS * Q4_K_BYTES;         // 288 B = 32 mod 128: conflict-free rows
constexpr int QMM_W_BYTES = QMM_ROWS * Q4K_SROW;      // weight part of a stage

__device__ __forceinline__ void mma_s8(int* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int byte_of(uint32_t w, int j) {  // zero-extended byte j (0..3)
    return (int)__byte_perm(w, 0u, 0x4440u + (uint32_t)j);
}

// packed Q4_K 6-bit scales / mins of one block header (ggml get_scale_min_k4, 4 per word)
template <int NT>
__global__ void __launch_bounds__(QMM_THREADS, NT >= 4 ? 1 : (NT >= 2 ? 2 : 3))
    qmm_q4k_kernel(const __grid_constant__ CUtensorMap wmap, int nb, int64_t n, ActQ a,
                   int64_t k, int m, float* __restrict__ y, float* __restrict__ part,
                   int* __restrict__ tickets, int S, int sps) {
    constexpr int XC = 8 * NT;                    // activation rows staged per CTA
    constexpr int SB_BYTES = QMM_W_BYTES;         // weights only: activations come through L1
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;             // [STAGES] bulk copies landed
    uint64_t* empty = full + QMM_STAGES;          // [STAGES] all warps done with the stage
    int* flag = (int*)(smem + 96);
    uint8_t* buf = smem + 128;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int rg = warp & 3;   // row group: rows 16*rg .. +15 of the CTA
    const int gh = warp >> 2;  // sub-block pairs g = 2*gh, 2*gh+1 (sub-blocks 4*gh .. 4*gh+3)
    // grid.x = activation column block (fastest: CTAs over the same weight rows run together and
    // share them through L2), grid.y = row block
    const int64_t r0 = (int64_t)blockIdx.y * QMM_ROWS;
    const int c0 = blockIdx.x * XC;
    const int split = blockIdx.z;
    const int sb0 = split * sps, sb1 = min(nb, sb0 + sps);
    const int nchunks = (sb1 - sb0 + QMM_KS - 1) / QMM_KS;
    const int rows_here = (int)((n - r0) < QMM_ROWS ? (n - r0) : QMM_ROWS);
    const int cols_here = min(XC, m - c0);

    pdl_wait();
    if (threadIdx.x == 0) {
        for (int s = 0; s < QMM_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], QMM_WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // warp 0: weight rows, activation rows and their Q8_K pair sums of chunk c -> stage c % STAGES
    auto issue = [&](int c) -> bool {
        const int st = c % QMM_STAGES;
        if (c >= QMM_STAGES && !mbar_wait(&empty[st], (uint32_t)(((c / QMM_STAGES) - 1) & 1), &g_qmm_error))
            return false;
        const int sbc = sb0 + c * QMM_KS;
        const int nsb = min(QMM_KS, sb1 - sbc);
        uint8_t* dst = buf + (size_t)st * SB_BYTES;
        // the weight box is always QMM_ROWS x QMM_KS blocks (rows past n / blocks past the row's end
        // are zero-filled and still counted)
        if (lane == 0) {
            mbar_arrive_expect_tx(&full[st], (uint32_t)QMM_W_BYTES);
            fence_proxy_async_smem();
            tma_load_2d(dst, &wmap, sbc * (Q4_K_BYTES / 4), (int)r0, &full[st]);
        }
        __syncwarp();
        return true;
    };
    bool ok = true;
    if (warp == 0)
        for (int c = 0; c < QMM_STAGES - 1 && c < nchunks; c++) ok = issue(c) && ok;

    float yacc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int i = 0; i < 4; i++) yacc[t][i] = 0.0f;

    const int nb_act = (int)(k / QK_K);
    const float* xd = (const float*)a.d;
    for (int c = 0; c < nchunks && ok; c++) {
        if (warp == 0 && c + QMM_STAGES - 1 < nchunks) ok = issue(c + QMM_STAGES - 1) && ok;
        const int sbc = sb0 + c * QMM_KS;
        const int nsb = min(QMM_KS, sb1 - sbc);
        // activation block scales of this chunk (global; overlaps the wait)
        float dxr[QMM_KS][NT][2];
#pragma unroll
        for (int s = 0; s < QMM_KS; s++)
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const int col = c0 + t * 8 + 2 * tig + cc;
                    dxr[s][t][cc] = (s < nsb && col < m) ? __ldg(&xd[(size_t)col * nb_act + sbc + s]) : 0.0f;
                }
        ok = mbar_wait(&full[c % QMM_STAGES], (uint32_t)((c / QMM_STAGES) & 1), &g_qmm_error) && ok;
        if (!ok) break;
        const uint8_t* stage = buf + (size_t)(c % QMM_STAGES) * SB_BYTES;
        // both super-blocks of the chunk, unconditionally (ILP): one that is absent (zero-filled by
        // the tensor copy) or belongs to the next split has dx = 0 and adds nothing
#pragma unroll
        for (int s = 0; s < QMM_KS; s++) {
            const uint8_t* rowA = stage + (rg * 16 + gid) * Q4K_SROW + s * Q4_K_BYTES;
            const uint8_t* rowB = rowA + 8 * Q4K_SROW;
            const uint4 hA = *(const uint4*)rowA, hB = *(const uint4*)rowB;
            const Q4kScales sA = q4k_unpack(hA), sB = q4k_unpack(hB);
            // scale folding: sc = 8*sh + sl (sh, sl in 0..7), q*sh and q*sl fit int8 and one 32-bit
            // multiply scales 4 nibbles at once, so all sub-blocks of the super-block accumulate in
            // two mma accumulators (no per-sub-block integer epilogue): isum = 8*Ch + Cl
            int ch[NT][4], cl[NT][4];
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
                for (int i = 0; i < 4; i++) ch[t][i] = cl[t][i] = 0;
#pragma unroll
            for (int gg = 0; gg < 2; gg++) {
                const int g = 2 * gh + gg;
                const uint2 wA = *(const uint2*)(rowA + 16 + 32 * g + 8 * tig);
                const uint2 wB = *(const uint2*)(rowB + 16 + 32 * g + 8 * tig);
                const uint32_t lo0 = wA.x & 0x0F0F0F0Fu, lo1 = wB.x & 0x0F0F0F0Fu;
                const uint32_t lo2 = wA.y & 0x0F0F0F0Fu, lo3 = wB.y & 0x0F0F0F0Fu;
                const uint32_t hi0 = (wA.x >> 4) & 0x0F0F0F0Fu, hi1 = (wB.x >> 4) & 0x0F0F0F0Fu;
                const uint32_t hi2 = (wA.y >> 4) & 0x0F0F0F0Fu, hi3 = (wB.y >> 4) & 0x0F0F0F0Fu;
                const uint32_t scw_A = gh == 0 ? sA.sc03 : sA.sc47, scw_B = gh == 0 ? sB.sc03 : sB.sc47;
                const uint32_t sA0 = byte_of(scw_A, (2 * g) & 3), sA1 = byte_of(scw_A, (2 * g + 1) & 3);
                const uint32_t sB0 = byte_of(scw_B, (2 * g) & 3), sB1 = byte_of(scw_B, (2 * g + 1) & 3);
                // sub-block 2g (low nibbles) and 2g+1 (high nibbles), rows A / B, high / low scale part
                const uint32_t h0a = lo0 * (sA0 >> 3), h0b = lo1 * (sB0 >> 3), h0c = lo2 * (sA0 >> 3), h0d = lo3 * (sB0 >> 3);
                const uint32_t l0a = lo0 * (sA0 & 7), l0b = lo1 * (sB0 & 7), l0c = lo2 * (sA0 & 7), l0d = lo3 * (sB0 & 7);
                const uint32_t h1a = hi0 * (sA1 >> 3), h1b = hi1 * (sB1 >> 3), h1c = hi2 * (sA1 >> 3), h1d = hi3 * (sB1 >> 3);
                const uint32_t l1a = hi0 * (sA1 & 7), l1b = hi1 * (sB1 & 7), l1c = hi2 * (sA1 & 7), l1d = hi3 * (sB1 & 7);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    uint2 x0 = make_uint2(0, 0), x1 = make_uint2(0, 0);
                    if (t * 8 + gid < cols_here && s < nsb) {
                        const int8_t* xp = a.qs + (size_t)(c0 + t * 8 + gid) * k + (size_t)(sbc + s) * QK_K +
                                           64 * g + 8 * tig;
                        x0 = __ldg((const uint2*)xp);
                        x1 = __ldg((const uint2*)(xp + 32));
                    }
                    mma_s8(ch[t], h0a, h0b, h0c, h0d, x0.x, x0.y);
                    mma_s8(cl[t], l0a, l0b, l0c, l0d, x0.x, x0.y);
                    mma_s8(ch[t], h1a, h1b, h1c, h1d, x1.x, x1.y);
                    mma_s8(cl[t], l1a, l1b, l1c, l1d, x1.x, x1.y);
                }
            }
            int isum[NT][4];
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
                for (int i = 0; i < 4; i++) isum[t][i] = 8 * ch[t][i] + cl[t][i];
            const float2 dA = __half22float2(*reinterpret_cast<const __half2*>(&hA.x));
            const float2 dB = __half22float2(*reinterpret_cast<const __half2*>(&hB.x));
#pragma unroll
            for (int t = 0; t < NT; t++) {
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const int lc = t * 8 + 2 * tig + cc;
                    if (lc >= cols_here) continue;
                    // this warp's half of the min term: sub-blocks 4*gh .. 4*gh+3
                    if (s >= nsb) continue;
                    const uint2 bs = __ldg((const uint2*)(a.bs32 + (size_t)(c0 + lc) * (k / 32) +
                                                          (size_t)(sbc + s) * 8 + 4 * gh));
                    const float dx = dxr[s][t][cc];
                    const uint32_t mnA = gh == 0 ? sA.mn03 : sA.mn47, mnB = gh == 0 ? sB.mn03 : sB.mn47;
                    const int mA = __dp2a_hi((int)bs.y, (int)mnA, __dp2a_lo((int)bs.x, (int)mnA, 0));
                    const int mB = __dp2a_hi((int)bs.y, (int)mnB, __dp2a_lo((int)bs.x, (int)mnB, 0));
                    yacc[t][cc] += dx * (dA.x * (float)isum[t][cc] - dA.y * (float)mA);
                    yacc[t][2 + cc] += dx * (dB.x * (float)isum[t][2 + cc] - dB.y * (float)mB);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[c % QMM_STAGES]);
    }
    pdl_trigger();
    ok = __syncthreads_and(ok);
    if (!ok) return;
    // combine the two super-block halves of each row group (stage buffers are free now)
    float* red = (float*)buf;
    if (gh == 1) {
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int i = 0; i < 4; i++) red[((rg * NT + t) * 4 + i) * 32 + lane] = yacc[t][i];
    }
    __syncthreads();
    const bool writer = gh == 0;  // the gh == 1 warps stay for the barriers below
    if (writer) {
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int i = 0; i < 4; i++) yacc[t][i] += red[((rg * NT + t) * 4 + i) * 32 + lane];
    }

    // ---- epilogue: c0/c1 -> row gid, cols 2tig,2tig+1; c2/c3 -> row gid+8 ----
    const int64_t rowA = r0 + rg * 16 + gid, rowB = rowA + 8;
    if (S == 1) {
        if (!writer) return;
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int col = c0 + t * 8 + 2 * tig + (i & 1);
                const int64_t row = i < 2 ? rowA : rowB;
                if (col < m && row < n) y[(size_t)col * n + row] = yacc[t][i];
            }
        return;
    }
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (!writer) break;
            const int col = c0 + t * 8 + 2 * tig + (i & 1);
            const int64_t row = i < 2 ? rowA : rowB;
            if (col < m && row < n) part[((size_t)split * m + col) * n + row] = yacc[t][i];
        }
    __threadfence();
    __syncthreads();
    int* ticket = &tickets[blockIdx.y * gridDim.x + blockIdx.x];
    if (threadIdx.x == 0) *flag = (atomicAdd(ticket, 1) == S - 1);
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    for (int i = threadIdx.x; i < cols_here * rows_here; i += blockDim.x) {
        const int col = c0 + i / rows_here;
        const int64_t row = r0 + i % rows_here;
        float sum = 0.0f;
        for (int q = 0; q < S; q++) sum += __ldcg(&part[((size_t)q * m + col) * n + row]);
        y[(size_t)col * n + row] = sum;
    }
    if (threadIdx.x == 0) *ticket = 0;
}

// ------------------------------------------------------------------------------------------
// M == 1 (decode GEMV): the mma's 8 columns carry the 8 sub-blocks of a super-block.
// k slots 4*tig..+3 of an mma hold 4 elements of sub-block 2*tig (low nibbles of qs pair group
// tig), slots 16+4*tig..+3 the same 4 elements of sub-block 2*tig+1 (high nibbles of the same
// bytes).  B column c carries the activation of sub-block c in exactly those slots and zeros
// elsewhere, so 8 chained mmas (elements 4i..4i+3 of every sub-block, i = 0..7) leave the exact
// int32 dot of row r with sub-block c in C[r][c].  Lane (gid, tig) thus ends a super-block holding
// the dots of sub-blocks 2*tig, 2*tig+1 for rows gid and gid+8 and applies their 6-bit scales and
// mins itself; only lanes with gid>>1 == tig feed nonzero activation bytes (others read a zero pad).
//
// The CTA's slice of the activation (its split's super-blocks) sits in shared memory for the whole
// launch: either quantized to Q8_K right here from the fp32 input (QX: dcg_mul_mat's fused path,
// the same arithmetic and bytes as the stand-alone quantize kernel) or copied from a quantized
// activation, by all five warps, while the producer warp's first weight fill is in flight.  The
// ring is then kept full by that producer warp.  The S split-K CTAs of a row block form one thread
// block cluster; rank 0 adds their 64-row partials in rank order through distributed shared memory
// (deterministic, no global partials, no tickets).
// ------------------------------------------------------------------------------------------
constexpr int M1_WARPS = 4;        // consumer warps; warp 4 only issues the copies
constexpr int M1_THREADS = 160;
// super-blocks per ring stage: one 2-D box of 64 rows x M1_SBS super-blocks (wider boxes move more
// bytes per row segment; 144-B rows, M1_SBS = 1, keep the consumer's loads free of bank conflicts)
#ifndef DCG_M1_SBS
#define DCG_M1_SBS 1
#endif
constexpr int M1_SBS = DCG_M1_SBS;
constexpr int M1_SROW = Q4_K_BYTES * M1_SBS;       // smem row stride of a stage
constexpr int M1_STAGE = QMM_ROWS * M1_SROW;       // M1_SBS super-blocks of 64 rows
constexpr int M1_HDR = 512;                        // barriers | zero pad | 64 row partials
constexpr int M1_XQ = QK_K + 16 + 4;               // per super-block: quants, pair sums, d
constexpr int M1_MAX_SPS = 32;                     // activation slice: at most 32 super-blocks
// resident CTAs per SM and weight ring depth (swept 2..6 x 2..7 on config 2; the macros exist only
// for such sweeps)
#ifndef DCG_M1_CTAS
#define DCG_M1_CTAS 4
#endif
#ifndef DCG_M1_STAGES
#define DCG_M1_STAGES 4
#endif
constexpr int M1_CTAS = DCG_M1_CTAS;
constexpr int M1_STAGES = DCG_M1_STAGES;
constexpr int M1_MAX_CLUSTER = 8;                  // portable cluster size bounds the splits

template <bool QX>
__global__ void __launch_bounds__(M1_THREADS, M1_CTAS)
    qmm_q4k_m1_kernel(const __grid_constant__ CUtensorMap wmap, int nb, int64_t n, ActQ a,
                      const float* __restrict__ x, float* __restrict__ y, int sps) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;
    uint64_t* empty = full + M1_STAGES;
    uint8_t* zpad = smem + 128;   // 64 zero bytes: the activation words of inactive lanes
    float* ypart = (float*)(smem + 256);
    uint8_t* ring = smem + M1_HDR;
    int8_t* xqs = (int8_t*)(ring + M1_STAGES * M1_STAGE);
    int16_t* xbs = (int16_t*)(xqs + (size_t)sps * QK_K);
    float* xd = (float*)(xbs + (size_t)sps * 8);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int64_t r0 = (int64_t)blockIdx.x * QMM_ROWS;
    const int sb0 = blockIdx.z * sps, sb1 = min(nb, sb0 + sps);
    const int nchunks = sb1 - sb0;                 // super-blocks of this split
    const int nst = (nchunks + M1_SBS - 1) / M1_SBS;   // ring stages

    if (threadIdx.x < 16) ((uint32_t*)zpad)[threadIdx.x] = 0u;
    if (threadIdx.x < QMM_ROWS) ypart[threadIdx.x] = 0.0f;
    if (threadIdx.x == 0) {
        for (int s = 0; s < M1_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], M1_WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // producer lane: the first ring fill, then all warps stage the activation slice
    const int pre = min(M1_STAGES, nst);
    auto issue = [&](int c) {
        const int st = c % M1_STAGES;
        mbar_arrive_expect_tx(&full[st], (uint32_t)M1_STAGE);
        fence_proxy_async_smem();
        tma_load_2d(ring + (size_t)st * M1_STAGE, &wmap, (sb0 + c * M1_SBS) * (Q4_K_BYTES / 4), (int)r0, &full[st]);
    };
    if (warp == M1_WARPS && lane == 0)
        for (int c = 0; c < pre; c++) issue(c);
    pdl_wait();
    constexpr int NW = M1_WARPS + 1;
    if (QX) {  // quantize: warp w takes super-blocks w, w + 5, ..., two at a time (loads overlap)
        for (int s = warp; s < nchunks; s += 2 * NW) {
            const int s2 = s + NW;
            const bool two = s2 < nchunks;  // warp-uniform
            const float4* p1 = (const float4*)(x + (size_t)(sb0 + s) * QK_K + lane * 8);
            const float4* p2 = (const float4*)(x + (size_t)(sb0 + (two ? s2 : s)) * QK_K + lane * 8);
            const float4 u0 = __ldg(p1), u1 = __ldg(p1 + 1), w0 = __ldg(p2), w1 = __ldg(p2 + 1);
            const float v1[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            const float v2[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            const Q8KLane q1 = warp_q8_K(v1, lane);
            const Q8KLane q2 = warp_q8_K(v2, lane);
            *(uint2*)(xqs + s * QK_K + lane * 8) = make_uint2(q1.w0, q1.w1);
            if ((lane & 3) == 0) xbs[s * 8 + (lane >> 2)] = (int16_t)q1.s32;
            if (lane == 0) xd[s] = q1.d;
            if (two) {
                *(uint2*)(xqs + s2 * QK_K + lane * 8) = make_uint2(q2.w0, q2.w1);
                if ((lane & 3) == 0) xbs[s2 * 8 + (lane >> 2)] = (int16_t)q2.s32;
                if (lane == 0) xd[s2] = q2.d;
            }
        }
    } else {   // copy the slice of an already quantized activation
        const int t = threadIdx.x;
        for (int i = t; i < nchunks * (QK_K / 16); i += M1_THREADS)
            ((uint4*)xqs)[i] = __ldg((const uint4*)(a.qs + (size_t)sb0 * QK_K) + i);
        for (int i = t; i < nchunks * 8; i += M1_THREADS) xbs[i] = a.bs32[(size_t)sb0 * 8 + i];
        for (int i = t; i < nchunks; i += M1_THREADS) xd[i] = ((const float*)a.d)[sb0 + i];
    }
    __syncthreads();

    bool ok = true;
    if (warp == M1_WARPS) {  // producer: keep the ring full
        if (lane == 0) {
            for (int c = pre; c < nst && ok; c++) {
                ok = mbar_wait(&empty[c % M1_STAGES], (uint32_t)(((c / M1_STAGES) - 1) & 1), &g_qmm_error);
                if (ok) issue(c);
            }
        }
    } else {
        const bool active = (gid >> 1) == tig;  // feeds column gid (sub-block gid) of every mma
        const bool odd = gid & 1;                // ... through b1 (odd sub-block) or b0 (even)
        float yA = 0.0f, yB = 0.0f;
        for (int c = 0; c < nst; c++) {
            ok = mbar_wait(&full[c % M1_STAGES], (uint32_t)((c / M1_STAGES) & 1), &g_qmm_error);
            if (!ok) break;
            const uint8_t* stage = ring + (size_t)(c % M1_STAGES) * M1_STAGE;
#pragma unroll
          for (int jj = 0; jj < M1_SBS; jj++) {
            const int cs = c * M1_SBS + jj;        // super-block within the split
            if (cs >= nchunks) break;
            const float dx = xd[cs];
            const uint8_t* rowA = stage + (warp * 16 + gid) * M1_SROW + jj * Q4_K_BYTES;
            const uint8_t* rowB = rowA + 8 * M1_SROW;
            const uint4 hA = *(const uint4*)rowA, hB = *(const uint4*)rowB;
            // weight words: pair group tig, elements 4i..4i+3 (i = 0..7) of rows gid / gid+8
            const uint4 a0 = *(const uint4*)(rowA + 16 + 32 * tig), a1 = *(const uint4*)(rowA + 32 + 32 * tig);
            const uint4 b0 = *(const uint4*)(rowB + 16 + 32 * tig), b1 = *(const uint4*)(rowB + 32 + 32 * tig);
            const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            // activation words of sub-block gid (active lanes) or zeros
            const uint8_t* xsrc = active ? (const uint8_t*)xqs + cs * QK_K + 32 * gid : zpad;
            const uint4 x0 = *(const uint4*)xsrc, x1 = *(const uint4*)(xsrc + 16);
            const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int acc[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t xv0 = odd ? 0u : xw[i], xv1 = odd ? xw[i] : 0u;
                mma_s8(acc, wa[i] & 0x0F0F0F0Fu, wb[i] & 0x0F0F0F0Fu, (wa[i] >> 4) & 0x0F0F0F0Fu,
                       (wb[i] >> 4) & 0x0F0F0F0Fu, xv0, xv1);
            }
            // acc: [0] row gid / sub-block 2tig, [1] row gid / 2tig+1, [2] row gid+8 / 2tig, [3] ...
            const Q4kScales sA = q4k_unpack(hA), sB = q4k_unpack(hB);
            const int sh = 16 * (tig & 1);
            const uint32_t scA = ((tig < 2 ? sA.sc03 : sA.sc47) >> sh) & 0xFFFFu;
            const uint32_t scB = ((tig < 2 ? sB.sc03 : sB.sc47) >> sh) & 0xFFFFu;
            const uint32_t mnA = ((tig < 2 ? sA.mn03 : sA.mn47) >> sh) & 0xFFFFu;
            const uint32_t mnB = ((tig < 2 ? sB.mn03 : sB.mn47) >> sh) & 0xFFFFu;
            const int isA = (int)(scA & 0xFF) * acc[0] + (int)(scA >> 8) * acc[1];
            const int isB = (int)(scB & 0xFF) * acc[2] + (int)(scB >> 8) * acc[3];
            const int bsp = *(const int*)(xbs + cs * 8 + 2 * tig);  // pair sums of sub-blocks 2tig, 2tig+1
            const int msA = __dp2a_lo(bsp, (int)mnA, 0), msB = __dp2a_lo(bsp, (int)mnB, 0);
            const float2 dA = __half22float2(*reinterpret_cast<const __half2*>(&hA.x));
            const float2 dB = __half22float2(*reinterpret_cast<const __half2*>(&hB.x));
            yA += dx * (dA.x * (float)isA - dA.y * (float)msA);
            yB += dx * (dB.x * (float)isB - dB.y * (float)msB);
          }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[c % M1_STAGES]);
        }
        yA += __shfl_xor_sync(0xffffffffu, yA, 1);
        yA += __shfl_xor_sync(0xffffffffu, yA, 2);
        yB += __shfl_xor_sync(0xffffffffu, yB, 1);
        yB += __shfl_xor_sync(0xffffffffu, yB, 2);
        if (tig == 0) {
            ypart[warp * 16 + gid] = yA;
            ypart[warp * 16 + gid + 8] = yB;
        }
    }
    // every thread of every CTA of the cluster reaches both barriers, on the error path too
    cluster_sync_all();
    if (cluster_rank() == 0 && threadIdx.x < QMM_ROWS && r0 + threadIdx.x < n) {
        float sum = 0.0f;
        for (uint32_t r = 0; r < gridDim.z; r++) sum += ld_cluster_f32(ypart + threadIdx.x, r);
        y[r0 + threadIdx.x] = sum;
    }
    cluster_sync_all();   // keeps every CTA's partials alive until rank 0 has read them
    pdl_trigger();
}

// split-K count: as many splits as still fit one wave of resident CTAs (ctas_per_sm x 148 SMs),
// keeping >= 2 super-blocks per split
static int qmm_splits(int tiles, int nb, int ctas_per_sm = 3) {
    const int slots = ctas_per_sm * 148;
    int S = slots / tiles;
    S = S < 1 ? 1 : S;
    S = S > nb / 2 ? (nb / 2 > 0 ? nb / 2 : 1) : S;
    const int sps = (nb + S - 1) / S;
    return (nb + sps - 1) / sps;
}

int qmm_ticket_count(int type, int64_t n, int64_t m) {
    (void)type;
    const int rb = (int)((n + QMM_ROWS - 1) / QMM_ROWS);
    const int nt = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
    const int cb = (int)((m + 8 * nt - 1) / (8 * nt));
    return rb * cb;
}

size_t qmm_scratch_bytes(int type, int64_t n, int64_t k, int64_t m) {
    (void)type;
    const int nb = (int)(k / QK_K);
    const int rb = (int)((n + QMM_ROWS - 1) / QMM_ROWS);
    const int nt = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
    const int cb = (int)((m + 8 * nt - 1) / (8 * nt));
    const int S = qmm_splits(rb * cb, nb);  // M == 1 needs none of it unless it falls back
    return align256((size_t)rb * cb * 4) + (S > 1 ? align256((size_t)S * m * n * 4) : 0);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// weight rows as a 2-D u32 tensor [n][row_bytes/4]; box = QMM_KS blocks x QMM_ROWS rows
static cudaError_t make_wmap(CUtensorMap* map, const void* W, int64_t n, size_t row_bytes,
                             int box_blocks = QMM_KS) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(box_blocks * Q4_K_BYTES / 4), (cuuint32_t)QMM_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(W), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int NT>
static cudaError_t launch_q4k_t(const uint8_t* W, int64_t n, int64_t k, const ActQ& a, int m, float* y,
                                void* scratch, cudaStream_t st) {
    const size_t smem = 128 + (size_t)M1_STAGES * QMM_W_BYTES;
    cudaError_t e = DCG_SMEM_ATTR((qmm_q4k_kernel<NT>), smem);
    if (e != cudaSuccess) return e;
    const int nb = (int)(k / QK_K);
    const int rb = (int)((n + QMM_ROWS - 1) / QMM_ROWS);
    const int cb = (m + 8 * NT - 1) / (8 * NT);
    int S = qmm_splits(rb * cb, nb);
    const int sps = (nb + S - 1) / S;
    S = (nb + sps - 1) / sps;
    int* tickets = (int*)scratch;
    float* part = (float*)((uint8_t*)scratch + align256((size_t)rb * cb * 4));
    CUtensorMap wmap;
    e = make_wmap(&wmap, W, n, (size_t)nb * Q4_K_BYTES);
    if (e != cudaSuccess) return e;
    dim3 grid(cb, rb, S);
    return launch_pdl(qmm_q4k_kernel<NT>, grid, dim3(QMM_THREADS), smem, st, wmap, nb, n, a, k, m, y,
                      part, tickets, S, sps);
}

// M == 1 grid: row blocks x S splits (one cluster of S CTAs per row block), S <= 8 and each
// split's activation slice <= M1_MAX_SPS super-blocks; cudaErrorNotSupported when K is too long.
static bool m1_plan(int64_t n, int64_t k, int* rb, int* S, int* sps) {
    const int nb = (int)(k / QK_K);
    *rb = (int)((n + QMM_ROWS - 1) / QMM_ROWS);
    int s = qmm_splits(*rb, nb, M1_CTAS);
    s = std::min(s, M1_MAX_CLUSTER);
    s = std::max(s, (nb + M1_MAX_SPS - 1) / M1_MAX_SPS);
    if (s > M1_MAX_CLUSTER) return false;
    *sps = (nb + s - 1) / s;
    *sps = (*sps + M1_SBS - 1) / M1_SBS * M1_SBS;   // splits start on a stage boundary
    if (*sps > M1_MAX_SPS) return false;
    *S = (nb + *sps - 1) / *sps;
    return true;
}

template <bool QX>
static cudaError_t launch_q4k_m1(const uint8_t* W, int64_t n, int64_t k, const ActQ& a, const float* x,
                                 float* y, cudaStream_t st) {
    int rb, S, sps;
    if (!m1_plan(n, k, &rb, &S, &sps)) return cudaErrorNotSupported;
    const size_t smem_max = M1_HDR + (size_t)M1_STAGES * M1_STAGE + (size_t)M1_MAX_SPS * M1_XQ;
    cudaError_t e = DCG_SMEM_ATTR((qmm_q4k_m1_kernel<QX>), smem_max);
    if (e != cudaSuccess) return e;
    const int nb = (int)(k / QK_K);
    CUtensorMap wmap;
    e = make_wmap(&wmap, W, n, (size_t)nb * Q4_K_BYTES, M1_SBS);
    if (e != cudaSuccess) return e;
    // A programmatic dependent whose own dependents are released only at its exit (after the
    // cluster reduction).  Released earlier, the next grid's clusters landed in a GPU still
    // holding this one and a config-2 step measured 28.3 us; in plain stream order 20.6 us; with
    // the release at exit 19.5 us (the next launch overlaps this one's drain).
    const size_t smem = M1_HDR + (size_t)M1_STAGES * M1_STAGE + (size_t)sps * M1_XQ;
    return launch_ex(qmm_q4k_m1_kernel<QX>, dim3(rb, 1, S), dim3(M1_THREADS), smem, st, (unsigned)S,
                     wmap, nb, n, a, x, y, sps);
}

bool qmm_m1_fused_supports(int type, int64_t n, int64_t k, int64_t m) {
    int rb, S, sps;
    return type == DCG_TYPE_Q4_K && m == 1 && m1_plan(n, k, &rb, &S, &sps);
}

cudaError_t launch_qmm_m1_fused(const void* packed_w, int64_t n, int64_t k, const float* x, float* y,
                                cudaStream_t st) {
    return launch_q4k_m1<true>((const uint8_t*)packed_w, n, k, ActQ{}, x, y, st);
}

bool qmm_supports(int type) { return type == DCG_TYPE_Q4_K; }

cudaError_t launch_qmm(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                       int64_t m, float* y, void* scratch, cudaStream_t st) {
    if (type != DCG_TYPE_Q4_K) return cudaErrorNotSupported;
    const ActQ a = act_view(DCG_TYPE_Q8_K, const_cast<void*>(act), m, k);
    const uint8_t* W = (const uint8_t*)packed_w;
    if (m == 1) {
        const cudaError_t e = launch_q4k_m1<false>(W, n, k, a, nullptr, y, st);
        if (e != cudaErrorNotSupported) return e;
    }
    if (m <= 8) return launch_q4k_t<1>(W, n, k, a, (int)m, y, scratch, st);
    if (m <= 16) return launch_q4k_t<2>(W, n, k, a, (int)m, y, scratch, st);
    return launch_q4k_t<4>(W, n, k, a, (int)m, y, scratch, st);
}

}  // namespace dcg
