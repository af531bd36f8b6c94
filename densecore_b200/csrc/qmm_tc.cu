// qmm_tc.cu -- Q4_K / Q6_K weight x Q8_K activation matmul on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in tensor memory) for every M >= 2: batched decode and
// prefill.  Replaces ggml_mul_mat's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K row loops for these
// shapes (core/src/inference.cpp:1063, :1794-1797, :1817; the dot products of simd_ops.cpp:82-93).
//
// Work decomposition (stream-K).  A unit is one 128-row weight tile x one N-column activation tile
// x one K super-block (256).  The units are ordered tile by tile (column tiles of a row tile next
// to each other, so their shared weights come from L2) and split into G contiguous ranges, one per
// CTA (G <= number of SMs, one CTA per SM): every SM streams the same number of weight bytes,
// whatever the tile count, and its pipeline never drains between tiles.  A tile whose units span
// several CTAs is finished by the last of them to arrive (atomic ticket): each writes its partial
// tile to scratch, and the last sums all partials in CTA order, so results are deterministic.
//
// Per unit (super-block), warp-specialised:
//   warp 0      TMA: the 128-row weight tile (Q4_K 144 B, Q6_K 208 B per row) into a WS-deep ring
//   warp 1      TMA: the N x 256 B Q8_K activation tile as one 3-D box in the K-major no-swizzle
//               core-matrix layout the MMA reads, into an AS-deep ring; its lanes stage the
//               columns' scales dx (and the Q4_K min-term pair sums) in a metadata ring
//   warp 2      one thread issues per K half 4 k-steps x 2 planes of M128 x N x K32 MMAs into
//               C_H, C_L (double-buffered across units) and releases stages with tcgen05.commit
//   warps 4-19  expand unit i's weights and drain unit i-1's accumulators (tcgen05.ld), in one of
//               three forms (TcCfg):
//     SB8 (Q4_K, N <= 32)  one plane of the unscaled 4-bit quants as int8 in shared memory, one
//               MMA per 32-element sub-block into its own accumulator region; the drain forms
//               isum = sum_j sc_j C_j in integers, y += dx (d isum - dmin sum_j m_j bsum32_j)
//     TA (Q4_K N = 64, Q6_K N <= 64)  two int8 planes with q * scale = SHIFT * H + L exactly,
//               stored into tensor memory (tcgen05.st) and read there by the MMAs:
//                 Q4_K  sc = 8 sh + sl (sh, sl <= 7): H = q sh, L = q sl (q <= 15), SHIFT = 8
//                 Q6_K  p = (u - 32) sc (u the unsigned 6-bit quant, sc the signed 8-bit sub-block
//                       scale): H = p >> 7, L = p & 127, SHIFT = 128 (the -32 offset is folded in)
//               the drain forms isum = SHIFT C_H + C_L, y += dx (d isum [- dmin msum])
//     N = 128 (prefill)  the same two planes in shared memory
//               In SB8 and TA warps 4-11 only expand and warps 12-19 only drain, so the expansion
//               of unit i+1 overlaps the drain of unit i; for N = 128 all 16 do both.
// Every wait is bounded (device error flag); tensor memory is always freed before exit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace dcg {

__device__ int g_tc_error = 0;

// Pipeline timeline for tuning, compiled in only with -DDCG_TC_TRACE (never in the library build):
// clock64 stamps of 12 events for the first 64 units of CTAs 0-3 (g_tc_trace[cta][unit][event]).
#ifdef DCG_TC_TRACE
__device__ long long g_tc_trace[4][64][12];
#define TC_TRACE(i, ev)                                                                            \
    do {                                                                                           \
        if (blockIdx.x < 4 && (i) < 64) g_tc_trace[blockIdx.x][(i)][(ev)] = clock64();             \
    } while (0)
extern "C" int dcg_debug_tc_trace(void* out) {
    return (int)cudaMemcpyFromSymbol(out, g_tc_trace, sizeof(g_tc_trace));
}
#else
#define TC_TRACE(i, ev) \
    do {                \
    } while (0)
#endif

cudaError_t qmm_tc_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_tc_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int TC_ROWS = 128;      // weight rows per tile (the MMA's M)
constexpr int TC_THREADS = 640;   // 20 warps: 0 weight TMA, 1 activation TMA, 2 MMA, 3 spare, 4-19 prep + epilogue
constexpr int TC_WORK0 = 4;
constexpr int TC_WORKERS = 16;
constexpr int TC_HPLANE = TC_ROWS * 128;   // one int8 plane of a K half: 16 KB
constexpr int TC_HSBO = 8 * 128;           // plane: 8-row groups 1 KB apart, 16-B K chunks 128 B apart
constexpr int TC_MS = 4;                   // metadata slots (dx, pair sums, row scales)
constexpr int TC_SMEM_MAX = 232448;        // 227 KB opt-in

template <int TYPE>
struct TcW;
template <>
struct TcW<DCG_TYPE_Q4_K> {
    static constexpr int ROWB = Q4_K_BYTES;     // bytes per row per super-block in the device layout
    static constexpr int SHIFT = 8;
};
template <>
struct TcW<DCG_TYPE_Q6_K> {
    static constexpr int ROWB = Q6_K_PAYLOAD;   // ql | qh | scales (fp16 d is a separate array)
    static constexpr int SHIFT = 128;
};

template <int TYPE, int N>
struct TcCfg {
    static constexpr int WT = TC_ROWS * TcW<TYPE>::ROWB;          // weight tile per unit
    static constexpr int AT = N * QK_K;                            // activation tile per unit
    static constexpr int AS = N >= 128 ? 2 : (N >= 64 ? 3 : 4);    // activation ring
    static constexpr int META = N * 4 + N * 16;                    // per column: dx, 8 pair sums
    static constexpr int OFF_BAR = 0;                              // barriers, flag, TMEM slot
    // plane buffers: two (units alternate, so the prep of unit i+1 need not wait for unit i's
    // MMAs) where shared memory allows, else one
    // TA: the planes live in tensor memory (A operand read from TMEM), for N <= 64, where they fit
    // beside the accumulators: columns [0, 4N) accumulators, [TMEM_PL + 128 pb + 64 h, +32) H and
    // [+32, +64) L of plane buffer pb, K half h (three buffers for N <= 32, two for N = 64).
    // Otherwise in shared memory.
    // SB8 (Q4_K, N <= 32): one unscaled plane (the 4-bit quants as int8) in shared memory and one
    // MMA per sub-block into its own accumulator region, [2 buffers][8 sub-blocks] x N columns; the
    // drain applies the 6-bit scales as integers.  Half the MMAs of the two-plane form.
    static constexpr bool SB8 = TYPE == DCG_TYPE_Q4_K && N <= 32;
    static constexpr bool TA = !SB8 && N <= 64;
    static constexpr int PB = SB8 ? 2 : (TA ? (N <= 32 ? 3 : 2) : (N <= 32 ? 2 : 1));
    static constexpr int OFF_PL = 1024;                            // planes [buffer][K half][H, L]
    static constexpr int PL_BYTES = SB8 ? PB * 2 * TC_HPLANE : (TA ? 0 : PB * 4 * TC_HPLANE);
    static constexpr int OFF_ACT = OFF_PL + PL_BYTES;
    static constexpr int OFF_META = OFF_ACT + AS * AT;
    static constexpr int OFF_ROWP = OFF_META + TC_MS * META;       // [slot][128 rows] 16 B
    static constexpr int OFF_RAW = OFF_ROWP + TC_MS * TC_ROWS * 16;
    static constexpr int WS_FIT = (TC_SMEM_MAX - OFF_RAW) / WT;
    static constexpr int WS = WS_FIT > 8 ? 8 : WS_FIT;             // weight ring
    static constexpr int SMEM = OFF_RAW + WS * WT;
    static constexpr int TMEM_COLS = SB8 ? 16 * N : (TA ? 512 : 4 * N);   // accumulators (+ planes)
    static constexpr int TMEM_PL = 512 - PB * 128;                // first plane column (TA)
    static_assert(WS >= 2, "weight ring too shallow");
    static_assert(SMEM <= TC_SMEM_MAX, "shared memory");
};

// cp.async of 4 / 16 bytes global -> shared (src_bytes = 0: zero fill), and an arrive on an
// mbarrier once this thread's earlier cp.asyncs have landed (counted as one expected arrival)
__device__ __forceinline__ void cp_async4(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// named barrier of the draining warps: all 16 workers, or the 8 epilogue-only warps (SPLIT)
template <bool SPLIT>
__device__ __forceinline__ void work_bar() {
    if (SPLIT) asm volatile("bar.sync 1, 256;" ::: "memory");
    else asm volatile("bar.sync 1, 512;" ::: "memory");
}

// ---- prep: one weight row of one super-block (in shared memory) -> the two planes' 4 K chunks
// (16 elements each) of quarter p: K half h = p / 2, chunks j = 4 (p % 2) .. +3 of that half ----
// Q4_K quarter p = sub-blocks 2p (low nibbles of byte group p) and 2p + 1 (its high nibbles)
template <int TYPE, typename std::enable_if<TYPE == DCG_TYPE_Q4_K, int>::type = 0>
__device__ __forceinline__ void prep_quarter(const uint8_t* row, int p, uint32_t (&H)[16], uint32_t (&L)[16]) {
    const uint4 hdr = *(const uint4*)row;
    const uint4 g0 = *(const uint4*)(row + 16 + 32 * p), g1 = *(const uint4*)(row + 32 + 32 * p);
    const Q4kScales sc = q4k_unpack(hdr);
    const uint32_t w[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int sbk = 2 * p + (c >> 1);   // chunks 0, 1: sub-block 2p; 2, 3: sub-block 2p + 1
        const uint32_t scs = ((sbk < 4 ? sc.sc03 : sc.sc47) >> (8 * (sbk & 3))) & 0x3Fu;
        const uint32_t sh = scs >> 3, sl = scs & 7u;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t word = w[(c & 1) * 4 + t];
            const uint32_t nib = (c >> 1) ? (word >> 4) & 0x0F0F0F0Fu : word & 0x0F0F0F0Fu;
            H[4 * c + t] = nib * sh;
            L[4 * c + t] = nib * sl;
        }
    }
}

// Q6_K chunk j of K half h (elements 128h + 16j .. +15) = sub-block 8h + j, group grp = j/2,
// l-range 16 (j & 1) .. +15; u = low nibble of ql[64h + 32 (grp & 1) + l] (shifted by 4 (grp >> 1))
// | 2 bits of qh[32h + l] (shifted by 2 grp) << 4.  p = (u - 32) sc is formed two elements per
// 32-bit word (16-bit lanes, biased by 32768 so no lane borrows): V = (u0 | u1 << 16) sc + K with
// K = (32768 - 32 sc) in both lanes; then L = V & 127 and H = (V >> 7) & 255 per lane.
template <int TYPE, typename std::enable_if<TYPE == DCG_TYPE_Q6_K, int>::type = 0>
__device__ __forceinline__ void prep_quarter(const uint8_t* row, int p, uint32_t (&H)[16], uint32_t (&L)[16]) {
    const int h = p >> 1, j0 = 4 * (p & 1);
    const uint32_t scw = *(const uint32_t*)(row + 192 + 8 * h + j0);   // scales of chunks j0 .. j0+3
    uint4 ql[4], qh[2];
#pragma unroll
    for (int c = 0; c < 4; c++) {   // chunk j0 + c: group (j0 + c) / 2, l0 = 16 (c & 1)
        const int grp = (j0 + c) >> 1;
        ql[c] = *(const uint4*)(row + 64 * h + 32 * (grp & 1) + 16 * (c & 1));
    }
    qh[0] = *(const uint4*)(row + 128 + 32 * h);
    qh[1] = *(const uint4*)(row + 128 + 32 * h + 16);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int j = j0 + c, grp = j >> 1;
        const int sc = (int)(int8_t)((scw >> (8 * c)) & 0xFF);
        const uint32_t kk = (uint32_t)(32768 - 32 * sc) * 0x10001u;
        const uint32_t* qlw = (const uint32_t*)&ql[c];
        const uint32_t* qhw = (const uint32_t*)&qh[c & 1];
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t u = ((qlw[t] >> (4 * (grp >> 1))) & 0x0F0F0F0Fu) | (((qhw[t] >> (2 * grp)) & 0x03030303u) << 4);
            const uint32_t v01 = __byte_perm(u, 0u, 0x4140u) * (uint32_t)sc + kk;
            const uint32_t v23 = __byte_perm(u, 0u, 0x4342u) * (uint32_t)sc + kk;
            L[4 * c + t] = __byte_perm(v01 & 0x007F007Fu, v23 & 0x007F007Fu, 0x6420u);
            H[4 * c + t] = __byte_perm((v01 >> 7) & 0x00FF00FFu, (v23 >> 7) & 0x00FF00FFu, 0x6420u);
        }
    }
}

// the 4 chunks of quarter p (chunks 4 (p % 2) .. +3 of its K half) into shared-memory planes laid out
// as core matrices: 16-B K chunks 128 B apart
__device__ __forceinline__ void planes_store(const uint32_t (&H)[16], const uint32_t (&L)[16], int p, uint8_t* pH,
                                             uint8_t* pL) {
    const int j0 = 4 * (p & 1);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        *(uint4*)(pH + (j0 + c) * 128) = make_uint4(H[4 * c], H[4 * c + 1], H[4 * c + 2], H[4 * c + 3]);
        *(uint4*)(pL + (j0 + c) * 128) = make_uint4(L[4 * c], L[4 * c + 1], L[4 * c + 2], L[4 * c + 3]);
    }
}

// ---- the kernel ----
template <int TYPE, int N>
__global__ void __launch_bounds__(TC_THREADS, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                  const __half* __restrict__ wd, int nb, int64_t n, ActQ a, int m, float* __restrict__ y,
                  int ct_tiles, int64_t T, float* __restrict__ part, int* __restrict__ tickets) {
    using C = TcCfg<TYPE, N>;
    constexpr int WS = C::WS, AS = C::AS, MS = TC_MS;
    constexpr bool Q4 = TYPE == DCG_TYPE_Q4_K;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* w_full = (uint64_t*)smem;        // [WS] weight tile landed (tx)
    uint64_t* w_empty = w_full + WS;           // [WS] 16 prep warps read it
    uint64_t* a_full = w_empty + WS;           // [AS] activation tile landed (tx)
    uint64_t* a_empty = a_full + AS;           // [AS] MMAs that read it done
    uint64_t* pl_full = a_empty + AS;          // [PB][2] K-half planes written (256 prep threads)
    uint64_t* pl_empty = pl_full + 2 * C::PB;  // [PB][2] MMAs that read them done
    uint64_t* acc_full = pl_empty + 2 * C::PB; // [2] accumulators complete
    uint64_t* acc_empty = acc_full + 2;        // [2] 16 epilogue warps read them
    uint64_t* meta_full = acc_empty + 2;       // [MS] column metadata staged (32 producer lanes)
    uint64_t* row_full = meta_full + MS;       // [MS] row scales staged (128 prep threads)
    uint64_t* meta_empty = row_full + MS;      // [MS] 16 epilogue warps done with the slot
    uint64_t* mma_done = meta_empty + MS;      // [1] every MMA retired
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
    int* last_flag = (int*)(tmem_slot + 1);
    uint8_t* planes = smem + C::OFF_PL;
    uint8_t* act = smem + C::OFF_ACT;
    uint8_t* meta = smem + C::OFF_META;        // [MS][dx: N floats | pair sums: N x 8 int16]
    uint4* rowp = (uint4*)(smem + C::OFF_ROWP);
    uint8_t* raw = smem + C::OFF_RAW;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x, bid = blockIdx.x;
    const int64_t u0 = sk_begin(bid, T, G), u1 = sk_begin(bid + 1, T, G);
    const int nu = (int)(u1 - u0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < WS; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], (C::TA || C::SB8) ? TC_WORKERS / 2 : TC_WORKERS);
        }
        for (int s = 0; s < AS; s++) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2 * C::PB; b++) {
            mbar_init(&pl_full[b], (C::TA || C::SB8) ? 128 : 256);
            mbar_init(&pl_empty[b], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], (C::TA || C::SB8) ? TC_WORKERS / 2 : TC_WORKERS);
        }
        for (int s = 0; s < MS; s++) {
            mbar_init(&meta_full[s], 32);
            mbar_init(&row_full[s], 128);
            mbar_init(&meta_empty[s], (C::TA || C::SB8) ? TC_WORKERS / 2 : TC_WORKERS);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        // ---------------- weight producer (constant data: may run ahead of pdl_wait) ----------------
        if (lane == 0) {
            for (int i = 0; i < nu && ok; i++) {
                const int64_t u = u0 + i, tile = u / nb;
                const int s = (int)(u % nb), st = i % WS;
                const int rt = (int)(tile / ct_tiles);
                if (i >= WS) ok = mbar_wait(&w_empty[st], (uint32_t)(((i / WS) - 1) & 1), &g_tc_error);
                if (!ok) break;
                TC_TRACE(i, 0);
                mbar_arrive_expect_tx(&w_full[st], (uint32_t)C::WT);
                tma_load_2d(raw + (size_t)st * C::WT, &wmap, s * (TcW<TYPE>::ROWB / 4), rt * TC_ROWS, &w_full[st]);
            }
        }
        pdl_wait();
    } else if (warp == 1) {
        // ---------------- activation producer + column metadata ----------------
        // lane c stages columns c, c + 32, ...: their dx (and Q4_K pair sums) arrive by cp.async
        // straight into the metadata slot, which this lane's completion arrival marks full
        pdl_wait();
        constexpr int CPL = (N + 31) / 32;   // columns per lane
        for (int i = 0; i < nu && ok; i++) {
            const int64_t u = u0 + i, tile = u / nb;
            const int s = (int)(u % nb), st = i % AS, ms = i % MS;
            const int c0 = (int)(tile % ct_tiles) * N;
            if (i >= AS) ok = mbar_wait(&a_empty[st], (uint32_t)(((i / AS) - 1) & 1), &g_tc_error);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            if (lane == 0) {
                TC_TRACE(i, 1);
                mbar_arrive_expect_tx(&a_full[st], (uint32_t)C::AT);
                tma_load_3d(act + (size_t)st * C::AT, &amap, 0, c0, s * 16, &a_full[st]);
            }
            if (i >= MS) ok = mbar_wait(&meta_empty[ms], (uint32_t)(((i / MS) - 1) & 1), &g_tc_error);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            float* mdx = (float*)(meta + (size_t)ms * C::META);
            uint4* mbs = (uint4*)(mdx + N);
#pragma unroll
            for (int j = 0; j < CPL; j++) {
                const int c = lane + 32 * j, col = c0 + c;
                if (c < N) {
                    const bool live = col < m;
                    const size_t e = live ? (size_t)col * nb + s : 0;
                    cp_async4(&mdx[c], (const float*)a.d + e, live ? 4u : 0u);
                    if (Q4) cp_async16(&mbs[c], a.bs32 + e * 8, live ? 16u : 0u);
                }
            }
            cp_async_arrive(&meta_full[ms]);
        }
    } else if (warp == 2) {
        // ---------------- MMA issue ----------------
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8<TC_ROWS, N>();
            for (int i = 0; i < nu && ok; i++) {
                const int st = i % AS, b = i & 1;
                ok = mbar_wait(&a_full[st], (uint32_t)((i / AS) & 1), &g_tc_error) &&
                     (i < 2 || mbar_wait(&acc_empty[b], (uint32_t)(((i >> 1) - 1) & 1), &g_tc_error));
                TC_TRACE(i, 4);
                const uint32_t pa = smem_u32(act + (size_t)st * C::AT);
                const uint32_t dH = tmem + (uint32_t)(b * 2 * N), dL = dH + N;
                const uint32_t dS = tmem + (uint32_t)(b * 8 * N);   // SB8: sub-block regions
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int pb = i % C::PB;
                    ok = ok && mbar_wait(&pl_full[pb * 2 + h], (uint32_t)((i / C::PB) & 1), &g_tc_error);
                    if (!ok) break;
                    TC_TRACE(i, 8 + h);
                    tc_fence_after();
                    if (C::SB8) {
                        const uint32_t pQ = smem_u32(planes + (size_t)(pb * 2 + h) * TC_HPLANE);
#pragma unroll
                        for (int j = 0; j < 4; j++) {   // sub-block 4h + j: K chunks 8h + 2j, 8h + 2j + 1
                            const uint64_t bd = umma_desc(pa + (h * 4 + j) * 2 * N * 16, N * 16, 128);
                            mma_i8(dS + (uint32_t)((h * 4 + j) * N), umma_desc(pQ + j * 256, 128, TC_HSBO), bd, idesc, 0u);
                        }
                    } else if (C::TA) {
                        const uint32_t tH = tmem + (uint32_t)(C::TMEM_PL + pb * 128 + h * 64), tL = tH + 32;
#pragma unroll
                        for (int j = 0; j < 4; j++) {   // k-step: K elements 32j .. +31 of the half
                            const uint64_t bd = umma_desc(pa + (h * 4 + j) * 2 * N * 16, N * 16, 128);
                            const uint32_t accum = (h | j) ? 1u : 0u;
                            mma_i8_ta(dH, tH + 8 * j, bd, idesc, accum);
                            mma_i8_ta(dL, tL + 8 * j, bd, idesc, accum);
                        }
                    } else {
                        const uint32_t pH = smem_u32(planes + (size_t)(pb * 4 + 2 * h) * TC_HPLANE), pL = pH + TC_HPLANE;
#pragma unroll
                        for (int j = 0; j < 4; j++) {   // k-step: K chunks 8h + 2j, 8h + 2j + 1
                            const uint64_t bd = umma_desc(pa + (h * 4 + j) * 2 * N * 16, N * 16, 128);
                            const uint32_t accum = (h | j) ? 1u : 0u;
                            mma_i8(dH, umma_desc(pH + j * 256, 128, TC_HSBO), bd, idesc, accum);
                            mma_i8(dL, umma_desc(pL + j * 256, 128, TC_HSBO), bd, idesc, accum);
                        }
                    }
                    tc_commit(&pl_empty[pb * 2 + h]);
                }
                if (!ok) break;
                tc_commit(&a_empty[st]);
                tc_commit(&acc_full[b]);
                TC_TRACE(i, 5);
            }
            tc_commit(mma_done);
            mbar_wait(mma_done, 0, &g_tc_error);
        }
    } else if (warp >= TC_WORK0) {
        // ---------------- prep + epilogue: thread <-> (weight row, quarter) ----------------
        // Iteration i expands unit i's weights (quarter qp of its row's K) and then drains unit
        // i-1's accumulators (quarter qp of the columns): unit i's MMAs run while unit i-1 is
        // drained.
        // SPLIT (planes in tensor memory): warps 4-11 only expand (thread = row x K half, two K
        // quarters) and warps 12-19 only drain (thread = row x half of the columns), so the prep of
        // unit i+1 overlaps the drain of unit i instead of following it.  Otherwise each of the 16
        // warps does both, for a K quarter and a quarter of the columns.
        constexpr bool SPLIT = C::TA || C::SB8;
        constexpr int NH = SPLIT ? N / 2 : N / 4;      // columns per thread
        const int quarter = warp & 3, grp = (warp - TC_WORK0) >> 2;   // TMEM lane group, warp group
        const bool do_prep = !SPLIT || grp < 2, do_epi = !SPLIT || grp >= 2;
        const int qp = SPLIT ? (do_prep ? 2 * grp : 0) : grp;   // (first) K quarter this thread expands
        const int half = qp >> 1;                     // the K half this thread's prep writes
        const int cq = SPLIT ? grp - 2 : grp;         // column part this thread drains
        const int row = quarter * 32 + lane;
        const int et = threadIdx.x - (SPLIT ? TC_WORK0 + 8 : TC_WORK0) * 32;   // among the draining threads
        pdl_wait();   // y, the partials and the tickets may be in use by the previous kernel
        // Q6_K: the row's fp16 d of unit i, fetched two units ahead by cp.async as the aligned pair of
        // halves holding it (the epilogue picks the half) into the unit's row slot, whose row_full
        // arrival is that copy's completion
        auto fetch_d = [&](int i) {
            if (Q4 || i >= nu) return;
            const int64_t u = u0 + i, tile = u / nb;
            const int64_t r = (tile / ct_tiles) * TC_ROWS + row;
            const size_t e = r < n ? (size_t)(r * nb + (u % nb)) & ~(size_t)1 : 0;
            cp_async4(&rowp[(i % MS) * TC_ROWS + row], wd + e, r < n ? 4u : 0u);
            cp_async_arrive(&row_full[i % MS]);
        };
        if (!Q4 && do_prep && qp == 0) {
            fetch_d(0);
            fetch_d(1);
        }
        float yacc[NH];
        int seg_s0 = 0;
        for (int i = 0; i <= nu; i++) {
            // ---- prep of unit i ----
            if (do_prep && i < nu && ok) {
                const int st = i % WS, ms = i % MS;
                ok = mbar_wait(&w_full[st], (uint32_t)((i / WS) & 1), &g_tc_error);
                if (warp == TC_WORK0 && lane == 0) TC_TRACE(i, 2);
                if (ok && qp == 0 && i >= MS)
                    ok = mbar_wait(&meta_empty[ms], (uint32_t)(((i / MS) - 1) & 1), &g_tc_error);
                const int pb = i % C::PB;
                if (ok && i >= C::PB)
                    ok = mbar_wait(&pl_empty[pb * 2 + half], (uint32_t)(((i / C::PB) - 1) & 1), &g_tc_error);
                ok = __all_sync(0xffffffffu, ok);
                
                if (ok) {
                    const uint8_t* src = raw + (size_t)st * C::WT + (size_t)row * TcW<TYPE>::ROWB;
                    if (qp == 0) {   // the row's scales of this unit, for the epilogue
                        if (Q4) {
                            const uint4 hdr = *(const uint4*)src;
                            const Q4kScales sc = q4k_unpack(hdr);
                            rowp[ms * TC_ROWS + row] = C::SB8 ? hdr : make_uint4(hdr.x, sc.mn03, sc.mn47, 0u);
                            mbar_arrive(&row_full[ms]);
                        } else if (i + 2 < nu) {   // the slot of unit i + 2 held unit i - 2
                            const int m2 = (i + 2) % MS;
                            if (i + 2 >= MS)
                                ok = mbar_wait(&meta_empty[m2], (uint32_t)((((i + 2) / MS) - 1) & 1), &g_tc_error);
                            fetch_d(i + 2);
                        }
                    }
                    uint32_t hv[16], lv[16];
                    if (C::TA) {
                        // the MMAs that read this plane buffer have retired (pl_empty); order the
                        // stores after them, and the next MMAs after the stores
                        tc_fence_after();
#pragma unroll
                        for (int q2 = 0; q2 < (SPLIT ? 2 : 1); q2++) {
                            prep_quarter<TYPE>(src, qp + q2, hv, lv);
                            const uint32_t tH = tmem + ((uint32_t)(quarter * 32) << 16) +
                                                (uint32_t)(C::TMEM_PL + pb * 128 + half * 64 + 16 * ((qp + q2) & 1));
                            tmem_st16(tH, hv);
                            tmem_st16(tH + 32, lv);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                    } else if (C::SB8) {
                        // quants as int8 (no scale), K half `half` of plane buffer pb
                        uint8_t* pQ = planes + (size_t)(pb * 2 + half) * TC_HPLANE + (size_t)(row >> 3) * TC_HSBO + (row & 7) * 16;
#pragma unroll
                        for (int q2 = 0; q2 < 2; q2++) {
                            const int p4 = qp + q2;   // quarter: sub-blocks 2 p4 (low nibbles), 2 p4 + 1 (high)
                            const uint4 g0 = *(const uint4*)(src + 16 + 32 * p4), g1 = *(const uint4*)(src + 32 + 32 * p4);
                            const int j0 = 4 * (p4 & 1);
                            const uint32_t m4 = 0x0F0F0F0Fu;
                            *(uint4*)(pQ + (j0 + 0) * 128) = make_uint4(g0.x & m4, g0.y & m4, g0.z & m4, g0.w & m4);
                            *(uint4*)(pQ + (j0 + 1) * 128) = make_uint4(g1.x & m4, g1.y & m4, g1.z & m4, g1.w & m4);
                            *(uint4*)(pQ + (j0 + 2) * 128) = make_uint4((g0.x >> 4) & m4, (g0.y >> 4) & m4, (g0.z >> 4) & m4, (g0.w >> 4) & m4);
                            *(uint4*)(pQ + (j0 + 3) * 128) = make_uint4((g1.x >> 4) & m4, (g1.y >> 4) & m4, (g1.z >> 4) & m4, (g1.w >> 4) & m4);
                        }
                    } else {
                        prep_quarter<TYPE>(src, qp, hv, lv);
                        uint8_t* pH = planes + (size_t)(pb * 4 + 2 * half) * TC_HPLANE + (size_t)(row >> 3) * TC_HSBO + (row & 7) * 16;
                        planes_store(hv, lv, qp, pH, pH + TC_HPLANE);
                    }
                    
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&w_empty[st]);
                    if (!C::TA) fence_proxy_async_smem();   // generic-proxy plane stores -> the MMA's reads
                    mbar_arrive(&pl_full[pb * 2 + half]);
                    if (warp == TC_WORK0 && lane == 0) TC_TRACE(i, 3);
                }
            }
            if (i == 0 || !do_epi) continue;
            // ---- epilogue of unit e = i - 1 ----
            const int e = i - 1;
            const int64_t u = u0 + e, tile = u / nb;
            const int s = (int)(u % nb), b = e & 1, ms = e % MS;
            if (e == 0 || s == 0) {
                seg_s0 = s;
#pragma unroll
                for (int c = 0; c < NH; c++) yacc[c] = 0.0f;
            }
            if (ok) {
                if (warp == TC_WORK0 + (SPLIT ? 8 : 0) && lane == 0) TC_TRACE(e, 6);
                ok = mbar_wait(&acc_full[b], (uint32_t)((e >> 1) & 1), &g_tc_error) &&
                     mbar_wait(&meta_full[ms], (uint32_t)((e / MS) & 1), &g_tc_error) &&
                     mbar_wait(&row_full[ms], (uint32_t)((e / MS) & 1), &g_tc_error);
                ok = __all_sync(0xffffffffu, ok);   // warp-uniform: the TMEM loads are .sync.aligned
            }
            if (warp == TC_WORK0 + (SPLIT ? 8 : 0) && lane == 0) TC_TRACE(e, 10);
            if (ok) {
                tc_fence_after();
                if constexpr (C::SB8) {
                    // sub-block j's int32 dots C_j: isum = sum_j sc_j C_j exactly (ggml's integer sum)
                    const uint4 hdr = rowp[ms * TC_ROWS + row];
                    const Q4kScales sc = q4k_unpack(hdr);
                    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));
                    const int mp0 = (int)(sc.mn03 & 0xFFu) | (int)((sc.mn03 >> 8) & 0xFFu) << 8;
                    const int mp1 = (int)((sc.mn03 >> 16) & 0xFFu) | (int)(sc.mn03 >> 24) << 8;
                    const int mp2 = (int)(sc.mn47 & 0xFFu) | (int)((sc.mn47 >> 8) & 0xFFu) << 8;
                    const int mp3 = (int)((sc.mn47 >> 16) & 0xFFu) | (int)(sc.mn47 >> 24) << 8;
                    const float* mdx = (const float*)(meta + (size_t)ms * C::META) + cq * NH;
                    const uint4* mbs = (const uint4*)((const float*)(meta + (size_t)ms * C::META) + N) + cq * NH;
                    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 8 * N + cq * NH);
                    int isum[NH];
#pragma unroll
                    for (int c = 0; c < NH; c++) isum[c] = 0;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int scj = (int)(((j < 4 ? sc.sc03 : sc.sc47) >> (8 * (j & 3))) & 0xFFu);
                        uint32_t v[16];
                        if (NH == 16) tmem_ld16(lane_addr + (uint32_t)(j * N), v);
                        else tmem_ld8(lane_addr + (uint32_t)(j * N), v);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < NH; c++) isum[c] += scj * (int)v[c];
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
#pragma unroll
                    for (int c = 0; c < NH; c++) {
                        const uint4 bs = mbs[c];
                        int msum = __dp2a_lo((int)bs.x, mp0, 0);
                        msum = __dp2a_lo((int)bs.y, mp1, msum);
                        msum = __dp2a_lo((int)bs.z, mp2, msum);
                        msum = __dp2a_lo((int)bs.w, mp3, msum);
                        yacc[c] += mdx[c] * (dd.x * __int2float_rn(isum[c]) - dd.y * i2f_exact22(msum));
                    }
                } else {
                    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 2 * N + cq * NH);
                    const uint4 rp = rowp[ms * TC_ROWS + row];
                    const float* mdx = (const float*)(meta + (size_t)ms * C::META) + cq * NH;
                    const uint4* mbs = (const uint4*)((const float*)(meta + (size_t)ms * C::META) + N) + cq * NH;
                    float2 dd = make_float2(0.0f, 0.0f);
                    if (!Q4) {   // the fetched pair of halves; this unit's d is the one at an odd index or not
                        const int64_t r = (tile / ct_tiles) * TC_ROWS + row;
                        const __half2 pr = *reinterpret_cast<const __half2*>(&rp.x);
                        dd.x = ((r * nb + s) & 1) ? __high2float(pr) : __low2float(pr);
                    }
                    int mp0 = 0, mp1 = 0, mp2 = 0, mp3 = 0;
                    if (Q4) {
                        dd = __half22float2(*reinterpret_cast<const __half2*>(&rp.x));
                        // mins as (m0, m1), (m2, m3), ... pairs in the low bytes for dp2a
                        mp0 = (int)(rp.y & 0xFFu) | (int)((rp.y >> 8) & 0xFFu) << 8;
                        mp1 = (int)((rp.y >> 16) & 0xFFu) | (int)(rp.y >> 24) << 8;
                        mp2 = (int)(rp.z & 0xFFu) | (int)((rp.z >> 8) & 0xFFu) << 8;
                        mp3 = (int)((rp.z >> 16) & 0xFFu) | (int)(rp.z >> 24) << 8;
                    }
                    constexpr int CH = NH < 16 ? NH : 16;
    #pragma unroll
                    for (int cc = 0; cc < NH; cc += CH) {
                        uint32_t hv[16], lv[16];
                        if (CH == 16) {
                            tmem_ld16(lane_addr + cc, hv);
                            tmem_ld16(lane_addr + N + cc, lv);
                        } else if (CH == 8) {
                            tmem_ld8(lane_addr + cc, hv);
                            tmem_ld8(lane_addr + N + cc, lv);
                        } else {
                            tmem_ld4(lane_addr + cc, hv);
                            tmem_ld4(lane_addr + N + cc, lv);
                        }
                        tmem_wait_ld();
                        if (cc == 0 && warp == TC_WORK0 + (SPLIT ? 8 : 0) && lane == 0) TC_TRACE(e, 11);
                        if (cc + CH == NH) {   // every read of this buffer issued and complete
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&acc_empty[b]);
                        }
    #pragma unroll
                        for (int j = 0; j < CH; j++) {
                            const float dx = mdx[cc + j];   // 0 for columns past m
                            // isum = SHIFT C_H + C_L as one correctly rounded fp32 value (what
                            // (float)isum gives), from exact conversions of |C_H|, |C_L| < 2^22
                            const float fsum = fmaf(i2f_exact22((int)hv[j]), (float)TcW<TYPE>::SHIFT,
                                                    i2f_exact22((int)lv[j]));
                            if (Q4) {
                                const uint4 bs = mbs[cc + j];
                                int msum = __dp2a_lo((int)bs.x, mp0, 0);
                                msum = __dp2a_lo((int)bs.y, mp1, msum);
                                msum = __dp2a_lo((int)bs.z, mp2, msum);
                                msum = __dp2a_lo((int)bs.w, mp3, msum);
                                yacc[cc + j] += dx * (dd.x * fsum - dd.y * i2f_exact22(msum));
                            } else {
                                yacc[cc + j] += dx * (dd.x * fsum);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&meta_empty[ms]);
                if (warp == TC_WORK0 + (SPLIT ? 8 : 0) && lane == 0) TC_TRACE(e, 7);
            }
            // ---- end of a tile segment: direct store, or partial + ticket (last arriver sums) ----
            if (e == nu - 1 || s == nb - 1) {
                const int64_t rt = tile / ct_tiles;
                const int ct = (int)(tile % ct_tiles);
                const int64_t r = rt * TC_ROWS + row;
                const int cbase = ct * N + cq * NH;
                if (seg_s0 == 0 && s == nb - 1) {
                    if (ok && r < n)
#pragma unroll
                        for (int c = 0; c < NH; c++)
                            if (cbase + c < m) y[(size_t)(cbase + c) * n + r] = yacc[c];
                } else {
                    const int64_t t0 = tile * nb;
                    const int slot = sk_begin(bid, T, G) > t0 ? 0 : 1;
                    float* P = part + (size_t)(bid * 2 + slot) * N * TC_ROWS;
#pragma unroll
                    for (int c = 0; c < NH; c++) P[(cq * NH + c) * TC_ROWS + row] = yacc[c];
                    __threadfence();
                    work_bar<SPLIT>();
                    const int64_t cf = sk_owner(t0, T, G), cl = sk_owner(t0 + nb - 1, T, G);
                    if (et == 0) {
                        const int old = atomicAdd(&tickets[tile], 1);
                        const int last = old == (int)(cl - cf);
                        if (last) tickets[tile] = 0;   // every contributor has arrived: ready for the next call
                        *last_flag = last;
                    }
                    work_bar<SPLIT>();
                    const int last = *last_flag;
                    if (last) {
                        __threadfence();
                        // the partials in CTA order (this CTA's own one re-read from scratch too)
#pragma unroll
                        for (int c = 0; c < NH; c++) yacc[c] = 0.0f;
                        for (int64_t q = cf; q <= cl; q++) {
                            const int sq = sk_begin(q, T, G) > t0 ? 0 : 1;
                            const float* Q = part + (size_t)(q * 2 + sq) * N * TC_ROWS;
#pragma unroll
                            for (int c = 0; c < NH; c++) yacc[c] += __ldcg(&Q[(cq * NH + c) * TC_ROWS + row]);
                        }
                        if (ok && r < n)
#pragma unroll
                            for (int c = 0; c < NH; c++)
                                if (cbase + c < m) y[(size_t)(cbase + c) * n + r] = yacc[c];
                    }
                    work_bar<SPLIT>();   // last_flag is reused by the next segment
                }
            }
        }
    }

    // ---------------- teardown ----------------
    tc_fence_before();
    __syncthreads();   // every MMA retired (mma_done) and every TMEM read done
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
    }
    pdl_trigger();   // dependents are released only after this CTA's tensor memory is free
}

// ---- host side ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();  // qmm.cu

static cudaError_t tc_maps(CUtensorMap* wm, CUtensorMap* am, int type, const void* W, int64_t n, int64_t k,
                           const void* qs, int64_t m, int N) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int rowb = type == DCG_TYPE_Q4_K ? Q4_K_BYTES : Q6_K_PAYLOAD;
    const size_t row_bytes = (size_t)(k / QK_K) * rowb;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)n};
        const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
        const cuuint32_t box[2] = {(cuuint32_t)(rowb / 4), (cuuint32_t)TC_ROWS};
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

// column tile for m activation rows: the smallest of 16 / 32 / 64 / 128 that holds them (128 beyond)
static int tc_n(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128)); }

struct TcPlan {
    int N, ct;
    int64_t rt, T, G;
};
static TcPlan tc_plan(int64_t n, int64_t k, int64_t m) {
    TcPlan p;
    p.N = tc_n(m);
    p.ct = (int)((m + p.N - 1) / p.N);
    p.rt = (n + TC_ROWS - 1) / TC_ROWS;
    p.T = p.rt * p.ct * (k / QK_K);
    const int64_t sms = num_sms();
    // at least sk_min_units() units per CTA (tuning knob DCG_SK_MIN_UNITS), at most one CTA per SM
    const int64_t mu = sk_min_units();
    const int64_t want = (p.T + mu - 1) / mu;
    p.G = want < sms ? want : sms;
    return p;
}

size_t qmm_tc_scratch_bytes(int type, int64_t n, int64_t k, int64_t m) {
    (void)type;
    const TcPlan p = tc_plan(n, k, m);
    return align256((size_t)p.rt * p.ct * 4) + (size_t)p.G * 2 * p.N * TC_ROWS * 4;
}
int qmm_tc_ticket_count(int type, int64_t n, int64_t k, int64_t m) {
    (void)type;
    const TcPlan p = tc_plan(n, k, m);
    return (int)(p.rt * p.ct);
}

template <int TYPE, int N>
static cudaError_t launch_tc_t(const void* W, const __half* wd, int64_t n, int64_t k, const ActQ& a, int m,
                               float* y, void* scratch, const TcPlan& p, cudaStream_t st) {
    using C = TcCfg<TYPE, N>;
    cudaError_t e = DCG_SMEM_ATTR((qmm_tc_kernel<TYPE, N>), C::SMEM);
    if (e != cudaSuccess) return e;
    CUtensorMap wm, am;
    e = tc_maps(&wm, &am, TYPE, W, n, k, a.qs, m, N);
    if (e != cudaSuccess) return e;
    int* tickets = (int*)scratch;
    float* part = (float*)((uint8_t*)scratch + align256((size_t)p.rt * p.ct * 4));
    return launch_pdl(qmm_tc_kernel<TYPE, N>, dim3((unsigned)p.G), dim3(TC_THREADS), (size_t)C::SMEM, st, wm, am,
                      wd, (int)(k / QK_K), n, a, m, y, p.ct, p.T, part, tickets);
}

bool qmm_tc_supports(int type, int64_t n, int64_t k, int64_t m) {
    return (type == DCG_TYPE_Q4_K || type == DCG_TYPE_Q6_K) && m >= 2 && k % QK_K == 0 && n > 0;
}

cudaError_t launch_qmm_tc(int type, const void* packed_w, int64_t n, int64_t k, const void* act, int64_t m,
                          float* y, void* scratch, cudaStream_t st) {
    const ActQ a = act_view(DCG_TYPE_Q8_K, const_cast<void*>(act), m, k);
    const TcPlan p = tc_plan(n, k, m);
    const int mi = (int)m;
    if (type == DCG_TYPE_Q4_K) {
        switch (p.N) {
            case 16: return launch_tc_t<DCG_TYPE_Q4_K, 16>(packed_w, nullptr, n, k, a, mi, y, scratch, p, st);
            case 32: return launch_tc_t<DCG_TYPE_Q4_K, 32>(packed_w, nullptr, n, k, a, mi, y, scratch, p, st);
            case 64: return launch_tc_t<DCG_TYPE_Q4_K, 64>(packed_w, nullptr, n, k, a, mi, y, scratch, p, st);
            default: return launch_tc_t<DCG_TYPE_Q4_K, 128>(packed_w, nullptr, n, k, a, mi, y, scratch, p, st);
        }
    }
    const PackedW w = packed_view(DCG_TYPE_Q6_K, packed_w, n, k);
    switch (p.N) {
        case 16: return launch_tc_t<DCG_TYPE_Q6_K, 16>(packed_w, w.d, n, k, a, mi, y, scratch, p, st);
        case 32: return launch_tc_t<DCG_TYPE_Q6_K, 32>(packed_w, w.d, n, k, a, mi, y, scratch, p, st);
        case 64: return launch_tc_t<DCG_TYPE_Q6_K, 64>(packed_w, w.d, n, k, a, mi, y, scratch, p, st);
        default: return launch_tc_t<DCG_TYPE_Q6_K, 128>(packed_w, w.d, n, k, a, mi, y, scratch, p, st);
    }
}

}  // namespace dcg
