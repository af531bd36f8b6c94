// qmm_q8tc.cu -- Q8_0 weight x Q8_0 activation matmul on the 5th-generation tensor cores
// (tcgen05.mma kind::i8) for M >= 2: the batched-decode and prefill form of ggml_mul_mat's
// vec_dot_q8_0_q8_0 row loop (core/src/inference.cpp:1063, :1794-1797, :1817; the dot of
// simd_ops.cpp:82-93): y[c][r] = sum_b fp16(dw[r][b]) fp16(dx[c][b]) sum_{i<32} qw[r][32b+i] qx[c][32b+i].
//
// Q8_0 weights need no expansion: the device layout's int8 payload rows are the MMA's A operand,
// and its fp16 block scales a separate [n][k/32] array.  Both operands and both scale arrays come
// in by TMA (128-byte-swizzled K-major boxes for the int8 tiles).  Every 32-element block has its
// own pair of scales, so every block's MMA (M128 x N x K32) writes its own tensor-memory region;
// the epilogue drains them, y += (dw dx) * dot, with an exact two-operation int -> float
// conversion (|dot| <= 32 * 127 * 127 < 2^22).
//
// Work split as in qmm_tc.cu (stream-K over 128-row x N-column x 256-K units, one CTA per SM,
// deterministic last-arriver fixup of tiles shared by several CTAs).  Warps:
//   warp 0      TMA: weight tile (two 128 x 128 B swizzled boxes) + its 128 x 8 block scales
//   warp 1      TMA: activation tile (two N x 128 B swizzled boxes) + its N x 8 block scales
//   warp 2      MMA issue: per accumulator group of BPB blocks, one MMA per block into its region
//   warp 3      widens each activation stage's fp16 block scales into a float table of (dx, -dx B)
//               pairs, B = 1.5 * 2^23, so the epilogue turns a dot into dx * dot with one integer
//               add and one fma: fma(dx, float_bits(0x4B400000 + dot), -dx B) = dx * dot, rounded once
//   warps 4-19  epilogue: thread (row, column quarter) drains its rows of each group
// A stage is released when its MMAs have completed and the epilogue has read its scales.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace dcg {

__device__ int g_q8tc_error = 0;

cudaError_t qmm_q8tc_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_q8tc_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_q8tc_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int Q8T_ROWS = 128;
constexpr int Q8T_THREADS = 640;       // 20 warps: 0 weight TMA, 1 activation TMA, 2 MMA, 3 spare, 4-19 epilogue
constexpr int Q8T_EPI0 = 4;
constexpr int Q8T_WHALF = Q8T_ROWS * 128;            // one swizzled K half of the weight tile: 16 KB
constexpr int Q8T_WSTAGE = 2 * Q8T_WHALF + 2048;     // + the 128 x 8 fp16 block scales (1 KB aligned)
constexpr int Q8T_SMEM_MAX = 232448;

template <int N>
struct Q8tCfg {
    static constexpr int AHALF = N * 128;                                    // swizzled K half
    static constexpr int ASC = (N * 16 + 1023) / 1024 * 1024;                // N x 8 fp16 scales
    static constexpr int ATAB = 8 * N * 8;                                   // [8 blocks][N] (dx, -dx 1.5 2^23)
    static constexpr int ASTAGE = 2 * AHALF + ASC + ATAB;
    static constexpr int AS = N >= 128 ? 2 : (N >= 64 ? 3 : 4);
    static constexpr int OFF_ACT = 1024;
    static constexpr int OFF_W = OFF_ACT + AS * ASTAGE;
    static constexpr int WS_FIT = (Q8T_SMEM_MAX - 1024 - OFF_W) / Q8T_WSTAGE;   // 1 KB alignment slack
    static constexpr int WS = WS_FIT > 6 ? 6 : WS_FIT;
    static constexpr int SMEM = OFF_W + WS * Q8T_WSTAGE + 1024;
    static constexpr int BPB = N >= 128 ? 2 : (N >= 64 ? 4 : 8);            // blocks per accumulator group
    static constexpr int GPU = 8 / BPB;                                       // groups per unit
    static constexpr int TMEM_COLS = 2 * BPB * N;                             // two groups in flight
    static constexpr int NQ = N / 4;                                          // columns per epilogue thread
    static_assert(WS >= 2, "weight ring too shallow");
    static_assert(TMEM_COLS <= 512, "tensor memory");
};

__device__ __forceinline__ void q8_epi_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

template <int N>
__global__ void __launch_bounds__(Q8T_THREADS, 1)
    qmm_q8tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap wdmap,
                    const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap admap, int nb,
                    int64_t n, int m, float* __restrict__ y, int ct_tiles, int64_t T, float* __restrict__ part,
                    int* __restrict__ tickets) {
    using C = Q8tCfg<N>;
    constexpr int WS = C::WS, AS = C::AS, BPB = C::BPB, GPU = C::GPU, NQ = C::NQ;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // SWIZZLE_128B boxes need 1 KB-aligned destinations
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* w_full = (uint64_t*)smem;       // [WS] tx
    uint64_t* w_empty = w_full + WS;          // [WS] MMA commit + 16 epilogue warps
    uint64_t* a_full = w_empty + WS;          // [AS] tx
    uint64_t* a_empty = a_full + AS;          // [AS] MMA commit + 16 epilogue warps
    uint64_t* a_tab = a_empty + AS;           // [AS] scale table written (32 lanes of warp 3)
    uint64_t* acc_full = a_tab + AS;          // [2] commit
    uint64_t* acc_empty = acc_full + 2;       // [2] 16 epilogue warps
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
    int* last_flag = (int*)(tmem_slot + 1);
    uint8_t* act = smem + C::OFF_ACT;
    uint8_t* wst = smem + C::OFF_W;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x, bid = blockIdx.x;
    const int64_t u0 = sk_begin(bid, T, G), u1 = sk_begin(bid + 1, T, G);
    const int nu = (int)(u1 - u0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < WS; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], 17);
        }
        for (int s = 0; s < AS; s++) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 17);
            mbar_init(&a_tab[s], 32);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 16);
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
        // ---------------- weight producer (constant data) ----------------
        if (lane == 0) {
            for (int i = 0; i < nu && ok; i++) {
                const int64_t u = u0 + i, tile = u / nb;
                const int s = (int)(u % nb), st = i % WS;
                const int r0 = (int)(tile / ct_tiles) * Q8T_ROWS;
                if (i >= WS) ok = mbar_wait(&w_empty[st], (uint32_t)(((i / WS) - 1) & 1), &g_q8tc_error);
                if (!ok) break;
                uint8_t* d = wst + (size_t)st * Q8T_WSTAGE;
                mbar_arrive_expect_tx(&w_full[st], (uint32_t)(2 * Q8T_WHALF + Q8T_ROWS * 16));
                tma_load_2d(d, &wmap, s * 256, r0, &w_full[st]);
                tma_load_2d(d + Q8T_WHALF, &wmap, s * 256 + 128, r0, &w_full[st]);
                tma_load_2d(d + 2 * Q8T_WHALF, &wdmap, s * 8, r0, &w_full[st]);
            }
        }
    } else if (warp == 1) {
        // ---------------- activation producer ----------------
        pdl_wait();
        if (lane == 0) {
            for (int i = 0; i < nu && ok; i++) {
                const int64_t u = u0 + i, tile = u / nb;
                const int s = (int)(u % nb), st = i % AS;
                const int c0 = (int)(tile % ct_tiles) * N;
                if (i >= AS) ok = mbar_wait(&a_empty[st], (uint32_t)(((i / AS) - 1) & 1), &g_q8tc_error);
                if (!ok) break;
                uint8_t* d = act + (size_t)st * C::ASTAGE;
                mbar_arrive_expect_tx(&a_full[st], (uint32_t)(2 * C::AHALF + N * 16));
                tma_load_2d(d, &amap, s * 256, c0, &a_full[st]);
                tma_load_2d(d + C::AHALF, &amap, s * 256 + 128, c0, &a_full[st]);
                tma_load_2d(d + 2 * C::AHALF, &admap, s * 8, c0, &a_full[st]);
            }
        }
    } else if (warp == 3) {
        // ---------------- activation scale table ----------------
        pdl_wait();
        for (int i = 0; i < nu && ok; i++) {
            const int st = i % AS;
            ok = __all_sync(0xffffffffu, mbar_wait(&a_full[st], (uint32_t)((i / AS) & 1), &g_q8tc_error));
            if (!ok) break;
            const uint8_t* d = act + (size_t)st * C::ASTAGE;
            const __half* dxh = (const __half*)(d + 2 * C::AHALF);       // [N][8]
            float2* tab = (float2*)(d + 2 * C::AHALF + C::ASC);           // [8][N]
            for (int e = lane; e < N * 8; e += 32) {
                const int c = e >> 3, j = e & 7;
                const float dx = __half2float(dxh[e]);
                tab[j * N + c] = make_float2(dx, -dx * 12582912.0f);
            }
            mbar_arrive(&a_tab[st]);
        }
    } else if (warp == 2) {
        // ---------------- MMA issue ----------------
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8<Q8T_ROWS, N>();
            for (int i = 0; i < nu && ok; i++) {
                const int ws = i % WS, as = i % AS;
                ok = mbar_wait(&w_full[ws], (uint32_t)((i / WS) & 1), &g_q8tc_error) &&
                     mbar_wait(&a_full[as], (uint32_t)((i / AS) & 1), &g_q8tc_error);
                const uint32_t pw = smem_u32(wst + (size_t)ws * Q8T_WSTAGE);
                const uint32_t pa = smem_u32(act + (size_t)as * C::ASTAGE);
                for (int g = 0; g < GPU && ok; g++) {
                    const int q = i * GPU + g, b = q & 1;
                    if (q >= 2) ok = mbar_wait(&acc_empty[b], (uint32_t)(((q >> 1) - 1) & 1), &g_q8tc_error);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int bl = 0; bl < BPB; bl++) {
                        const int j = g * BPB + bl;                       // block within the unit
                        const uint32_t off = (uint32_t)((j & 3) * 32);   // k-step within its 128-B half row
                        const uint64_t ad = umma_desc_sw128(pw + (j >> 2) * Q8T_WHALF + off);
                        const uint64_t bd = umma_desc_sw128(pa + (j >> 2) * C::AHALF + off);
                        mma_i8(tmem + (uint32_t)((b * BPB + bl) * N), ad, bd, idesc, 0u);
                    }
                    tc_commit(&acc_full[b]);
                }
                if (!ok) break;
                tc_commit(&w_empty[ws]);
                tc_commit(&a_empty[as]);
            }
            tc_commit(mma_done);
            mbar_wait(mma_done, 0, &g_q8tc_error);
        }
    } else if (warp >= Q8T_EPI0) {
        // ---------------- epilogue: thread <-> (weight row, column quarter) ----------------
        const int quarter = warp & 3, cq = (warp - Q8T_EPI0) >> 2;
        const int row = quarter * 32 + lane;
        const int et = threadIdx.x - Q8T_EPI0 * 32;   // 0..511
        pdl_wait();
        float yacc[NQ];
        int seg_s0 = 0;
        for (int i = 0; i < nu; i++) {
            const int64_t u = u0 + i, tile = u / nb;
            const int s = (int)(u % nb), ws = i % WS, as = i % AS;
            if (i == 0 || s == 0) {
                seg_s0 = s;
#pragma unroll
                for (int c = 0; c < NQ; c++) yacc[c] = 0.0f;
            }
            if (ok) {
                ok = mbar_wait(&w_full[ws], (uint32_t)((i / WS) & 1), &g_q8tc_error) &&
                     mbar_wait(&a_tab[as], (uint32_t)((i / AS) & 1), &g_q8tc_error);
                ok = __all_sync(0xffffffffu, ok);
            }
            if (ok) {
                // this row's 8 weight block scales; the columns' (dx, -dx B) table
                const uint4 dwv = *(const uint4*)(wst + (size_t)ws * Q8T_WSTAGE + 2 * Q8T_WHALF + row * 16);
                const __half* dws = (const __half*)&dwv;
                const float2* tab = (const float2*)(act + (size_t)as * C::ASTAGE + 2 * C::AHALF + C::ASC) + cq * NQ;
                for (int g = 0; g < GPU && ok; g++) {
                    const int q = i * GPU + g, b = q & 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (uint32_t)((q >> 1) & 1), &g_q8tc_error));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int bl = 0; bl < BPB; bl++) {
                        const int j = g * BPB + bl;
                        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) +
                                               (uint32_t)((b * BPB + bl) * N + cq * NQ);
                        const float dw = __half2float(dws[j]);
                        const float4* tj = (const float4*)(tab + j * N);   // two columns per float4
                        constexpr int CH = NQ < 16 ? NQ : 16;
#pragma unroll
                        for (int cc = 0; cc < NQ; cc += CH) {
                            uint32_t v[16];
                            if (CH == 16) tmem_ld16(taddr + cc, v);
                            else if (CH == 8) tmem_ld8(taddr + cc, v);
                            else tmem_ld4(taddr + cc, v);
                            tmem_wait_ld();
                            if (bl == BPB - 1 && cc + CH == NQ) {   // every read of this group done
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&acc_empty[b]);
                            }
#pragma unroll
                            for (int c = 0; c < CH; c += 2) {
                                const float4 t = tj[(cc + c) >> 1];
                                const float p0 = fmaf(t.x, __int_as_float(0x4B400000 + (int)v[c]), t.y);
                                const float p1 = fmaf(t.z, __int_as_float(0x4B400000 + (int)v[c + 1]), t.w);
                                yacc[cc + c] = fmaf(dw, p0, yacc[cc + c]);
                                yacc[cc + c + 1] = fmaf(dw, p1, yacc[cc + c + 1]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {   // this unit's scales are read: its stages may be refilled
                mbar_arrive(&w_empty[ws]);
                mbar_arrive(&a_empty[as]);
            }
            // ---- end of a tile segment: direct store, or partial + ticket (last arriver sums) ----
            if (i == nu - 1 || s == nb - 1) {
                const int64_t r = (tile / ct_tiles) * Q8T_ROWS + row;
                const int cbase = (int)(tile % ct_tiles) * N + cq * NQ;
                if (seg_s0 == 0 && s == nb - 1) {
                    if (ok && r < n)
#pragma unroll
                        for (int c = 0; c < NQ; c++)
                            if (cbase + c < m) y[(size_t)(cbase + c) * n + r] = yacc[c];
                } else {
                    const int64_t t0 = tile * nb;
                    const int slot = sk_begin(bid, T, G) > t0 ? 0 : 1;
                    float* P = part + (size_t)(bid * 2 + slot) * N * Q8T_ROWS;
#pragma unroll
                    for (int c = 0; c < NQ; c++) P[(cq * NQ + c) * Q8T_ROWS + row] = yacc[c];
                    __threadfence();
                    q8_epi_bar();
                    const int64_t cf = sk_owner(t0, T, G), cl = sk_owner(t0 + nb - 1, T, G);
                    if (et == 0) {
                        const int old = atomicAdd(&tickets[tile], 1);
                        const int last = old == (int)(cl - cf);
                        if (last) tickets[tile] = 0;
                        *last_flag = last;
                    }
                    q8_epi_bar();
                    if (*last_flag) {
                        __threadfence();
#pragma unroll
                        for (int c = 0; c < NQ; c++) yacc[c] = 0.0f;
                        for (int64_t qq = cf; qq <= cl; qq++) {
                            const int sq = sk_begin(qq, T, G) > t0 ? 0 : 1;
                            const float* Q = part + (size_t)(qq * 2 + sq) * N * Q8T_ROWS;
#pragma unroll
                            for (int c = 0; c < NQ; c++) yacc[c] += __ldcg(&Q[(cq * NQ + c) * Q8T_ROWS + row]);
                        }
                        if (ok && r < n)
#pragma unroll
                            for (int c = 0; c < NQ; c++)
                                if (cbase + c < m) y[(size_t)(cbase + c) * n + r] = yacc[c];
                    }
                    q8_epi_bar();
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
    }
    pdl_trigger();
}

// ---- host side ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();  // qmm.cu

static cudaError_t map2d(CUtensorMap* mp, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                         uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)(inner * esize)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(mp, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? cudaSuccess
               : cudaErrorInvalidValue;
}

static int q8tc_n(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128)); }

struct Q8tPlan {
    int N, ct;
    int64_t rt, T, G;
};
static Q8tPlan q8tc_plan(int64_t n, int64_t k, int64_t m) {
    Q8tPlan p;
    p.N = q8tc_n(m);
    p.ct = (int)((m + p.N - 1) / p.N);
    p.rt = (n + Q8T_ROWS - 1) / Q8T_ROWS;
    p.T = p.rt * p.ct * (k / 256);
    const int64_t sms = num_sms();
    // at least sk_min_units() units per CTA (tuning knob DCG_SK_MIN_UNITS), at most one CTA per SM
    const int64_t mu = sk_min_units();
    const int64_t want = (p.T + mu - 1) / mu;
    p.G = want < sms ? want : sms;
    return p;
}

bool qmm_q8tc_supports(int type, int64_t n, int64_t k, int64_t m) {
    return type == DCG_TYPE_Q8_0 && m >= 2 && k % 256 == 0 && n > 0;
}
size_t qmm_q8tc_scratch_bytes(int64_t n, int64_t k, int64_t m) {
    const Q8tPlan p = q8tc_plan(n, k, m);
    return align256((size_t)p.rt * p.ct * 4) + (size_t)p.G * 2 * p.N * Q8T_ROWS * 4;
}
int qmm_q8tc_ticket_count(int64_t n, int64_t k, int64_t m) {
    const Q8tPlan p = q8tc_plan(n, k, m);
    return (int)(p.rt * p.ct);
}

template <int N>
static cudaError_t launch_q8tc_t(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m, float* y,
                                 void* scratch, const Q8tPlan& p, cudaStream_t st) {
    using C = Q8tCfg<N>;
    cudaError_t e = DCG_SMEM_ATTR((qmm_q8tc_kernel<N>), C::SMEM);
    if (e != cudaSuccess) return e;
    CUtensorMap wm, wdm, am, adm;
    const uint64_t nb32 = (uint64_t)(k / 32);
    if ((e = map2d(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.payload, (uint64_t)k, (uint64_t)n, 128, Q8T_ROWS,
                   CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
        return e;
    if ((e = map2d(&wdm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, nb32, (uint64_t)n, 8, Q8T_ROWS,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) != cudaSuccess)
        return e;
    if ((e = map2d(&am, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.qs, (uint64_t)k, (uint64_t)m, 128, N,
                   CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
        return e;
    if ((e = map2d(&adm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.d, nb32, (uint64_t)m, 8, N,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) != cudaSuccess)
        return e;
    int* tickets = (int*)scratch;
    float* part = (float*)((uint8_t*)scratch + align256((size_t)p.rt * p.ct * 4));
    return launch_pdl(qmm_q8tc_kernel<N>, dim3((unsigned)p.G), dim3(Q8T_THREADS), (size_t)C::SMEM, st, wm, wdm, am,
                      adm, (int)(k / 256), n, m, y, p.ct, p.T, part, tickets);
}

cudaError_t launch_qmm_q8tc(const void* packed_w, int64_t n, int64_t k, const void* act, int64_t m, float* y,
                            void* scratch, cudaStream_t st) {
    const PackedW w = packed_view(DCG_TYPE_Q8_0, packed_w, n, k);
    const ActQ a = act_view(DCG_TYPE_Q8_0, const_cast<void*>(act), m, k);
    const Q8tPlan p = q8tc_plan(n, k, m);
    switch (p.N) {
        case 16: return launch_q8tc_t<16>(w, n, k, a, (int)m, y, scratch, p, st);
        case 32: return launch_q8tc_t<32>(w, n, k, a, (int)m, y, scratch, p, st);
        case 64: return launch_q8tc_t<64>(w, n, k, a, (int)m, y, scratch, p, st);
        default: return launch_q8tc_t<128>(w, n, k, a, (int)m, y, scratch, p, st);
    }
}

}  // namespace dcg
