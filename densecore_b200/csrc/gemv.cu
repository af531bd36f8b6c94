// gemv.cu -- memory-bound quantized mat-vec (M <= 8 activation rows per launch).
//
// Replaces the row loop of DenseCore's cb_gemv_custom (core/src/inference.cpp:916-924), which calls
// ggml vec_dot_{q8_0_q8_0,q4_K_q8_K,q6_K_q8_K} once per output row.  Here every lane streams
// 16-byte vectors of weight payload (ld.global.nc, no L1 allocation), unpacks them to int8 lanes in
// registers, takes dp4a int32 dot products per sub-block, applies the integer sub-block scales,
// and converts to fp32 once per (lane, super-block) with the fp16/f32 block scales.
//
// Work mapping (one CTA = 8 warps):
//   * a "unit" is the span of one row that one warp covers with one 16-B load per lane:
//       Q8_0: 16 blocks of 32 (512 weights; lane = (block, half-block));
//       Q4_K / Q6_K: 4 super-blocks of 256 (1024 weights; 8 lanes per super-block).
//   * warp w owns R consecutive rows and the K-slice ks = w % S (units ks, ks+S, ...);
//     the S partial sums of a row are combined through shared memory at the end.
// The activation rows (SoA Q8_0 / Q8_K, common.cuh) are read through L1: every warp of the SM
// reads the same few KB.
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

#include <algorithm>

namespace dcg {

template <int TYPE>
struct UnitInfo;
template <>
struct UnitInfo<DCG_TYPE_Q8_0> { static constexpr int BLOCKS = 16; };
template <>
struct UnitInfo<DCG_TYPE_Q4_K> { static constexpr int BLOCKS = 4; };
template <>
struct UnitInfo<DCG_TYPE_Q6_K> { static constexpr int BLOCKS = 4; };

// weight registers of one (unit, row) for one lane
struct WReg {
    uint4 a;  // Q8_0: 16 qs | Q4_K: 16 nibble bytes | Q6_K: ql
    uint4 b;  // Q4_K: block header (d, dmin, scales) | Q6_K: qh
    uint4 c;  // Q6_K: scales
    float d;  // Q8_0 / Q6_K: block scale (fp16 -> f32); Q4_K: d
    float dmin;
};

template <bool SMEM>
__device__ __forceinline__ uint4 ldw(const uint8_t* p) {
    if (SMEM) return *(const uint4*)p;
    return ld_stream_v4(p);
}

// lane's weight registers of block `blk` of one row; rowp = start of the row's payload (global
// or shared), drow = the row's fp16 block scales (Q8_0 / Q6_K; global)
template <int TYPE, bool SMEM>
__device__ __forceinline__ void load_w_row(const uint8_t* rowp, const __half* drow, int blk, int lane,
                                           WReg& r) {
    if (TYPE == DCG_TYPE_Q8_0) {
        r.a = ldw<SMEM>(rowp + (size_t)blk * QK8_0 + (lane & 1) * 16);
        r.d = __half2float(drow[blk]);
    } else if (TYPE == DCG_TYPE_Q4_K) {
        const uint8_t* p = rowp + (size_t)blk * Q4_K_BYTES;
        r.b = ldw<SMEM>(p);
        r.a = ldw<SMEM>(p + 16 + (lane & 7) * 16);
    } else {
        const int i = lane & 7, h = i >> 2, c = (i >> 1) & 1, half = i & 1;
        const uint8_t* p = rowp + (size_t)blk * Q6_K_PAYLOAD;
        r.a = ldw<SMEM>(p + h * 64 + c * 32 + half * 16);
        r.b = ldw<SMEM>(p + 128 + h * 32 + half * 16);
        r.c = ldw<SMEM>(p + 192);
        r.d = __half2float(drow[blk]);
    }
}

template <int TYPE>
__device__ __forceinline__ void load_w(const PackedW& w, int64_t row, int blk, int lane, WReg& r) {
    load_w_row<TYPE, false>(w.payload + row * w.row_bytes, w.d ? w.d + row * w.nb : nullptr, blk,
                            lane, r);
}

__device__ __forceinline__ uint32_t u4(const uint4& v, int t) {
    return t == 0 ? v.x : (t == 1 ? v.y : (t == 2 ? v.z : v.w));
}

// one lane's contribution of one (unit, row) against activation row m
template <int TYPE>
__device__ __forceinline__ float lane_dot(const WReg& r, const ActQ& a, int64_t k, int nb, int m,
                                          int blk, int lane) {
    if (TYPE == DCG_TYPE_Q8_0) {
        const size_t e0 = (size_t)m * k + (size_t)blk * QK8_0 + (lane & 1) * 16;
        const uint4 xv = ld_act_v4(a.qs + e0);
        int s = 0;
        s = dp4a((int)r.a.x, (int)xv.x, s);
        s = dp4a((int)r.a.y, (int)xv.y, s);
        s = dp4a((int)r.a.z, (int)xv.z, s);
        s = dp4a((int)r.a.w, (int)xv.w, s);
        const float dx = __half2float(((const __half*)a.d)[(size_t)m * nb + blk]);
        return __fmul_rn(r.d, dx) * (float)s;
    } else if (TYPE == DCG_TYPE_Q4_K) {
        const int i = lane & 7, g = i >> 1, half = i & 1;
        const int j0 = 2 * g, j1 = 2 * g + 1;
        const int8_t* xq = a.qs + (size_t)m * k + (size_t)blk * QK_K + j0 * 32 + half * 16;
        const uint4 xl = ld_act_v4(xq);
        const uint4 xh = ld_act_v4(xq + 32);
        int d0 = 0, d1 = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t q = u4(r.a, t);
            d0 = dp4a((int)(q & 0x0F0F0F0Fu), (int)u4(xl, t), d0);
            d1 = dp4a((int)((q >> 4) & 0x0F0F0F0Fu), (int)u4(xh, t), d1);
        }
        int sc0, m0, sc1, m1;
        q4k_scale_min(r.b.y, r.b.z, r.b.w, j0, sc0, m0);
        q4k_scale_min(r.b.y, r.b.z, r.b.w, j1, sc1, m1);
        const int isum = sc0 * d0 + sc1 * d1;
        const int16_t* bs = a.bsums + (size_t)m * (k / 16) + (size_t)blk * 16;
        const int msum = m0 * (int)bs[2 * j0 + half] + m1 * (int)bs[2 * j1 + half];
        const float dx = ((const float*)a.d)[(size_t)m * nb + blk];
        const __half2 dd = *reinterpret_cast<const __half2*>(&r.b.x);
        const float dw = __low2float(dd), dmin = __high2float(dd);
        return dx * (dw * (float)isum - dmin * (float)msum);
    } else {
        const int i = lane & 7, h = i >> 2, c = (i >> 1) & 1, half = i & 1;
        const int s_lo = h * 8 + c * 2 + half, s_hi = s_lo + 4;
        const int8_t* xq = a.qs + (size_t)m * k + (size_t)blk * QK_K + h * 128 + c * 32 + half * 16;
        const uint4 xl = ld_act_v4(xq);
        const uint4 xh = ld_act_v4(xq + 64);
        int d0 = 0, d1 = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t ql = u4(r.a, t), qh = u4(r.b, t);
            const uint32_t lo = (ql & 0x0F0F0F0Fu) | (((qh >> (2 * c)) & 0x03030303u) << 4);
            const uint32_t hi = ((ql >> 4) & 0x0F0F0F0Fu) | (((qh >> (2 * c + 4)) & 0x03030303u) << 4);
            d0 = dp4a((int)__vsub4(lo, 0x20202020u), (int)u4(xl, t), d0);
            d1 = dp4a((int)__vsub4(hi, 0x20202020u), (int)u4(xh, t), d1);
        }
        const int sc_lo = (int)(int8_t)((u4(r.c, s_lo >> 2) >> (8 * (s_lo & 3))) & 0xFF);
        const int sc_hi = (int)(int8_t)((u4(r.c, s_hi >> 2) >> (8 * (s_hi & 3))) & 0xFF);
        const int isum = sc_lo * d0 + sc_hi * d1;
        const float dx = ((const float*)a.d)[(size_t)m * nb + blk];
        return __fmul_rn(r.d, dx) * (float)isum;
    }
}

template <int TYPE, int M, int R>
__global__ void __launch_bounds__(256) gemv_kernel(PackedW w, int64_t n, int64_t k, ActQ a,
                                                   int m0, float* __restrict__ y, int S) {
    pdl_wait();
    pdl_trigger();
    constexpr int PER = UnitInfo<TYPE>::BLOCKS;
    constexpr int U = 2;  // units in flight per warp
    __shared__ float red[8][R * M];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int rg = wid / S, ks = wid % S;
    const int rows_per_cta = (8 / S) * R;
    const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta + (int64_t)rg * R;
    const int nb = w.nb;
    const int n_units = (nb + PER - 1) / PER;
    const int lane_blk = (TYPE == DCG_TYPE_Q8_0) ? (lane >> 1) : (lane >> 3);

    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int mm = 0; mm < M; mm++) acc[r][mm] = 0.0f;

    for (int u0 = ks; u0 < n_units; u0 += S * U) {
        WReg wr[U][R];
        bool ok[U][R];
#pragma unroll
        for (int uu = 0; uu < U; uu++) {
            const int u = u0 + uu * S;
            const int blk = u * PER + lane_blk;
#pragma unroll
            for (int r = 0; r < R; r++) {
                ok[uu][r] = (u < n_units) && (blk < nb) && (row0 + r < n);
                if (ok[uu][r]) load_w<TYPE>(w, row0 + r, blk, lane, wr[uu][r]);
            }
        }
#pragma unroll
        for (int uu = 0; uu < U; uu++) {
            const int blk = (u0 + uu * S) * PER + lane_blk;
#pragma unroll
            for (int mm = 0; mm < M; mm++)
#pragma unroll
                for (int r = 0; r < R; r++)
                    if (ok[uu][r]) acc[r][mm] += lane_dot<TYPE>(wr[uu][r], a, k, nb, m0 + mm, blk, lane);
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int mm = 0; mm < M; mm++) {
            float v = acc[r][mm];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[wid][r * M + mm] = v;
        }
    __syncthreads();
    for (int t = threadIdx.x; t < (8 / S) * R * M; t += blockDim.x) {
        const int g = t / (R * M), rm = t % (R * M);
        const int r = rm / M, mm = rm % M;
        const int64_t row = (int64_t)blockIdx.x * rows_per_cta + (int64_t)g * R + r;
        if (row >= n) continue;
        float s = 0.0f;
        for (int q = 0; q < S; q++) s += red[g * S + q][rm];
        y[(size_t)(m0 + mm) * n + row] = s;
    }
}

// ------------------------------------------------------------------------------------------
// TMA-streamed GEMV.  Tiles of TR consecutive whole rows (contiguous bytes of the row-major
// payload) are copied global -> shared by the bulk-copy engine through a STAGES-deep ring of
// buffers completing on mbarriers; the 8 warps decode from shared memory.  Thread 0 keeps
// STAGES-1 tiles in flight; a __syncthreads at the end of each tile frees its buffer.
//   TR >= 8: warp w reduces rows w, w+8, ... of the tile on its own;
//   TR <  8: 8/TR warps split one row's units and combine partials in a fixed order.
// ------------------------------------------------------------------------------------------
// error flag of the bounded waits in this file (read back by dcg_device_error)
__device__ int g_gemv_error = 0;

cudaError_t gemv_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int TMA_STAGES = 4;
constexpr int TMA_TILE = 24 * 1024;  // bytes per stage; 2 CTAs (2 x ~97 KB) fit one SM

template <int TYPE, int M>
__global__ void __launch_bounds__(256, 2) gemv_tma_kernel(PackedW w, int64_t n, int64_t k, ActQ a,
                                                          int m0, float* __restrict__ y, int TR) {
    pdl_wait();
    pdl_trigger();
    constexpr int PER = UnitInfo<TYPE>::BLOCKS;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;                                    // [STAGES]
    float* red = (float*)(smem + 64);                                    // [2][8][M]
    uint8_t* buf = smem + 64 + ((2 * 8 * M * 4 + 127) & ~127);           // [STAGES][TILE]
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nb = w.nb;
    const int upr = (nb + PER - 1) / PER;  // units per row
    const int lane_blk = (TYPE == DCG_TYPE_Q8_0) ? (lane >> 1) : (lane >> 3);
    const int64_t n_tiles = (n + TR - 1) / TR;
    const int my_tiles = (int)((n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < TMA_STAGES; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int i) {  // tile i of this CTA into stage i % STAGES
        const int64_t t = blockIdx.x + (int64_t)i * gridDim.x;
        const int64_t r0 = t * TR;
        const int rows = (int)((n - r0) < TR ? (n - r0) : TR);
        const uint32_t bytes = (uint32_t)(rows * w.row_bytes);
        uint64_t* bar = &full[i % TMA_STAGES];
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(buf + (size_t)(i % TMA_STAGES) * TMA_TILE, w.payload + r0 * w.row_bytes, bytes, bar);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < TMA_STAGES - 1 && i < my_tiles; i++) issue(i);

    const int wpr = TR >= 8 ? 1 : 8 / TR;  // warps per row
    for (int i = 0; i < my_tiles; i++) {
        if (threadIdx.x == 0 && i + TMA_STAGES - 1 < my_tiles) {
            fence_proxy_async_smem();
            issue(i + TMA_STAGES - 1);
        }
        const int64_t r0 = (blockIdx.x + (int64_t)i * gridDim.x) * TR;
        const int rows = (int)((n - r0) < TR ? (n - r0) : TR);
        bool ok = mbar_wait(&full[i % TMA_STAGES], (uint32_t)((i / TMA_STAGES) & 1), &g_gemv_error);
        const uint8_t* tile = buf + (size_t)(i % TMA_STAGES) * TMA_TILE;
        float* redb = red + (i & 1) * 8 * M;
        for (int rr = wid / wpr; rr < rows; rr += 8 / wpr) {
            const int64_t row = r0 + rr;
            const uint8_t* rowp = tile + (size_t)rr * w.row_bytes;
            const __half* drow = w.d ? w.d + row * nb : nullptr;
            float acc[M];
#pragma unroll
            for (int mm = 0; mm < M; mm++) acc[mm] = 0.0f;
            for (int u = wid % wpr; u < upr; u += wpr) {
                const int blk = u * PER + lane_blk;
                if (blk < nb) {
                    WReg r;
                    load_w_row<TYPE, true>(rowp, drow, blk, lane, r);
#pragma unroll
                    for (int mm = 0; mm < M; mm++) acc[mm] += lane_dot<TYPE>(r, a, k, nb, m0 + mm, blk, lane);
                }
            }
#pragma unroll
            for (int mm = 0; mm < M; mm++) {
                float v = acc[mm];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[mm] = v;
            }
            if (lane == 0) {
                if (wpr == 1) {
#pragma unroll
                    for (int mm = 0; mm < M; mm++) y[(size_t)(m0 + mm) * n + row] = acc[mm];
                } else {
#pragma unroll
                    for (int mm = 0; mm < M; mm++) redb[wid * M + mm] = acc[mm];
                }
            }
        }
        ok = __syncthreads_and(ok);  // frees this stage for the next issue; uniform exit on error
        if (!ok) return;
        if (wpr > 1 && threadIdx.x < rows * M) {
            const int rr = threadIdx.x / M, mm = threadIdx.x % M;
            float s = 0.0f;
            for (int q = 0; q < wpr; q++) s += redb[(rr * wpr + q) * M + mm];
            y[(size_t)(m0 + mm) * n + r0 + rr] = s;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Register-resident-activation variant (M <= 2).  A lane always decodes the same K positions of
// every row it touches (its slot inside a super-block / block and the units u = sub + j*wpr of
// its warp), so its slice of the quantized activation -- payload bytes, block scale and (Q4_K)
// the two Q8_K block sums it needs -- is loaded into registers once per kernel.  The loop body is
// then shared-memory weight loads, nibble unpacking, dp4a and a few fp32 ops.
// ------------------------------------------------------------------------------------------
struct XReg {
    uint4 lo, hi;  // Q8_0: lo only; Q4_K: sub-blocks j0 / j1; Q6_K: low / high nibble elements
    float d;       // activation block scale
    int b0, b1;    // Q4_K: Q8_K bsums of this lane's 16-element halves of sub-blocks j0 / j1
};

template <int TYPE>
__device__ __forceinline__ void load_x(const ActQ& a, int64_t k, int nb, int m, int blk, int lane,
                                       XReg& x) {
    if (TYPE == DCG_TYPE_Q8_0) {
        x.lo = ld_act_v4(a.qs + (size_t)m * k + (size_t)blk * QK8_0 + (lane & 1) * 16);
        x.d = __half2float(((const __half*)a.d)[(size_t)m * nb + blk]);
    } else if (TYPE == DCG_TYPE_Q4_K) {
        const int i = lane & 7, g = i >> 1, half = i & 1;
        const int8_t* xq = a.qs + (size_t)m * k + (size_t)blk * QK_K + 64 * g + half * 16;
        x.lo = ld_act_v4(xq);
        x.hi = ld_act_v4(xq + 32);
        x.d = ((const float*)a.d)[(size_t)m * nb + blk];
        const int16_t* bs = a.bsums + (size_t)m * (k / 16) + (size_t)blk * 16;
        x.b0 = bs[4 * g + half];
        x.b1 = bs[4 * g + 2 + half];
    } else {
        const int i = lane & 7, h = i >> 2, c = (i >> 1) & 1, half = i & 1;
        const int8_t* xq = a.qs + (size_t)m * k + (size_t)blk * QK_K + h * 128 + c * 32 + half * 16;
        x.lo = ld_act_v4(xq);
        x.hi = ld_act_v4(xq + 64);
        x.d = ((const float*)a.d)[(size_t)m * nb + blk];
    }
}

// Q4_K: the (scale, min) pairs of sub-blocks j0 = 2g and j1 = 2g+1, branch-free; returns
// sc0 | sc1 << 8 in *sc and m0 | m1 << 8 in *mn (ggml get_scale_min_k4 layout)
__device__ __forceinline__ void q4k_pair(const uint4& hdr, int g, uint32_t& sc, uint32_t& mn) {
    const int sh = 16 * (g & 1);  // bytes (2g)&3 and (2g+1)&3 of each scale word
    const uint32_t a0 = (hdr.y >> sh) & 0xFFFFu, a1 = (hdr.z >> sh) & 0xFFFFu, a2 = (hdr.w >> sh) & 0xFFFFu;
    const uint32_t sc_lo = a0 & 0x3F3Fu, mn_lo = a1 & 0x3F3Fu;
    const uint32_t sc_hi = (a2 & 0x0F0Fu) | ((a0 >> 2) & 0x3030u);
    const uint32_t mn_hi = ((a2 >> 4) & 0x0F0Fu) | ((a1 >> 2) & 0x3030u);
    sc = g >= 2 ? sc_hi : sc_lo;
    mn = g >= 2 ? mn_hi : mn_lo;
}

template <int TYPE>
__device__ __forceinline__ float xr_dot(const uint4& wa, const uint4& wb, const uint4& wc, float wd,
                                        const XReg& x, int lane) {
    if (TYPE == DCG_TYPE_Q8_0) {
        int s = dp4a((int)wa.x, (int)x.lo.x, 0);
        s = dp4a((int)wa.y, (int)x.lo.y, s);
        s = dp4a((int)wa.z, (int)x.lo.z, s);
        s = dp4a((int)wa.w, (int)x.lo.w, s);
        return (wd * x.d) * (float)s;
    } else if (TYPE == DCG_TYPE_Q4_K) {
        int d0 = 0, d1 = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t q = u4(wa, t);
            d0 = dp4a((int)(q & 0x0F0F0F0Fu), (int)u4(x.lo, t), d0);
            d1 = dp4a((int)((q >> 4) & 0x0F0F0F0Fu), (int)u4(x.hi, t), d1);
        }
        uint32_t sc, mn;
        q4k_pair(wb, (lane & 7) >> 1, sc, mn);
        const int isum = (int)(sc & 0xFF) * d0 + (int)(sc >> 8) * d1;
        const int msum = (int)(mn & 0xFF) * x.b0 + (int)(mn >> 8) * x.b1;
        const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&wb.x));
        return x.d * (dd.x * (float)isum - dd.y * (float)msum);
    } else {
        const int i = lane & 7, h = i >> 2, c = (i >> 1) & 1, half = i & 1;
        int d0 = 0, d1 = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t ql = u4(wa, t), qh = u4(wb, t);
            const uint32_t lo = (ql & 0x0F0F0F0Fu) | (((qh >> (2 * c)) & 0x03030303u) << 4);
            const uint32_t hi = ((ql >> 4) & 0x0F0F0F0Fu) | (((qh >> (2 * c + 4)) & 0x03030303u) << 4);
            d0 = dp4a((int)__vsub4(lo, 0x20202020u), (int)u4(x.lo, t), d0);
            d1 = dp4a((int)__vsub4(hi, 0x20202020u), (int)u4(x.hi, t), d1);
        }
        const int s_lo = h * 8 + c * 2 + half;  // scales s_lo (word s_lo/4) and s_lo + 4 (next word)
        const int sc_lo = (int)(int8_t)(u4(wc, s_lo >> 2) >> (8 * (s_lo & 3)));
        const int sc_hi = (int)(int8_t)(u4(wc, (s_lo >> 2) + 1) >> (8 * (s_lo & 3)));
        return (wd * x.d) * (float)(sc_lo * d0 + sc_hi * d1);
    }
}

// 3 CTAs of 8 warps per SM: 3 stages of 20 KB each, <= 85 registers per thread
constexpr int XR_STAGES = 3;
constexpr int XR_TILE = 20 * 1024;
constexpr int XR_CTAS = 3;

template <int TYPE, int M, int UW>
__global__ void __launch_bounds__(256, (UW <= 4 ? XR_CTAS : 2)) gemv_tma_xr_kernel(PackedW w, int64_t n, int64_t k, ActQ a,
                                                             int m0, float* __restrict__ y, int TR) {
    constexpr int PER = UnitInfo<TYPE>::BLOCKS;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;
    float* red = (float*)(smem + 64);
    uint8_t* buf = smem + 64 + ((2 * 8 * M * 4 + 127) & ~127);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nb = w.nb;
    const int upr = (nb + PER - 1) / PER;
    const int lane_blk = (TYPE == DCG_TYPE_Q8_0) ? (lane >> 1) : (lane >> 3);
    const int64_t n_tiles = (n + TR - 1) / TR;
    const int my_tiles = (int)((n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x);
    const int wpr = TR >= 8 ? 1 : 8 / TR;
    const int sub = wid % wpr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < XR_STAGES; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int i) {
        const int64_t t = blockIdx.x + (int64_t)i * gridDim.x;
        const int64_t r0 = t * TR;
        const int rows = (int)((n - r0) < TR ? (n - r0) : TR);
        const uint32_t bytes = (uint32_t)(rows * w.row_bytes);
        uint64_t* bar = &full[i % XR_STAGES];
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(buf + (size_t)(i % XR_STAGES) * XR_TILE, w.payload + r0 * w.row_bytes, bytes, bar);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < XR_STAGES - 1 && i < my_tiles; i++) issue(i);
    // the weight tiles are constant: requested before the wait on the kernel producing the activation
    pdl_wait();
    pdl_trigger();

    // this lane's activation slice, once (overlaps the first bulk copies)
    XReg xr[UW][M];
    bool uok[UW];
#pragma unroll
    for (int j = 0; j < UW; j++) {
        const int u = sub + j * wpr;
        const int blk = u * PER + lane_blk;
        uok[j] = (u < upr) && (blk < nb);
#pragma unroll
        for (int mm = 0; mm < M; mm++)
            if (uok[j]) load_x<TYPE>(a, k, nb, m0 + mm, blk, lane, xr[j][mm]);
    }

    for (int i = 0; i < my_tiles; i++) {
        if (threadIdx.x == 0 && i + XR_STAGES - 1 < my_tiles) {
            fence_proxy_async_smem();
            issue(i + XR_STAGES - 1);
        }
        const int64_t r0 = (blockIdx.x + (int64_t)i * gridDim.x) * TR;
        const int rows = (int)((n - r0) < TR ? (n - r0) : TR);
        bool ok = mbar_wait(&full[i % XR_STAGES], (uint32_t)((i / XR_STAGES) & 1), &g_gemv_error);
        const uint8_t* tile = buf + (size_t)(i % XR_STAGES) * XR_TILE;
        float* redb = red + (i & 1) * 8 * M;
        for (int rr = wid / wpr; rr < rows; rr += 8 / wpr) {
            const int64_t row = r0 + rr;
            const uint8_t* rowp = tile + (size_t)rr * w.row_bytes;
            float wdv[UW];
            if (TYPE != DCG_TYPE_Q4_K) {
#pragma unroll
                for (int j = 0; j < UW; j++)
                    wdv[j] = uok[j] ? __half2float(w.d[row * nb + (sub + j * wpr) * PER + lane_blk]) : 0.0f;
            }
            float acc[M];
#pragma unroll
            for (int mm = 0; mm < M; mm++) acc[mm] = 0.0f;
#pragma unroll
            for (int j = 0; j < UW; j++) {
                if (!uok[j]) continue;
                const int blk = (sub + j * wpr) * PER + lane_blk;
                uint4 wa, wb = make_uint4(0, 0, 0, 0), wc = make_uint4(0, 0, 0, 0);
                if (TYPE == DCG_TYPE_Q8_0) {
                    wa = *(const uint4*)(rowp + (size_t)blk * QK8_0 + (lane & 1) * 16);
                } else if (TYPE == DCG_TYPE_Q4_K) {
                    const uint8_t* p = rowp + (size_t)blk * Q4_K_BYTES;
                    wb = *(const uint4*)p;
                    wa = *(const uint4*)(p + 16 + (lane & 7) * 16);
                } else {
                    const int li = lane & 7, h = li >> 2, c = (li >> 1) & 1, half = li & 1;
                    const uint8_t* p = rowp + (size_t)blk * Q6_K_PAYLOAD;
                    wa = *(const uint4*)(p + h * 64 + c * 32 + half * 16);
                    wb = *(const uint4*)(p + 128 + h * 32 + half * 16);
                    wc = *(const uint4*)(p + 192);
                }
#pragma unroll
                for (int mm = 0; mm < M; mm++)
                    acc[mm] += xr_dot<TYPE>(wa, wb, wc, TYPE == DCG_TYPE_Q4_K ? 0.0f : wdv[j], xr[j][mm], lane);
            }
#pragma unroll
            for (int mm = 0; mm < M; mm++) {
                float v = acc[mm];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[mm] = v;
            }
            if (lane == 0) {
                if (wpr == 1) {
#pragma unroll
                    for (int mm = 0; mm < M; mm++) y[(size_t)(m0 + mm) * n + row] = acc[mm];
                } else {
#pragma unroll
                    for (int mm = 0; mm < M; mm++) redb[wid * M + mm] = acc[mm];
                }
            }
        }
        ok = __syncthreads_and(ok);
        if (!ok) return;
        if (wpr > 1 && threadIdx.x < rows * M) {
            const int rr = threadIdx.x / M, mm = threadIdx.x % M;
            float s = 0.0f;
            for (int q = 0; q < wpr; q++) s += redb[(rr * wpr + q) * M + mm];
            y[(size_t)(m0 + mm) * n + r0 + rr] = s;
        }
    }
}

template <int TYPE, int M, int UW>
static cudaError_t launch_xr(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m0, float* y,
                             int TR, int grid, cudaStream_t st) {
    const size_t smem = 64 + ((2 * 8 * M * 4 + 127) & ~127) + (size_t)XR_STAGES * XR_TILE;
    cudaError_t e = DCG_SMEM_ATTR((gemv_tma_xr_kernel<TYPE, M, UW>), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(gemv_tma_xr_kernel<TYPE, M, UW>, dim3((unsigned)grid), dim3(256), smem, st, w, n, k, a,
                      m0, y, TR);
}

// returns cudaErrorNotSupported when the shape needs more than 8 units per warp
template <int TYPE, int M>
static cudaError_t launch_gemv_xr_t(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m0,
                                    float* y, cudaStream_t st) {
    constexpr int PER = UnitInfo<TYPE>::BLOCKS;
    int TR = 1;
    while (TR * 2 * (int64_t)w.row_bytes <= XR_TILE && TR < 64) TR *= 2;
    const int wpr = TR >= 8 ? 1 : 8 / TR;
    const int upr = (w.nb + PER - 1) / PER;
    const int uw = (upr + wpr - 1) / wpr;
    const int64_t n_tiles = (n + TR - 1) / TR;
    const int grid = (int)std::min<int64_t>(n_tiles, (int64_t)num_sms() * XR_CTAS);
    if (uw <= 1) return launch_xr<TYPE, M, 1>(w, n, k, a, m0, y, TR, grid, st);
    if (uw <= 2) return launch_xr<TYPE, M, 2>(w, n, k, a, m0, y, TR, grid, st);
    if (uw <= 4) return launch_xr<TYPE, M, 4>(w, n, k, a, m0, y, TR, grid, st);
    if constexpr (M == 1) {  // 8 units x 2 activation rows would spill
        if (uw <= 8) return launch_xr<TYPE, M, 8>(w, n, k, a, m0, y, TR, grid, st);
    }
    return cudaErrorNotSupported;
}

template <int TYPE, int M>
static cudaError_t launch_gemv_tma_t(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m0,
                                     float* y, cudaStream_t st) {
    const size_t smem = 64 + ((2 * 8 * M * 4 + 127) & ~127) + (size_t)TMA_STAGES * TMA_TILE;
    cudaError_t e = DCG_SMEM_ATTR((gemv_tma_kernel<TYPE, M>), smem);
    if (e != cudaSuccess) return e;
    int TR = 1;
    while (TR * 2 * (int64_t)w.row_bytes <= TMA_TILE && TR < 64) TR *= 2;
    const int64_t n_tiles = (n + TR - 1) / TR;
    const int64_t grid = std::min<int64_t>(n_tiles, (int64_t)num_sms() * 2);
    return launch_pdl(gemv_tma_kernel<TYPE, M>, dim3((unsigned)grid), dim3(256), smem, st, w, n, k, a, m0, y,
                      TR);
}

template <int TYPE, int M>
static cudaError_t launch_gemv_t(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m0,
                                 float* y, cudaStream_t st) {
    constexpr int R = (M <= 2) ? 4 : 2;
    constexpr int PER = UnitInfo<TYPE>::BLOCKS;
    const int n_units = (w.nb + PER - 1) / PER;
    // smallest K-split that still gives >= 4 CTAs per SM, keeping >= 2 units per warp
    int S = 1;
    while (S < 8) {
        const int64_t ctas = (n + (8 / S) * R - 1) / ((8 / S) * R);
        if (ctas >= 4 * 148 || n_units < 4 * S) break;
        S *= 2;
    }
    const int64_t ctas = (n + (8 / S) * R - 1) / ((8 / S) * R);
    return launch_pdl(gemv_kernel<TYPE, M, R>, dim3((unsigned)ctas), dim3(256), 0, st, w, n, k, a, m0, y, S);
}

template <int TYPE>
static cudaError_t dispatch_m(const PackedW& w, int64_t n, int64_t k, const ActQ& a, int m0, int m,
                              float* y, cudaStream_t st) {
    if (w.row_bytes <= (size_t)TMA_TILE && w.row_bytes % 16 == 0) {
        if (m <= 2) {
            cudaError_t e = m == 1 ? launch_gemv_xr_t<TYPE, 1>(w, n, k, a, m0, y, st)
                                   : launch_gemv_xr_t<TYPE, 2>(w, n, k, a, m0, y, st);
            if (e != cudaErrorNotSupported) return e;
        }
        switch (m) {
            case 1: return launch_gemv_tma_t<TYPE, 1>(w, n, k, a, m0, y, st);
            case 2: return launch_gemv_tma_t<TYPE, 2>(w, n, k, a, m0, y, st);
            case 3: return launch_gemv_tma_t<TYPE, 3>(w, n, k, a, m0, y, st);
            case 4: return launch_gemv_tma_t<TYPE, 4>(w, n, k, a, m0, y, st);
            case 5: return launch_gemv_tma_t<TYPE, 5>(w, n, k, a, m0, y, st);
            case 6: return launch_gemv_tma_t<TYPE, 6>(w, n, k, a, m0, y, st);
            case 7: return launch_gemv_tma_t<TYPE, 7>(w, n, k, a, m0, y, st);
            case 8: return launch_gemv_tma_t<TYPE, 8>(w, n, k, a, m0, y, st);
        }
    }
    switch (m) {
        case 1: return launch_gemv_t<TYPE, 1>(w, n, k, a, m0, y, st);
        case 2: return launch_gemv_t<TYPE, 2>(w, n, k, a, m0, y, st);
        case 3: return launch_gemv_t<TYPE, 3>(w, n, k, a, m0, y, st);
        case 4: return launch_gemv_t<TYPE, 4>(w, n, k, a, m0, y, st);
        case 5: return launch_gemv_t<TYPE, 5>(w, n, k, a, m0, y, st);
        case 6: return launch_gemv_t<TYPE, 6>(w, n, k, a, m0, y, st);
        case 7: return launch_gemv_t<TYPE, 7>(w, n, k, a, m0, y, st);
        case 8: return launch_gemv_t<TYPE, 8>(w, n, k, a, m0, y, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                        int64_t act_m, int64_t m0, int64_t m, float* y, cudaStream_t st) {
    if (m < 1 || m > 8) return cudaErrorInvalidValue;
    const PackedW w = packed_view(type, packed_w, n, k);
    const int act_type = type == DCG_TYPE_Q8_0 ? DCG_TYPE_Q8_0 : DCG_TYPE_Q8_K;
    const ActQ a = act_view(act_type, const_cast<void*>(act), act_m, k);
    switch (type) {
        case DCG_TYPE_Q8_0: return dispatch_m<DCG_TYPE_Q8_0>(w, n, k, a, (int)m0, (int)m, y, st);
        case DCG_TYPE_Q4_K: return dispatch_m<DCG_TYPE_Q4_K>(w, n, k, a, (int)m0, (int)m, y, st);
        case DCG_TYPE_Q6_K: return dispatch_m<DCG_TYPE_Q6_K>(w, n, k, a, (int)m0, (int)m, y, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace dcg
