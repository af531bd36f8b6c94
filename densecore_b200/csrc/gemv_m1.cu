// gemv_m1.cu -- single-row quantized mat-vec (M = 1, the decode GEMV) for Q4_K, Q6_K and Q8_0
// weights, with the activation quantized inside the kernel: the B200 form of cb_gemv_custom
// (core/src/inference.cpp:840-948: quantize x with from_float, then one vec_dot per output row).
//
// Layout of the work.  The grid has one CTA per SM.  CTA c owns the contiguous output rows
// [c n / G, (c+1) n / G) with their whole K, so its weights are one contiguous byte range of the
// device layout (a unit = one row x one 256-element super-block: 144 B Q4_K, 208 B Q6_K, 256 B
// Q8_0, stored row-major), plus the matching range of the separate fp16 scale array (Q6_K, Q8_0).
// Every SM therefore streams the same number of bytes, in 1-D bulk copies (TMA) of 32 units, into
// a ring as deep as shared memory allows.  The ring fill is issued before the kernel waits on its
// predecessor (weights are constant), and the copy warp releases this kernel's dependents as soon
// as it has issued its last copy, so the next mat-vec's CTAs (each CTA takes under half of an SM's
// shared memory) start streaming their own weights while this one drains.
//
// Meanwhile all warps quantize x (fp32) to the weight's vec_dot_type in shared memory, with the
// quantize kernels' arithmetic (ggml's quantize_row_q8_0 / q8_K); dcg_mul_mat_q's variant copies
// an already quantized activation instead.  Eight consumer warps then take 4 units each per stage,
// 8 lanes per unit:
//   Q4_K  lane j: 16 nibble bytes = 16 elements of sub-blocks 2g and 2g+1 (g = j / 2), dp4a with
//         the Q8_K quants; isum = sum sc_s dot_s and msum = sum m_s bsum32_s reduced over the 8
//         lanes as integers, then dx (d isum - dmin msum) once per unit (ggml's expression)
//   Q6_K  lane j: 16 ql + 16 qh bytes = two 16-element sub-blocks; isum reduced as an integer,
//         then d dx isum
//   Q8_0  lane j: block j of the unit (32 int8), (dw dx) dot, summed over the 8 blocks
// Each unit's value lands in a per-row slot array; at the end each row sums its units in K order
// (deterministic).
#include "common.cuh"
#include "kernels.h"
#include "quant_dev.cuh"
#include "tma.cuh"

namespace dcg {

__device__ int g_m1s_error = 0;

cudaError_t m1s_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_m1s_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_m1s_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int M1S_U = 32;                 // units per stage
constexpr int M1S_CONS = 8;               // consumer warps (4 units each per stage)
constexpr int M1S_THREADS = (M1S_CONS + 1) * 32;
constexpr int M1S_SMEM_MAX = 112 * 1024;  // two CTAs per SM: the next launch's CTA fits beside this one
constexpr int M1S_MIN_STAGES = 4;
constexpr int M1S_HDR = 512;              // barriers (up to 31 stages) and flags

template <int TYPE>
struct M1S;
template <>
struct M1S<DCG_TYPE_Q4_K> {
    static constexpr int UB = Q4_K_BYTES, DB = 0;   // payload / separate-scale bytes per unit
};
template <>
struct M1S<DCG_TYPE_Q6_K> {
    static constexpr int UB = Q6_K_PAYLOAD, DB = 2;
};
template <>
struct M1S<DCG_TYPE_Q8_0> {
    static constexpr int UB = 256, DB = 16;
};

// stage bytes: payload, then the unit scales (Q6_K: copied from a 16-B aligned start, +32 B slack)
template <int TYPE>
__host__ __device__ constexpr int m1s_stage_bytes() {
    return M1S_U * M1S<TYPE>::UB + (M1S<TYPE>::DB ? ((M1S_U * M1S<TYPE>::DB + 32 + 15) / 16) * 16 : 0);
}

// shared-memory layout of the activation: quants [k], scales (float) [k/32 or k/256], Q4_K pair sums
__host__ __device__ inline size_t m1s_x_bytes(int type, int64_t k) {
    const size_t q = align256((size_t)k);
    if (type == DCG_TYPE_Q8_0) return q + align256((size_t)(k / 32) * 4);
    return q + align256((size_t)(k / QK_K) * 4) + align256((size_t)(k / 32) * 2);
}

struct M1SPlan {
    int G, rows, stages;   // CTAs, max rows per CTA, ring depth
    size_t smem;
};

template <int TYPE, bool QX>
__global__ void __launch_bounds__(M1S_THREADS, 2)
    gemv_m1s_kernel(const uint8_t* __restrict__ W, const uint8_t* __restrict__ Wd, int nb, int64_t n, int64_t k,
                    const float* __restrict__ x, ActQ a, float* __restrict__ y, int stages) {
    constexpr int UB = M1S<TYPE>::UB, DB = M1S<TYPE>::DB;
    constexpr int SB = m1s_stage_bytes<TYPE>();
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = (uint64_t*)smem;
    uint64_t* empty = full + stages;
    int8_t* xq = (int8_t*)(smem + M1S_HDR);
    float* xd = (float*)((uint8_t*)xq + align256((size_t)k));
    int16_t* xbs = (int16_t*)((uint8_t*)xd + align256((size_t)(k / (TYPE == DCG_TYPE_Q8_0 ? 32 : QK_K)) * 4));
    float* part = (float*)(smem + M1S_HDR + m1s_x_bytes(TYPE, k));
    const int64_t G = gridDim.x, c = blockIdx.x;
    const int64_t r0 = c * n / G, r1 = (c + 1) * n / G;
    const int rows = (int)(r1 - r0);
    uint8_t* ring = (uint8_t*)part + align256((size_t)rows * nb * 4);
    const int64_t gu0 = r0 * nb, nunits = (int64_t)rows * nb;
    const int nst = (int)((nunits + M1S_U - 1) / M1S_U);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], M1S_CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // stage t: units [gu0 + t U, +U) -> ring slot t % stages
    auto issue = [&](int t) {
        const int st = t % stages;
        const int64_t ua = gu0 + (int64_t)t * M1S_U;
        const int cnt = (int)min((int64_t)M1S_U, gu0 + nunits - ua);
        uint8_t* dst = ring + (size_t)st * SB;
        uint32_t bytes = (uint32_t)cnt * UB;
        uint32_t dbytes = 0;
        const uint8_t* dsrc = nullptr;
        if (DB) {
            const uintptr_t s0 = (uintptr_t)(Wd + ua * DB) & ~(uintptr_t)15;
            const uintptr_t s1 = ((uintptr_t)(Wd + (ua + cnt) * DB) + 15) & ~(uintptr_t)15;
            dsrc = (const uint8_t*)s0;
            dbytes = (uint32_t)(s1 - s0);
        }
        mbar_arrive_expect_tx(&full[st], bytes + dbytes);
        bulk_g2s(dst, W + ua * UB, bytes, &full[st]);
        if (DB) bulk_g2s(dst + M1S_U * UB, dsrc, dbytes, &full[st]);
    };
    const int pre = min(stages, nst);
    if (warp == M1S_CONS && lane == 0)
        for (int t = 0; t < pre; t++) issue(t);
    pdl_wait();

    // ---- the activation, quantized (or copied) into shared memory by all warps ----
    if (QX) {
        constexpr int NW = M1S_CONS + 1;
        for (int b = warp; b < (int)(k / QK_K); b += NW) {   // 256 elements per warp pass, 8 per lane
            const float4* p = (const float4*)(x + (size_t)b * QK_K + lane * 8);
            const float4 u0 = __ldg(p), u1 = __ldg(p + 1);
            const float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            if (TYPE == DCG_TYPE_Q8_0) {   // 8 blocks of 32: lanes 4j .. 4j+3 hold block j
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                uint32_t w0 = 0, w1 = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    w0 |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i], id)) << (8 * i);
                    w1 |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i + 4], id)) << (8 * i);
                }
                *(uint2*)(xq + (size_t)b * QK_K + lane * 8) = make_uint2(w0, w1);
                // the scale as the device layout stores it (fp16), widened once for the dots
                if ((lane & 3) == 0) xd[b * 8 + (lane >> 2)] = __half2float(__float2half_rn(d));
            } else {
                const Q8KLane q = warp_q8_K(v, lane);
                *(uint2*)(xq + (size_t)b * QK_K + lane * 8) = make_uint2(q.w0, q.w1);
                if (TYPE == DCG_TYPE_Q4_K && (lane & 3) == 0) xbs[b * 8 + (lane >> 2)] = (int16_t)q.s32;
                if (lane == 0) xd[b] = q.d;
            }
        }
    } else {
        for (int i = threadIdx.x; i < (int)(k / 16); i += M1S_THREADS) ((uint4*)xq)[i] = __ldg((const uint4*)a.qs + i);
        if (TYPE == DCG_TYPE_Q8_0) {
            for (int i = threadIdx.x; i < (int)(k / 32); i += M1S_THREADS) xd[i] = __half2float(((const __half*)a.d)[i]);
        } else {
            for (int i = threadIdx.x; i < (int)(k / QK_K); i += M1S_THREADS) xd[i] = ((const float*)a.d)[i];
            if (TYPE == DCG_TYPE_Q4_K)
                for (int i = threadIdx.x; i < (int)(k / 32); i += M1S_THREADS) xbs[i] = a.bs32[i];
        }
    }
    __syncthreads();

    bool ok = true;
    if (warp == M1S_CONS) {
        // ---- copy warp: keep the ring full, then release the dependents ----
        if (lane == 0) {
            for (int t = pre; t < nst && ok; t++) {
                ok = mbar_wait(&empty[t % stages], (uint32_t)(((t / stages) - 1) & 1), &g_m1s_error);
                if (ok) issue(t);
            }
            pdl_trigger();
        }
    } else {
        const int gq = lane >> 3, j = lane & 7;
        for (int t = 0; t < nst && ok; t++) {
            const int st = t % stages;
            ok = mbar_wait(&full[st], (uint32_t)((t / stages) & 1), &g_m1s_error);
            if (!ok) break;
            const uint8_t* stage = ring + (size_t)st * SB;
            const int ui = warp * 4 + gq;                              // unit within the stage
            const int64_t lu = (int64_t)t * M1S_U + ui;                // unit within the CTA
            const bool live = lu < nunits;                             // group-uniform
            const int sb = (int)(lu % nb);
            const uint8_t* up = stage + (size_t)ui * UB;
            float val = 0.0f;
            if (TYPE == DCG_TYPE_Q4_K) {
                int isum = 0, msum = 0;
                float d = 0.0f, dmin = 0.0f;
                if (live) {
                    const uint4 hdr = *(const uint4*)up;
                    const uint4 q = *(const uint4*)(up + 16 + 16 * j);
                    const int g = j >> 1, half = j & 1;
                    const int8_t* xb = xq + (size_t)sb * QK_K + (2 * g) * 32 + half * 16;
                    const uint4 xl = *(const uint4*)xb, xh = *(const uint4*)(xb + 32);
                    int dl = 0, dh = 0;
                    dl = dp4a((int)(q.x & 0x0F0F0F0Fu), (int)xl.x, dl);
                    dl = dp4a((int)(q.y & 0x0F0F0F0Fu), (int)xl.y, dl);
                    dl = dp4a((int)(q.z & 0x0F0F0F0Fu), (int)xl.z, dl);
                    dl = dp4a((int)(q.w & 0x0F0F0F0Fu), (int)xl.w, dl);
                    dh = dp4a((int)((q.x >> 4) & 0x0F0F0F0Fu), (int)xh.x, dh);
                    dh = dp4a((int)((q.y >> 4) & 0x0F0F0F0Fu), (int)xh.y, dh);
                    dh = dp4a((int)((q.z >> 4) & 0x0F0F0F0Fu), (int)xh.z, dh);
                    dh = dp4a((int)((q.w >> 4) & 0x0F0F0F0Fu), (int)xh.w, dh);
                    int sc0, m0, sc1, m1, scj, mj;
                    q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * g, sc0, m0);
                    q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * g + 1, sc1, m1);
                    q4k_scale_min(hdr.y, hdr.z, hdr.w, j, scj, mj);
                    isum = sc0 * dl + sc1 * dh;
                    msum = mj * (int)xbs[sb * 8 + j];
                    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));
                    d = dd.x;
                    dmin = dd.y;
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    isum += __shfl_xor_sync(0xffffffffu, isum, o);
                    msum += __shfl_xor_sync(0xffffffffu, msum, o);
                }
                val = xd[sb] * (d * (float)isum - dmin * (float)msum);
            } else if (TYPE == DCG_TYPE_Q6_K) {
                int isum = 0;
                float d = 0.0f;
                if (live) {
                    const int h = j >> 2, cc = (j >> 1) & 1, half = j & 1;
                    const uint4 ql = *(const uint4*)(up + h * 64 + cc * 32 + half * 16);
                    const uint4 qh = *(const uint4*)(up + 128 + h * 32 + half * 16);
                    const uint4 scv = *(const uint4*)(up + 192);
                    const int8_t* xb = xq + (size_t)sb * QK_K + h * 128 + cc * 32 + half * 16;
                    const uint4 xl = *(const uint4*)xb, xh = *(const uint4*)(xb + 64);
                    const uint32_t qlw[4] = {ql.x, ql.y, ql.z, ql.w}, qhw[4] = {qh.x, qh.y, qh.z, qh.w};
                    const uint32_t xlw[4] = {xl.x, xl.y, xl.z, xl.w}, xhw[4] = {xh.x, xh.y, xh.z, xh.w};
                    int d0 = 0, d1 = 0;
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        const uint32_t lo = (qlw[w] & 0x0F0F0F0Fu) | (((qhw[w] >> (2 * cc)) & 0x03030303u) << 4);
                        const uint32_t hi = ((qlw[w] >> 4) & 0x0F0F0F0Fu) | (((qhw[w] >> (2 * cc + 4)) & 0x03030303u) << 4);
                        d0 = dp4a((int)__vsub4(lo, 0x20202020u), (int)xlw[w], d0);
                        d1 = dp4a((int)__vsub4(hi, 0x20202020u), (int)xhw[w], d1);
                    }
                    const int s_lo = h * 8 + cc * 2 + half, s_hi = s_lo + 4;
                    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
                    const int sc_lo = (int)(int8_t)((scw[s_lo >> 2] >> (8 * (s_lo & 3))) & 0xFF);
                    const int sc_hi = (int)(int8_t)((scw[s_hi >> 2] >> (8 * (s_hi & 3))) & 0xFF);
                    isum = sc_lo * d0 + sc_hi * d1;
                    // unit scales were copied from a 16-B aligned start below the stage's first unit
                    const int skew = (int)(((uintptr_t)(Wd + (gu0 + (int64_t)t * M1S_U) * DB) & 15) / (DB ? DB : 1));
                    d = __half2float(((const __half*)(stage + M1S_U * UB))[skew + ui]);
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
                val = __fmul_rn(d, xd[sb]) * (float)isum;
            } else {   // Q8_0: lane j takes block j of the unit
                if (live) {
                    const uint4 w0 = *(const uint4*)(up + 32 * j), w1 = *(const uint4*)(up + 32 * j + 16);
                    const int8_t* xb = xq + (size_t)sb * QK_K + 32 * j;
                    const uint4 x0 = *(const uint4*)xb, x1 = *(const uint4*)(xb + 16);
                    int s = 0;
                    s = dp4a((int)w0.x, (int)x0.x, s);
                    s = dp4a((int)w0.y, (int)x0.y, s);
                    s = dp4a((int)w0.z, (int)x0.z, s);
                    s = dp4a((int)w0.w, (int)x0.w, s);
                    s = dp4a((int)w1.x, (int)x1.x, s);
                    s = dp4a((int)w1.y, (int)x1.y, s);
                    s = dp4a((int)w1.z, (int)x1.z, s);
                    s = dp4a((int)w1.w, (int)x1.w, s);
                    const float dw = __half2float(((const __half*)(stage + M1S_U * UB))[ui * 8 + j]);
                    val = __fmul_rn(dw, xd[sb * 8 + j]) * (float)s;
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) val += __shfl_xor_sync(0xffffffffu, val, o);
            }
            if (live && j == 0) part[lu] = val;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
    ok = __syncthreads_and(ok);
    // ---- each row sums its units in K order ----
    if (ok)
        for (int r = threadIdx.x; r < rows; r += M1S_THREADS) {
            float s = 0.0f;
            for (int b = 0; b < nb; b++) s += part[(size_t)r * nb + b];
            y[r0 + r] = s;
        }
}

static bool m1s_plan(int type, int64_t n, int64_t k, M1SPlan* p) {
    if (k % QK_K) return false;
    const int64_t nb = k / QK_K;
    const int sms = num_sms();
    p->G = (int)(n < sms ? n : sms);
    p->rows = (int)((n + p->G - 1) / p->G);
    const size_t sb = type == DCG_TYPE_Q4_K ? m1s_stage_bytes<DCG_TYPE_Q4_K>()
                      : type == DCG_TYPE_Q6_K ? m1s_stage_bytes<DCG_TYPE_Q6_K>() : m1s_stage_bytes<DCG_TYPE_Q8_0>();
    const size_t fixed = M1S_HDR + m1s_x_bytes(type, k) + align256((size_t)p->rows * nb * 4);
    if (fixed + M1S_MIN_STAGES * sb > (size_t)M1S_SMEM_MAX) return false;
    int st = (int)((M1S_SMEM_MAX - fixed) / sb);
    // no deeper than the CTA's stage count, and within the barrier header (2 x 8 B per stage)
    const int64_t nst = ((int64_t)p->rows * nb + M1S_U - 1) / M1S_U;
    if (st > nst) st = (int)nst;
    if (st > 31) st = 31;
    p->stages = st;
    p->smem = fixed + (size_t)st * sb;
    return true;
}

bool m1s_supports(int type, int64_t n, int64_t k) {
    M1SPlan p;
    return (type == DCG_TYPE_Q4_K || type == DCG_TYPE_Q6_K || type == DCG_TYPE_Q8_0) && n > 0 && m1s_plan(type, n, k, &p);
}

template <int TYPE, bool QX>
static cudaError_t launch_m1s_t(const void* packed_w, int64_t n, int64_t k, const float* x, const ActQ& a, float* y,
                                const M1SPlan& p, cudaStream_t st) {
    cudaError_t e = DCG_SMEM_ATTR((gemv_m1s_kernel<TYPE, QX>), M1S_SMEM_MAX);
    if (e != cudaSuccess) return e;
    const PackedW w = packed_view(TYPE, packed_w, n, k);
    return launch_pdl(gemv_m1s_kernel<TYPE, QX>, dim3((unsigned)p.G), dim3(M1S_THREADS), p.smem, st,
                      (const uint8_t*)w.payload, (const uint8_t*)w.d, (int)(k / QK_K), n, k, x, a, y, p.stages);
}

// x: fp32 activation row (quantized in the kernel), or null and act: the SoA quantized activation
cudaError_t launch_m1s(int type, const void* packed_w, int64_t n, int64_t k, const float* x, const void* act,
                       float* y, cudaStream_t st) {
    M1SPlan p;
    if (!m1s_plan(type, n, k, &p)) return cudaErrorNotSupported;
    const int at = type == DCG_TYPE_Q8_0 ? DCG_TYPE_Q8_0 : DCG_TYPE_Q8_K;
    const ActQ a = act ? act_view(at, const_cast<void*>(act), 1, k) : ActQ{};
    switch (type) {
        case DCG_TYPE_Q4_K:
            return x ? launch_m1s_t<DCG_TYPE_Q4_K, true>(packed_w, n, k, x, a, y, p, st)
                     : launch_m1s_t<DCG_TYPE_Q4_K, false>(packed_w, n, k, x, a, y, p, st);
        case DCG_TYPE_Q6_K:
            return x ? launch_m1s_t<DCG_TYPE_Q6_K, true>(packed_w, n, k, x, a, y, p, st)
                     : launch_m1s_t<DCG_TYPE_Q6_K, false>(packed_w, n, k, x, a, y, p, st);
        default:
            return x ? launch_m1s_t<DCG_TYPE_Q8_0, true>(packed_w, n, k, x, a, y, p, st)
                     : launch_m1s_t<DCG_TYPE_Q8_0, false>(packed_w, n, k, x, a, y, p, st);
    }
}

}  // namespace dcg
