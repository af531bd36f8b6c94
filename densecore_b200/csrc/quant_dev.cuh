// quant_dev.cuh -- warp-level activation quantizers writing the SoA activation layout
// (common.cuh), shared by the fused pre-matmul kernels.  Same arithmetic as quant.cu's
// quantize_q8_0_kernel / quantize_q8_K_kernel (ggml's reference Q8_0 / Q8_K quantizers).
#pragma once
#include "common.cuh"

namespace dcg {

// Q8_0 block b of the activation (32 elements, one per lane)
__device__ __forceinline__ void warp_q8_0_store(float v, int lane, const ActQ& a, int64_t b) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    a.qs[b * QK8_0 + lane] = (int8_t)(int)roundf(__fmul_rn(v, id));
    if (lane == 0) ((__half*)a.d)[b] = __float2half_rn(d);
}

// Q8_K of one 256-element block, 8 consecutive elements per lane (lane*8 .. +7): the lane's 8
// quants packed in w0 (elements 0-3) / w1 (4-7), the 16-element sum of lanes 2j, 2j+1 in s16 (valid
// on even lanes), the 32-element sum of lanes 4j..4j+3 in s32 (valid on lanes 4j), and d.
struct Q8KLane {
    uint32_t w0, w1;
    int s16, s32;
    float d;
};

__device__ __forceinline__ Q8KLane warp_q8_K(const float* v, int lane) {
    float amax = -1.0f, vmax = 0.0f;
    int imax = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float x = fabsf(v[i]);
        if (x > amax) { amax = x; vmax = v[i]; imax = lane * 8 + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, o);
        const int oi = __shfl_xor_sync(0xffffffffu, imax, o);
        if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
    }
    int8_t q[8];
    Q8KLane r;
    r.d = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, vmax);
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = (int8_t)min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
        r.d = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
    r.w0 = 0;
    r.w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        s += q[i] + q[i + 4];
        r.w0 |= (uint32_t)(uint8_t)q[i] << (8 * i);
        r.w1 |= (uint32_t)(uint8_t)q[i + 4] << (8 * i);
    }
    r.s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    r.s32 = r.s16 + __shfl_xor_sync(0xffffffffu, r.s16, 2);
    return r;
}

// Q8_K block b of the activation
__device__ __forceinline__ void warp_q8_K_store(const float* v, int lane, const ActQ& a, int64_t b) {
    const Q8KLane r = warp_q8_K(v, lane);
    *(uint2*)(a.qs + b * QK_K + lane * 8) = make_uint2(r.w0, r.w1);
    if ((lane & 1) == 0) a.bsums[b * 16 + (lane >> 1)] = (int16_t)r.s16;
    if ((lane & 3) == 0) a.bs32[b * 8 + (lane >> 2)] = (int16_t)r.s32;
    if (lane == 0) ((float*)a.d)[b] = r.d;
}

}  // namespace dcg
