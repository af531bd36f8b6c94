// quant.cu -- activation quantizers (ggml from_float for Q8_0 / Q8_K), the weight encoders used
// for synthetic checkpoints (Q8_0 / Q4_K / Q6_K), and the upload-time repack of ggml weight rows
// into the device layout described in common.cuh.
//
// Activation quantization must be byte-identical to ggml's reference quantizers:
//   Q8_0: d = amax/127 (IEEE divide), stored fp16 (RNE); id = d ? 1/d : 0; q = roundf(x*id).
//   Q8_K: max = first element of largest |x|; iscale = -127/max; q = min(127, rint(iscale*x));
//         d = 1/iscale (f32); bsums = sums of 16 q.
// Every product below is a single rounded multiply (__fmul_rn) so no FMA contraction can change
// a rounding step.
#include "common.cuh"
#include "kernels.h"

namespace dcg {

// ------------------------------------------------------------------------------------------
// Q8_0: one warp per 32-element block, one element per lane.
// out_soa: false -> ggml blocks (34 B); true -> SoA activation layout of common.cuh.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ x,
                                                            uint8_t* __restrict__ y,
                                                            int64_t n_blocks, int64_t m, int64_t k,
                                                            bool out_soa, int* zero, int nzero) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nzero; i += (int64_t)gridDim.x * blockDim.x)
        zero[i] = 0;
    if (b >= n_blocks) return;
    const float v = x[b * QK8_0 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int8_t q = (int8_t)(int)roundf(__fmul_rn(v, id));
    const __half dh = __float2half_rn(d);
    if (!out_soa) {
        uint8_t* blk = y + b * Q8_0_BYTES;
        blk[2 + lane] = (uint8_t)q;
        if (lane == 0) *(__half*)blk = dh;  // 34*b is even: 2-B aligned
    } else {
        ActQ a = act_view(DCG_TYPE_Q8_0, y, m, k);
        a.qs[b * QK8_0 + lane] = q;
        if (lane == 0) ((__half*)a.d)[b] = dh;
    }
}

// ------------------------------------------------------------------------------------------
// Q8_K: one warp per 256-element block, 8 consecutive elements per lane.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_q8_K_kernel(const float* __restrict__ x,
                                                            uint8_t* __restrict__ y,
                                                            int64_t n_blocks, int64_t m, int64_t k,
                                                            bool out_soa, int* zero, int nzero) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nzero; i += (int64_t)gridDim.x * blockDim.x)
        zero[i] = 0;
    if (b >= n_blocks) return;
    const float4* xp = (const float4*)(x + b * QK_K + lane * 8);
    const float4 v0 = xp[0], v1 = xp[1];
    float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    // largest magnitude; ties go to the lowest index (ggml scans with a strict '>')
    float amax = -1.0f, vmax = 0.0f;
    int imax = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float a = fabsf(v[i]);
        if (a > amax) { amax = a; vmax = v[i]; imax = lane * 8 + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, o);
        const int oi = __shfl_xor_sync(0xffffffffu, imax, o);
        if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
    }
    int8_t q[8];
    float d = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, vmax);
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = (int8_t)min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
        d = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) s += q[i];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        w0 |= (uint32_t)(uint8_t)q[i] << (8 * i);
        w1 |= (uint32_t)(uint8_t)q[i + 4] << (8 * i);
    }
    if (!out_soa) {
        uint8_t* blk = y + b * Q8_K_BYTES;  // 292*b is only 4-B aligned: two 4-B stores
        uint32_t* qw = (uint32_t*)(blk + 4 + lane * 8);
        qw[0] = w0;
        qw[1] = w1;
        if ((lane & 1) == 0) *(int16_t*)(blk + 260 + lane) = (int16_t)s;
        if (lane == 0) *(float*)blk = d;
    } else {
        ActQ a = act_view(DCG_TYPE_Q8_K, y, m, k);
        *(uint2*)(a.qs + b * QK_K + lane * 8) = make_uint2(w0, w1);
        if ((lane & 1) == 0) a.bsums[b * 16 + (lane >> 1)] = (int16_t)s;
        const int s32 = s + __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) a.bs32[b * 8 + (lane >> 2)] = (int16_t)s32;
        if (lane == 0) ((float*)a.d)[b] = d;
    }
}

}  // namespace dcg

namespace dcg {

// ------------------------------------------------------------------------------------------
// Weight encoders (synthetic checkpoints): one warp per 256-element super-block, 8 consecutive
// elements per lane, ggml block bytes out.  The arithmetic is the simple min/max encoding the CPU
// checker uses (any valid Q4_K / Q6_K encoding is acceptable to DenseCore's loader).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void __launch_bounds__(256) encode_q4_K_kernel(const float* __restrict__ x,
                                                          uint8_t* __restrict__ y, int64_t n_blocks) {
    __shared__ uint8_t L[8][QK_K];
    __shared__ uint8_t LS[8][8], LM[8][8];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = (int64_t)blockIdx.x * 8 + wid;
    if (b >= n_blocks) return;  // whole warp exits together
    const float4* xp = (const float4*)(x + b * QK_K + lane * 8);
    const float4 v0 = xp[0], v1 = xp[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float lo = 0.0f, hi = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) { lo = fminf(lo, v[i]); hi = fmaxf(hi, v[i]); }
    // sub-block j = lane/4 spans lanes 4j..4j+3
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    const float scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    const float mn = lo < 0.0f ? -lo : 0.0f;  // +0 (never -0) when the sub-block has no negatives
    float max_scale = scale, max_min = mn;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
        max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    const float inv_s = max_scale > 0.0f ? __fdiv_rn(63.0f, max_scale) : 0.0f;
    const float inv_m = max_min > 0.0f ? __fdiv_rn(63.0f, max_min) : 0.0f;
    const int ls = clampi((int)roundf(__fmul_rn(inv_s, scale)), 0, 63);
    const int lm = clampi((int)roundf(__fmul_rn(inv_m, mn)), 0, 63);
    const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
    const __half dmh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
    const float dl = __fmul_rn(__half2float(dh), (float)ls);
    const float dm = __fmul_rn(__half2float(dmh), (float)lm);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = 0;
        if (dl != 0.0f) q = clampi((int)roundf(__fdiv_rn(__fadd_rn(v[i], dm), dl)), 0, 15);
        L[wid][lane * 8 + i] = (uint8_t)q;
    }
    if ((lane & 3) == 0) { LS[wid][lane >> 2] = (uint8_t)ls; LM[wid][lane >> 2] = (uint8_t)lm; }
    __syncwarp();
    uint8_t* blk = y + b * Q4_K_BYTES;
    // 128 nibble bytes: byte g*32+l = L[64g+l] | L[64g+32+l] << 4; four bytes per lane
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const int byte = lane * 4 + t, g = byte >> 5, l = byte & 31;
        blk[16 + byte] = (uint8_t)(L[wid][64 * g + l] | (L[wid][64 * g + 32 + l] << 4));
    }
    if (lane < 12) {  // packed 6-bit scales/mins (inverse of get_scale_min_k4)
        const uint8_t* s = LS[wid];
        const uint8_t* mm = LM[wid];
        uint8_t o;
        if (lane < 4) o = (uint8_t)(s[lane] | ((s[lane + 4] >> 4) << 6));
        else if (lane < 8) o = (uint8_t)(mm[lane - 4] | ((mm[lane] >> 4) << 6));
        else o = (uint8_t)((s[lane - 4] & 0xF) | ((mm[lane - 4] & 0xF) << 4));
        blk[4 + lane] = o;
    }
    if (lane == 0) { *(__half*)blk = dh; *(__half*)(blk + 2) = dmh; }
}

__global__ void __launch_bounds__(256) encode_q6_K_kernel(const float* __restrict__ x,
                                                          uint8_t* __restrict__ y, int64_t n_blocks) {
    __shared__ uint8_t L[8][QK_K];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = (int64_t)blockIdx.x * 8 + wid;
    if (b >= n_blocks) return;
    const float4* xp = (const float4*)(x + b * QK_K + lane * 8);
    const float4 v0 = xp[0], v1 = xp[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));  // sub-block s = lane/2
    const float scale = __fdiv_rn(amax, 31.0f);
    float max_scale = scale;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
    const float inv = max_scale > 0.0f ? __fdiv_rn(127.0f, max_scale) : 0.0f;
    const int sc = clampi((int)roundf(__fmul_rn(inv, scale)), 0, 127);
    const __half dh = __float2half_rn(__fdiv_rn(max_scale, 127.0f));
    const float dl = __fmul_rn(__half2float(dh), (float)sc);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = 0;
        if (dl != 0.0f) q = clampi((int)roundf(__fdiv_rn(v[i], dl)), -32, 31);
        L[wid][lane * 8 + i] = (uint8_t)(q + 32);
    }
    __syncwarp();
    uint8_t* blk = y + b * Q6_K_BYTES;
    const uint8_t* Lw = L[wid];
    // ql: 128 bytes, 4 per lane
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const int byte = lane * 4 + t, h = byte >> 6, r = byte & 63;
        const uint8_t* Lh = Lw + 128 * h;
        const int e = r & 31, c = r >> 5;  // c=0: elements e and e+64; c=1: e+32 and e+96
        blk[byte] = (uint8_t)((Lh[e + 32 * c] & 0xF) | ((Lh[e + 64 + 32 * c] & 0xF) << 4));
    }
    // qh: 64 bytes, 2 per lane
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int byte = lane * 2 + t, h = byte >> 5, l = byte & 31;
        const uint8_t* Lh = Lw + 128 * h;
        blk[128 + byte] = (uint8_t)((Lh[l] >> 4) | ((Lh[l + 32] >> 4) << 2) |
                                    ((Lh[l + 64] >> 4) << 4) | ((Lh[l + 96] >> 4) << 6));
    }
    if ((lane & 1) == 0) blk[192 + (lane >> 1)] = (uint8_t)(int8_t)sc;
    if (lane == 0) *(__half*)(blk + 208) = dh;
}

// ------------------------------------------------------------------------------------------
// Upload-time repack ggml rows <-> device layout (one thread per block; runs once per weight).
// ------------------------------------------------------------------------------------------
__global__ void pack_kernel(int type, const uint8_t* __restrict__ src, size_t src_stride,
                            uint8_t* __restrict__ dst, int64_t n, int64_t k, bool unpack) {
    const int nb = blocks_per_row(type, k);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nb) return;
    const int64_t row = i / nb;
    const int blk = (int)(i % nb);
    PackedW w = packed_view(type, dst, n, k);
    uint8_t* pay = (uint8_t*)w.payload + row * w.row_bytes;
    __half* dd = (__half*)w.d;
    if (type == DCG_TYPE_Q8_0) {
        uint8_t* g = (uint8_t*)src + row * src_stride + (size_t)blk * Q8_0_BYTES;
        uint8_t* p = pay + (size_t)blk * QK8_0;
        for (int t = 0; t < QK8_0; t++) {
            if (unpack) g[2 + t] = p[t]; else p[t] = g[2 + t];
        }
        if (unpack) memcpy(g, &dd[row * nb + blk], 2); else memcpy(&dd[row * nb + blk], g, 2);
    } else if (type == DCG_TYPE_Q6_K) {
        uint8_t* g = (uint8_t*)src + row * src_stride + (size_t)blk * Q6_K_BYTES;
        uint8_t* p = pay + (size_t)blk * Q6_K_PAYLOAD;
        for (int t = 0; t < Q6_K_PAYLOAD; t++) {
            if (unpack) g[t] = p[t]; else p[t] = g[t];
        }
        if (unpack) memcpy(g + 208, &dd[row * nb + blk], 2); else memcpy(&dd[row * nb + blk], g + 208, 2);
    } else {  // Q4_K: identical bytes
        uint8_t* g = (uint8_t*)src + row * src_stride + (size_t)blk * Q4_K_BYTES;
        uint8_t* p = pay + (size_t)blk * Q4_K_BYTES;
        for (int t = 0; t < Q4_K_BYTES; t++) {
            if (unpack) g[t] = p[t]; else p[t] = g[t];
        }
    }
}

// ------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------
cudaError_t launch_quantize_act(int act_type, const float* x, void* y, int64_t m, int64_t k,
                                bool soa, cudaStream_t st, int* zero, int nzero) {
    const int64_t nblk = m * k / (act_type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K);
    if (nblk == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((nblk + 7) / 8);
    if (act_type == DCG_TYPE_Q8_0)
        return launch_pdl(quantize_q8_0_kernel, dim3(grid), dim3(256), 0, st, x, (uint8_t*)y, nblk, m, k, soa, zero, nzero);
    else
        return launch_pdl(quantize_q8_K_kernel, dim3(grid), dim3(256), 0, st, x, (uint8_t*)y, nblk, m, k, soa, zero, nzero);
    return cudaGetLastError();
}

cudaError_t launch_encode_weights(int type, const float* x, void* y, int64_t n, int64_t k,
                                  cudaStream_t st) {
    if (type == DCG_TYPE_Q8_0) return launch_quantize_act(DCG_TYPE_Q8_0, x, y, n, k, false, st);
    const int64_t nblk = n * k / QK_K;
    if (nblk == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((nblk + 7) / 8);
    if (type == DCG_TYPE_Q4_K) encode_q4_K_kernel<<<grid, 256, 0, st>>>(x, (uint8_t*)y, nblk);
    else encode_q6_K_kernel<<<grid, 256, 0, st>>>(x, (uint8_t*)y, nblk);
    return cudaGetLastError();
}

cudaError_t launch_pack(int type, const void* src, size_t src_stride, void* dst, int64_t n,
                        int64_t k, bool unpack, cudaStream_t st) {
    const int64_t total = n * blocks_per_row(type, k);
    if (total == 0) return cudaSuccess;
    pack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(type, (const uint8_t*)src, src_stride,
                                                                (uint8_t*)dst, n, k, unpack);
    return cudaGetLastError();
}

}  // namespace dcg
