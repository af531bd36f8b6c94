// fused.cu -- the element-wise work around the matmuls of a decode step, fused into the kernels
// that produce the matmul inputs (the reference fuses the same steps on CPU: AddRMSNorm and the
// QKV path of simd_ops.h, and BuildTransformerGraph's rms_norm / QK-norm / RoPE / SwiGLU nodes,
// core/src/inference.cpp:1124-1313, :1790-1797):
//
//   add_rmsnorm_quant_kernel   x += delta (optional); act = quantize(x * rsqrt(mean(x^2)+eps) * w)
//   swiglu_quant_kernel        act = quantize(silu(gate) * up)
//   qk_rope_append_kernel      q, k: per-head RMSNorm (Qwen3 QK-norm) and NeoX RoPE at the
//                              sequence's position; q -> q_out, k and v -> fp16 paged KV slots
//
// The quantized activation goes straight to the SoA layout the matmuls read.
#include <math.h>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"
#include "quant_dev.cuh"

namespace dcg {

constexpr int FUSE_THREADS = 256;

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
    __syncthreads();
    return t;
}

// ggml's rms_norm scale: the fp32 squares summed in double, mean rounded to fp32, then
// 1.0f / sqrtf(mean + eps) with IEEE-rounded fp32 operations (the sum's order differs from the
// CPU's sequential one only far below fp32 resolution)
__device__ __forceinline__ float rms_scale(double sumsq, int64_t k, float eps) {
    const float mean = (float)(sumsq / (double)k);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// one CTA per activation row, the row staged in shared memory: every thread issues all of its
// 16-byte loads of x (and delta) before it uses one, so a row costs one memory latency instead of one
// per element; the norm weight (constant) is staged before the wait on the producing kernel.
// x, delta and weight 16-byte aligned, k <= RMS_MAX_K.
constexpr int RMS_MAX_K = 8192;
__global__ void __launch_bounds__(FUSE_THREADS) add_rmsnorm_quant_v4_kernel(
    float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w, float eps,
    int64_t k, int act_type, ActQ a) {
    __shared__ double red[FUSE_THREADS / 32];
    extern __shared__ float4 rms_sm[];   // [k/4] x, then [k/4] weight
    const int k4 = (int)(k / 4);
    float4* xs = rms_sm;
    float4* ws = rms_sm + k4;
    for (int i = threadIdx.x; i < k4; i += FUSE_THREADS) ws[i] = __ldg((const float4*)w + i);
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    float4* xr = (float4*)(x + row * k);
    const float4* dr = delta ? (const float4*)(delta + row * k) : nullptr;
    double ss = 0.0;
    constexpr int U = RMS_MAX_K / 4 / FUSE_THREADS;   // 16-byte vectors per thread at most
    float4 v[U], d[U];
#pragma unroll
    for (int j = 0; j < U; j++) {
        const int i = threadIdx.x + j * FUSE_THREADS;
        if (i < k4) {
            v[j] = xr[i];
            if (dr) d[j] = dr[i];
        }
    }
#pragma unroll
    for (int j = 0; j < U; j++) {
        const int i = threadIdx.x + j * FUSE_THREADS;
        if (i < k4) {
            float4 t = v[j];
            if (dr) {
                t.x = __fadd_rn(t.x, d[j].x);
                t.y = __fadd_rn(t.y, d[j].y);
                t.z = __fadd_rn(t.z, d[j].z);
                t.w = __fadd_rn(t.w, d[j].w);
                xr[i] = t;
            }
            xs[i] = t;
            ss += (double)__fmul_rn(t.x, t.x);
            ss += (double)__fmul_rn(t.y, t.y);
            ss += (double)__fmul_rn(t.z, t.z);
            ss += (double)__fmul_rn(t.w, t.w);
        }
    }
    const float rs = rms_scale(block_sum(ss, red), k, eps);  // block_sum's barrier publishes xs
    const float* xf = (const float*)xs;
    const float* wf = (const float*)ws;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (act_type == DCG_TYPE_Q8_0) {
        for (int64_t b = warp; b < k / QK8_0; b += nw) {
            const int64_t i = b * QK8_0 + lane;
            warp_q8_0_store(__fmul_rn(__fmul_rn(xf[i], rs), wf[i]), lane, a, row * (k / QK8_0) + b);
        }
    } else {
        for (int64_t b = warp; b < k / QK_K; b += nw) {
            float vv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int64_t i = b * QK_K + lane * 8 + j;
                vv[j] = __fmul_rn(__fmul_rn(xf[i], rs), wf[i]);
            }
            warp_q8_K_store(vv, lane, a, row * (k / QK_K) + b);
        }
    }
}

// general form (any alignment, any k): one CTA per activation row
__global__ void __launch_bounds__(FUSE_THREADS) add_rmsnorm_quant_kernel(
    float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w, float eps,
    int64_t k, int act_type, ActQ a) {
    __shared__ double red[FUSE_THREADS / 32];
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    float* xr = x + row * k;
    double ss = 0.0;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        float v = xr[i];
        if (delta) {
            v = __fadd_rn(v, delta[row * k + i]);
            xr[i] = v;
        }
        ss += (double)__fmul_rn(v, v);
    }
    const float rs = rms_scale(block_sum(ss, red), k, eps);  // block_sum also orders the x writes above
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (act_type == DCG_TYPE_Q8_0) {
        for (int64_t b = warp; b < k / QK8_0; b += nw) {
            const int64_t i = b * QK8_0 + lane;
            warp_q8_0_store(__fmul_rn(__fmul_rn(xr[i], rs), w[i]), lane, a, row * (k / QK8_0) + b);
        }
    } else {
        for (int64_t b = warp; b < k / QK_K; b += nw) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int64_t i = b * QK_K + lane * 8 + j;
                v[j] = __fmul_rn(__fmul_rn(xr[i], rs), w[i]);
            }
            warp_q8_K_store(v, lane, a, row * (k / QK_K) + b);
        }
    }
}

// act = quantize(silu(g) * u); g, u rows of `ffn` with row stride ld; one warp per block
__global__ void __launch_bounds__(FUSE_THREADS) swiglu_quant_kernel(
    const float* __restrict__ g, const float* __restrict__ u, int64_t ld, int64_t m, int64_t ffn,
    int act_type, ActQ a) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t per_row = act_type == DCG_TYPE_Q8_0 ? ffn / QK8_0 : ffn / QK_K;
    if (gw >= m * per_row) return;
    const int64_t row = gw / per_row, b = gw % per_row;
    const float* gr = g + row * ld;
    const float* ur = u + row * ld;
    if (act_type == DCG_TYPE_Q8_0) {
        const int64_t i = b * QK8_0 + lane;
        const float gv = gr[i];
        warp_q8_0_store(__fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), ur[i]), lane, a, row * per_row + b);
    } else {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int64_t i = b * QK_K + lane * 8 + j;
            const float gv = gr[i];
            v[j] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), ur[i]);
        }
        warp_q8_K_store(v, lane, a, row * per_row + b);
    }
}

// one warp per (row, head) over hq + hkv heads; lane owns dims {2l, 2l+1, 64+2l, 65+2l}.  Row s is
// one token: sequence s itself (decode), or sequence seq_ids[s] (several tokens of one sequence)
__global__ void __launch_bounds__(FUSE_THREADS) qk_rope_append_kernel(
    const float* __restrict__ q, int64_t ldq, const float* __restrict__ k, int64_t ldk,
    const float* __restrict__ v, int64_t ldv, int n_seqs, int hq, int hkv, const float* __restrict__ qw,
    const float* __restrict__ kw, float eps, float theta_scale, const int* __restrict__ pos,
    float* __restrict__ q_out, __half* __restrict__ karena, __half* __restrict__ varena, int n_layer,
    int layer, const int* __restrict__ bt, int mbs, const int* __restrict__ seq_ids) {
    constexpr int D = 128;
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int gw = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int heads = hq + hkv;
    if (gw >= n_seqs * heads) return;
    const int s = gw / heads, h = gw % heads;
    const bool is_q = h < hq;
    const int hh = is_q ? h : h - hq;
    const float* src = is_q ? q + (int64_t)s * ldq + hh * D : k + (int64_t)s * ldk + hh * D;
    const float* nw = is_q ? qw : kw;
    const int d0 = 2 * lane, d1 = 64 + 2 * lane;
    float x0 = src[d0], x1 = src[d0 + 1], y0 = src[d1], y1 = src[d1 + 1];
    if (nw) {  // QK-norm (Qwen3), the rms_norm of the head as above; skipped without weights (Llama)
        double ss = (double)__fmul_rn(x0, x0) + (double)__fmul_rn(x1, x1) + (double)__fmul_rn(y0, y0) +
                    (double)__fmul_rn(y1, y1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rms_scale(ss, D, eps);
        x0 = __fmul_rn(__fmul_rn(x0, rs), nw[d0]);
        x1 = __fmul_rn(__fmul_rn(x1, rs), nw[d0 + 1]);
        y0 = __fmul_rn(__fmul_rn(y0, rs), nw[d1]);
        y1 = __fmul_rn(__fmul_rn(y1, rs), nw[d1 + 1]);
    }
    // NeoX rotate-half: (x_i, x_{i+64}) at angle theta_i, with ggml's fp32 recurrence
    // theta_0 = p, theta_{i+1} = theta_i * theta_scale (theta_scale = powf(base, -2/D), from the host)
    float t0 = (float)pos[s];
    for (int i = 0; i < d0; i++) t0 = __fmul_rn(t0, theta_scale);
    const float t1 = __fmul_rn(t0, theta_scale);
    const float c0 = cosf(t0), s0 = sinf(t0), c1 = cosf(t1), s1 = sinf(t1);
    // ggml's rotation: x0 cos - x1 sin, x0 sin + x1 cos, each product rounded
    const float r0 = __fsub_rn(__fmul_rn(x0, c0), __fmul_rn(y0, s0)), r1 = __fsub_rn(__fmul_rn(x1, c1), __fmul_rn(y1, s1));
    const float r2 = __fadd_rn(__fmul_rn(x0, s0), __fmul_rn(y0, c0)), r3 = __fadd_rn(__fmul_rn(x1, s1), __fmul_rn(y1, c1));
    if (is_q) {
        float* dst = q_out + ((int64_t)s * hq + hh) * D;
        *(float2*)(dst + d0) = make_float2(r0, r1);
        *(float2*)(dst + d1) = make_float2(r2, r3);
        return;
    }
    const int ps = pos[s];
    const int phys = bt[(int64_t)(seq_ids ? seq_ids[s] : s) * mbs + ps / 16];   // row s's sequence
    const size_t slot = (((size_t)phys * n_layer + layer) * 16 + (ps % 16)) * (size_t)hkv * D + (size_t)hh * D;
    *(__half2*)(karena + slot + d0) = __floats2half2_rn(r0, r1);
    *(__half2*)(karena + slot + d1) = __floats2half2_rn(r2, r3);
    const float* vr = v + (int64_t)s * ldv + hh * D;
    *(__half2*)(varena + slot + d0) = __floats2half2_rn(vr[d0], vr[d0 + 1]);
    *(__half2*)(varena + slot + d1) = __floats2half2_rn(vr[d1], vr[d1 + 1]);
}

cudaError_t launch_add_rmsnorm_quant(float* x, const float* delta, const float* w, float eps, int64_t m,
                                     int64_t k, int act_type, void* act, cudaStream_t st) {
    const ActQ a = act_view(act_type, act, m, k);
    const bool a16 = ((uintptr_t)x | (uintptr_t)delta | (uintptr_t)w) % 16 == 0;
    if (a16 && k <= RMS_MAX_K && k % 4 == 0) {
        const size_t smem = (size_t)k * 8;
        cudaError_t e = DCG_SMEM_ATTR(add_rmsnorm_quant_v4_kernel, RMS_MAX_K * 8);
        if (e != cudaSuccess) return e;
        return launch_pdl(add_rmsnorm_quant_v4_kernel, dim3((unsigned)m), dim3(FUSE_THREADS), smem, st, x, delta, w,
                          eps, k, act_type, a);
    }
    return launch_pdl(add_rmsnorm_quant_kernel, dim3((unsigned)m), dim3(FUSE_THREADS), 0, st, x, delta, w, eps,
                      k, act_type, a);
}

cudaError_t launch_swiglu_quant(const float* g, const float* u, int64_t ld, int64_t m, int64_t ffn,
                                int act_type, void* act, cudaStream_t st) {
    const ActQ a = act_view(act_type, act, m, ffn);
    const int64_t warps = m * (act_type == DCG_TYPE_Q8_0 ? ffn / QK8_0 : ffn / QK_K);
    const unsigned grid = (unsigned)((warps * 32 + FUSE_THREADS - 1) / FUSE_THREADS);
    return launch_pdl(swiglu_quant_kernel, dim3(grid), dim3(FUSE_THREADS), 0, st, g, u, ld, m, ffn, act_type, a);
}

cudaError_t launch_qk_rope_append(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                  int64_t ldv, int n_seqs, int hq, int hkv, const float* qw, const float* kw,
                                  float eps, float theta, const int* pos, float* q_out, void* karena,
                                  void* varena, int n_layer, int layer, const int* bt, int mbs,
                                  cudaStream_t st, const int* seq_ids) {
    const int64_t warps = (int64_t)n_seqs * (hq + hkv);
    const unsigned grid = (unsigned)((warps * 32 + FUSE_THREADS - 1) / FUSE_THREADS);
    // ggml's per-dimension angle ratio powf(freq_base, -2 / n_dims), computed once on the host (libm)
    const float theta_scale = powf(theta, -2.0f / 128.0f);
    return launch_pdl(qk_rope_append_kernel, dim3(grid), dim3(FUSE_THREADS), 0, st, q, ldq, k, ldk, v, ldv,
                      n_seqs, hq, hkv, qw, kw, eps, theta_scale, pos, q_out, (__half*)karena, (__half*)varena,
                      n_layer, layer, bt, mbs, seq_ids);
}

}  // namespace dcg
