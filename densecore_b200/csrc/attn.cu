// attn.cu -- decode GQA attention over DenseCore's paged fp16 KV cache, and the KV slot append.
//
// Reference: the attention selector and flash path of BuildTransformerGraph
// (core/src/inference.cpp:1506-1573), fed by cb_kv_manage's gather of PagedKVCache slots
// (inference.cpp:556-643; layout kv_cache.cpp:353-370).  Here each sequence attends to its own
// positions 0..ctx_len-1 through its own block table (the reference's batched path reads only
// seq_id[0]'s history; the per-sequence semantics are the oracle's), reading the fp16 arena in
// place -- no gather copy.
//
// Arena element (block, layer, slot, head, dim) = ((block*n_layer + layer)*16 + slot)*hkv*D +
// head*D + dim, fp16.
//
// paged_attn_split_kernel<NREP>: one CTA (4 warps) per (sequence, kv head, split of the KV
// blocks); the NREP query heads that share the kv head are served together so every K/V byte is
// read once.  Per 16-token block a warp computes the scores with lane pairs per token (64 dims
// each), updates an exp2-domain online softmax, and accumulates P.V with 4 dims per lane.  The 4
// warps merge in shared memory; the split's unnormalised output and (max, sum) go to scratch, or
// straight to `out` when there is a single split.  attn_combine_kernel merges the splits.
#include <math.h>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"

namespace dcg {

constexpr int HD = 128;        // head_dim (all BASELINE configs)
constexpr int KVB = 16;        // tokens per KV block
constexpr int ATT_WARPS = 4;
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void h8_to_f(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

template <int NREP>
__global__ void __launch_bounds__(ATT_WARPS * 32) paged_attn_split_kernel(
    const float* __restrict__ q, const __half* __restrict__ karena, const __half* __restrict__ varena,
    int n_layer, int layer, const int* __restrict__ bt, int mbs, const int* __restrict__ ctx, int hq,
    int hkv, float scale_log2, int bps, int splits, float* __restrict__ part_o,
    float* __restrict__ part_ml, float* __restrict__ out) {
    __shared__ __align__(16) float qs[NREP][HD];
    __shared__ __align__(16) float pb[ATT_WARPS][KVB][NREP];
    __shared__ float wm[ATT_WARPS][NREP], wl[ATT_WARPS][NREP];
    __shared__ __align__(16) float wacc[ATT_WARPS][NREP][HD];

    pdl_wait();
    const int seq = blockIdx.x / hkv, kvh = blockIdx.x % hkv, split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L = ctx[seq];
    const int nblk = (L + KVB - 1) / KVB;
    const int b0 = split * bps, b1 = min(nblk, b0 + bps);
    const size_t pidx = ((size_t)blockIdx.x * splits + split) * NREP;

    // query heads kvh*NREP .. +NREP-1, pre-scaled into the log2 domain
    for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        const int r = i / HD, dd = i % HD;
        qs[r][dd] = q[((size_t)seq * hq + kvh * NREP + r) * HD + dd] * scale_log2;
    }
    __syncthreads();

    float m[NREP], l[NREP], acc[NREP][4];
#pragma unroll
    for (int r = 0; r < NREP; r++) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[r][j] = 0.0f;
    }
    const size_t tok_stride = (size_t)hkv * HD;  // halfs between consecutive slots
    const int t = lane >> 1, half = lane & 1;

    for (int b = b0 + warp; b < b1; b += ATT_WARPS) {
        const int phys = bt[(size_t)seq * mbs + b];
        const size_t base = ((size_t)phys * n_layer + layer) * KVB * tok_stride + (size_t)kvh * HD;
        const int ntok = min(KVB, L - b * KVB);
        // ---- scores: lane pair (t, half) covers token t, dims {i*16 + half*8 .. +8} ----
        float s[NREP];
#pragma unroll
        for (int r = 0; r < NREP; r++) s[r] = 0.0f;
        if (t < ntok) {
            const __half* krow = karena + base + (size_t)t * tok_stride;
            uint4 kv[8];
#pragma unroll
            for (int i = 0; i < 8; i++) kv[i] = __ldg((const uint4*)(krow + i * 16 + half * 8));
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float kf[8];
                h8_to_f(kv[i], kf);
#pragma unroll
                for (int r = 0; r < NREP; r++) {
                    const float4 q0 = *(const float4*)&qs[r][i * 16 + half * 8];
                    const float4 q1 = *(const float4*)&qs[r][i * 16 + half * 8 + 4];
                    s[r] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] +
                            q1.x * kf[4] + q1.y * kf[5] + q1.z * kf[6] + q1.w * kf[7];
                }
            }
        }
#pragma unroll
        for (int r = 0; r < NREP; r++) {
            s[r] += __shfl_xor_sync(0xffffffffu, s[r], 1);
            if (t >= ntok) s[r] = -INFINITY;
        }
        // ---- online softmax over this block ----
#pragma unroll
        for (int r = 0; r < NREP; r++) {
            float mx = s[r];
#pragma unroll
            for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(m[r], mx);  // finite: the block has >= 1 token
            const float corr = exp2f(m[r] - mn);
            const float p = (t < ntok) ? exp2f(s[r] - mn) : 0.0f;
            float ps = half == 0 ? p : 0.0f;
#pragma unroll
            for (int o = 2; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[r] = l[r] * corr + ps;
            m[r] = mn;
#pragma unroll
            for (int j = 0; j < 4; j++) acc[r][j] *= corr;
            if (half == 0) pb[warp][t][r] = p;
        }
        __syncwarp();
        // ---- P.V: lane owns dims lane*4 .. +3 ----
        const __half* vb = varena + base + lane * 4;
        for (int tt = 0; tt < ntok; tt++) {
            const uint2 vv = __ldg((const uint2*)(vb + (size_t)tt * tok_stride));
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vv.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vv.y));
#pragma unroll
            for (int r = 0; r < NREP; r++) {
                const float p = pb[warp][tt][r];
                acc[r][0] += p * v01.x;
                acc[r][1] += p * v01.y;
                acc[r][2] += p * v23.x;
                acc[r][3] += p * v23.y;
            }
        }
        __syncwarp();
    }
    pdl_trigger();
    // ---- merge the warps ----
#pragma unroll
    for (int r = 0; r < NREP; r++) {
        if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
        *(float4*)&wacc[warp][r][lane * 4] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        const int r = i / HD, dd = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, wm[w][r]);
        float Ls = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < ATT_WARPS; w++) {
                const float f = wl[w][r] > 0.0f ? exp2f(wm[w][r] - M) : 0.0f;
                Ls += wl[w][r] * f;
                O += wacc[w][r][dd] * f;
            }
        }
        if (out) {  // single split: normalise in place
            out[((size_t)seq * hq + kvh * NREP + r) * HD + dd] = Ls > 0.0f ? O / Ls : 0.0f;
        } else {
            part_o[(pidx + r) * HD + dd] = O;
            if (dd == 0) {
                part_ml[(pidx + r) * 2] = M;
                part_ml[(pidx + r) * 2 + 1] = Ls;
            }
        }
    }
}

// out[seq][h][:] = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M); one CTA of 128 threads per (seq, h)
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                    float* __restrict__ out, int hq, int hkv, int nrep, int splits) {
    pdl_wait();
    pdl_trigger();
    const int seq = blockIdx.x / hq, h = blockIdx.x % hq;
    const int kvh = h / nrep, r = h % nrep;
    const int dd = threadIdx.x;
    const size_t base = ((size_t)(seq * hkv + kvh) * splits) * nrep + r;
    float M = -INFINITY;
    for (int s = 0; s < splits; s++) {
        const size_t p = base + (size_t)s * nrep;
        if (part_ml[p * 2 + 1] > 0.0f) M = fmaxf(M, part_ml[p * 2]);
    }
    float Ls = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
        for (int s = 0; s < splits; s++) {
            const size_t p = base + (size_t)s * nrep;
            const float l = part_ml[p * 2 + 1];
            if (l > 0.0f) {
                const float f = exp2f(part_ml[p * 2] - M);
                Ls += l * f;
                O += part_o[p * HD + dd] * f;
            }
        }
    }
    out[((size_t)seq * hq + h) * HD + dd] = Ls > 0.0f ? O / Ls : 0.0f;
}

// KV append: token i of sequence seq_ids[i] at position positions[i]; f32 -> fp16 (RNE), the
// PagedKVCache::WriteKSlot / WriteVSlot conversion (kv_cache.cpp:566-598).
__global__ void kv_append_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                 __half* __restrict__ karena, __half* __restrict__ varena, int n_layer,
                                 int layer, const int* __restrict__ bt, int mbs,
                                 const int* __restrict__ seq_ids, const int* __restrict__ pos,
                                 int n_tok, int hkv, int hd) {
    pdl_wait();
    pdl_trigger();
    const int per = hkv * hd;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_tok * per) return;
    const int tok = (int)(i / per), e = (int)(i % per);
    const int s = seq_ids[tok], p = pos[tok];
    const int phys = bt[(size_t)s * mbs + p / KVB];
    const size_t dst = (((size_t)phys * n_layer + layer) * KVB + (p % KVB)) * per + e;
    karena[dst] = __float2half_rn(k[i]);
    varena[dst] = __float2half_rn(v[i]);
}

void attn_plan(int n_seqs, int hkv, int max_ctx, int* splits, int* bps) {
    const int max_nblk = max(1, (max_ctx + KVB - 1) / KVB);
    int sp = max(1, (4 * 148 + n_seqs * hkv - 1) / (n_seqs * hkv));
    sp = max(sp, (max_nblk + 31) / 32);  // at most 32 blocks (512 tokens) per CTA
    sp = min(sp, max_nblk);
    *splits = sp;
    *bps = (max_nblk + sp - 1) / sp;
}

size_t attn_scratch_bytes(int n_seqs, int hq, int hkv, int max_ctx) {
    int splits, bps;
    attn_plan(n_seqs, hkv, max_ctx, &splits, &bps);
    if (splits == 1) return 0;
    const size_t parts = (size_t)n_seqs * hq * splits;  // hkv * nrep == hq
    return align256(parts * HD * 4) + align256(parts * 2 * 4);
}

cudaError_t launch_paged_attn(const float* q, const void* karena, const void* varena, int n_layer,
                              int layer, const int* bt, int mbs, const int* ctx, int n_seqs, int hq,
                              int hkv, int max_ctx, float scale, float* out, void* scratch,
                              cudaStream_t st) {
    int splits, bps;
    attn_plan(n_seqs, hkv, max_ctx, &splits, &bps);
    const int nrep = hq / hkv;
    const size_t parts = (size_t)n_seqs * hq * splits;
    float* po = (float*)scratch;
    float* pml = splits > 1 ? (float*)((uint8_t*)scratch + align256(parts * HD * 4)) : nullptr;
    dim3 grid(n_seqs * hkv, splits);
    const float sl2 = scale * LOG2E;
    const __half* K = (const __half*)karena;
    const __half* V = (const __half*)varena;
    float* direct = splits == 1 ? out : nullptr;
    cudaError_t e = cudaSuccess;
#define DCG_ATT(NR)                                                                                  \
    e = launch_pdl(paged_attn_split_kernel<NR>, grid, dim3(ATT_WARPS * 32), 0, st, q, K, V, n_layer, \
                   layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct)
    switch (nrep) {
        case 1: DCG_ATT(1); break;
        case 2: DCG_ATT(2); break;
        case 4: DCG_ATT(4); break;
        case 8: DCG_ATT(8); break;
        default: return cudaErrorInvalidValue;
    }
#undef DCG_ATT
    if (e != cudaSuccess || splits == 1) return e;
    return launch_pdl(attn_combine_kernel, dim3(n_seqs * hq), dim3(HD), 0, st, (const float*)po,
                      (const float*)pml, out, hq, hkv, nrep, splits);
}

cudaError_t launch_kv_append(const float* k, const float* v, void* karena, void* varena, int n_layer,
                             int layer, const int* bt, int mbs, const int* seq_ids, const int* pos,
                             int n_tok, int hkv, int hd, cudaStream_t st) {
    const int64_t total = (int64_t)n_tok * hkv * hd;
    if (total == 0) return cudaSuccess;
    return launch_pdl(kv_append_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, k, v,
                      (__half*)karena, (__half*)varena, n_layer, layer, bt, mbs, seq_ids, pos, n_tok, hkv, hd);
}

}  // namespace dcg
