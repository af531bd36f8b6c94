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
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

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

// ------------------------------------------------------------------------------------------
// TMA-pipelined variant (the one launched): a producer warp streams each KV block's K and V tiles
// (16 slots x 128 dims of one kv head, 4 KB each, read in place from the arena through a 3-D
// tensor map: dim 0 = head_dim, dim 1 = kv head, dim 2 = slot of the whole arena) into an
// 8-stage shared-memory ring; consumer warp w takes blocks w, w+8, ... of the CTA's split.
// Scores: lane pair (t, half) covers token t; at step i it reads 16-byte chunk (i + t) % 8 of its
// half so the 16 token rows (256 B apart) hit distinct banks.  P.V: lane owns dims 4*lane..+3.
// ------------------------------------------------------------------------------------------
__device__ int g_attn_error = 0;

cudaError_t attn_device_error(int* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_attn_error, sizeof(int));
    if (e == cudaSuccess && clear && *out) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_attn_error, &zero, sizeof(int));
    }
    return e;
}

constexpr int AT_STAGES = 8;
constexpr int AT_CONS = 8;  // consumer warps (+1 producer warp)
constexpr int AT_TILE = KVB * HD * 2;  // 4 KB: one kv head of one block

__device__ __forceinline__ void tma_load_3d(void* dst, const void* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

template <int NREP>
__global__ void __launch_bounds__((AT_CONS + 1) * 32) paged_attn_tma_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
    const float* __restrict__ q, int n_layer, int layer, const int* __restrict__ bt, int mbs,
    const int* __restrict__ ctx, int hq, int hkv, float scale_log2, int bps, int splits,
    float* __restrict__ part_o, float* __restrict__ part_ml, float* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t dsm[];
    uint64_t* full = (uint64_t*)dsm;
    uint64_t* empty = full + AT_STAGES;
    uint8_t* ring = dsm + 256;  // [AT_STAGES][K tile | V tile]
    __shared__ __align__(16) float qs[NREP][HD];
    __shared__ __align__(16) float pb[AT_CONS][KVB][NREP];
    __shared__ float wm[AT_CONS][NREP], wl[AT_CONS][NREP];
    float (*wacc)[NREP][HD] = reinterpret_cast<float (*)[NREP][HD]>(ring);  // after the ring drains

    pdl_wait();
    const int seq = blockIdx.x / hkv, kvh = blockIdx.x % hkv, split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L = ctx[seq];
    const int nblk = (L + KVB - 1) / KVB;
    const int b0 = split * bps, b1 = min(nblk, b0 + bps);
    const int nbh = max(0, b1 - b0);
    const size_t pidx = ((size_t)blockIdx.x * splits + split) * NREP;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AT_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        const int r = i / HD, dd = i % HD;
        qs[r][dd] = q[((size_t)seq * hq + kvh * NREP + r) * HD + dd] * scale_log2;
    }
    __syncthreads();

    bool ok = true;
    if (warp == AT_CONS) {  // producer
        if (lane == 0) {
            for (int i = 0; i < nbh && ok; i++) {
                const int st = i % AT_STAGES;
                if (i >= AT_STAGES)
                    ok = mbar_wait(&empty[st], (uint32_t)(((i / AT_STAGES) - 1) & 1), &g_attn_error);
                if (!ok) break;
                const int phys = bt[(size_t)seq * mbs + b0 + i];
                const int slot = (phys * n_layer + layer) * KVB;
                uint8_t* dst = ring + (size_t)st * 2 * AT_TILE;
                mbar_arrive_expect_tx(&full[st], 2 * AT_TILE);
                tma_load_3d(dst, &kmap, 0, kvh, slot, &full[st]);
                tma_load_3d(dst + AT_TILE, &vmap, 0, kvh, slot, &full[st]);
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }

    float m[NREP], l[NREP], acc[NREP][4];
#pragma unroll
    for (int r = 0; r < NREP; r++) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[r][j] = 0.0f;
    }
    const int t = lane >> 1, half = lane & 1;
    for (int i = warp; i < nbh && warp < AT_CONS && ok; i += AT_CONS) {
        const int st = i % AT_STAGES;
        ok = mbar_wait(&full[st], (uint32_t)((i / AT_STAGES) & 1), &g_attn_error);
        if (!ok) break;
        const uint8_t* kt = ring + (size_t)st * 2 * AT_TILE;
        const uint8_t* vt = kt + AT_TILE;
        const int ntok = min(KVB, L - (b0 + i) * KVB);
        float s[NREP];
#pragma unroll
        for (int r = 0; r < NREP; r++) s[r] = 0.0f;
        if (t < ntok) {
#pragma unroll
            for (int ii = 0; ii < 8; ii++) {
                const int ch = (ii + t) & 7;  // 16-dim chunk
                const uint4 kv = *(const uint4*)(kt + t * 256 + ch * 32 + half * 16);
                float kf[8];
                h8_to_f(kv, kf);
#pragma unroll
                for (int r = 0; r < NREP; r++) {
                    const float4 q0 = *(const float4*)&qs[r][ch * 16 + half * 8];
                    const float4 q1 = *(const float4*)&qs[r][ch * 16 + half * 8 + 4];
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
#pragma unroll
        for (int r = 0; r < NREP; r++) {
            float mx = s[r];
#pragma unroll
            for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(m[r], mx);
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
        for (int tt = 0; tt < ntok; tt++) {
            const uint2 vv = *(const uint2*)(vt + tt * 256 + lane * 8);
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
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    pdl_trigger();
    ok = __syncthreads_and(ok);
    if (!ok) return;
    if (warp < AT_CONS) {
#pragma unroll
        for (int r = 0; r < NREP; r++) {
            if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
            *(float4*)&wacc[warp][r][lane * 4] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        const int r = i / HD, dd = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < AT_CONS; w++) M = fmaxf(M, wm[w][r]);
        float Ls = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < AT_CONS; w++) {
                const float f = wl[w][r] > 0.0f ? exp2f(wm[w][r] - M) : 0.0f;
                Ls += wl[w][r] * f;
                O += wacc[w][r][dd] * f;
            }
        }
        if (out) {
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();  // qmm.cu

// arena as a 3-D fp16 tensor: [slots][hkv][HD]; box = 16 slots x 1 head x HD
static cudaError_t make_kv_map(CUtensorMap* map, const void* arena, int hkv, int64_t n_slots) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)hkv, (cuuint64_t)n_slots};
    const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)hkv * HD * 2};
    const cuuint32_t box[3] = {(cuuint32_t)HD, 1, (cuuint32_t)KVB};
    const cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(arena), dims, strides, box,
                    es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int NR>
static cudaError_t launch_attn_tma(dim3 grid, cudaStream_t st, const CUtensorMap& km, const CUtensorMap& vm,
                                   const float* q, int n_layer, int layer, const int* bt, int mbs,
                                   const int* ctx, int hq, int hkv, float sl2, int bps, int splits,
                                   float* po, float* pml, float* direct) {
    static bool attr = false;
    const size_t dyn = 256 + (size_t)AT_STAGES * 2 * AT_TILE;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(paged_attn_tma_kernel<NR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)dyn);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    return launch_pdl(paged_attn_tma_kernel<NR>, grid, dim3((AT_CONS + 1) * 32), dyn, st, km, vm, q, n_layer,
                      layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct);
}

cudaError_t launch_paged_attn(const float* q, const void* karena, const void* varena, int n_layer,
                              int layer, const int* bt, int mbs, const int* ctx, int n_seqs, int hq,
                              int hkv, int max_ctx, float scale, float* out, void* scratch,
                              cudaStream_t st, int64_t n_arena_blocks) {
    int splits, bps;
    attn_plan(n_seqs, hkv, max_ctx, &splits, &bps);
    const int nrep = hq / hkv;
    const size_t parts = (size_t)n_seqs * hq * splits;
    float* po = (float*)scratch;
    float* pml = splits > 1 ? (float*)((uint8_t*)scratch + align256(parts * HD * 4)) : nullptr;
    dim3 grid(n_seqs * hkv, splits);
    const float sl2 = scale * LOG2E;
    float* direct = splits == 1 ? out : nullptr;
    const int64_t n_slots = n_arena_blocks * n_layer * KVB;
    CUtensorMap km, vm;
    cudaError_t e = make_kv_map(&km, karena, hkv, n_slots);
    if (e == cudaSuccess) e = make_kv_map(&vm, varena, hkv, n_slots);
    if (e != cudaSuccess) return e;
    switch (nrep) {
        case 1: e = launch_attn_tma<1>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 2: e = launch_attn_tma<2>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 4: e = launch_attn_tma<4>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 8: e = launch_attn_tma<8>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        default: return cudaErrorInvalidValue;
    }
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
