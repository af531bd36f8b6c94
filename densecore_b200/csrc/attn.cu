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
// paged_attn_mma_kernel<NREP>: one CTA (3 consumer warps + 1 producer warp, 2 CTAs per SM) per
// (sequence, kv head, split of the KV blocks); consumer warp w takes blocks w, w+3, ... through
// ring stages that hold its next two blocks while it computes one; the NREP query heads that share the kv head are served
// together so every K/V byte is read once.  Scores and P.V run on the tensor cores with an
// exp2-domain online softmax; the warps merge in shared memory; the split's unnormalised output
// and (max, sum) go to scratch, or straight to `out` when there is a single split.
// attn_combine_kernel merges the splits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdlib.h>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace dcg {

constexpr int HD = 128;        // head_dim (Qwen3 and Llama-3 layouts; the entry points reject others)
constexpr int KVB = 16;        // tokens per KV block
constexpr float LOG2E = 1.4426950408889634f;

// ------------------------------------------------------------------------------------------
// Pipeline: a producer warp streams each KV block's K and V tiles (16 slots x 128 dims of one kv
// head, read in place from the arena through a 3-D tensor map: dim 0 = head_dim, dim 1 = kv head,
// dim 2 = slot of the whole arena) into a shared-memory ring; consumer warp w takes blocks
// w, w+8, ... of the CTA's split.
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

// ------------------------------------------------------------------------------------------
// Per 16-token KV block, per consumer warp:
//   S^T[rep][t] = Q K^T : mma m16n8k16 f16 -> f32, A = Q (NREP query heads as rows, zero-padded to
//                 16; k = 16 dims per step; held in registers), B = K rows via ldmatrix.x4;
//   online softmax on the S^T accumulators (each lane: one head, 4 tokens);
//   O += P V   : the S^T accumulator layout is the A-fragment layout of P (FlashAttention-2's
//                register reuse), B = V via ldmatrix.x4.trans.
// Q and P enter the f16 mma as hi + lo halves (x = hi + lo exactly to ~2^-22), K and V are exact
// fp16, accumulation is fp32: results match an fp32 computation to ~1e-6.
// Tiles arrive by TMA with 128-byte swizzle (two 64-dim halves per tile) so every ldmatrix is
// bank-conflict free: 16-byte chunk c of row r sits at chunk c ^ (r & 7).
// ------------------------------------------------------------------------------------------
constexpr int MA_CONS = 3;                 // consumer warps (+1 producer): 3 x 9 stages, 2 CTAs per SM
constexpr int MA_STAGES = 9;                // 3 per consumer warp: its next blocks load while it computes
constexpr int MA_HALF = KVB * 64 * 2;      // 2 KB: 16 rows x 64 dims
constexpr int MA_STAGE = 4 * MA_HALF;      // K lo | K hi | V lo | V hi = 8 KB

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (x0, x1) -> hi = fp16x2(x), lo = fp16x2(x - hi)
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// smem byte address of 16-byte chunk c (0..15 over 128 dims) of row r in a swizzled half pair
__device__ __forceinline__ uint32_t swz(uint32_t tile, int r, int c) {
    const uint32_t half = tile + (uint32_t)(c >> 3) * MA_HALF;
    return half + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

template <int NREP>
__global__ void __launch_bounds__((MA_CONS + 1) * 32, 2) paged_attn_mma_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
    const float* __restrict__ q, int n_layer, int layer, const int* __restrict__ bt, int mbs,
    const int* __restrict__ ctx, int hq, int hkv, float scale_log2, int bps, int splits,
    float* __restrict__ part_o, float* __restrict__ part_ml, float* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t dsm[];
    uint64_t* full = (uint64_t*)dsm;
    uint64_t* empty = full + MA_STAGES;
    // ring at the first 1024-byte boundary past the barriers: the 128-byte swizzle repeats per 1 KB
    const uint32_t dsm_s = smem_u32(dsm);
    uint8_t* ring = dsm + ((((dsm_s + 256 + 1023) & ~1023u)) - dsm_s);
    __shared__ float wm[MA_CONS][NREP], wl[MA_CONS][NREP];
    __shared__ __align__(16) uint4 qfrag[8][32];  // per k-step, per lane: {hi a0, hi a2, lo a0, lo a2}

    pdl_wait();
    const int seq = blockIdx.x / hkv, kvh = blockIdx.x % hkv, split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int L = ctx[seq];
    const int nblk = (L + KVB - 1) / KVB;
    const int b0 = split * bps, b1 = min(nblk, b0 + bps);
    const int nbh = max(0, b1 - b0);
    const size_t pidx = ((size_t)blockIdx.x * splits + split) * NREP;

    if (threadIdx.x == 0) {
        for (int s = 0; s < MA_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // Q as the mma A operand: row gid = query head kvh*NREP + gid (zero rows beyond NREP);
    // k-step j covers dims 16j .. 16j+15: a0 <- dims 16j+2tig,+1 ; a2 <- dims 16j+8+2tig,+1.
    // Built once by warp 0 into shared memory (registers go to the O accumulators).
    if (warp == 0) {
        const float* qr = q + ((size_t)seq * hq + kvh * NREP + (gid < NREP ? gid : 0)) * HD;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t h[2], l[2];
#pragma unroll
            for (int hlf = 0; hlf < 2; hlf++) {
                const int d = 16 * j + 8 * hlf + 2 * tig;
                float x0 = 0.0f, x1 = 0.0f;
                if (gid < NREP) {
                    x0 = qr[d] * scale_log2;
                    x1 = qr[d + 1] * scale_log2;
                }
                split_h2(x0, x1, h[hlf], l[hlf]);
            }
            qfrag[j][lane] = make_uint4(h[0], h[1], l[0], l[1]);
        }
    }
    __syncthreads();

    bool ok = true;
    if (warp == MA_CONS) {  // producer: K and V tiles of each block, one box each
        if (lane == 0) {
            for (int i = 0; i < nbh && ok; i++) {
                const int st = i % MA_STAGES;
                if (i >= MA_STAGES)
                    ok = mbar_wait(&empty[st], (uint32_t)(((i / MA_STAGES) - 1) & 1), &g_attn_error);
                if (!ok) break;
                const int phys = bt[(size_t)seq * mbs + b0 + i];
                const int slot = (phys * n_layer + layer) * KVB;
                uint8_t* dst = ring + (size_t)st * MA_STAGE;
                mbar_arrive_expect_tx(&full[st], MA_STAGE);
                // one box per tile: 64 dims x 16 tokens x 2 halves -> the two swizzled half-tiles
                tma_load_4d(dst, &kmap, 0, slot, 0, kvh, &full[st]);
                tma_load_4d(dst + 2 * MA_HALF, &vmap, 0, slot, 0, kvh, &full[st]);
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }

    float o[16][2];  // O[head gid][dims 8n + 2tig, +1]
#pragma unroll
    for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = 0.0f;
    float mrow = -INFINITY, lrow = 0.0f;
    const uint32_t ring_s = smem_u32(ring);
    // ldmatrix lane roles: matrix mi = lane >> 3, row within matrix = lane & 7
    const int mi = lane >> 3, mr = lane & 7;

    for (int i = warp; i < nbh && warp < MA_CONS && ok; i += MA_CONS) {
        const int st = i % MA_STAGES;
        ok = mbar_wait(&full[st], (uint32_t)((i / MA_STAGES) & 1), &g_attn_error);
        if (!ok) break;
        const uint32_t kt = ring_s + (uint32_t)st * MA_STAGE;
        const uint32_t vt = kt + 2 * MA_HALF;
        const int ntok = min(KVB, L - (b0 + i) * KVB);
        // ---- S^T = Q K^T: two token tiles (0-7, 8-15) ----
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            // matrices: m0 tok 0-7 dims 16j.., m1 tok 0-7 dims 16j+8.., m2 tok 8-15 dims 16j.., m3 tok 8-15 dims 16j+8..
            const int tok = (mi >> 1) * 8 + mr, ch = 2 * j + (mi & 1);
            uint32_t k0, k1, k2, k3;
            ldsm_x4(swz(kt, tok, ch), k0, k1, k2, k3);
            const uint4 qf = qfrag[j][lane];
            mma_f16(sacc[0], qf.x, 0u, qf.y, 0u, k0, k1);
            mma_f16(sacc[0], qf.z, 0u, qf.w, 0u, k0, k1);
            mma_f16(sacc[1], qf.x, 0u, qf.y, 0u, k2, k3);
            mma_f16(sacc[1], qf.z, 0u, qf.w, 0u, k2, k3);
        }
        // lane: head gid, tokens 2tig, 2tig+1 (tile 0) and 8+2tig, 9+2tig (tile 1)
        float sv[4] = {sacc[0][0], sacc[0][1], sacc[1][0], sacc[1][1]};
        const int tk[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (tk[u] >= ntok) sv[u] = -INFINITY;
            mx = fmaxf(mx, sv[u]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(mrow, mx);  // finite: the block has >= 1 token
        const float corr = exp2f(mrow - mn);
        float p[4], ps = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            p[u] = tk[u] < ntok ? exp2f(sv[u] - mn) : 0.0f;
            ps += p[u];
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        lrow = lrow * corr + ps;
        mrow = mn;
#pragma unroll
        for (int n = 0; n < 16; n++) {
            o[n][0] *= corr;
            o[n][1] *= corr;
        }
        // ---- O += P V: A = P (head rows, k = 16 tokens), B = V^T via ldmatrix.trans ----
        uint32_t ph0, pl0, ph1, pl1;
        split_h2(p[0], p[1], ph0, pl0);   // a0: tokens 2tig, 2tig+1
        split_h2(p[2], p[3], ph1, pl1);   // a2: tokens 8+2tig, 9+2tig
        // slots past the context hold whatever the arena held (possibly NaN / Inf bit patterns):
        // P is 0 there, but 0 * NaN is NaN, so their V halves are zeroed as well (B fragment:
        // low half = the lower token of each pair)
        const uint32_t vm01 = (tk[0] < ntok ? 0x0000FFFFu : 0u) | (tk[1] < ntok ? 0xFFFF0000u : 0u);
        const uint32_t vm23 = (tk[2] < ntok ? 0x0000FFFFu : 0u) | (tk[3] < ntok ? 0xFFFF0000u : 0u);
#pragma unroll
        for (int n2 = 0; n2 < 8; n2++) {
            // matrices: m0 tok 0-7 dims 16n2.., m1 tok 8-15 dims 16n2.., m2 tok 0-7 dims 16n2+8.., m3 tok 8-15 dims 16n2+8..
            const int tok = (mi & 1) * 8 + mr, ch = 2 * n2 + (mi >> 1);
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(swz(vt, tok, ch), v0, v1, v2, v3);
            if (ntok < KVB) {   // the last, partial block of the sequence
                v0 &= vm01;
                v2 &= vm01;
                v1 &= vm23;
                v3 &= vm23;
            }
            float c0[4] = {o[2 * n2][0], o[2 * n2][1], 0.f, 0.f};
            float c1[4] = {o[2 * n2 + 1][0], o[2 * n2 + 1][1], 0.f, 0.f};
            mma_f16(c0, ph0, 0u, ph1, 0u, v0, v1);
            mma_f16(c0, pl0, 0u, pl1, 0u, v0, v1);
            mma_f16(c1, ph0, 0u, ph1, 0u, v2, v3);
            mma_f16(c1, pl0, 0u, pl1, 0u, v2, v3);
            o[2 * n2][0] = c0[0];
            o[2 * n2][1] = c0[1];
            o[2 * n2 + 1][0] = c1[0];
            o[2 * n2 + 1][1] = c1[1];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    pdl_trigger();
    ok = __syncthreads_and(ok);
    if (!ok) return;
    // ---- merge the consumer warps (stage ring reused as [warp][head][dim]) ----
    float* wacc = (float*)ring;
    if (warp < MA_CONS && gid < NREP) {
        if (tig == 0) { wm[warp][gid] = mrow; wl[warp][gid] = lrow; }
#pragma unroll
        for (int n = 0; n < 16; n++)
            *(float2*)&wacc[((size_t)warp * NREP + gid) * HD + 8 * n + 2 * tig] = make_float2(o[n][0], o[n][1]);
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < NREP * HD; idx += blockDim.x) {
        const int r = idx / HD, dd = idx % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < MA_CONS; w++) M = fmaxf(M, wm[w][r]);
        float Ls = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < MA_CONS; w++) {
                const float f = wl[w][r] > 0.0f ? exp2f(wm[w][r] - M) : 0.0f;
                Ls += wl[w][r] * f;
                O += wacc[((size_t)w * NREP + r) * HD + dd] * f;
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

// ------------------------------------------------------------------------------------------
// Multi-token (prefill / chunked prompt) causal attention over the same paged cache: the flash
// path of inference.cpp:1519-1573 with its host-built causal mask (query i of a batch of N new
// tokens sees keys 0 .. n_past + i, :1538-1558; the tiled path's diag_mask_inf, :1590-1711), made
// per sequence.  Sequence s's new tokens are rows seq_starts[s] .. seq_starts[s+1]-1 of q / out;
// token i of n_s sits at position ctx_lens[s] - n_s + i (its K/V already appended) and attends to
// keys 0 .. that position.
//
// One CTA per (tile of PF_ROWS / NREP tokens of one sequence, kv head): its rows are the (token,
// query head) pairs of that group, 16 per consumer warp (the mma's M), so each K/V byte is read
// once per tile for all NREP heads.  A producer warp streams the tiles of KV blocks
// 0 .. (last position) / 16 (TMA, 128-byte swizzle, as the decode kernel); every consumer warp
// consumes every block: S = Q K^T (Q as fp16 hi + lo, K exact fp16), causal mask per row, exp2
// online softmax, O += P V (P as hi + lo) -- fp32-accurate like the decode kernel.
// ------------------------------------------------------------------------------------------
constexpr int PF_CONS = 4;                  // consumer warps
constexpr int PF_ROWS = 16 * PF_CONS;       // (token, head) rows per CTA
constexpr int PF_STAGES = 8;

template <int NREP>
__global__ void __launch_bounds__((PF_CONS + 1) * 32, 2) paged_attn_prefill_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
    const float* __restrict__ q, int n_layer, int layer, const int* __restrict__ bt, int mbs,
    const int* __restrict__ seq_starts, const int* __restrict__ ctx, int hq, int hkv, float scale_log2,
    float* __restrict__ out) {
    constexpr int TQ = PF_ROWS / NREP;      // tokens per CTA
    extern __shared__ __align__(128) uint8_t dsm[];
    uint64_t* full = (uint64_t*)dsm;
    uint64_t* empty = full + PF_STAGES;
    const uint32_t dsm_s = smem_u32(dsm);
    uint8_t* ring = dsm + ((((dsm_s + 256 + 1023) & ~1023u)) - dsm_s);

    pdl_wait();
    const int seq = blockIdx.y, kvh = blockIdx.z;
    const int s0 = seq_starts[seq], ns = seq_starts[seq + 1] - s0;
    const int t0 = blockIdx.x * TQ;                 // first token of the tile within the sequence
    if (t0 >= ns) return;                           // CTA-uniform
    const int L = ctx[seq];
    const int pos0 = L - ns;                        // position of the sequence's first new token
    const int tq = min(TQ, ns - t0);
    const int last_pos = pos0 + t0 + tq - 1;
    const int nbh = last_pos / KVB + 1;             // KV blocks this tile reads
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;

    if (threadIdx.x == 0) {
        for (int st = 0; st < PF_STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], PF_CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    bool ok = true;
    if (warp == PF_CONS) {   // producer
        if (lane == 0) {
            for (int i = 0; i < nbh && ok; i++) {
                const int st = i % PF_STAGES;
                if (i >= PF_STAGES)
                    ok = mbar_wait(&empty[st], (uint32_t)(((i / PF_STAGES) - 1) & 1), &g_attn_error);
                if (!ok) break;
                const int phys = bt[(size_t)seq * mbs + i];
                const int slot = (phys * n_layer + layer) * KVB;
                uint8_t* dst = ring + (size_t)st * MA_STAGE;
                mbar_arrive_expect_tx(&full[st], MA_STAGE);
                tma_load_4d(dst, &kmap, 0, slot, 0, kvh, &full[st]);
                tma_load_4d(dst + 2 * MA_HALF, &vmap, 0, slot, 0, kvh, &full[st]);
            }
        }
    } else {
        // rows of this warp: r = 16 warp + gid (A rows gid) and r + 8 (A rows gid + 8);
        // row r <-> token t0 + r / NREP, query head kvh NREP + r % NREP
        int rpos[2];
        const float* qrow[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int r = 16 * warp + gid + 8 * h;
            const int t = t0 + r / NREP;
            rpos[h] = t < ns ? pos0 + t : -1;      // -1: a padding row, every key masked
            qrow[h] = q + ((size_t)(s0 + (t < ns ? t : 0)) * hq + kvh * NREP + r % NREP) * HD;
        }
        // Q fragments for the 8 k-steps (dims 16j ..): a0/a2 rows gid, a1/a3 rows gid + 8
        uint32_t qh[8][4], ql[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int a = 0; a < 4; a++) {
                const int h = a & 1, d = 16 * j + 8 * (a >> 1) + 2 * tig;
                float x0 = 0.0f, x1 = 0.0f;
                if (rpos[h] >= 0) {
                    const float2 v = *(const float2*)(qrow[h] + d);
                    x0 = v.x * scale_log2;
                    x1 = v.y * scale_log2;
                }
                split_h2(x0, x1, qh[j][a], ql[j][a]);
            }
        float o[16][4];   // [dim tile n][c0, c1 (row gid), c2, c3 (row gid + 8)]
#pragma unroll
        for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
        float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
        const uint32_t ring_s = smem_u32(ring);
        const int mi = lane >> 3, mr = lane & 7;
        for (int i = 0; i < nbh && ok; i++) {
            const int st = i % PF_STAGES;
            ok = mbar_wait(&full[st], (uint32_t)((i / PF_STAGES) & 1), &g_attn_error);
            if (!ok) break;
            const uint32_t kt = ring_s + (uint32_t)st * MA_STAGE, vt = kt + 2 * MA_HALF;
            const int kb = i * KVB;   // first key of the block
            // ---- S = Q K^T for keys kb .. kb + 15 (tiles of 8) ----
            float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int tok = (mi >> 1) * 8 + mr, ch = 2 * j + (mi & 1);
                uint32_t k0, k1, k2, k3;
                ldsm_x4(swz(kt, tok, ch), k0, k1, k2, k3);
                mma_f16(sacc[0], qh[j][0], qh[j][1], qh[j][2], qh[j][3], k0, k1);
                mma_f16(sacc[0], ql[j][0], ql[j][1], ql[j][2], ql[j][3], k0, k1);
                mma_f16(sacc[1], qh[j][0], qh[j][1], qh[j][2], qh[j][3], k2, k3);
                mma_f16(sacc[1], ql[j][0], ql[j][1], ql[j][2], ql[j][3], k2, k3);
            }
            // lane: rows gid (c0, c1) and gid + 8 (c2, c3); keys kb + 8 tile + 2 tig + {0, 1}
            float p[2][4];   // [tile][c]
            float corr[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float mx = -INFINITY;
#pragma unroll
                for (int tl = 0; tl < 2; tl++)
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int key = kb + 8 * tl + 2 * tig + e;
                        float& v = sacc[tl][2 * h + e];
                        if (key > rpos[h]) v = -INFINITY;
                        mx = fmaxf(mx, v);
                    }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mn = fmaxf(mrow[h], mx);
                // a row that has seen no key yet (mn = -inf) keeps O = 0, l = 0
                corr[h] = mn == -INFINITY ? 1.0f : exp2f(mrow[h] - mn);
                float ps = 0.0f;
#pragma unroll
                for (int tl = 0; tl < 2; tl++)
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const float v = sacc[tl][2 * h + e];
                        const float pv = v == -INFINITY ? 0.0f : exp2f(v - mn);
                        p[tl][2 * h + e] = pv;
                        ps += pv;
                    }
                ps += __shfl_xor_sync(0xffffffffu, ps, 1);
                ps += __shfl_xor_sync(0xffffffffu, ps, 2);
                lrow[h] = lrow[h] * corr[h] + ps;
                mrow[h] = mn;
            }
#pragma unroll
            for (int n = 0; n < 16; n++) {
                o[n][0] *= corr[0];
                o[n][1] *= corr[0];
                o[n][2] *= corr[1];
                o[n][3] *= corr[1];
            }
            // ---- O += P V: A = P (a0: row gid keys 2tig.., a1: row gid+8, a2/a3: keys 8+2tig..) ----
            uint32_t ph[4], pl[4];
            split_h2(p[0][0], p[0][1], ph[0], pl[0]);
            split_h2(p[0][2], p[0][3], ph[1], pl[1]);
            split_h2(p[1][0], p[1][1], ph[2], pl[2]);
            split_h2(p[1][2], p[1][3], ph[3], pl[3]);
            // slots past the context (the last block) may hold NaN / Inf bit patterns: zero their V
            const int nval = min(KVB, L - kb);
            const uint32_t vm01 = (2 * tig < nval ? 0x0000FFFFu : 0u) | (2 * tig + 1 < nval ? 0xFFFF0000u : 0u);
            const uint32_t vm23 = (8 + 2 * tig < nval ? 0x0000FFFFu : 0u) | (9 + 2 * tig < nval ? 0xFFFF0000u : 0u);
#pragma unroll
            for (int n2 = 0; n2 < 8; n2++) {
                const int tok = (mi & 1) * 8 + mr, ch = 2 * n2 + (mi >> 1);
                uint32_t v0, v1, v2, v3;
                ldsm_x4_t(swz(vt, tok, ch), v0, v1, v2, v3);
                if (nval < KVB) {
                    v0 &= vm01;
                    v2 &= vm01;
                    v1 &= vm23;
                    v3 &= vm23;
                }
                mma_f16(o[2 * n2], ph[0], ph[1], ph[2], ph[3], v0, v1);
                mma_f16(o[2 * n2], pl[0], pl[1], pl[2], pl[3], v0, v1);
                mma_f16(o[2 * n2 + 1], ph[0], ph[1], ph[2], ph[3], v2, v3);
                mma_f16(o[2 * n2 + 1], pl[0], pl[1], pl[2], pl[3], v2, v3);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        // ---- normalise and store: lane owns rows gid / gid + 8, dims 8n + 2tig, +1 ----
        if (ok) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (rpos[h] < 0) continue;
                const int r = 16 * warp + gid + 8 * h;
                const float inv = lrow[h] > 0.0f ? 1.0f / lrow[h] : 0.0f;
                float* orow = out + ((size_t)(s0 + t0 + r / NREP) * hq + kvh * NREP + r % NREP) * HD;
#pragma unroll
                for (int n = 0; n < 16; n++)
                    *(float2*)(orow + 8 * n + 2 * tig) = make_float2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
            }
        }
    }
    pdl_trigger();
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

// split planner: enough CTAs for `target` (default 4 x 148) and at most `maxb` (default 64) KV blocks per CTA
// (DCG_ATTN_TARGET / DCG_ATTN_MAXB override both, for tuning)
void attn_plan(int n_seqs, int hkv, int max_ctx, int* splits, int* bps) {
    static const int target = getenv("DCG_ATTN_TARGET") ? atoi(getenv("DCG_ATTN_TARGET")) : 4 * 148;
    static const int maxb = getenv("DCG_ATTN_MAXB") ? atoi(getenv("DCG_ATTN_MAXB")) : 64;
    const int max_nblk = max(1, (max_ctx + KVB - 1) / KVB);
    int sp = max(1, (target + n_seqs * hkv - 1) / (n_seqs * hkv));
    sp = max(sp, (max_nblk + maxb - 1) / maxb);
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

// arena as a 3-D fp16 tensor: [slots][hkv][HD]; box = 16 slots x 1 head x 64 dims, 128-byte swizzle
static cudaError_t make_kv_map(CUtensorMap* map, const void* arena, int hkv, int64_t n_slots) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    // (64 dims of a half, slot, half, kv head): one box of 64 x 16 tokens x 2 halves fills the
    // [half][token][64] smem tile, each 128-B row swizzled
    const cuuint64_t dims[4] = {64u, (cuuint64_t)n_slots, 2u, (cuuint64_t)hkv};
    const cuuint64_t strides[3] = {(cuuint64_t)hkv * HD * 2, 128u, (cuuint64_t)HD * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)KVB, 2, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(arena), dims, strides, box,
                    es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int NR>
static cudaError_t launch_attn_mma(dim3 grid, cudaStream_t st, const CUtensorMap& km, const CUtensorMap& vm,
                                   const float* q, int n_layer, int layer, const int* bt, int mbs,
                                   const int* ctx, int hq, int hkv, float sl2, int bps, int splits,
                                   float* po, float* pml, float* direct) {
    const size_t dyn = 2048 + (size_t)MA_STAGES * MA_STAGE;
    cudaError_t e = DCG_SMEM_ATTR((paged_attn_mma_kernel<NR>), dyn);
    if (e != cudaSuccess) return e;
    return launch_pdl(paged_attn_mma_kernel<NR>, grid, dim3((MA_CONS + 1) * 32), dyn, st, km, vm, q, n_layer,
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
        case 1: e = launch_attn_mma<1>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 2: e = launch_attn_mma<2>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 4: e = launch_attn_mma<4>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
        case 8: e = launch_attn_mma<8>(grid, st, km, vm, q, n_layer, layer, bt, mbs, ctx, hq, hkv, sl2, bps, splits, po, pml, direct); break;
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


template <int NR>
static cudaError_t launch_prefill_t(dim3 grid, cudaStream_t st, const CUtensorMap& km, const CUtensorMap& vm,
                                    const float* q, int n_layer, int layer, const int* bt, int mbs,
                                    const int* seq_starts, const int* ctx, int hq, int hkv, float sl2, float* out) {
    const size_t dyn = 2048 + (size_t)PF_STAGES * MA_STAGE;
    cudaError_t e = DCG_SMEM_ATTR((paged_attn_prefill_kernel<NR>), dyn);
    if (e != cudaSuccess) return e;
    return launch_pdl(paged_attn_prefill_kernel<NR>, grid, dim3((PF_CONS + 1) * 32), dyn, st, km, vm, q, n_layer,
                      layer, bt, mbs, seq_starts, ctx, hq, hkv, sl2, out);
}

cudaError_t launch_paged_attn_prefill(const float* q, const void* karena, const void* varena, int n_layer,
                                      int layer, const int* bt, int mbs, const int* seq_starts, const int* ctx,
                                      int n_seqs, int max_seq_tokens, int hq, int hkv, float scale, float* out,
                                      cudaStream_t st, int64_t n_arena_blocks) {
    const int nrep = hq / hkv;
    const int tq = PF_ROWS / nrep;
    const dim3 grid((unsigned)((max_seq_tokens + tq - 1) / tq), (unsigned)n_seqs, (unsigned)hkv);
    const int64_t n_slots = n_arena_blocks * n_layer * KVB;
    CUtensorMap km, vm;
    cudaError_t e = make_kv_map(&km, karena, hkv, n_slots);
    if (e == cudaSuccess) e = make_kv_map(&vm, varena, hkv, n_slots);
    if (e != cudaSuccess) return e;
    const float sl2 = scale * LOG2E;
    switch (nrep) {
        case 1: return launch_prefill_t<1>(grid, st, km, vm, q, n_layer, layer, bt, mbs, seq_starts, ctx, hq, hkv, sl2, out);
        case 2: return launch_prefill_t<2>(grid, st, km, vm, q, n_layer, layer, bt, mbs, seq_starts, ctx, hq, hkv, sl2, out);
        case 4: return launch_prefill_t<4>(grid, st, km, vm, q, n_layer, layer, bt, mbs, seq_starts, ctx, hq, hkv, sl2, out);
        case 8: return launch_prefill_t<8>(grid, st, km, vm, q, n_layer, layer, bt, mbs, seq_starts, ctx, hq, hkv, sl2, out);
    }
    return cudaErrorInvalidValue;
}

}  // namespace dcg
