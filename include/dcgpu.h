/*
 * dcgpu.h -- C ABI of libdcgpu.so, the B200 (sm_100a) implementation of DenseCore's quantized
 * weight matmul and paged decode attention.
 *
 * Plain C: pointers, sizes, ints.  Every entry point returns DCG_OK (0) or a negative DCG_E* code
 * (DenseCore's C API convention, core/include/densecore.h:244); no C++ exception crosses it.
 * dcg_last_error() gives the message of the calling thread's last failure.
 *
 * Two families:
 *  (1) device entry points (suffix-free): all buffers are device pointers, work is enqueued on the
 *      given cudaStream_t (passed as void*, NULL = legacy default stream) and nothing synchronizes.
 *      These are what an engine with device-resident weights and KV cache calls per step.
 *  (2) host entry points (dcg_ctx_*): the drop-in for the CPU call sites.  Weights are uploaded
 *      once (dcg_ctx_weight_register) and stay resident; each call copies its host activations in
 *      and its host results out and returns when they are ready.
 *
 * Type ids are ggml's enum ggml_type values.
 */
#ifndef DCGPU_H
#define DCGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DCG_OK 0
#define DCG_EINVAL (-1)       /* bad argument: null pointer, unsupported type, bad shape */
#define DCG_ECUDA (-2)        /* CUDA runtime error (message in dcg_last_error) */
#define DCG_ENOMEM (-3)       /* device allocation failed */
#define DCG_ESCRATCH (-4)     /* caller-provided scratch too small */
#define DCG_ENOTFOUND (-5)    /* weight handle / host pointer not registered */

#define DCG_TYPE_F32 0
#define DCG_TYPE_F16 1
#define DCG_TYPE_Q8_0 8
#define DCG_TYPE_Q4_K 12
#define DCG_TYPE_Q6_K 14
#define DCG_TYPE_Q8_K 15

#define DCG_KV_BLOCK_SIZE 16 /* tokens per KV block (core/include/kv_cache.h:17) */

int dcg_version(void);

/* Programmatic dependent launch (on by default): each kernel of this library may start its
 * prologue while the previous kernel in the stream drains, and reads that kernel's outputs only
 * after it has completed.  enable = 0 makes every later launch plainly stream-ordered, for streams
 * (or captured graphs) where this library's kernels sit next to kernels of another library, such
 * as NCCL collectives of a tensor-parallel step.  Process-wide; returns the previous setting.
 * Launches already captured into a graph keep the setting they were captured with.  No counterpart
 * in the reference (its operators run on CPU threads). */
int dcg_set_programmatic_launch(int enable);
const char* dcg_strerror(int code);
const char* dcg_last_error(void);

/* Status of the kernels' bounded waits: *code = 0, or DCG_DEVERR_TIMEOUT when a kernel gave up
 * waiting for a bulk copy and returned early (its outputs are then invalid).  clear != 0 resets
 * it.  The flag is read with a blocking copy, so call it between steps. */
#define DCG_DEVERR_TIMEOUT 1
int dcg_device_error(int* code, int clear);

/* ---------------------------------------------------------------------------------------------
 * Sizes
 * ------------------------------------------------------------------------------------------- */
/* ggml row bytes of k elements of `type` (ggml_row_size; inference.cpp:983, kv_cache.cpp:341). */
size_t dcg_row_size(int type, int64_t k);
/* bytes of an n x k weight in the device layout (see dcg_weight_pack). */
size_t dcg_packed_weight_size(int type, int64_t n, int64_t k);
/* scratch bytes dcg_mul_mat needs for an n x k weight and m activation rows. */
size_t dcg_mul_mat_scratch_size(int type, int64_t n, int64_t k, int64_t m);
/* scratch bytes dcg_mul_mat_q needs (0 when the kernel takes none). */
size_t dcg_mul_mat_q_scratch_size(int type, int64_t n, int64_t k, int64_t m);

/* ---------------------------------------------------------------------------------------------
 * Activation quantization -- ggml type-trait from_float for the vec_dot_type of the weight
 * (replaces from_float(x, q, N) at core/src/inference.cpp:889-892).  Output: ggml block bytes,
 * m rows of dcg_row_size(type, k).  Byte-identical to ggml's reference quantizers.
 * ------------------------------------------------------------------------------------------- */
int dcg_quantize_row_q8_0(const float* x, void* y, int64_t m, int64_t k, void* stream);
int dcg_quantize_row_q8_K(const float* x, void* y, int64_t m, int64_t k, void* stream);

/* Weight encoder f32 -> ggml Q8_0 / Q4_K / Q6_K rows (offline-quantizer role of
 * core/src/quantize.cpp; used to build seeded synthetic checkpoints on the device). */
int dcg_quantize_weights(int type, const float* x, void* rows, int64_t n, int64_t k, void* stream);

/* Upload-time repack of n ggml rows (row_stride bytes apart; ggml tensor nb[1]) into the device
 * layout the matmul streams: Q4_K unchanged; Q8_0 and Q6_K with the fp16 block scales moved to a
 * separate array so every payload row is 16-byte aligned.  dcg_weight_unpack inverts it. */
int dcg_weight_pack(int type, const void* rows, size_t row_stride, int64_t n, int64_t k,
                    void* packed, void* stream);
int dcg_weight_unpack(int type, const void* packed, int64_t n, int64_t k, void* rows,
                      size_t row_stride, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Quantized matmul -- the mul_mat op on a quantized weight (smart_mul_mat / ggml_mul_mat_gemv /
 * cb_gemv_custom, core/src/inference.cpp:1043-1064, :958-1033, :840-948; ggml_mul_mat at
 * :1063, :1794-1797, :1817).
 *   y[m][n] = sum_k W[n][k] * x[m][k], x quantized on the fly to Q8_0 (Q8_0 weights) or Q8_K
 *   (Q4_K / Q6_K weights), integer block dots, fp32 scaling and accumulation.
 * w: device layout (dcg_weight_pack) of an n x k weight; k % 256 == 0 (k % 32 for Q8_0).
 * scratch: >= dcg_mul_mat_scratch_size(type, n, k, m) bytes of device memory, 256-B aligned.
 * ------------------------------------------------------------------------------------------- */
int dcg_mul_mat(int type, const void* w, int64_t n, int64_t k, const float* x, int64_t m, float* y,
                void* scratch, size_t scratch_bytes, void* stream);

/* The two stages of dcg_mul_mat, for callers that quantize one activation once and multiply it by
 * several weights (the Q/K/V projections share one input, inference.cpp:1128-1130).
 * dcg_quantize_act writes the activation in the device layout (int8 payload rows, then block
 * scales, then Q8_K block sums) that dcg_mul_mat_q reads; act_type is the vec_dot_type
 * (DCG_TYPE_Q8_0 or DCG_TYPE_Q8_K); act must hold dcg_act_size(act_type, m, k) bytes, 256-B
 * aligned.  dcg_mul_mat_q is ComputeDotProductBatch's job (core/src/simd_ops.cpp:140-197) for all
 * rows and all m activation rows at once.  Its scratch (dcg_mul_mat_q_scratch_size bytes) must be
 * zero-filled before its first use; every call leaves it ready for the next (dcg_mul_mat needs no
 * such preparation). */
size_t dcg_act_size(int act_type, int64_t m, int64_t k);
int dcg_quantize_act(int act_type, const float* x, void* act, int64_t m, int64_t k, void* stream);
int dcg_mul_mat_q(int type, const void* w, int64_t n, int64_t k, const void* act, int64_t m,
                  float* y, void* scratch, size_t scratch_bytes, void* stream);

/* dcg_mul_mat without scratch: for callers that cannot allocate device memory where they run the
 * matmul (a ggml custom-op callback inside the compute thread pool, a plugin host that forbids
 * allocation after start-up, a step that must not synchronize on cudaMalloc).  No counterpart in
 * the reference.  The quantized activation lives in a fixed 1 MiB device array owned by the
 * library (held on every GPU that loads it until exit); calls needing more than that
 * (dcg_act_size of the vec_dot_type > 1 MiB: m*k above about 986,000 for Q8_0 weights or 871,000
 * for Q4_K / Q6_K weights, e.g. m <= 68 / 60 at k = 14336) fail with DCG_EINVAL.  w must be
 * 256-byte, x 16-byte and y 4-byte aligned (DCG_EINVAL otherwise).  All calls share the array:
 * calls that overlap on the GPU race, so keep them on one stream.  The first call on each device
 * resolves the array's address; make it before any stream capture.  Allocates nothing. */
int dcg_mul_mat_noalloc(int type, const void* w, int64_t n, int64_t k, const float* x, int64_t m,
                        float* y, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Paged decode attention -- the attention op the runtime selector dispatches for a decode step
 * (inference.cpp:1506-1573: scale = 1/sqrt(head_dim), softmax(q.K^T * scale).V, GQA with
 * kv_head = h / (hq/hkv)), reading PagedKVCache's fp16 arena in place instead of cb_kv_manage's
 * gather (inference.cpp:556-643).  One query token per sequence; sequence s attends to its own
 * positions 0..ctx_lens[s]-1 (the current token already appended).
 *   q            [n_seqs][hq][head_dim] f32
 *   k/v_arena    fp16, element (block, layer, slot, head, dim) at
 *                ((block*n_layer + layer)*16 + slot)*hkv*head_dim + head*head_dim + dim
 *                (kv_cache.cpp:353-370, the declared WriteKSlot(block_id, layer, ...) order)
 *   n_arena_blocks  physical blocks in each arena (PagedKVCache max_blocks, kv_cache.h:164); every
 *                block id in block_tables must be < n_arena_blocks
 *   block_tables [n_seqs][max_blocks_per_seq] int32 physical block ids
 *   ctx_lens     [n_seqs] int32, each <= max_ctx and <= 16*max_blocks_per_seq
 *   out          [n_seqs][hq][head_dim] f32
 * head_dim must be 128 and hq/hkv one of 1, 2, 4, 8.  scratch: dcg_paged_attn_scratch_size bytes
 * (0 is valid when that size is 0), 256-B aligned.  All pointers are device pointers. */
size_t dcg_paged_attn_scratch_size(int n_seqs, int hq, int hkv, int head_dim, int max_ctx);
int dcg_paged_attn_decode(const float* q, const void* k_arena, const void* v_arena,
                          int64_t n_arena_blocks, int n_layer, int layer,
                          const int32_t* block_tables, int max_blocks_per_seq,
                          const int32_t* ctx_lens, int n_seqs, int hq, int hkv, int head_dim,
                          int max_ctx, float scale, float* out, void* scratch, size_t scratch_bytes,
                          void* stream);

/* Multi-token causal attention over the same cache: the prefill / prompt-chunk branch of the
 * attention selector (the flash path with its host-built causal mask, inference.cpp:1519-1573 and
 * :1538-1558 -- query i of N new tokens sees keys 0 .. n_past + i -- and the tiled path's
 * diag_mask_inf, :1590-1711), made per sequence.  Sequence s's new tokens are rows
 * seq_starts[s] .. seq_starts[s+1]-1 of q / out ([n_tok][hq][head_dim] f32); token i of its n_s
 * new tokens sits at position ctx_lens[s] - n_s + i, its K/V already appended, and attends to keys
 * 0 .. that position.  max_seq_tokens >= every n_s.  seq_starts and ctx_lens are device int32
 * arrays; the rest as dcg_paged_attn_decode.  Needs no scratch. */
int dcg_paged_attn_prefill(const float* q, const void* k_arena, const void* v_arena, int64_t n_arena_blocks,
                           int n_layer, int layer, const int32_t* block_tables, int max_blocks_per_seq,
                           const int32_t* seq_starts, const int32_t* ctx_lens, int n_seqs, int max_seq_tokens,
                           int hq, int hkv, int head_dim, int max_ctx, float scale, float* out, void* stream);

/* KV append -- PagedKVCache::WriteKSlot / WriteVSlot (kv_cache.cpp:566-598) for n_tok tokens at
 * once: token i (k, v: [n_tok][hkv][head_dim] f32) goes to slot positions[i] of sequence
 * seq_ids[i] through its block table, converted to fp16 (round to nearest even). */
int dcg_kv_append(const float* k, const float* v, void* k_arena, void* v_arena, int n_layer,
                  int layer, const int32_t* block_tables, int max_blocks_per_seq,
                  const int32_t* seq_ids, const int32_t* positions, int n_tok, int hkv,
                  int head_dim, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Fused element-wise producers of the matmul inputs (the reference's AddRMSNorm / fused QKV on CPU,
 * core/include/simd_ops.h:2437-2763, and the rms_norm / QK-norm / RoPE / SwiGLU graph nodes of
 * BuildTransformerGraph, core/src/inference.cpp:1124-1313, :1790-1797).  All device pointers.
 *
 * dcg_add_rmsnorm_quantize: x[m][k] += delta (if delta != NULL; x updated in place), then
 *   act = quantize(x * rsqrt(mean(x^2) + eps) * weight) in the dcg_quantize_act layout of act_type.
 * dcg_swiglu_quantize: act = quantize(silu(gate) * up); gate/up rows of ffn values, row stride ld
 *   (they may be the two halves of one stacked matmul output).
 * dcg_qk_norm_rope_kv_append: for each sequence s, query heads and key heads of q/k (row strides
 *   ldq/ldk, head_dim 128) get a per-head RMSNorm (weights q_norm_w / k_norm_w, Qwen3 QK-norm; both
 *   NULL skips it, as for Llama) and
 *   NeoX (rotate-half) RoPE at positions[s] with base rope_theta; q goes to q_out[n_seqs][hq][128],
 *   k and v (row stride ldv) are written as fp16 to slot positions[s] of sequence s (the
 *   dcg_kv_append layout). */
/* dcg_qk_norm_rope_kv_append for n_tok token rows of any sequences: row i is a token of sequence
 * seq_ids[i] at positions[i] (several rows may share a sequence: a prompt chunk). */
int dcg_qk_norm_rope_kv_append_tokens(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                      int64_t ldv, int n_tok, int hq, int hkv, int head_dim,
                                      const float* q_norm_w, const float* k_norm_w, float eps, float rope_theta,
                                      const int32_t* seq_ids, const int32_t* positions, float* q_out,
                                      void* k_arena, void* v_arena, int n_layer, int layer,
                                      const int32_t* block_tables, int max_blocks_per_seq, void* stream);
int dcg_add_rmsnorm_quantize(float* x, const float* delta, const float* weight, float eps, int64_t m,
                             int64_t k, int act_type, void* act, void* stream);
int dcg_swiglu_quantize(const float* gate, const float* up, int64_t ld, int64_t m, int64_t ffn,
                        int act_type, void* act, void* stream);
int dcg_qk_norm_rope_kv_append(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                               int64_t ldv, int n_seqs, int hq, int hkv, int head_dim,
                               const float* q_norm_w, const float* k_norm_w, float eps, float rope_theta,
                               const int32_t* positions, float* q_out, void* k_arena, void* v_arena,
                               int n_layer, int layer, const int32_t* block_tables,
                               int max_blocks_per_seq, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Host boundary (drop-in for the CPU call sites; synchronous).
 * ------------------------------------------------------------------------------------------- */
typedef struct dcg_ctx dcg_ctx;
typedef struct dcg_weight dcg_weight;

/* One context per device (InitEngine-time, engine.cpp:122-278).  Thread-safe: calls serialize on
 * an internal mutex. */
int dcg_ctx_create(int device, dcg_ctx** out);
int dcg_ctx_destroy(dcg_ctx* ctx);

/* Upload one ggml weight tensor (n rows of k, ggml row stride) and keep it resident.  The host
 * pointer is the key dcg_ctx_find_weight looks up (the weight_tensor->data of cb_gemv_custom).
 * Registering a pointer again returns the resident copy when type, n and k match, and DCG_EINVAL
 * when they differ.  The device copy is not refreshed from host memory: release a weight before
 * its host buffer is freed or rewritten. */
int dcg_ctx_weight_register(dcg_ctx* ctx, int type, const void* host_rows, size_t row_stride,
                            int64_t n, int64_t k, dcg_weight** out);
int dcg_ctx_weight_release(dcg_ctx* ctx, dcg_weight* w);
int dcg_ctx_find_weight(dcg_ctx* ctx, const void* host_rows, dcg_weight** out);

/* cb_gemv_custom / ggml_mul_mat replacement: y_host[m][n] = W . x_host[m] (x f32, k per row). */
int dcg_ctx_mul_mat(dcg_ctx* ctx, dcg_weight* w, const float* x_host, int64_t m, float* y_host);

#ifdef __cplusplus
}
#endif
#endif /* DCGPU_H */
