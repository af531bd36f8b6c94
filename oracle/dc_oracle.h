/*
 * dc_oracle.h -- CPU restatement of DenseCore's quantized-matmul and decode-attention
 * arithmetic.  TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py as the checker.  The product (libdcgpu.so) never
 * links or calls it.
 *
 * DenseCore delegates this arithmetic to ggml (git submodule core/third_party/ggml, url
 * github.com/ggerganov/ggml, no pinned commit; absent from the reference tree).  The functions
 * below restate ggml's published block formats and reference (scalar) algorithms in our own
 * code, anchored on DenseCore's call sites:
 *   - from_float -> quantize_row_q8_0 / quantize_row_q8_K : core/src/inference.cpp:887-894
 *   - vec_dot_{q8_0_q8_0,q4_K_q8_K,q6_K_q8_K}            : core/src/inference.cpp:916-924,
 *                                                          core/src/simd_ops.cpp:82-93
 *   - row-sliced GEMV (cb_gemv_custom)                     : core/src/inference.cpp:840-948
 *   - paged fp16 KV layout                                 : core/src/kv_cache.cpp:353-370
 *   - decode attention (flash path semantics)              : core/src/inference.cpp:1519-1573
 * Parity pins: Q8_0 quantize bytes and Q8_0/Q4_K/Q6_K dequantization are checked against the
 * `gguf` Python package's implementation (tests/golden/make_golden.py); attention is checked
 * against DenseCore's own FlashAttentionGQA compiled from its sources (oracle/build_ref.sh).
 */
#ifndef DC_ORACLE_H
#define DC_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (ggml.h enum ggml_type values) */
enum { DCO_F32 = 0, DCO_F16 = 1, DCO_Q8_0 = 8, DCO_Q4_K = 12, DCO_Q6_K = 14, DCO_Q8_K = 15 };

uint16_t dco_fp32_to_fp16(float f);
float dco_fp16_to_fp32(uint16_t h);

size_t dco_row_size(int type, int64_t k);

/* activation / weight quantizers: k elements -> k/blk blocks */
void dco_quantize_row_q8_0(const float* x, void* y, int64_t k);
void dco_quantize_row_q8_K(const float* x, void* y, int64_t k);
void dco_quantize_row_q4_K(const float* x, void* y, int64_t k);
void dco_quantize_row_q6_K(const float* x, void* y, int64_t k);

void dco_dequantize_row(int type, const void* x, float* y, int64_t k);

/* vec_dot: one weight row (type) against one pre-quantized activation row */
void dco_vec_dot(int type, int n, float* s, const void* w, const void* xq);

/* per-block int32 dots (bit-exact checks).  Q8_0: n/32 values.  Q4_K: n/32 values of
 * sc_j * dot_j and n/256 values of sum_j m_j * bsum_j.  Q6_K: n/16 values of
 * (q-32).q8 per 16-element sub-block (unscaled). */
void dco_block_dots(int type, int n, const void* w, const void* xq, int32_t* out, int32_t* out2);

/* GEMV/GEMM: y[m][n_rows] = W[n_rows] . xq[m]; rows split over nthreads like cb_gemv_custom */
void dco_mul_mat(int type, const void* w, size_t row_stride, int64_t n_rows, int64_t k,
                 const void* xq, int64_t m, float* y, int nthreads);

/* The same with a SIMD restatement of the Q4_K dot (bit-identical results; the CPU baseline's
 * compute): isa = DCO_ISA_VNNI (AVX-512 VNNI vpdpbusd), DCO_ISA_AVX2 (maddubs), or 0 for the best
 * the host supports.  Returns the ISA that ran (0: the scalar dots). */
#define DCO_ISA_AVX2 1
#define DCO_ISA_VNNI 2
int dco_simd_isa(void);
int dco_mul_mat_simd(int type, const void* w, size_t row_stride, int64_t n_rows, int64_t k,
                     const void* xq, int64_t m, float* y, int nthreads, int isa);

/* fp16 paged-KV decode attention, one query token per sequence.
 * q [n_seqs][hq][d] f32; k_arena/v_arena fp16 laid out [(block*n_layer+layer)][16][hkv][d];
 * block_tables [n_seqs][max_blocks_per_seq]; ctx_lens[n_seqs]; out [n_seqs][hq][d]. */
void dco_paged_attn_decode(const float* q, const uint16_t* k_arena, const uint16_t* v_arena,
                           int n_layer, int layer, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* ctx_lens, int n_seqs, int hq,
                           int hkv, int d, float scale, float* out, int nthreads);

/* KV append: write n_tok tokens' K/V (f32 [n_tok][hkv][d]) into fp16 slots at positions pos[i]
 * of sequence seq[i] through its block table. */
void dco_kv_append(const float* k, const float* v, uint16_t* k_arena, uint16_t* v_arena,
                   int n_layer, int layer, const int32_t* block_tables, int max_blocks_per_seq,
                   const int32_t* seq_ids, const int32_t* positions, int n_tok, int hkv, int d);

#ifdef __cplusplus
}
#endif
#endif
