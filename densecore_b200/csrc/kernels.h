// kernels.h -- internal launchers shared between the .cu files and the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dcg {

// also zeroes zero[0 .. nzero) (the matmul's split-K tickets) in the same launch
cudaError_t launch_quantize_act(int act_type, const float* x, void* y, int64_t m, int64_t k,
                                bool soa, cudaStream_t st, int* zero = nullptr, int nzero = 0);
cudaError_t launch_encode_weights(int type, const float* x, void* y, int64_t n, int64_t k,
                                  cudaStream_t st);
cudaError_t launch_pack(int type, const void* src, size_t src_stride, void* dst, int64_t n,
                        int64_t k, bool unpack, cudaStream_t st);

// y[m][n] = W[n] . act[m]; act in the SoA activation layout; m <= 8 per launch.
cudaError_t launch_gemv(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                        int64_t act_m, int64_t m0, int64_t m, float* y, cudaStream_t st);

// tensor-core quantized matmul (qmm.cu); cudaErrorNotSupported for types it does not cover
size_t qmm_scratch_bytes(int type, int64_t n, int64_t k, int64_t m);
// ints at the start of the qmm scratch that must be zero when a qmm launch starts (left zero)
int qmm_ticket_count(int type, int64_t n, int64_t m);
// M == 1 Q4_K with the activation quantized inside the matmul kernel (no scratch)
bool qmm_m1_fused_supports(int type, int64_t n, int64_t k, int64_t m);
cudaError_t launch_qmm_m1_fused(const void* packed_w, int64_t n, int64_t k, const float* x, float* y,
                                cudaStream_t st);
cudaError_t launch_qmm(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                       int64_t m, float* y, void* scratch, cudaStream_t st);
// tcgen05 Q4_K / Q6_K GEMM for m >= 2 (qmm_tc.cu); scratch: tickets (zero at launch, left zero)
// followed by the stream-K partial tiles
bool qmm_tc_supports(int type, int64_t n, int64_t k, int64_t m);
size_t qmm_tc_scratch_bytes(int type, int64_t n, int64_t k, int64_t m);
int qmm_tc_ticket_count(int type, int64_t n, int64_t k, int64_t m);
cudaError_t launch_qmm_tc(int type, const void* packed_w, int64_t n, int64_t k, const void* act, int64_t m,
                          float* y, void* scratch, cudaStream_t st);
cudaError_t qmm_tc_device_error(int* out, bool clear);
cudaError_t qmm_device_error(int* out, bool clear);
bool qmm_supports(int type);

// tcgen05 Q8_0 GEMM for m >= 2, k % 256 == 0 (qmm_q8tc.cu); scratch as for qmm_tc
bool qmm_q8tc_supports(int type, int64_t n, int64_t k, int64_t m);
size_t qmm_q8tc_scratch_bytes(int64_t n, int64_t k, int64_t m);
int qmm_q8tc_ticket_count(int64_t n, int64_t k, int64_t m);
cudaError_t launch_qmm_q8tc(const void* packed_w, int64_t n, int64_t k, const void* act, int64_t m, float* y,
                            void* scratch, cudaStream_t st);
cudaError_t qmm_q8tc_device_error(int* out, bool clear);

// M = 1 streaming mat-vec for Q4_K / Q6_K / Q8_0 (gemv_m1.cu): x = fp32 row quantized in the kernel,
// or x = null and act = the SoA quantized activation; no scratch
bool m1s_supports(int type, int64_t n, int64_t k);
cudaError_t launch_m1s(int type, const void* packed_w, int64_t n, int64_t k, const float* x, const void* act,
                       float* y, cudaStream_t st);
cudaError_t m1s_device_error(int* out, bool clear);

// register-direct tensor-core matmul for Q8_0 / Q6_K (qmm_rd.cu), M >= 2, k % 256 == 0
bool qmm_rd_supports(int type, int64_t k, int64_t m);
cudaError_t launch_qmm_rd(int type, const void* packed_w, int64_t n, int64_t k, const void* act,
                          int64_t m, float* y, cudaStream_t st);

// paged decode attention (attn.cu); n_arena_blocks = physical KV blocks in the arena
cudaError_t attn_device_error(int* out, bool clear);
void attn_plan(int n_seqs, int hkv, int max_ctx, int* splits, int* bps);
size_t attn_scratch_bytes(int n_seqs, int hq, int hkv, int max_ctx);
cudaError_t launch_paged_attn(const float* q, const void* karena, const void* varena, int n_layer,
                              int layer, const int* bt, int mbs, const int* ctx, int n_seqs, int hq,
                              int hkv, int max_ctx, float scale, float* out, void* scratch,
                              cudaStream_t st, int64_t n_arena_blocks);
// multi-token causal attention (prefill / prompt chunks) over the paged cache (attn.cu)
cudaError_t launch_paged_attn_prefill(const float* q, const void* karena, const void* varena, int n_layer,
                                      int layer, const int* bt, int mbs, const int* seq_starts, const int* ctx,
                                      int n_seqs, int max_seq_tokens, int hq, int hkv, float scale, float* out,
                                      cudaStream_t st, int64_t n_arena_blocks);
cudaError_t launch_kv_append(const float* k, const float* v, void* karena, void* varena, int n_layer,
                             int layer, const int* bt, int mbs, const int* seq_ids, const int* pos,
                             int n_tok, int hkv, int hd, cudaStream_t st);

// fused pre-matmul element-wise kernels (fused.cu)
cudaError_t launch_add_rmsnorm_quant(float* x, const float* delta, const float* w, float eps, int64_t m,
                                     int64_t k, int act_type, void* act, cudaStream_t st);
cudaError_t launch_swiglu_quant(const float* g, const float* u, int64_t ld, int64_t m, int64_t ffn,
                                int act_type, void* act, cudaStream_t st);
cudaError_t launch_qk_rope_append(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                  int64_t ldv, int n_seqs, int hq, int hkv, const float* qw, const float* kw,
                                  float eps, float theta, const int* pos, float* q_out, void* karena,
                                  void* varena, int n_layer, int layer, const int* bt, int mbs,
                                  cudaStream_t st, const int* seq_ids = nullptr);

// error flag of the bounded waits of the GEMV kernels (0 = none); optionally cleared
cudaError_t gemv_device_error(int* out, bool clear);

}  // namespace dcg
