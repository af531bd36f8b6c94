// capi.cu -- the extern "C" boundary of libdcgpu.so (declarations and citations: include/dcgpu.h).
#include <mutex>
#include <string>
#include <unordered_map>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
int cuda_fail(cudaError_t e, const char* where) {
    g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return DCG_ECUDA;
}
#define DCG_CUDA(call, where)                              \
    do {                                                   \
        cudaError_t _e = (call);                           \
        if (_e != cudaSuccess) return cuda_fail(_e, where); \
    } while (0)

bool weight_type_ok(int t) {
    return t == DCG_TYPE_Q8_0 || t == DCG_TYPE_Q4_K || t == DCG_TYPE_Q6_K;
}
int check_shape(int type, int64_t n, int64_t k) {
    if (!weight_type_ok(type)) return fail(DCG_EINVAL, "unsupported weight type " + std::to_string(type));
    if (n < 0 || k <= 0) return fail(DCG_EINVAL, "bad shape");
    const int64_t blk = type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K;
    if (k % blk) return fail(DCG_EINVAL, "k=" + std::to_string(k) + " is not a multiple of the block size " + std::to_string(blk));
    return DCG_OK;
}
int act_type_of(int wtype) { return wtype == DCG_TYPE_Q8_0 ? DCG_TYPE_Q8_0 : DCG_TYPE_Q8_K; }
bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace

namespace dcg_internal {
void set_error(const std::string& m) { g_last_error = m; }
}  // namespace dcg_internal

// ------------------------------------------------------------------------------------------
// internal: enqueue quantize + GEMV chunks (no checks beyond shapes; scratch already sized)
// ------------------------------------------------------------------------------------------
// scratch of dcg_mul_mat: [quantized activation | matmul tickets + split-K partials]
// (the matmul part: the tcgen05 kernel for m >= 2 Q4_K / Q6_K, the Q4_K M = 1 kernel's fallback)
// Batches up to DCG_MMA_MAX_M (default 0: none) take the register-fed mma.sync kernels instead of the
// tcgen05 ones, for side-by-side measurement
static int64_t mma_max_m() {
    static const int64_t v = [] {
        const char* e = getenv("DCG_MMA_MAX_M");
        return e ? (int64_t)atoll(e) : (int64_t)0;
    }();
    return v;
}
static bool use_tc(int type, int64_t n, int64_t k, int64_t m) {
    return m > mma_max_m() && dcg::qmm_tc_supports(type, n, k, m);
}
// Q8_0 weights of up to 16M elements at m <= 64 (the projections of a small model's decode step)
// run faster on the register-fed mma.sync kernel (qmm_rd.cu): measured on B200 at m = 64, 4096x1024
// 8.1 vs 11.7 us, 6144x1024 11.7 vs 19.7 us, 1024x3072 12.9 vs 14.9 us; the tcgen05 kernel keeps
// the large ones (151936x1024: 106 vs 176 us)
static bool use_q8tc(int type, int64_t n, int64_t k, int64_t m) {
    if (type == DCG_TYPE_Q8_0 && m <= 64 && n * k <= (int64_t)16 << 20 && dcg::qmm_rd_supports(type, k, m))
        return false;
    return m > mma_max_m() && dcg::qmm_q8tc_supports(type, n, k, m);
}
static size_t qmm_part(int type, int64_t n, int64_t k, int64_t m) {
    if (use_tc(type, n, k, m)) return dcg::qmm_tc_scratch_bytes(type, n, k, m);
    if (use_q8tc(type, n, k, m)) return dcg::qmm_q8tc_scratch_bytes(n, k, m);
    return dcg::qmm_supports(type) ? dcg::qmm_scratch_bytes(type, n, k, m) : 0;
}
static int qmm_tickets(int type, int64_t n, int64_t k, int64_t m) {
    if (use_tc(type, n, k, m)) return dcg::qmm_tc_ticket_count(type, n, k, m);
    if (use_q8tc(type, n, k, m)) return dcg::qmm_q8tc_ticket_count(n, k, m);
    return dcg::qmm_supports(type) ? dcg::qmm_ticket_count(type, n, m) : 0;
}

// M = 1 kernel choice: the per-type kernels (qmm.cu, gemv.cu); DCG_M1_KERNEL=stream selects the
// streaming mat-vec (gemv_m1.cu) instead, for side-by-side measurement
static bool use_m1s(int type, int64_t n, int64_t k, int64_t m) {
    static const bool stream = [] {
        const char* e = getenv("DCG_M1_KERNEL");
        return e && strcmp(e, "stream") == 0;
    }();
    return m == 1 && stream && dcg::m1s_supports(type, n, k);
}

static int enqueue_mul_mat_q(int type, const void* w, int64_t n, int64_t k, const void* act, int64_t m,
                             float* y, void* qscratch, cudaStream_t st) {
    if (use_m1s(type, n, k, m)) {
        DCG_CUDA(dcg::launch_m1s(type, w, n, k, nullptr, act, y, st), "gemv_m1");
        return DCG_OK;
    }
    if (use_tc(type, n, k, m)) {
        DCG_CUDA(dcg::launch_qmm_tc(type, w, n, k, act, m, y, qscratch, st), "qmm_tc");
        return DCG_OK;
    }
    if (use_q8tc(type, n, k, m)) {
        DCG_CUDA(dcg::launch_qmm_q8tc(w, n, k, act, m, y, qscratch, st), "qmm_q8tc");
        return DCG_OK;
    }
    if (dcg::qmm_supports(type)) {
        DCG_CUDA(dcg::launch_qmm(type, w, n, k, act, m, y, qscratch, st), "qmm");
        return DCG_OK;
    }
    if (dcg::qmm_rd_supports(type, k, m)) {
        DCG_CUDA(dcg::launch_qmm_rd(type, w, n, k, act, m, y, st), "qmm_rd");
        return DCG_OK;
    }
    for (int64_t m0 = 0; m0 < m; m0 += 8) {
        const int64_t mc = (m - m0) < 8 ? (m - m0) : 8;
        DCG_CUDA(dcg::launch_gemv(type, w, n, k, act, m, m0, mc, y, st), "gemv");
    }
    return DCG_OK;
}

static int enqueue_mul_mat(int type, const void* w, int64_t n, int64_t k, const float* x,
                           int64_t m, float* y, void* scratch, cudaStream_t st) {
    if (use_m1s(type, n, k, m)) {
        DCG_CUDA(dcg::launch_m1s(type, w, n, k, x, nullptr, y, st), "gemv_m1");
        return DCG_OK;
    }
    if (dcg::qmm_m1_fused_supports(type, n, k, m)) {
        DCG_CUDA(dcg::launch_qmm_m1_fused(w, n, k, x, y, st), "qmm m1");
        return DCG_OK;
    }
    void* qs = (uint8_t*)scratch + dcg::act_bytes(act_type_of(type), m, k);
    const int nt = qmm_tickets(type, n, k, m);
    DCG_CUDA(dcg::launch_quantize_act(act_type_of(type), x, scratch, m, k, true, st, (int*)qs, nt),
             "quantize");
    return enqueue_mul_mat_q(type, w, n, k, scratch, m, y, qs, st);
}

extern "C" {

int dcg_version(void) { return 100; }

int dcg_set_programmatic_launch(int enable) {
    return dcg::pdl_flag().exchange(enable ? 1 : 0) ? 1 : 0;
}

const char* dcg_strerror(int code) {
    switch (code) {
        case DCG_OK: return "ok";
        case DCG_EINVAL: return "invalid argument";
        case DCG_ECUDA: return "CUDA error";
        case DCG_ENOMEM: return "out of device memory";
        case DCG_ESCRATCH: return "scratch buffer too small";
        case DCG_ENOTFOUND: return "not registered";
    }
    return "unknown error";
}

const char* dcg_last_error(void) { return g_last_error.c_str(); }

size_t dcg_row_size(int type, int64_t k) {
    switch (type) {
        case DCG_TYPE_Q8_0: return (size_t)(k / QK8_0) * Q8_0_BYTES;
        case DCG_TYPE_Q4_K: return (size_t)(k / QK_K) * Q4_K_BYTES;
        case DCG_TYPE_Q6_K: return (size_t)(k / QK_K) * Q6_K_BYTES;
        case DCG_TYPE_Q8_K: return (size_t)(k / QK_K) * Q8_K_BYTES;
        case DCG_TYPE_F16: return (size_t)k * 2;
        case DCG_TYPE_F32: return (size_t)k * 4;
    }
    return 0;
}

size_t dcg_packed_weight_size(int type, int64_t n, int64_t k) {
    if (!weight_type_ok(type)) return 0;
    return dcg::packed_weight_bytes(type, n, k);
}

size_t dcg_mul_mat_scratch_size(int type, int64_t n, int64_t k, int64_t m) {
    if (!weight_type_ok(type) || n < 0 || k <= 0 || m < 0) return 0;
    return dcg::act_bytes(act_type_of(type), m, k) + qmm_part(type, n, k, m);
}

size_t dcg_mul_mat_q_scratch_size(int type, int64_t n, int64_t k, int64_t m) {
    if (!weight_type_ok(type) || n < 0 || k <= 0 || m < 0) return 0;
    return qmm_part(type, n, k, m);
}

static int quantize_rows(int act_type, const float* x, void* y, int64_t m, int64_t k, void* stream) {
    const int64_t blk = act_type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K;
    if (!x || !y) return fail(DCG_EINVAL, "null pointer");
    if (m < 0 || k <= 0 || k % blk) return fail(DCG_EINVAL, "k must be a positive multiple of the block size");
    if (!aligned(x, 16)) return fail(DCG_EINVAL, "x must be 16-byte aligned");
    if (act_type == DCG_TYPE_Q8_K && !aligned(y, 4)) return fail(DCG_EINVAL, "y must be 4-byte aligned");
    if (act_type == DCG_TYPE_Q8_0 && !aligned(y, 2)) return fail(DCG_EINVAL, "y must be 2-byte aligned");
    DCG_CUDA(dcg::launch_quantize_act(act_type, x, y, m, k, false, (cudaStream_t)stream), "quantize");
    return DCG_OK;
}

int dcg_quantize_row_q8_0(const float* x, void* y, int64_t m, int64_t k, void* stream) {
    return quantize_rows(DCG_TYPE_Q8_0, x, y, m, k, stream);
}
int dcg_quantize_row_q8_K(const float* x, void* y, int64_t m, int64_t k, void* stream) {
    return quantize_rows(DCG_TYPE_Q8_K, x, y, m, k, stream);
}

int dcg_quantize_weights(int type, const float* x, void* rows, int64_t n, int64_t k, void* stream) {
    int rc = check_shape(type, n, k);
    if (rc) return rc;
    if (!x || !rows) return fail(DCG_EINVAL, "null pointer");
    if (!aligned(x, 16) || !aligned(rows, 4)) return fail(DCG_EINVAL, "misaligned buffer");
    DCG_CUDA(dcg::launch_encode_weights(type, x, rows, n, k, (cudaStream_t)stream), "encode");
    return DCG_OK;
}

int dcg_weight_pack(int type, const void* rows, size_t row_stride, int64_t n, int64_t k,
                    void* packed, void* stream) {
    int rc = check_shape(type, n, k);
    if (rc) return rc;
    if (!rows || !packed) return fail(DCG_EINVAL, "null pointer");
    if (row_stride < dcg_row_size(type, k)) return fail(DCG_EINVAL, "row_stride smaller than a row");
    if (!aligned(packed, 256)) return fail(DCG_EINVAL, "packed buffer must be 256-byte aligned");
    DCG_CUDA(dcg::launch_pack(type, rows, row_stride, packed, n, k, false, (cudaStream_t)stream), "pack");
    return DCG_OK;
}

int dcg_weight_unpack(int type, const void* packed, int64_t n, int64_t k, void* rows,
                      size_t row_stride, void* stream) {
    int rc = check_shape(type, n, k);
    if (rc) return rc;
    if (!rows || !packed) return fail(DCG_EINVAL, "null pointer");
    if (row_stride < dcg_row_size(type, k)) return fail(DCG_EINVAL, "row_stride smaller than a row");
    DCG_CUDA(dcg::launch_pack(type, rows, row_stride, const_cast<void*>(packed), n, k, true,
                              (cudaStream_t)stream), "unpack");
    return DCG_OK;
}

int dcg_mul_mat(int type, const void* w, int64_t n, int64_t k, const float* x, int64_t m, float* y,
                void* scratch, size_t scratch_bytes, void* stream) {
    int rc = check_shape(type, n, k);
    if (rc) return rc;
    if (m < 0) return fail(DCG_EINVAL, "m < 0");
    if (m == 0 || n == 0) return DCG_OK;
    if (!w || !x || !y || !scratch) return fail(DCG_EINVAL, "null pointer");
    if (!aligned(w, 256) || !aligned(scratch, 256)) return fail(DCG_EINVAL, "w and scratch must be 256-byte aligned");
    if (!aligned(x, 16) || !aligned(y, 4)) return fail(DCG_EINVAL, "x must be 16-byte aligned, y 4-byte aligned");
    const size_t need = dcg_mul_mat_scratch_size(type, n, k, m);
    if (scratch_bytes < need)
        return fail(DCG_ESCRATCH, "scratch needs " + std::to_string(need) + " bytes, got " + std::to_string(scratch_bytes));
    return enqueue_mul_mat(type, w, n, k, x, m, y, scratch, (cudaStream_t)stream);
}

int dcg_device_error(int* code, int clear) {
    if (!code) return fail(DCG_EINVAL, "null pointer");
    int a = 0, b = 0, c = 0, d = 0, f = 0, g = 0;
    DCG_CUDA(dcg::qmm_q8tc_device_error(&f, clear != 0), "read device error flag");
    DCG_CUDA(dcg::m1s_device_error(&g, clear != 0), "read device error flag");
    DCG_CUDA(dcg::gemv_device_error(&a, clear != 0), "read device error flag");
    DCG_CUDA(dcg::qmm_device_error(&b, clear != 0), "read device error flag");
    DCG_CUDA(dcg::attn_device_error(&c, clear != 0), "read device error flag");
    DCG_CUDA(dcg::qmm_tc_device_error(&d, clear != 0), "read device error flag");
    *code = a ? a : (b ? b : (c ? c : (d ? d : (f ? f : g))));
    return DCG_OK;
}

size_t dcg_paged_attn_scratch_size(int n_seqs, int hq, int hkv, int head_dim, int max_ctx) {
    if (n_seqs <= 0 || hq <= 0 || hkv <= 0 || head_dim != 128 || max_ctx < 0) return 0;
    return dcg::attn_scratch_bytes(n_seqs, hq, hkv, max_ctx);
}

int dcg_paged_attn_decode(const float* q, const void* k_arena, const void* v_arena,
                          int64_t n_arena_blocks, int n_layer, int layer,
                          const int32_t* block_tables, int max_blocks_per_seq,
                          const int32_t* ctx_lens, int n_seqs, int hq, int hkv, int head_dim,
                          int max_ctx, float scale, float* out, void* scratch, size_t scratch_bytes,
                          void* stream) {
    if (n_seqs < 0) return fail(DCG_EINVAL, "n_seqs < 0");
    if (n_seqs == 0) return DCG_OK;
    if (!q || !k_arena || !v_arena || !block_tables || !ctx_lens || !out)
        return fail(DCG_EINVAL, "null pointer");
    if (head_dim != 128) return fail(DCG_EINVAL, "head_dim must be 128");
    if (hkv <= 0 || hq <= 0 || hq % hkv) return fail(DCG_EINVAL, "hq must be a multiple of hkv");
    const int nrep = hq / hkv;
    if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8) return fail(DCG_EINVAL, "hq/hkv must be 1, 2, 4 or 8");
    if (n_layer <= 0 || layer < 0 || layer >= n_layer) return fail(DCG_EINVAL, "bad layer");
    if (n_arena_blocks <= 0) return fail(DCG_EINVAL, "n_arena_blocks must be > 0");
    if (max_ctx < 0 || max_ctx > 16 * max_blocks_per_seq) return fail(DCG_EINVAL, "max_ctx exceeds the block table");
    if (!aligned(k_arena, 16) || !aligned(v_arena, 16) || !aligned(q, 16) || !aligned(out, 16))
        return fail(DCG_EINVAL, "q, out and the arenas must be 16-byte aligned");
    const size_t need = dcg::attn_scratch_bytes(n_seqs, hq, hkv, max_ctx);
    if (scratch_bytes < need || (need && !scratch))
        return fail(DCG_ESCRATCH, "attention scratch needs " + std::to_string(need) + " bytes");
    if (need && !aligned(scratch, 256)) return fail(DCG_EINVAL, "scratch must be 256-byte aligned");
    DCG_CUDA(dcg::launch_paged_attn(q, k_arena, v_arena, n_layer, layer, block_tables,
                                    max_blocks_per_seq, ctx_lens, n_seqs, hq, hkv, max_ctx, scale, out,
                                    scratch, (cudaStream_t)stream, n_arena_blocks), "paged_attn_decode");
    return DCG_OK;
}

int dcg_paged_attn_prefill(const float* q, const void* k_arena, const void* v_arena, int64_t n_arena_blocks,
                           int n_layer, int layer, const int32_t* block_tables, int max_blocks_per_seq,
                           const int32_t* seq_starts, const int32_t* ctx_lens, int n_seqs, int max_seq_tokens,
                           int hq, int hkv, int head_dim, int max_ctx, float scale, float* out, void* stream) {
    if (n_seqs < 0 || max_seq_tokens < 0) return fail(DCG_EINVAL, "n_seqs and max_seq_tokens must be >= 0");
    if (n_seqs == 0 || max_seq_tokens == 0) return DCG_OK;
    if (!q || !k_arena || !v_arena || !block_tables || !seq_starts || !ctx_lens || !out)
        return fail(DCG_EINVAL, "null pointer");
    if (head_dim != 128) return fail(DCG_EINVAL, "head_dim must be 128");
    if (hkv <= 0 || hq <= 0 || hq % hkv) return fail(DCG_EINVAL, "hq must be a multiple of hkv");
    const int nrep = hq / hkv;
    if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8) return fail(DCG_EINVAL, "hq/hkv must be 1, 2, 4 or 8");
    if (n_layer <= 0 || layer < 0 || layer >= n_layer) return fail(DCG_EINVAL, "bad layer");
    if (n_arena_blocks <= 0) return fail(DCG_EINVAL, "n_arena_blocks must be > 0");
    if (max_ctx < 0 || max_ctx > 16 * max_blocks_per_seq) return fail(DCG_EINVAL, "max_ctx exceeds the block table");
    if (!aligned(k_arena, 16) || !aligned(v_arena, 16) || !aligned(q, 16) || !aligned(out, 16))
        return fail(DCG_EINVAL, "q, out and the arenas must be 16-byte aligned");
    DCG_CUDA(dcg::launch_paged_attn_prefill(q, k_arena, v_arena, n_layer, layer, block_tables, max_blocks_per_seq,
                                            seq_starts, ctx_lens, n_seqs, max_seq_tokens, hq, hkv, scale, out,
                                            (cudaStream_t)stream, n_arena_blocks),
             "paged_attn_prefill");
    return DCG_OK;
}

int dcg_kv_append(const float* k, const float* v, void* k_arena, void* v_arena, int n_layer,
                  int layer, const int32_t* block_tables, int max_blocks_per_seq,
                  const int32_t* seq_ids, const int32_t* positions, int n_tok, int hkv,
                  int head_dim, void* stream) {
    if (n_tok < 0) return fail(DCG_EINVAL, "n_tok < 0");
    if (n_tok == 0) return DCG_OK;
    if (!k || !v || !k_arena || !v_arena || !block_tables || !seq_ids || !positions)
        return fail(DCG_EINVAL, "null pointer");
    if (hkv <= 0 || head_dim <= 0 || n_layer <= 0 || layer < 0 || layer >= n_layer || max_blocks_per_seq <= 0)
        return fail(DCG_EINVAL, "bad shape");
    if (!aligned(k_arena, 2) || !aligned(v_arena, 2)) return fail(DCG_EINVAL, "arenas must be 2-byte aligned");
    DCG_CUDA(dcg::launch_kv_append(k, v, k_arena, v_arena, n_layer, layer, block_tables,
                                   max_blocks_per_seq, seq_ids, positions, n_tok, hkv, head_dim,
                                   (cudaStream_t)stream), "kv_append");
    return DCG_OK;
}

static bool act_shape_ok(int act_type, int64_t k) {
    return (act_type == DCG_TYPE_Q8_0 && k % QK8_0 == 0) || (act_type == DCG_TYPE_Q8_K && k % QK_K == 0);
}

int dcg_add_rmsnorm_quantize(float* x, const float* delta, const float* weight, float eps, int64_t m,
                             int64_t k, int act_type, void* act, void* stream) {
    if (!x || !weight || !act) return fail(DCG_EINVAL, "null pointer");
    if (m < 0 || k <= 0 || !act_shape_ok(act_type, k)) return fail(DCG_EINVAL, "bad shape or act_type");
    if (m == 0) return DCG_OK;
    if (!aligned(act, 256)) return fail(DCG_EINVAL, "act must be 256-byte aligned");
    DCG_CUDA(dcg::launch_add_rmsnorm_quant(x, delta, weight, eps, m, k, act_type, act, (cudaStream_t)stream),
             "add_rmsnorm_quantize");
    return DCG_OK;
}

int dcg_swiglu_quantize(const float* gate, const float* up, int64_t ld, int64_t m, int64_t ffn,
                        int act_type, void* act, void* stream) {
    if (!gate || !up || !act) return fail(DCG_EINVAL, "null pointer");
    if (m < 0 || ffn <= 0 || ld < ffn || !act_shape_ok(act_type, ffn)) return fail(DCG_EINVAL, "bad shape or act_type");
    if (m == 0) return DCG_OK;
    if (!aligned(act, 256)) return fail(DCG_EINVAL, "act must be 256-byte aligned");
    DCG_CUDA(dcg::launch_swiglu_quant(gate, up, ld, m, ffn, act_type, act, (cudaStream_t)stream), "swiglu_quantize");
    return DCG_OK;
}

static int qk_rope_common(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                               int64_t ldv, int n_seqs, int hq, int hkv, int head_dim,
                               const float* q_norm_w, const float* k_norm_w, float eps, float rope_theta,
                               const int32_t* positions, float* q_out, void* k_arena, void* v_arena,
                               int n_layer, int layer, const int32_t* block_tables,
                               int max_blocks_per_seq, void* stream, const int32_t* seq_ids) {
    if (!q || !k || !v || !positions || !q_out || !k_arena || !v_arena || !block_tables)
        return fail(DCG_EINVAL, "null pointer");
    if (!q_norm_w != !k_norm_w) return fail(DCG_EINVAL, "give both QK-norm weights or neither");
    if (head_dim != 128) return fail(DCG_EINVAL, "head_dim must be 128");
    if (n_seqs < 0 || hq <= 0 || hkv <= 0 || n_layer <= 0 || layer < 0 || layer >= n_layer || max_blocks_per_seq <= 0)
        return fail(DCG_EINVAL, "bad shape");
    if (n_seqs == 0) return DCG_OK;
    DCG_CUDA(dcg::launch_qk_rope_append(q, ldq, k, ldk, v, ldv, n_seqs, hq, hkv, q_norm_w, k_norm_w, eps,
                                        rope_theta, positions, q_out, k_arena, v_arena, n_layer, layer,
                                        block_tables, max_blocks_per_seq, (cudaStream_t)stream, seq_ids),
             "qk_norm_rope_kv_append");
    return DCG_OK;
}

int dcg_qk_norm_rope_kv_append(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                               int64_t ldv, int n_seqs, int hq, int hkv, int head_dim,
                               const float* q_norm_w, const float* k_norm_w, float eps, float rope_theta,
                               const int32_t* positions, float* q_out, void* k_arena, void* v_arena,
                               int n_layer, int layer, const int32_t* block_tables,
                               int max_blocks_per_seq, void* stream) {
    return qk_rope_common(q, ldq, k, ldk, v, ldv, n_seqs, hq, hkv, head_dim, q_norm_w, k_norm_w, eps, rope_theta,
                          positions, q_out, k_arena, v_arena, n_layer, layer, block_tables, max_blocks_per_seq,
                          stream, nullptr);
}

int dcg_qk_norm_rope_kv_append_tokens(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                      int64_t ldv, int n_tok, int hq, int hkv, int head_dim,
                                      const float* q_norm_w, const float* k_norm_w, float eps, float rope_theta,
                                      const int32_t* seq_ids, const int32_t* positions, float* q_out,
                                      void* k_arena, void* v_arena, int n_layer, int layer,
                                      const int32_t* block_tables, int max_blocks_per_seq, void* stream) {
    if (!seq_ids) return fail(DCG_EINVAL, "null pointer");
    return qk_rope_common(q, ldq, k, ldk, v, ldv, n_tok, hq, hkv, head_dim, q_norm_w, k_norm_w, eps, rope_theta,
                          positions, q_out, k_arena, v_arena, n_layer, layer, block_tables, max_blocks_per_seq,
                          stream, seq_ids);
}

size_t dcg_act_size(int act_type, int64_t m, int64_t k) {
    if (act_type != DCG_TYPE_Q8_0 && act_type != DCG_TYPE_Q8_K) return 0;
    return dcg::act_bytes(act_type, m, k);
}

int dcg_quantize_act(int act_type, const float* x, void* act, int64_t m, int64_t k, void* stream) {
    if (act_type != DCG_TYPE_Q8_0 && act_type != DCG_TYPE_Q8_K)
        return fail(DCG_EINVAL, "act_type must be Q8_0 or Q8_K");
    const int64_t blk = act_type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K;
    if (!x || !act) return fail(DCG_EINVAL, "null pointer");
    if (m < 0 || k <= 0 || k % blk) return fail(DCG_EINVAL, "k must be a positive multiple of the block size");
    if (!aligned(x, 16) || !aligned(act, 256)) return fail(DCG_EINVAL, "x must be 16-byte and act 256-byte aligned");
    DCG_CUDA(dcg::launch_quantize_act(act_type, x, act, m, k, true, (cudaStream_t)stream), "quantize");
    return DCG_OK;
}

int dcg_mul_mat_q(int type, const void* w, int64_t n, int64_t k, const void* act, int64_t m,
                  float* y, void* scratch, size_t scratch_bytes, void* stream) {
    int rc = check_shape(type, n, k);
    if (rc) return rc;
    if (m < 0) return fail(DCG_EINVAL, "m < 0");
    if (m == 0 || n == 0) return DCG_OK;
    if (!w || !act || !y) return fail(DCG_EINVAL, "null pointer");
    if (!aligned(w, 256) || !aligned(act, 256) || !aligned(y, 4)) return fail(DCG_EINVAL, "misaligned buffer");
    const size_t need = qmm_part(type, n, k, m);
    if (need && (!scratch || scratch_bytes < need))
        return fail(DCG_ESCRATCH, "mul_mat_q scratch needs " + std::to_string(need) + " bytes");
    if (need && !aligned(scratch, 256)) return fail(DCG_EINVAL, "scratch must be 256-byte aligned");
    return enqueue_mul_mat_q(type, w, n, k, act, m, y, scratch, (cudaStream_t)stream);
}

}  // extern "C"
