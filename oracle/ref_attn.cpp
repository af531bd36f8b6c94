// C entry over DenseCore's FlashAttentionGQA (core/include/flash_attention.h:239-272), built from
// the reference sources by oracle/Makefile.  Test infrastructure: attention cross-check and the
// reference CPU attention timing.  Layouts are the reference's: Q [B,Hq,Sq,D], K/V [B,Hkv,Skv,D].
#include <immintrin.h>
#include "flash_attention.h"

extern "C" void ggml_fp32_to_fp16_row(const float* x, ggml_fp16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = _cvtss_sh(x[i], 0);
}
extern "C" void ggml_fp16_to_fp32_row(const ggml_fp16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = _cvtsh_ss(x[i]);
}

extern "C" int ref_flash_attention_gqa(const float* Q, const float* K, const float* V, float* O,
                                       int batch, int hq, int hkv, int sq, int skv, int d,
                                       float scale, int causal, int ith, int nth) {
    densecore::FlashAttentionConfig cfg;
    cfg.scale = scale;
    cfg.causal = causal != 0;
    densecore::FlashAttentionGQA(Q, K, V, O, batch, hq, hkv, sq, skv, d, cfg, ith, nth);
    return 0;
}
