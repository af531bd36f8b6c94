/* Stand-in for ggml.h when compiling DenseCore's flash_attention.h / simd_ops.h: they only need
 * the fp16 storage type and the two row converters (simd_ops.h:82, :925-934). */
#pragma once
#include <stdint.h>
typedef uint16_t ggml_fp16_t;
#ifdef __cplusplus
extern "C" {
#endif
void ggml_fp32_to_fp16_row(const float* x, ggml_fp16_t* y, int64_t n);
void ggml_fp16_to_fp32_row(const ggml_fp16_t* x, float* y, int64_t n);
#ifdef __cplusplus
}
#endif
