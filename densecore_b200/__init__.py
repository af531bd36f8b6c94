"""densecore_b200 -- B200 (sm_100a) implementation of DenseCore's quantized weight matmul and
paged decode attention, behind a C ABI (include/dcgpu.h, libdcgpu.so).

Python surface (ops.py) mirrors the reference operator names: quantize_row_q8_0 /
quantize_row_q8_K (ggml from_float), mul_mat (smart_mul_mat / ggml_mul_mat on a quantized
weight), paged_attn_decode and kv_append (the decode attention over PagedKVCache).
"""
from .ggml_types import (F16, F32, Q4_K, Q6_K, Q8_0, Q8_K, VEC_DOT_TYPE, block_size,  # noqa: F401
                         row_size, type_size)

__all__ = ["ops", "F32", "F16", "Q8_0", "Q4_K", "Q6_K", "Q8_K", "VEC_DOT_TYPE", "row_size"]
