"""ggml type ids and block geometry used at the boundary (ggml enum ggml_type; GGUF block sizes)."""
F32, F16, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 8, 12, 14, 15

_BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210),
          Q8_K: (256, 292)}

# ggml type_traits_cpu[...].vec_dot_type: the activation format each weight type dots against
# (selected at core/src/inference.cpp:970-983)
VEC_DOT_TYPE = {Q8_0: Q8_0, Q4_K: Q8_K, Q6_K: Q8_K}


def block_size(t: int) -> int:
    return _BLOCK[t][0]


def type_size(t: int) -> int:
    return _BLOCK[t][1]


def row_size(t: int, k: int) -> int:
    """ggml_row_size(t, k)."""
    bs, ts = _BLOCK[t]
    if k % bs:
        raise ValueError(f"k={k} is not a multiple of the block size {bs} of type {t}")
    return k // bs * ts
