"""ctypes/numpy front of the CPU checker (dc_oracle.c) and of DenseCore's own FlashAttentionGQA
built from its sources (oracle/_ref/libref_attn.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs as
the checker; the product (densecore_b200) never imports it.  Function citations are in
dc_oracle.h / dc_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

F32, F16, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 8, 12, 14, 15
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q8_K: (256, 292)}
VEC_DOT_TYPE = {Q8_0: Q8_0, Q4_K: Q8_K, Q6_K: Q8_K}

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        vp, i64, i32, f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.dco_fp32_to_fp16.restype = ctypes.c_uint16
        L.dco_fp32_to_fp16.argtypes = [f]
        L.dco_row_size.restype = ctypes.c_size_t
        L.dco_row_size.argtypes = [i32, i64]
        for n in ("dco_quantize_row_q8_0", "dco_quantize_row_q8_K", "dco_quantize_row_q4_K",
                  "dco_quantize_row_q6_K"):
            getattr(L, n).argtypes = [vp, vp, i64]
        L.dco_dequantize_row.argtypes = [i32, vp, vp, i64]
        L.dco_vec_dot.argtypes = [i32, i32, vp, vp, vp]
        L.dco_block_dots.argtypes = [i32, i32, vp, vp, vp, vp]
        L.dco_mul_mat.argtypes = [i32, vp, ctypes.c_size_t, i64, i64, vp, i64, vp, i32]
        L.dco_mul_mat_simd.argtypes = [i32, vp, ctypes.c_size_t, i64, i64, vp, i64, vp, i32, i32]
        L.dco_mul_mat_simd.restype = i32
        L.dco_simd_isa.restype = i32
        L.dco_paged_attn_decode.argtypes = [vp, vp, vp, i32, i32, vp, i32, vp, i32, i32, i32, i32,
                                            f, vp, i32]
        L.dco_kv_append.argtypes = [vp, vp, vp, vp, i32, i32, vp, i32, vp, vp, i32, i32, i32]
        _lib = L
    return _lib


def ref_lib():
    """DenseCore's FlashAttentionGQA, or None when it was never built here."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref_attn.so")
        if not os.path.exists(path):
            return None
        R = ctypes.CDLL(path)
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        R.ref_flash_attention_gqa.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32,
                                              ctypes.c_float, i32, i32, i32]
        _ref = R
    return _ref


def ref_int4_gemv(shapes, group: int, threads: int, budget_s: float) -> dict | None:
    """Times DenseCore's own INT4 decode GEMV (core/src/kernels/cpu_int4.cpp, runtime ISA dispatch)
    over the (n, k) shapes for about budget_s seconds; None when it was never built here."""
    path = os.path.join(HERE, "_ref", "libref_int4.so")
    if not os.path.exists(path):
        return None
    R = ctypes.CDLL(path)
    R.ref_int4_isa.restype = ctypes.c_char_p
    R.ref_int4_time.restype = ctypes.c_long
    R.ref_int4_time.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_double, ctypes.c_void_p]
    ns = (ctypes.c_int * len(shapes))(*[n for n, _ in shapes])
    ks = (ctypes.c_int * len(shapes))(*[k for _, k in shapes])
    sec = ctypes.c_double()
    passes = R.ref_int4_time(ns, ks, len(shapes), group, threads, budget_s, ctypes.byref(sec))
    # bytes per row: K/2 packed nibbles + an f32 scale and zero per group
    wbytes = sum(n * (k // 2 + 8 * (k // group)) for n, k in shapes)
    return {"passes": int(passes), "seconds": sec.value, "weight_bytes_per_pass": wbytes,
            "isa": R.ref_int4_isa().decode()}


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def row_size(qtype: int, k: int) -> int:
    blk, nb = BLOCK[qtype]
    assert k % blk == 0
    return k // blk * nb


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    """[rows, k] f32 -> [rows, row_size] uint8 in ggml block layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros((rows, row_size(qtype, k)), dtype=np.uint8)
    fn = {Q8_0: "dco_quantize_row_q8_0", Q8_K: "dco_quantize_row_q8_K",
          Q4_K: "dco_quantize_row_q4_K", Q6_K: "dco_quantize_row_q6_K"}[qtype]
    getattr(lib(), fn)(_p(x), _p(out), rows * k)
    return out


def dequantize(q: np.ndarray, qtype: int, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows = q.size // row_size(qtype, k)
    out = np.zeros((rows, k), dtype=np.float32)
    lib().dco_dequantize_row(qtype, _p(q), _p(out), rows * k)
    return out


def vec_dot(wtype: int, k: int, w_row: np.ndarray, xq_row: np.ndarray) -> float:
    s = np.zeros(1, dtype=np.float32)
    lib().dco_vec_dot(wtype, k, _p(s), _p(np.ascontiguousarray(w_row)),
                      _p(np.ascontiguousarray(xq_row)))
    return float(s[0])


def block_dots(wtype: int, k: int, w_row: np.ndarray, xq_row: np.ndarray):
    """Per-block int32 dots: Q8_0 -> (k/32,), Q4_K -> ((k/32,) sc*dot, (k/256,) min sums),
    Q6_K -> (k/16,) unscaled sub-block dots."""
    n1 = {Q8_0: k // 32, Q4_K: k // 32, Q6_K: k // 16}[wtype]
    a = np.zeros(n1, dtype=np.int32)
    b = np.zeros(max(1, k // 256), dtype=np.int32)
    lib().dco_block_dots(wtype, k, _p(np.ascontiguousarray(w_row)),
                         _p(np.ascontiguousarray(xq_row)), _p(a), _p(b))
    return (a, b) if wtype == Q4_K else a


ISA_NAMES = {0: "scalar", 1: "avx2", 2: "avx512vnni"}


def mul_mat(wtype: int, w: np.ndarray, k: int, xq: np.ndarray, m: int, nthreads: int = 1,
            simd=False):
    """y[m, n_rows] = W . xq (row-sliced over nthreads, like cb_gemv_custom).  simd: Q4_K dots by
    a SIMD restatement (bit-identical; the CPU baseline's compute): True = the best the host has
    (AVX-512 VNNI, else AVX2), or "avx2" / "avx512vnni"."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rs = row_size(wtype, k)
    n_rows = w.size // rs
    y = np.zeros((m, n_rows), dtype=np.float32)
    args = (wtype, _p(w), rs, n_rows, k, _p(np.ascontiguousarray(xq)), m, _p(y), nthreads)
    if simd:
        isa = {True: 0, "avx2": 1, "avx512vnni": 2}[simd]
        lib().dco_mul_mat_simd(*args, isa)
    else:
        lib().dco_mul_mat(*args)
    return y


def simd_isa() -> str:
    """The ISA mul_mat(..., simd=True) uses for Q4_K dots on this CPU: avx512vnni, avx2 or scalar."""
    return ISA_NAMES[int(lib().dco_simd_isa())]


def simd_available() -> bool:
    """Whether mul_mat(..., simd=True) runs SIMD Q4_K dots on this CPU."""
    return simd_isa() != "scalar"


def paged_attn_decode(q, k_arena, v_arena, n_layer, layer, block_tables, ctx_lens, hkv,
                      scale, nthreads=1):
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_seqs, hq, d = q.shape
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    cl = np.ascontiguousarray(ctx_lens, dtype=np.int32)
    out = np.zeros_like(q)
    lib().dco_paged_attn_decode(_p(q), _p(np.ascontiguousarray(k_arena).view(np.uint16)),
                                _p(np.ascontiguousarray(v_arena).view(np.uint16)), n_layer, layer,
                                _p(bt), bt.shape[1], _p(cl), n_seqs, hq, hkv, d, scale, _p(out),
                                nthreads)
    return out


def kv_append(k, v, k_arena, v_arena, n_layer, layer, block_tables, seq_ids, positions):
    """In place on k_arena / v_arena (float16 arrays)."""
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n_tok, hkv, d = k.shape
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    lib().dco_kv_append(_p(k), _p(v), _p(k_arena), _p(v_arena), n_layer, layer, _p(bt),
                        bt.shape[1], _p(np.ascontiguousarray(seq_ids, dtype=np.int32)),
                        _p(np.ascontiguousarray(positions, dtype=np.int32)), n_tok, hkv, d)


def paged_attn_prefill(q, k_arena, v_arena, n_layer, layer, block_tables, seq_starts, ctx_lens, hkv,
                       scale, nthreads=1):
    """Causal multi-token attention: sequence s's new tokens are rows seq_starts[s] ..
    seq_starts[s+1]-1 of q; token i of its n_s sits at position ctx_lens[s] - n_s + i and attends to
    keys 0 .. that position -- which is decode attention of that token with a context of
    position + 1 keys (inference.cpp:1538-1558 mask semantics, per sequence)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    bt = np.asarray(block_tables, dtype=np.int32)
    rows_bt, ctx_tok = [], []
    for s in range(len(seq_starts) - 1):
        n_s = int(seq_starts[s + 1] - seq_starts[s])
        for i in range(n_s):
            rows_bt.append(bt[s])
            ctx_tok.append(int(ctx_lens[s]) - n_s + i + 1)
    return paged_attn_decode(q, k_arena, v_arena, n_layer, layer, np.stack(rows_bt),
                             np.array(ctx_tok, np.int32), hkv, scale, nthreads)


def ref_flash_attention_gqa(Q, K, V, scale, causal=False):
    """DenseCore FlashAttentionGQA on dense [B,H,S,D] f32 arrays (None if not built)."""
    R = ref_lib()
    if R is None:
        return None
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    B, hq, sq, d = Q.shape
    _, hkv, skv, _ = K.shape
    O = np.zeros_like(Q)
    R.ref_flash_attention_gqa(_p(Q), _p(K), _p(V), _p(O), B, hq, hkv, sq, skv, d, scale,
                              int(causal), 0, 1)
    return O
