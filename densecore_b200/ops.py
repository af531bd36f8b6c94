"""Torch-facing operators over libdcgpu.so.  torch only provides device memory and the current
stream; all arithmetic runs in the sm_100a kernels.  Names follow the reference operator surface:

  quantize_row_q8_0 / quantize_row_q8_K  ggml from_float (core/src/inference.cpp:887-894)
  mul_mat                                 smart_mul_mat / cb_gemv_custom / ggml_mul_mat on a
                                          quantized weight (inference.cpp:1043-1064, :840-948)
  QuantWeight                             a weight tensor resident on the device (the
                                          weight_tensor->data of cb_gemv_custom, uploaded once)
  HostContext                             the synchronous host-pointer boundary (dcg_ctx_*)
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .ggml_types import Q4_K, Q6_K, Q8_0, Q8_K, VEC_DOT_TYPE, block_size, row_size


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _check_cuda(t: torch.Tensor, name: str, dtype=None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def _quantize_rows(fn: str, qtype: int, x: torch.Tensor, out: torch.Tensor | None):
    _check_cuda(x, "x", torch.float32)
    k = x.shape[-1]
    m = x.numel() // k
    if out is None:
        out = torch.empty((m, row_size(qtype, k)), dtype=torch.uint8, device=x.device)
    _lib.check(getattr(_lib.load(), fn)(_ptr(x), _ptr(out), m, k, _stream()), fn)
    return out


def quantize_row_q8_0(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """f32 [..., k] -> ggml Q8_0 rows (uint8 [m, k/32*34])."""
    return _quantize_rows("dcg_quantize_row_q8_0", Q8_0, x, out)


def quantize_row_q8_K(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """f32 [..., k] -> ggml Q8_K rows (uint8 [m, k/256*292])."""
    return _quantize_rows("dcg_quantize_row_q8_K", Q8_K, x, out)


def quantize_weights(x: torch.Tensor, qtype: int) -> torch.Tensor:
    """Encode an f32 [n, k] weight as ggml Q8_0 / Q4_K / Q6_K rows on the device."""
    _check_cuda(x, "x", torch.float32)
    n, k = x.shape
    out = torch.empty((n, row_size(qtype, k)), dtype=torch.uint8, device=x.device)
    _lib.check(_lib.load().dcg_quantize_weights(qtype, _ptr(x), _ptr(out), n, k, _stream()),
               "dcg_quantize_weights")
    return out


class QuantWeight:
    """An n x k quantized weight in the device layout the matmul streams (dcg_weight_pack)."""

    def __init__(self, qtype: int, n: int, k: int, packed: torch.Tensor):
        self.qtype, self.n, self.k, self.packed = qtype, n, k, packed

    @classmethod
    def from_ggml(cls, rows: torch.Tensor, qtype: int, k: int) -> "QuantWeight":
        """rows: uint8 [n, >=row_size] ggml rows on the device (tensor nb[1] = rows.stride(0))."""
        _check_cuda(rows, "rows", torch.uint8)
        n = rows.shape[0]
        L = _lib.load()
        nbytes = L.dcg_packed_weight_size(qtype, n, k)
        if nbytes == 0:
            raise ValueError(f"unsupported weight type {qtype}")
        packed = torch.empty(nbytes, dtype=torch.uint8, device=rows.device)
        _lib.check(L.dcg_weight_pack(qtype, _ptr(rows), rows.stride(0), n, k, _ptr(packed),
                                     _stream()), "dcg_weight_pack")
        return cls(qtype, n, k, packed)

    @classmethod
    def from_float(cls, w: torch.Tensor, qtype: int) -> "QuantWeight":
        return cls.from_ggml(quantize_weights(w, qtype), qtype, w.shape[1])

    def to_ggml(self) -> torch.Tensor:
        rows = torch.empty((self.n, row_size(self.qtype, self.k)), dtype=torch.uint8,
                           device=self.packed.device)
        _lib.check(_lib.load().dcg_weight_unpack(self.qtype, _ptr(self.packed), self.n, self.k,
                                                 _ptr(rows), rows.stride(0), _stream()),
                   "dcg_weight_unpack")
        return rows

    @property
    def nbytes(self) -> int:
        """Algorithmic bytes (ggml block bytes) of the weight."""
        return self.n * row_size(self.qtype, self.k)


def mul_mat_scratch_size(qtype: int, n: int, k: int, m: int) -> int:
    return int(_lib.load().dcg_mul_mat_scratch_size(qtype, n, k, m))


def mul_mat_q_scratch_size(qtype: int, n: int, k: int, m: int) -> int:
    return int(_lib.load().dcg_mul_mat_q_scratch_size(qtype, n, k, m))


def mul_mat(w: QuantWeight, x: torch.Tensor, out: torch.Tensor | None = None,
            scratch: torch.Tensor | None = None) -> torch.Tensor:
    """y[m, n] = x[m, k] . W[n, k]^T with x quantized on the fly to W's vec_dot_type."""
    _check_cuda(x, "x", torch.float32)
    if x.shape[-1] != w.k:
        raise ValueError(f"x has k={x.shape[-1]}, weight has k={w.k}")
    m = x.numel() // w.k
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=x.device)
    need = mul_mat_scratch_size(w.qtype, w.n, w.k, m)
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
    _lib.check(_lib.load().dcg_mul_mat(w.qtype, _ptr(w.packed), w.n, w.k, _ptr(x), m, _ptr(out),
                                       _ptr(scratch), scratch.numel(), _stream()), "dcg_mul_mat")
    return out


def quantize_act(x: torch.Tensor, act_type: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """f32 [m, k] -> device-layout activation (dcg_quantize_act) for mul_mat_q."""
    _check_cuda(x, "x", torch.float32)
    k = x.shape[-1]
    m = x.numel() // k
    L = _lib.load()
    if out is None:
        out = torch.empty(L.dcg_act_size(act_type, m, k), dtype=torch.uint8, device=x.device)
    _lib.check(L.dcg_quantize_act(act_type, _ptr(x), _ptr(out), m, k, _stream()), "dcg_quantize_act")
    return out


def mul_mat_q(w: QuantWeight, act: torch.Tensor, m: int, out: torch.Tensor | None = None,
              scratch: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """y[m, n] = W . act with act from quantize_act(x, VEC_DOT_TYPE[w.qtype])."""
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=act.device)
    if scratch is None:
        scratch = torch.zeros(max(1, mul_mat_q_scratch_size(w.qtype, w.n, w.k, m)),
                              dtype=torch.uint8, device=act.device)
    _lib.check(_lib.load().dcg_mul_mat_q(w.qtype, _ptr(w.packed), w.n, w.k, _ptr(act), m,
                                         _ptr(out), _ptr(scratch), scratch.numel(),
                                         _stream(stream)), "dcg_mul_mat_q")
    return out


def paged_attn_scratch_size(n_seqs: int, hq: int, hkv: int, max_ctx: int, head_dim: int = 128) -> int:
    return int(_lib.load().dcg_paged_attn_scratch_size(n_seqs, hq, hkv, head_dim, max_ctx))


def paged_attn_decode(q: torch.Tensor, k_arena: torch.Tensor, v_arena: torch.Tensor, n_layer: int,
                      layer: int, block_tables: torch.Tensor, ctx_lens: torch.Tensor, hkv: int,
                      max_ctx: int, scale: float | None = None, out: torch.Tensor | None = None,
                      scratch: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention of one query token per sequence over the paged fp16 KV arena.

    q [n_seqs, hq, 128] f32; k/v_arena fp16 (any shape, layout of dcgpu.h); block_tables
    [n_seqs, max_blocks] int32; ctx_lens [n_seqs] int32 (<= max_ctx)."""
    _check_cuda(q, "q", torch.float32)
    for t, nm in ((k_arena, "k_arena"), (v_arena, "v_arena")):
        _check_cuda(t, nm, torch.float16)
    _check_cuda(block_tables, "block_tables", torch.int32)
    _check_cuda(ctx_lens, "ctx_lens", torch.int32)
    n_seqs, hq, hd = q.shape
    if scale is None:
        scale = 1.0 / float(hd) ** 0.5
    if out is None:
        out = torch.empty_like(q)
    need = paged_attn_scratch_size(n_seqs, hq, hkv, max_ctx, hd)
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    n_arena_blocks = k_arena.numel() // (16 * hkv * hd * n_layer)
    _lib.check(_lib.load().dcg_paged_attn_decode(
        _ptr(q), _ptr(k_arena), _ptr(v_arena), n_arena_blocks, n_layer, layer, _ptr(block_tables),
        block_tables.shape[1], _ptr(ctx_lens), n_seqs, hq, hkv, hd, max_ctx, scale, _ptr(out),
        _ptr(scratch), scratch.numel(), _stream()), "dcg_paged_attn_decode")
    return out


def paged_attn_prefill(q: torch.Tensor, k_arena: torch.Tensor, v_arena: torch.Tensor, n_layer: int,
                       layer: int, block_tables: torch.Tensor, seq_starts: torch.Tensor, ctx_lens: torch.Tensor,
                       hkv: int, max_seq_tokens: int, max_ctx: int, scale: float | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of several new tokens per sequence over the paged fp16 KV arena.

    q [n_tok, hq, 128] f32, sequence s's tokens are rows seq_starts[s] .. seq_starts[s+1]-1
    (seq_starts [n_seqs + 1] int32); its i-th new token sits at position ctx_lens[s] - n_s + i
    (K/V already appended) and attends to keys 0 .. that position."""
    _check_cuda(q, "q", torch.float32)
    for t, nm in ((k_arena, "k_arena"), (v_arena, "v_arena")):
        _check_cuda(t, nm, torch.float16)
    for t, nm in ((block_tables, "block_tables"), (seq_starts, "seq_starts"), (ctx_lens, "ctx_lens")):
        _check_cuda(t, nm, torch.int32)
    n_tok, hq, hd = q.shape
    n_seqs = seq_starts.numel() - 1
    if scale is None:
        scale = 1.0 / float(hd) ** 0.5
    if out is None:
        out = torch.empty_like(q)
    n_arena_blocks = k_arena.numel() // (16 * hkv * hd * n_layer)
    _lib.check(_lib.load().dcg_paged_attn_prefill(
        _ptr(q), _ptr(k_arena), _ptr(v_arena), n_arena_blocks, n_layer, layer, _ptr(block_tables),
        block_tables.shape[1], _ptr(seq_starts), _ptr(ctx_lens), n_seqs, max_seq_tokens, hq, hkv, hd, max_ctx,
        scale, _ptr(out), _stream()), "dcg_paged_attn_prefill")
    return out


def kv_append(k: torch.Tensor, v: torch.Tensor, k_arena: torch.Tensor, v_arena: torch.Tensor,
              n_layer: int, layer: int, block_tables: torch.Tensor, seq_ids: torch.Tensor,
              positions: torch.Tensor) -> None:
    """Write n_tok tokens' K/V ([n_tok, hkv, hd] f32) into their fp16 slots (in place)."""
    for t, nm in ((k, "k"), (v, "v")):
        _check_cuda(t, nm, torch.float32)
    n_tok, hkv, hd = k.shape
    _lib.check(_lib.load().dcg_kv_append(
        _ptr(k), _ptr(v), _ptr(k_arena), _ptr(v_arena), n_layer, layer, _ptr(block_tables),
        block_tables.shape[1], _ptr(seq_ids), _ptr(positions), n_tok, hkv, hd, _stream()),
        "dcg_kv_append")


def add_rmsnorm_quantize(x: torch.Tensor, weight: torch.Tensor, eps: float, act_type: int,
                         act: torch.Tensor, delta: torch.Tensor | None = None) -> torch.Tensor:
    """x += delta (in place, optional); act = quantize(rmsnorm(x) * weight)."""
    m, k = x.shape
    _lib.check(_lib.load().dcg_add_rmsnorm_quantize(
        _ptr(x), _ptr(delta) if delta is not None else None, _ptr(weight), eps, m, k, act_type,
        _ptr(act), _stream()), "dcg_add_rmsnorm_quantize")
    return act


def swiglu_quantize(gate: torch.Tensor, up: torch.Tensor, ld: int, m: int, ffn: int, act_type: int,
                    act: torch.Tensor) -> torch.Tensor:
    """act = quantize(silu(gate) * up) over rows of `ffn` values with row stride `ld`."""
    _lib.check(_lib.load().dcg_swiglu_quantize(_ptr(gate), _ptr(up), ld, m, ffn, act_type, _ptr(act),
                                               _stream()), "dcg_swiglu_quantize")
    return act


def qk_norm_rope_kv_append(q, ldq, k, ldk, v, ldv, n_seqs, hq, hkv, q_norm_w, k_norm_w, eps, theta,
                           positions, q_out, k_arena, v_arena, n_layer, layer, block_tables):
    """Per-head RMSNorm + NeoX RoPE of q and k; q -> q_out, k/v -> fp16 paged slots."""
    _lib.check(_lib.load().dcg_qk_norm_rope_kv_append(
        _ptr(q), ldq, _ptr(k), ldk, _ptr(v), ldv, n_seqs, hq, hkv, 128,
        _ptr(q_norm_w) if q_norm_w is not None else None,
        _ptr(k_norm_w) if k_norm_w is not None else None,
        eps, theta, _ptr(positions), _ptr(q_out), _ptr(k_arena), _ptr(v_arena), n_layer, layer,
        _ptr(block_tables), block_tables.shape[1], _stream()), "dcg_qk_norm_rope_kv_append")


def qk_norm_rope_kv_append_tokens(q, ldq, k, ldk, v, ldv, n_tok, hq, hkv, q_norm_w, k_norm_w, eps, theta,
                                  seq_ids, positions, q_out, k_arena, v_arena, n_layer, layer, block_tables):
    """qk_norm_rope_kv_append for token rows of any sequences (row i: sequence seq_ids[i])."""
    _lib.check(_lib.load().dcg_qk_norm_rope_kv_append_tokens(
        _ptr(q), ldq, _ptr(k), ldk, _ptr(v), ldv, n_tok, hq, hkv, 128,
        _ptr(q_norm_w) if q_norm_w is not None else None,
        _ptr(k_norm_w) if k_norm_w is not None else None,
        eps, theta, _ptr(seq_ids), _ptr(positions), _ptr(q_out), _ptr(k_arena), _ptr(v_arena), n_layer, layer,
        _ptr(block_tables), block_tables.shape[1], _stream()), "dcg_qk_norm_rope_kv_append_tokens")


class HostContext:
    """The synchronous host boundary: weights registered once by host pointer, per-call host
    activations in and host results out (dcg_ctx_*)."""

    def __init__(self, device: int = 0):
        self._L = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(self._L.dcg_ctx_create(device, ctypes.byref(h)), "dcg_ctx_create")
        self.h = h
        self._keep = {}
        self._mm = self._L.dcg_ctx_mul_mat

    def register(self, rows: np.ndarray, qtype: int, k: int):
        rows = np.ascontiguousarray(rows, dtype=np.uint8)
        n = rows.shape[0]
        w = ctypes.c_void_p()
        _lib.check(self._L.dcg_ctx_weight_register(self.h, qtype, rows.ctypes.data, rows.strides[0],
                                                   n, k, ctypes.byref(w)),
                   "dcg_ctx_weight_register")
        self._keep[w.value] = (rows, n, k)
        return w

    def mul_mat(self, w, x: np.ndarray) -> np.ndarray:
        rows, n, k = self._keep[w.value]
        if not (x.dtype == np.float32 and x.flags.c_contiguous):
            x = np.ascontiguousarray(x, dtype=np.float32)
        m = x.size // k
        if m * k != x.size:
            raise ValueError(f"x has {x.size} elements, not a multiple of k={k}")
        y = np.empty((m, n), dtype=np.float32)
        rc = self._mm(self.h, w, x.ctypes.data, m, y.ctypes.data)
        if rc:
            _lib.check(rc, "dcg_ctx_mul_mat")
        return y

    def close(self):
        if self.h:
            self._L.dcg_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
