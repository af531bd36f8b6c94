"""CPU reference of one decode step: chains the oracle ops (activation quantize + vec_dot mul_mat,
paged attention, fp16 KV append) with the element-wise glue restated in ggml's fp32 arithmetic, so
that the activations the quantizers see round the same way on both sides:
  rms_norm   fp32 squares summed in double, mean rounded to fp32, scale = 1.0f / sqrtf(mean + eps),
             y = (x * scale) * weight (each product rounded to fp32)
  rope       NeoX rotate-half; theta_0 = p, theta_{i+1} = theta_i * powf(base, -2 / n_dims) in fp32;
             x0 cos - x1 sin, x0 sin + x1 cos with fp32 cosf / sinf
  silu       g / (1 + expf(-g)) in fp32, then * up
  residuals  fp32 adds
Test infrastructure only (imported by the GPU decode tests)."""
import ctypes
import ctypes.util
import math
import os

import numpy as np

from oracle import oracle as O

NTHREADS = max(1, min(32, os.cpu_count() or 1))
_libm = ctypes.CDLL(ctypes.util.find_library("m"))
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
f32 = np.float32


def rms_norm(x, w=None, eps=1e-6):
    x = np.asarray(x, f32)
    sq = (x * x).astype(np.float64).sum(-1, keepdims=True)
    mean = (sq / x.shape[-1]).astype(f32)
    scale = (f32(1.0) / np.sqrt(mean + f32(eps))).astype(f32)
    y = (x * scale).astype(f32)
    return y if w is None else (y * np.asarray(w, f32)).astype(f32)


def rope_neox(x, pos, base):
    """x [B, heads, D] fp32, pos [B] int: ggml's fp32 angle recurrence and rotation."""
    D = x.shape[-1]
    ts = f32(_libm.powf(f32(base), f32(-2.0 / D)))
    theta = np.empty((len(pos), D // 2), f32)
    t = np.asarray(pos, f32)
    for i in range(D // 2):
        theta[:, i] = t
        t = (t * ts).astype(f32)
    c, s = np.cos(theta)[:, None, :].astype(f32), np.sin(theta)[:, None, :].astype(f32)
    x0, x1 = x[..., : D // 2], x[..., D // 2:]
    return np.concatenate([(x0 * c).astype(f32) - (x1 * s).astype(f32),
                           (x0 * s).astype(f32) + (x1 * c).astype(f32)], -1).astype(f32)


def reference_step(dec, tokens, ctx_lens, norms=None):
    """norms: GGUF-named norm weight vectors (default: ones, the random-init decoder's)."""
    cfg = dec.cfg
    nw = (lambda name: np.asarray(norms[name], f32)) if norms else (lambda name: None)
    B, D, hq, hkv = dec.batch, cfg.head_dim, cfg.n_head, cfg.n_head_kv
    ka = dec.k_arena.cpu().numpy().copy()
    va = dec.v_arena.cpu().numpy().copy()
    bt = dec.block_tables.cpu().numpy()
    pos = np.array(ctx_lens) - 1

    def mm(li, name, x):
        rows, t, kk = dec.ggml_rows(li, name) if li is not None else (
            dec.output.to_ggml().cpu().numpy(), dec.output.qtype, dec.output.k)
        rows = np.ascontiguousarray(rows)
        xq = O.quantize(np.asarray(x, f32), O.VEC_DOT_TYPE[t])
        return O.mul_mat(t, rows, kk, xq, x.shape[0], nthreads=NTHREADS, simd=True)

    x = dec.tok_embd.cpu().float().numpy().astype(f32)[tokens]
    for li in range(cfg.n_layer):
        p = f"blk.{li}."
        h = rms_norm(x, nw(p + "attn_norm.weight"), cfg.rms_eps)
        q = mm(li, "attn_q", h).reshape(B, hq, D)
        k = mm(li, "attn_k", h).reshape(B, hkv, D)
        v = mm(li, "attn_v", h).reshape(B, hkv, D)
        if cfg.qk_norm:
            q = rms_norm(q, nw(p + "attn_q_norm.weight"), cfg.rms_eps)
            k = rms_norm(k, nw(p + "attn_k_norm.weight"), cfg.rms_eps)
        q, k = rope_neox(q, pos, cfg.rope_theta), rope_neox(k, pos, cfg.rope_theta)
        O.kv_append(k, v.astype(f32), ka, va, cfg.n_layer, li, bt, np.arange(B, dtype=np.int32),
                    pos.astype(np.int32))
        att = O.paged_attn_decode(q, ka, va, cfg.n_layer, li, bt, np.array(ctx_lens, np.int32), hkv,
                                  1.0 / math.sqrt(D), nthreads=NTHREADS)
        x = (x + mm(li, "attn_output", att.reshape(B, hq * D))).astype(f32)
        h = rms_norm(x, nw(p + "ffn_norm.weight"), cfg.rms_eps)
        g = mm(li, "ffn_gate", h)
        u = mm(li, "ffn_up", h)
        silu = (g / (f32(1.0) + np.exp(-g).astype(f32))).astype(f32)
        x = (x + mm(li, "ffn_down", (silu * u).astype(f32))).astype(f32)
    return mm(None, None, rms_norm(x, nw("output_norm.weight"), cfg.rms_eps)).astype(np.float64)
