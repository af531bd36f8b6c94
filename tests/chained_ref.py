"""CPU reference of one decode step: chains the oracle ops (activation quantize + vec_dot mul_mat,
paged attention, fp16 KV append) with float64 glue for the norms, RoPE, SwiGLU and residuals.
Test infrastructure only (imported by the GPU decode tests)."""
import math
import os

import numpy as np

from oracle import oracle as O

NTHREADS = max(1, min(32, os.cpu_count() or 1))


def reference_step(dec, tokens, ctx_lens, norms=None):
    """norms: GGUF-named norm weight vectors (default: ones, the random-init decoder's)."""
    cfg = dec.cfg
    nw = (lambda name: norms[name].astype(np.float64)) if norms else (lambda name: 1.0)
    B, D, hq, hkv = dec.batch, cfg.head_dim, cfg.n_head, cfg.n_head_kv
    ka = dec.k_arena.cpu().numpy().copy()
    va = dec.v_arena.cpu().numpy().copy()
    bt = dec.block_tables.cpu().numpy()
    pos = np.array(ctx_lens) - 1
    inv = 1.0 / (cfg.rope_theta ** (np.arange(0, D, 2, dtype=np.float64) / D))

    def rms(x, w=1.0):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg.rms_eps) * w

    def rope(x):
        ang = pos[:, None].astype(np.float64) * inv[None, :]
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        x1, x2 = x[..., : D // 2], x[..., D // 2:]
        return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    def mm(li, name, x):
        rows, t, kk = dec.ggml_rows(li, name) if li is not None else (
            dec.output.to_ggml().cpu().numpy(), dec.output.qtype, dec.output.k)
        rows = np.ascontiguousarray(rows)
        xq = O.quantize(x.astype(np.float32), O.VEC_DOT_TYPE[t])
        return O.mul_mat(t, rows, kk, xq, x.shape[0], nthreads=NTHREADS, simd=True).astype(np.float64)

    x = dec.tok_embd.cpu().float().numpy().astype(np.float64)[tokens]
    for li in range(cfg.n_layer):
        p = f"blk.{li}."
        h = rms(x, nw(p + "attn_norm.weight"))
        q = mm(li, "attn_q", h).reshape(B, hq, D)
        k = mm(li, "attn_k", h).reshape(B, hkv, D)
        v = mm(li, "attn_v", h).reshape(B, hkv, D)
        if cfg.qk_norm:
            q, k = rms(q, nw(p + "attn_q_norm.weight")), rms(k, nw(p + "attn_k_norm.weight"))
        q, k = rope(q), rope(k)
        O.kv_append(k.astype(np.float32), v.astype(np.float32), ka, va, cfg.n_layer, li, bt,
                    np.arange(B, dtype=np.int32), pos.astype(np.int32))
        att = O.paged_attn_decode(q.astype(np.float32), ka, va, cfg.n_layer, li, bt,
                                  np.array(ctx_lens, np.int32), hkv, 1.0 / math.sqrt(D), nthreads=NTHREADS)
        x = x + mm(li, "attn_output", att.reshape(B, hq * D).astype(np.float64))
        h = rms(x, nw(p + "ffn_norm.weight"))
        g = mm(li, "ffn_gate", h)
        u = mm(li, "ffn_up", h)
        x = x + mm(li, "ffn_down", g / (1.0 + np.exp(-g)) * u)
    return mm(None, None, rms(x, nw("output_norm.weight")))
