"""End-to-end decode step of the Qwen3-architecture decoder vs a CPU reference that chains the oracle
ops (activation quantize + vec_dot mul_mat, paged attention, fp16 KV append) with float64 glue.
Bar: logits within 2e-3 relative (L2 per sequence), next tokens equal."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def tiny(wtype, q6k_alt=()):
    from densecore_b200.decoder import DecoderConfig
    return DecoderConfig("tiny", n_layer=2, hidden=256, n_head=4, n_head_kv=2, head_dim=128, ffn=512,
                         vocab=512, wtype=wtype, q6k_alternate=q6k_alt)


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
        return O.mul_mat(t, rows, kk, xq, x.shape[0], nthreads=8).astype(np.float64)

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
                                  np.array(ctx_lens, np.int32), hkv, 1.0 / math.sqrt(D), nthreads=8)
        x = x + mm(li, "attn_output", att.reshape(B, hq * D).astype(np.float64))
        h = rms(x, nw(p + "ffn_norm.weight"))
        g = mm(li, "ffn_gate", h)
        u = mm(li, "ffn_up", h)
        x = x + mm(li, "ffn_down", g / (1.0 + np.exp(-g)) * u)
    return mm(None, None, rms(x, nw("output_norm.weight")))


@pytest.mark.parametrize("layout", ["q8_0", "q4_k_m"])
def test_decode_step_matches_reference(layout):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200.decoder import Decoder
    from densecore_b200.ggml_types import Q4_K, Q8_0
    cfg = tiny(Q8_0) if layout == "q8_0" else tiny(Q4_K, ("attn_v", "ffn_down"))
    ctx = [5, 17, 33]
    dec = Decoder(cfg, batch=3, max_ctx=64, seed=11)
    dec.fill_kv_random(5)
    tokens = [7, 300, 511]
    dec.tokens.copy_(torch.tensor(tokens))
    dec.ctx_lens.copy_(torch.tensor(ctx, dtype=torch.int32))
    ref = reference_step(dec, tokens, ctx)       # reads the arena before the GPU step mutates it
    dec.replay()                                 # CUDA-graph path
    torch.cuda.synchronize()
    got = dec.logits.cpu().numpy().astype(np.float64)
    err = np.linalg.norm(got - ref, axis=-1) / np.linalg.norm(ref, axis=-1)
    assert err.max() < 2e-3, err
    assert np.array_equal(dec.next_tokens.cpu().numpy(), ref.argmax(-1))
