"""Batched decode step of a Qwen3-architecture decoder on the dcgpu kernels.

This is the caller side of the hot path -- what DenseCore's BuildTransformerGraph does per decode
step (core/src/inference.cpp:1116-1817) for every sequence of a continuous batch -- rebuilt around
the B200 kernels:

  per layer:  act = add_rmsnorm_quantize(x += delta)     (fused: residual, RMSNorm, Q8 quantize)
              qkv = mul_mat_q(W_q|W_k|W_v, act)           (one stacked tensor-core matmul)
              qk_norm_rope_kv_append(qkv)                 (fused: Qwen3 QK-norm, NeoX RoPE, fp16 slots)
              o = paged_attn_decode(q, cache)
              yo = mul_mat_q(W_o, quantize(o))
              act = add_rmsnorm_quantize(x += yo)
              gu = mul_mat_q(W_gate|W_up, act)            (one stacked matmul)
              delta = mul_mat_q(W_down, swiglu_quantize(gu))
  logits = mul_mat(W_out, rmsnorm(x += delta)) (tied embeddings); next = argmax(logits)
  (all dcgpu kernels; torch only gathers the embedding rows and takes the argmax)

Each sequence attends to its own history through its own block table (per-sequence semantics; the
reference's batched path reads seq_id[0]'s history for every sequence).  Weights are random-init
N(0, 0.02) of the named architecture, quantized on the device by the weight encoder; norm weights
are ones.  The step runs as one CUDA graph.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from . import ops
from .ggml_types import Q4_K, Q6_K, Q8_0, Q8_K, VEC_DOT_TYPE

KV_BLOCK = 16


@dataclasses.dataclass
class DecoderConfig:
    name: str
    n_layer: int
    hidden: int
    n_head: int
    n_head_kv: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    # per-layer weight types: default for every linear, overrides by (layer parity, name)
    wtype: int = Q8_0
    q6k_alternate: tuple = ()  # names that are Q6_K in even layers (Q4_K_M layout)


QWEN3_0_6B = DecoderConfig("Qwen3-0.6B", 28, 1024, 16, 8, 128, 3072, 151936, wtype=Q8_0)
QWEN3_4B = DecoderConfig("Qwen3-4B", 36, 2560, 32, 8, 128, 9728, 151936, wtype=Q4_K,
                         q6k_alternate=("attn_v", "ffn_down"))


def _wtype(cfg: DecoderConfig, layer: int, name: str) -> int:
    if name in cfg.q6k_alternate and layer % 2 == 0:
        return Q6_K
    return cfg.wtype


class Decoder:
    """Weights, paged KV cache and the captured decode step for `batch` sequences."""

    def __init__(self, cfg: DecoderConfig, batch: int, max_ctx: int, seed: int = 0,
                 device: str | torch.device = "cuda"):
        self.cfg, self.batch, self.max_ctx = cfg, batch, max_ctx
        dev = self.device = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim
        qd, kvd = cfg.n_head * D, cfg.n_head_kv * D

        def qw(n, k, t):
            w = torch.randn((n, k), generator=g, device=dev) * 0.02
            return ops.QuantWeight.from_float(w, t)

        self.layers = []
        for li in range(cfg.n_layer):
            t_q, t_k, t_v = (_wtype(cfg, li, nm) for nm in ("attn_q", "attn_k", "attn_v"))
            wq = torch.randn((qd, H), generator=g, device=dev) * 0.02
            wk = torch.randn((kvd, H), generator=g, device=dev) * 0.02
            wv = torch.randn((kvd, H), generator=g, device=dev) * 0.02
            L = {"qkv_split": t_v != t_q}
            if t_v == t_q:  # one stacked [q; k; v] weight: rows are quantized independently
                L["attn_qkv"] = ops.QuantWeight.from_float(torch.cat([wq, wk, wv]), t_q)
            else:
                L["attn_qk"] = ops.QuantWeight.from_float(torch.cat([wq, wk]), t_q)
                L["attn_v"] = ops.QuantWeight.from_float(wv, t_v)
            del wq, wk, wv
            L["attn_output"] = qw(H, qd, _wtype(cfg, li, "attn_output"))
            wg = torch.randn((cfg.ffn, H), generator=g, device=dev) * 0.02
            wu = torch.randn((cfg.ffn, H), generator=g, device=dev) * 0.02
            L["ffn_gate_up"] = ops.QuantWeight.from_float(torch.cat([wg, wu]), _wtype(cfg, li, "ffn_gate"))
            del wg, wu
            L["ffn_down"] = qw(H, cfg.ffn, _wtype(cfg, li, "ffn_down"))
            self.layers.append(L)
        # tied embeddings: the LM head is the quantized token embedding; lookups dequantize it
        self.output = qw(cfg.vocab, H, cfg.wtype if cfg.wtype == Q8_0 else Q6_K)
        self.tok_embd = self._dequant_rows(self.output)
        self.ones_h = torch.ones(H, device=dev)
        self.ones_d = torch.ones(D, device=dev)

        # paged KV arena (kv_cache.cpp:353-370 layout): [(block*n_layer + layer)][16][hkv][D] fp16
        self.blocks_per_seq = (max_ctx + KV_BLOCK - 1) // KV_BLOCK
        self.n_blocks = batch * self.blocks_per_seq
        shape = (self.n_blocks * cfg.n_layer, KV_BLOCK, cfg.n_head_kv, D)
        self.k_arena = torch.empty(shape, dtype=torch.float16, device=dev)
        self.v_arena = torch.empty(shape, dtype=torch.float16, device=dev)
        # each sequence owns a shuffled set of physical blocks
        perm = torch.randperm(self.n_blocks, generator=torch.Generator().manual_seed(seed + 1))
        self.block_tables = perm.view(batch, self.blocks_per_seq).to(torch.int32).to(dev)

        # step buffers (static for graph capture)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.ctx_lens = torch.zeros(batch, dtype=torch.int32, device=dev)  # incl. the new token
        self.seq_ids = torch.arange(batch, dtype=torch.int32, device=dev)
        self.next_tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.logits = torch.empty((batch, cfg.vocab), device=dev)
        self._scratch = {}
        self.graph = None

    # ---------------------------------------------------------------- helpers
    def _dequant_rows(self, w: ops.QuantWeight) -> torch.Tensor:
        rows = w.to_ggml()
        n, k = w.n, w.k
        if w.qtype == Q8_0:
            b = rows.view(n, k // 32, 34)
            d = b[..., :2].contiguous().view(torch.float16).float()
            q = b[..., 2:].contiguous().view(torch.int8).float()
            return (q * d).reshape(n, k).to(torch.float16)
        # Q6_K: ql[128] qh[64] sc[16] d[2] per 256 (gguf layout)
        b = rows.view(n, k // 256, 210)
        ql, qh = b[..., :128].to(torch.int32), b[..., 128:192].to(torch.int32)
        sc = b[..., 192:208].contiguous().view(torch.int8).float()
        d = b[..., 208:210].contiguous().view(torch.float16).float()
        out = torch.empty((n, k // 256, 256), device=rows.device)
        for h in range(2):
            for grp in range(4):
                lo = (ql[..., h * 64 + (grp & 1) * 32: h * 64 + (grp & 1) * 32 + 32] >> (4 * (grp >> 1))) & 15
                hi = (qh[..., h * 32: h * 32 + 32] >> (2 * grp)) & 3
                q = (lo | (hi << 4)) - 32
                e0 = h * 128 + grp * 32
                out[..., e0:e0 + 32] = q.float() * sc[..., (e0 // 16):(e0 // 16) + 2].repeat_interleave(16, -1)
        return (out * d).reshape(n, k).to(torch.float16)

    def _buf(self, key, shape, dtype=torch.float32, zero=False):
        t = self._scratch.get(key)
        if t is None or t.shape != torch.Size(shape):
            t = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=self.device)
            self._scratch[key] = t
        return t

    def _mm(self, key, w: ops.QuantWeight, act, m):
        out = self._buf(("y", key), (m, w.n))
        scr = self._buf(("qs", key), (max(1, ops.mul_mat_q_scratch_size(w.qtype, w.n, w.k, m)),),
                        torch.uint8, zero=True)
        return ops.mul_mat_q(w, act, m, out=out, scratch=scr)

    # ---------------------------------------------------------------- the step
    def ggml_rows(self, li: int, name: str):
        """(ggml rows as numpy, type, k) of one logical weight (unstacking the fused ones)."""
        cfg, D = self.cfg, self.cfg.head_dim
        qd, kvd = cfg.n_head * D, cfg.n_head_kv * D
        L = self.layers[li]
        spans = {"attn_q": (0, qd), "attn_k": (qd, qd + kvd), "attn_v": (qd + kvd, qd + 2 * kvd),
                 "ffn_gate": (0, cfg.ffn), "ffn_up": (cfg.ffn, 2 * cfg.ffn)}
        if name in ("attn_output", "ffn_down") or (name == "attn_v" and L["qkv_split"]):
            w = L[name]
            return w.to_ggml().cpu().numpy(), w.qtype, w.k
        key = "ffn_gate_up" if name.startswith("ffn") else ("attn_qk" if L["qkv_split"] else "attn_qkv")
        w = L[key]
        a, b = spans[name]
        return w.to_ggml().cpu().numpy()[a:b], w.qtype, w.k

    def step(self):
        """One decode token for every sequence: reads self.tokens / self.ctx_lens, writes
        self.next_tokens and self.logits, appends K/V at position ctx_len-1.  Per layer: fused
        add+RMSNorm+quantize, stacked QKV matmul, fused QK-norm+RoPE+KV append, paged attention,
        quantize, O matmul, fused add+RMSNorm+quantize, stacked gate|up matmul, fused
        SwiGLU+quantize, down matmul (its output is added by the next layer's norm kernel)."""
        cfg, B = self.cfg, self.batch
        D, hq, hkv, H = cfg.head_dim, cfg.n_head, cfg.n_head_kv, cfg.hidden
        qd, kvd = hq * D, hkv * D
        pos = self._buf("pos", (B,), torch.int32)
        torch.sub(self.ctx_lens, 1, out=pos)
        x = self._buf("x", (B, H))
        x.copy_(self.tok_embd[self.tokens])
        scale = 1.0 / math.sqrt(D)
        q_rot = self._buf("q_rot", (B, hq, D))
        attn_out = self._buf("attn_out", (B, hq, D))
        attn_scr = self._buf("attn_scr", (max(1, ops.paged_attn_scratch_size(B, hq, hkv, self.max_ctx)),),
                             torch.uint8)
        delta = None
        for li, L in enumerate(self.layers):
            wqk = L["attn_qk"] if L["qkv_split"] else L["attn_qkv"]
            act = self._actbuf(("attn", wqk.qtype), B, H, wqk.qtype)
            ops.add_rmsnorm_quantize(x, self.ones_h, cfg.rms_eps, VEC_DOT_TYPE[wqk.qtype], act, delta)
            yqk = self._mm(("qkv", li), wqk, act, B)
            if L["qkv_split"]:
                wv = L["attn_v"]
                act_v = act
                if VEC_DOT_TYPE[wv.qtype] != VEC_DOT_TYPE[wqk.qtype]:
                    act_v = self._actbuf(("attn_v", wv.qtype), B, H, wv.qtype)
                    ops.add_rmsnorm_quantize(x, self.ones_h, cfg.rms_eps, VEC_DOT_TYPE[wv.qtype], act_v)
                yv, ldv = self._mm(("v", li), wv, act_v, B), kvd
            else:
                yv, ldv = yqk[:, qd + kvd:], wqk.n
            ops.qk_norm_rope_kv_append(yqk, wqk.n, yqk[:, qd:], wqk.n, yv, ldv, B, hq, hkv, self.ones_d,
                                       self.ones_d, cfg.rms_eps, cfg.rope_theta, pos, q_rot,
                                       self.k_arena, self.v_arena, cfg.n_layer, li, self.block_tables)
            ops.paged_attn_decode(q_rot, self.k_arena, self.v_arena, cfg.n_layer, li, self.block_tables,
                                  self.ctx_lens, hkv, self.max_ctx, scale, out=attn_out, scratch=attn_scr)
            wo = L["attn_output"]
            act_o = self._actbuf(("o", wo.qtype), B, qd, wo.qtype)
            ops.quantize_act(attn_out.view(B, qd), VEC_DOT_TYPE[wo.qtype], out=act_o)
            yo = self._mm(("o", li), wo, act_o, B)
            wgu = L["ffn_gate_up"]
            act_f = self._actbuf(("ffn", wgu.qtype), B, H, wgu.qtype)
            ops.add_rmsnorm_quantize(x, self.ones_h, cfg.rms_eps, VEC_DOT_TYPE[wgu.qtype], act_f, yo)
            ygu = self._mm(("gu", li), wgu, act_f, B)
            wd = L["ffn_down"]
            act_d = self._actbuf(("down", wd.qtype), B, cfg.ffn, wd.qtype)
            ops.swiglu_quantize(ygu, ygu[:, cfg.ffn:], 2 * cfg.ffn, B, cfg.ffn, VEC_DOT_TYPE[wd.qtype], act_d)
            delta = self._mm(("down", li), wd, act_d, B)
        act_h = self._actbuf(("head", self.output.qtype), B, H, self.output.qtype)
        ops.add_rmsnorm_quantize(x, self.ones_h, cfg.rms_eps, VEC_DOT_TYPE[self.output.qtype], act_h, delta)
        self.logits.copy_(self._mm(("head",), self.output, act_h, B))
        self.next_tokens.copy_(torch.argmax(self.logits, dim=-1))

    def _actbuf(self, key, m, k, wtype):
        at = VEC_DOT_TYPE[wtype]
        return self._buf(("act", key, at, k), (int(ops._lib.load().dcg_act_size(at, m, k)),), torch.uint8)

    def capture(self):
        """Capture step() into a CUDA graph (buffers are static)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.step()  # allocates every scratch buffer outside the capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        return self.graph

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def fill_kv_random(self, seed: int = 3):
        """Seeded random history for every slot (stands in for prefill when timing decode)."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        self.k_arena.normal_(0.0, 1.0, generator=g)
        self.v_arena.normal_(0.0, 1.0, generator=g)

    # bytes one decode step must read at least (weights + KV history), for the roofline
    def step_bytes(self, ctx_lens) -> int:
        w = sum(wt.nbytes for L in self.layers for wt in L.values()
                if isinstance(wt, ops.QuantWeight)) + self.output.nbytes
        kv = int(sum(int(c) for c in ctx_lens)) * self.cfg.n_layer * 2 * self.cfg.n_head_kv * \
            self.cfg.head_dim * 2
        return w + kv
