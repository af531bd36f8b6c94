"""Batched decode step of a Qwen3-architecture decoder on the dcgpu kernels.

This is the caller side of the hot path -- what DenseCore's BuildTransformerGraph does per decode
step (core/src/inference.cpp:1116-1817) for every sequence of a continuous batch -- rebuilt around
the B200 kernels:

  per layer:  h = rmsnorm(x)                      (torch)
              act = quantize_act(h)                (dcgpu, one Q8 activation for q/k/v)
              q, k, v = mul_mat_q(W_q|W_k|W_v, act)  (dcgpu tensor-core matmul)
              q, k = qk_norm, rope(q, k)           (torch; Qwen3 per-head RMSNorm, NeoX RoPE)
              kv_append(k, v)                      (dcgpu, fp16 paged slots)
              o = paged_attn_decode(q, cache)      (dcgpu)
              x += mul_mat(W_o, o)
              h = rmsnorm(x); act = quantize_act(h)
              x += mul_mat(W_down, silu(mul_mat_q(W_gate, act)) * mul_mat_q(W_up, act))
  logits = mul_mat(W_out, rmsnorm(x)) (tied embeddings); next = argmax(logits)

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
            L = {
                "attn_q": qw(qd, H, _wtype(cfg, li, "attn_q")),
                "attn_k": qw(kvd, H, _wtype(cfg, li, "attn_k")),
                "attn_v": qw(kvd, H, _wtype(cfg, li, "attn_v")),
                "attn_output": qw(H, qd, _wtype(cfg, li, "attn_output")),
                "ffn_gate": qw(cfg.ffn, H, _wtype(cfg, li, "ffn_gate")),
                "ffn_up": qw(cfg.ffn, H, _wtype(cfg, li, "ffn_up")),
                "ffn_down": qw(H, cfg.ffn, _wtype(cfg, li, "ffn_down")),
            }
            self.layers.append(L)
        # tied embeddings: the LM head is the quantized token embedding; lookups dequantize it
        self.output = qw(cfg.vocab, H, cfg.wtype if cfg.wtype == Q8_0 else Q6_K)
        self.tok_embd = self._dequant_rows(self.output)
        self.ones_h = torch.ones(H, device=dev)
        self.ones_d = torch.ones(D, device=dev)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=dev, dtype=torch.float64) / D))
        self.inv_freq = inv.float()

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

    def _rms(self, x, w, eps):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _rope(self, x, pos):
        # NeoX rotate-half over head_dim; x [B, H, D], pos [B]
        ang = pos.float()[:, None] * self.inv_freq[None, :]  # [B, D/2]
        cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    def _mm(self, key, w: ops.QuantWeight, act, m):
        out = self._buf(("y", key), (m, w.n))
        scr = self._buf(("qs", key), (max(1, ops.mul_mat_q_scratch_size(w.qtype, w.n, w.k, m)),),
                        torch.uint8, zero=True)
        return ops.mul_mat_q(w, act, m, out=out, scratch=scr)

    def _act(self, key, x, qtype):
        at = VEC_DOT_TYPE[qtype]
        m, k = x.shape
        buf = self._buf(("act", key, at), (int(ops._lib.load().dcg_act_size(at, m, k)),), torch.uint8)
        return ops.quantize_act(x.contiguous(), at, out=buf)

    # ---------------------------------------------------------------- the step
    def step(self):
        """One decode token for every sequence: reads self.tokens / self.ctx_lens, writes
        self.next_tokens and self.logits, appends K/V at position ctx_len-1."""
        cfg, B = self.cfg, self.batch
        D, hq, hkv = cfg.head_dim, cfg.n_head, cfg.n_head_kv
        pos = (self.ctx_lens - 1).to(torch.int32)
        x = self.tok_embd[self.tokens].float()
        scale = 1.0 / math.sqrt(D)
        attn_out = self._buf("attn_out", (B, hq, D))
        attn_scr = self._buf("attn_scr", (max(1, ops.paged_attn_scratch_size(B, hq, hkv, self.max_ctx)),),
                             torch.uint8)
        for li, L in enumerate(self.layers):
            h = self._rms(x, self.ones_h, cfg.rms_eps)
            a_q = self._act(("attn", L["attn_q"].qtype), h, L["attn_q"].qtype)
            a_v = a_q if VEC_DOT_TYPE[L["attn_v"].qtype] == VEC_DOT_TYPE[L["attn_q"].qtype] else \
                self._act(("attn_v", L["attn_v"].qtype), h, L["attn_v"].qtype)
            q = self._mm(("q", li), L["attn_q"], a_q, B).view(B, hq, D)
            k = self._mm(("k", li), L["attn_k"], a_q, B).view(B, hkv, D)
            v = self._mm(("v", li), L["attn_v"], a_v, B).view(B, hkv, D)
            q = self._rope(self._rms(q, self.ones_d, cfg.rms_eps), pos).contiguous()
            k = self._rope(self._rms(k, self.ones_d, cfg.rms_eps), pos).contiguous()
            ops.kv_append(k, v.contiguous(), self.k_arena, self.v_arena, cfg.n_layer, li,
                          self.block_tables, self.seq_ids, pos)
            ops.paged_attn_decode(q, self.k_arena, self.v_arena, cfg.n_layer, li, self.block_tables,
                                  self.ctx_lens, hkv, self.max_ctx, scale, out=attn_out,
                                  scratch=attn_scr)
            a_o = self._act(("o", L["attn_output"].qtype), attn_out.view(B, hq * D), L["attn_output"].qtype)
            x = x + self._mm(("o", li), L["attn_output"], a_o, B)
            h = self._rms(x, self.ones_h, cfg.rms_eps)
            a_f = self._act(("ffn", L["ffn_gate"].qtype), h, L["ffn_gate"].qtype)
            gate = self._mm(("gate", li), L["ffn_gate"], a_f, B)
            up = self._mm(("up", li), L["ffn_up"], a_f, B)
            hf = torch.nn.functional.silu(gate) * up
            a_d = self._act(("down", L["ffn_down"].qtype), hf, L["ffn_down"].qtype)
            x = x + self._mm(("down", li), L["ffn_down"], a_d, B)
        h = self._rms(x, self.ones_h, cfg.rms_eps)
        a_h = self._act(("head", self.output.qtype), h, self.output.qtype)
        self.logits.copy_(self._mm(("head",), self.output, a_h, B))
        self.next_tokens.copy_(torch.argmax(self.logits, dim=-1))

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
        w = sum(wt.nbytes for L in self.layers for wt in L.values()) + self.output.nbytes
        kv = int(sum(int(c) for c in ctx_lens)) * self.cfg.n_layer * 2 * self.cfg.n_head_kv * \
            self.cfg.head_dim * 2
        return w + kv
