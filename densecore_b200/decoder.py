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
reference's batched path reads seq_id[0]'s history for every sequence).  Weights are either
random-init N(0, 0.02) of the named architecture, quantized on the device by the weight encoder
(norm weights ones), or a GGUF checkpoint's (Decoder.from_gguf).  The step runs as one CUDA graph.
"""
from __future__ import annotations

import dataclasses
import math
import warnings

import numpy as np
import torch

from . import ops
from .ggml_types import F16, F32, Q4_K, Q6_K, Q8_0, Q8_K, VEC_DOT_TYPE

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
    qk_norm: bool = True       # Qwen3 per-head RMSNorm of q and k
    tied: bool = True          # LM head = token embedding
    out_type: int = -1         # LM head type (-1: Q8_0 for Q8_0 models, else Q6_K)


QWEN3_0_6B = DecoderConfig("Qwen3-0.6B", 28, 1024, 16, 8, 128, 3072, 151936, wtype=Q8_0)
QWEN3_4B = DecoderConfig("Qwen3-4B", 36, 2560, 32, 8, 128, 9728, 151936, wtype=Q4_K,
                         q6k_alternate=("attn_v", "ffn_down"))
LLAMA3_70B = DecoderConfig("Llama-3-70B", 80, 8192, 64, 8, 128, 28672, 128256, rope_theta=5e5,
                           rms_eps=1e-5, wtype=Q4_K, qk_norm=False, tied=False, out_type=Q4_K)


def tp_plan(cfg: DecoderConfig, rank: int, size: int) -> dict:
    """Megatron-style tensor-parallel shard of every weight for rank `rank` of `size`:
    rows (output features) of q/k/v (by kv-head groups), gate/up and the LM head; columns (input
    features, 256-aligned so every Q4_K/Q6_K/Q8_0 block stays whole) of attn_output and ffn_down,
    which are followed by an all-reduce.  Values are (start, stop) half-open ranges."""
    D = cfg.head_dim
    if cfg.n_head_kv % size or cfg.n_head % size or cfg.ffn % size or cfg.vocab % size:
        raise ValueError(f"{cfg.name} does not split {size} ways")
    hq, hkv, ffn, voc = cfg.n_head // size, cfg.n_head_kv // size, cfg.ffn // size, cfg.vocab // size
    if (hq * D) % 256 or ffn % 256:
        raise ValueError("K-split shards must be multiples of 256")
    r = rank
    return {"q_rows": (r * hq * D, (r + 1) * hq * D), "kv_rows": (r * hkv * D, (r + 1) * hkv * D),
            "o_cols": (r * hq * D, (r + 1) * hq * D), "ffn_rows": (r * ffn, (r + 1) * ffn),
            "down_cols": (r * ffn, (r + 1) * ffn), "vocab_rows": (r * voc, (r + 1) * voc),
            "hq": hq, "hkv": hkv, "ffn": ffn, "vocab": voc}


def _wtype(cfg: DecoderConfig, layer: int, name: str) -> int:
    if name in cfg.q6k_alternate and layer % 2 == 0:
        return Q6_K
    return cfg.wtype


class Decoder:
    """Weights, paged KV cache and the captured decode step for `batch` sequences."""

    def __init__(self, cfg: DecoderConfig, batch: int, max_ctx: int, seed: int = 0,
                 device: str | torch.device = "cuda", tp_rank: int = 0, tp_size: int = 1,
                 tp_group=None, shard_init: str = "slice", seq_tokens=None, weights: dict | None = None):
        """tp_size > 1: this process holds shard tp_rank of every weight (tp_plan) and the KV heads
        of its query-head group; two all-reduces per layer (after attn_output and ffn_down) and an
        all-gather of the logits over tp_group (NCCL).  shard_init = "slice": every rank draws the
        full random weights and keeps its slice (bitwise the tp_size = 1 model); "local": each rank
        draws only its shard (faster; a different random model).  seq_tokens: per-sequence token
        capacity; the arena then holds exactly those blocks (default: max_ctx for every sequence).
        weights: GGUF-named tensors (gguf_file.decoder_weights) instead of random ones."""
        self.cfg, self.batch, self.max_ctx = cfg, batch, max_ctx
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        self.seed = seed
        dev = self.device = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed if shard_init == "slice" else seed * 1009 + tp_rank)
        H, D = cfg.hidden, cfg.head_dim
        plan = self.plan = tp_plan(cfg, tp_rank, tp_size)
        local = shard_init == "local"
        self.hq, self.hkv, self.ffn, self.vocab_r = plan["hq"], plan["hkv"], plan["ffn"], plan["vocab"]
        qd_full, kvd_full = cfg.n_head * D, cfg.n_head_kv * D
        qd, kvd = self.hq * D, self.hkv * D

        def draw(n, k, rows=None, cols=None):
            """fp32 N(0, 0.02) weight restricted to this rank's rows / cols."""
            if local:
                n2 = rows[1] - rows[0] if rows else n
                k2 = cols[1] - cols[0] if cols else k
                return torch.randn((n2, k2), generator=g, device=dev) * 0.02
            w = torch.randn((n, k), generator=g, device=dev) * 0.02
            if rows:
                w = w[rows[0]:rows[1]]
            if cols:
                w = w[:, cols[0]:cols[1]]
            return w.contiguous()

        def qw(n, k, t, rows=None, cols=None):
            return ops.QuantWeight.from_float(draw(n, k, rows, cols), t)

        self.ones_h = torch.ones(H, device=dev)
        self.ones_d = torch.ones(D, device=dev) if cfg.qk_norm else None
        if weights is not None:
            self._load_weights(weights)
            self._init_cache(batch, max_ctx, seq_tokens)
            return

        self.layers = []
        for li in range(cfg.n_layer):
            t_q, t_k, t_v = (_wtype(cfg, li, nm) for nm in ("attn_q", "attn_k", "attn_v"))
            wq = draw(qd_full, H, plan["q_rows"])
            wk = draw(kvd_full, H, plan["kv_rows"])
            wv = draw(kvd_full, H, plan["kv_rows"])
            L = {"qkv_split": t_v != t_q}
            if t_v == t_q:  # one stacked [q; k; v] weight: rows are quantized independently
                L["attn_qkv"] = ops.QuantWeight.from_float(torch.cat([wq, wk, wv]), t_q)
            else:
                L["attn_qk"] = ops.QuantWeight.from_float(torch.cat([wq, wk]), t_q)
                L["attn_v"] = ops.QuantWeight.from_float(wv, t_v)
            del wq, wk, wv
            L["attn_output"] = qw(H, qd_full, _wtype(cfg, li, "attn_output"), cols=plan["o_cols"])
            wg = draw(cfg.ffn, H, plan["ffn_rows"])
            wu = draw(cfg.ffn, H, plan["ffn_rows"])
            L["ffn_gate_up"] = ops.QuantWeight.from_float(torch.cat([wg, wu]), _wtype(cfg, li, "ffn_gate"))
            del wg, wu
            L["ffn_down"] = qw(H, cfg.ffn, _wtype(cfg, li, "ffn_down"), cols=plan["down_cols"])
            L["attn_norm"] = L["ffn_norm"] = self.ones_h
            L["attn_q_norm"] = L["attn_k_norm"] = self.ones_d
            self.layers.append(L)
        self.output_norm = self.ones_h
        out_t = cfg.out_type if cfg.out_type >= 0 else (Q8_0 if cfg.wtype == Q8_0 else Q6_K)
        if cfg.tied:
            # the LM head is the quantized token embedding; lookups dequantize it (all vocab rows)
            full = ops.QuantWeight.from_float(draw(cfg.vocab, H) if not local else
                                              torch.randn((cfg.vocab, H), generator=g, device=dev) * 0.02,
                                              out_t)
            self.tok_embd = self._dequant_rows(full)
            if tp_size == 1:
                self.output = full
            else:
                a, b = plan["vocab_rows"]
                self.output = ops.QuantWeight.from_ggml(full.to_ggml()[a:b].contiguous(), out_t, H)
            del full
        else:
            self.tok_embd = (torch.randn((cfg.vocab, H), generator=g, device=dev) * 0.02).half()
            self.output = qw(cfg.vocab, H, out_t, rows=plan["vocab_rows"])
        self._init_cache(batch, max_ctx, seq_tokens)

    def _load_weights(self, w: dict):
        """Weights from GGUF-named tensors: ggml rows go to the device as they are; q|k|v and
        gate|up are stacked by concatenating rows (rows are quantized independently).  With
        tp_size > 1 each rank keeps its tp_plan shard: whole rows, or whole blocks of columns."""
        from .gguf_file import shard_cols, shard_rows
        cfg, dev, H, plan = self.cfg, self.device, self.cfg.hidden, self.plan
        supported = (Q8_0, Q4_K, Q6_K)
        if self.tp_size > 1:
            w = dict(w)
            rows_of = {"attn_q": "q_rows", "attn_k": "kv_rows", "attn_v": "kv_rows", "ffn_gate": "ffn_rows",
                       "ffn_up": "ffn_rows"}
            cols_of = {"attn_output": "o_cols", "ffn_down": "down_cols"}
            for name, v in list(w.items()):
                if not isinstance(v, tuple) or not name.startswith("blk."):
                    continue
                base = name.split(".")[2]
                r, t, k = v
                if base in rows_of:
                    w[name] = (shard_rows(r, *plan[rows_of[base]]), t, k)
                elif base in cols_of:
                    sr, sk = shard_cols(r, t, k, *plan[cols_of[base]])
                    w[name] = (sr, t, sk)
            head = "output.weight" if "output.weight" in w else "token_embd.weight"
            r, t, k = w[head]
            w["output.weight"] = (shard_rows(r, *plan["vocab_rows"]), t, k)

        def to_dev(a):
            # tensors of a memory-mapped file are read-only views: only read here (copied to the device)
            with warnings.catch_warnings():
                warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
                return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        def rows(name):
            r, t, k = w[name]
            if t not in supported:
                raise ValueError(f"{name}: ggml type {t} is not a supported matmul weight type")
            return to_dev(r), t, k

        def stack(names):
            parts = [rows(n) for n in names]
            if len({t for _, t, _ in parts}) != 1:
                return None
            return ops.QuantWeight.from_ggml(torch.cat([r for r, _, _ in parts]), parts[0][1], parts[0][2])

        def vec(name):
            return torch.from_numpy(np.ascontiguousarray(w[name], dtype=np.float32)).to(dev)

        self.layers = []
        for li in range(cfg.n_layer):
            p = f"blk.{li}."
            L = {"qkv_split": False}
            qkv = stack([p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"])
            if qkv is not None:
                L["attn_qkv"] = qkv
            else:
                qk = stack([p + "attn_q.weight", p + "attn_k.weight"])
                if qk is None:
                    raise NotImplementedError(f"layer {li}: attn_q and attn_k of different types")
                L.update(qkv_split=True, attn_qk=qk, attn_v=ops.QuantWeight.from_ggml(*rows(p + "attn_v.weight")))
            L["attn_output"] = ops.QuantWeight.from_ggml(*rows(p + "attn_output.weight"))
            gu = stack([p + "ffn_gate.weight", p + "ffn_up.weight"])
            if gu is None:
                raise NotImplementedError(f"layer {li}: ffn_gate and ffn_up of different types")
            L["ffn_gate_up"] = gu
            L["ffn_down"] = ops.QuantWeight.from_ggml(*rows(p + "ffn_down.weight"))
            L["attn_norm"], L["ffn_norm"] = vec(p + "attn_norm.weight"), vec(p + "ffn_norm.weight")
            L["attn_q_norm"] = vec(p + "attn_q_norm.weight") if cfg.qk_norm else None
            L["attn_k_norm"] = vec(p + "attn_k_norm.weight") if cfg.qk_norm else None
            self.layers.append(L)
        self.output_norm = vec("output_norm.weight")
        er, et, ek = w["token_embd.weight"]
        er_dev = to_dev(er)
        if et in supported:
            emb = ops.QuantWeight.from_ggml(er_dev, et, ek)
            self.tok_embd = self._dequant_rows(emb)
        elif et in (F16, F32):
            self.tok_embd = er_dev.view(torch.float16 if et == F16 else torch.float32).reshape(-1, ek).half()
            emb = None
        else:
            raise ValueError(f"token_embd: ggml type {et} is not supported")
        if "output.weight" in w:   # untied, or this rank's vocabulary rows of a tied head
            self.output = ops.QuantWeight.from_ggml(*rows("output.weight"))
        elif emb is not None:      # tied: the LM head is the embedding matrix itself
            self.output = emb
        else:                      # tied fp embedding: quantized to Q8_0 for the head matmul
            self.output = ops.QuantWeight.from_float(self.tok_embd.float(), Q8_0)

    @classmethod
    def from_gguf(cls, path: str, batch: int, max_ctx: int, device: str | torch.device = "cuda",
                  seq_tokens=None, tp_rank: int = 0, tp_size: int = 1, tp_group=None) -> "Decoder":
        """A decoder holding the weights of a GGUF checkpoint (tensor names and hyper-parameter
        keys of DenseCore's loader, core/src/model_loader.cpp:154-403); with tp_size > 1, this
        rank's tensor-parallel shard of them."""
        from .gguf_file import GGUFFile, decoder_config, decoder_weights
        g = GGUFFile(path)
        return cls(decoder_config(g), batch, max_ctx, device=device, seq_tokens=seq_tokens,
                   weights=decoder_weights(g), tp_rank=tp_rank, tp_size=tp_size, tp_group=tp_group)

    def _init_cache(self, batch, max_ctx, seq_tokens):
        cfg, dev, H, D = self.cfg, self.device, self.cfg.hidden, self.cfg.head_dim

        # paged KV arena (kv_cache.cpp:353-370 layout): [(block*n_layer + layer)][16][hkv][D] fp16
        self.blocks_per_seq = (max_ctx + KV_BLOCK - 1) // KV_BLOCK
        if seq_tokens is None:
            nblk = [self.blocks_per_seq] * batch
        else:
            nblk = [(int(t) + KV_BLOCK - 1) // KV_BLOCK for t in seq_tokens]
        self.n_blocks = sum(nblk)
        shape = (self.n_blocks * cfg.n_layer, KV_BLOCK, self.hkv, D)
        self.k_arena = torch.empty(shape, dtype=torch.float16, device=dev)
        self.v_arena = torch.empty(shape, dtype=torch.float16, device=dev)
        # each sequence owns a shuffled set of physical blocks
        perm = torch.randperm(self.n_blocks, generator=torch.Generator().manual_seed(self.seed + 1))
        bt = torch.zeros((batch, self.blocks_per_seq), dtype=torch.int32)
        o = 0
        for i, nb in enumerate(nblk):
            bt[i, :nb] = perm[o:o + nb].to(torch.int32)
            o += nb
        self.block_tables = bt.to(dev)

        # step buffers (static for graph capture)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.ctx_lens = torch.zeros(batch, dtype=torch.int32, device=dev)  # incl. the new token
        self.seq_ids = torch.arange(batch, dtype=torch.int32, device=dev)
        self.next_tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.logits = torch.empty((batch, cfg.vocab), device=dev)
        self.logits_r = torch.empty((batch, self.vocab_r), device=dev)
        self.gathered = torch.empty((self.tp_size, batch, self.vocab_r), device=dev)
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
        if w.qtype == Q4_K:
            # d, dmin (fp16), 12 bytes of 6-bit scales / mins, 128 bytes of nibbles per 256
            b = rows.view(n, k // 256, 144)
            d = b[..., 0:2].contiguous().view(torch.float16).float()
            dmin = b[..., 2:4].contiguous().view(torch.float16).float()
            s = b[..., 4:16].to(torch.int32)
            sc = torch.cat([s[..., 0:4] & 63, (s[..., 8:12] & 15) | ((s[..., 0:4] >> 6) << 4)], -1).float()
            mn = torch.cat([s[..., 4:8] & 63, (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)], -1).float()
            qs = b[..., 16:144].to(torch.int32).view(n, k // 256, 4, 32)
            q = torch.stack([qs & 15, qs >> 4], 3).reshape(n, k // 256, 8, 32).float()
            out = d[..., None] * sc[..., None] * q - dmin[..., None] * mn[..., None]
            return out.reshape(n, k).to(torch.float16)
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
        # outputs are reused across layers (the stream orders every reuse after the last reader)
        key = (key[0], w.n, w.k, w.qtype)
        out = self._buf(("y", key), (m, w.n))
        scr = self._buf(("qs", key), (max(1, ops.mul_mat_q_scratch_size(w.qtype, w.n, w.k, m)),),
                        torch.uint8, zero=True)
        return ops.mul_mat_q(w, act, m, out=out, scratch=scr)

    # ---------------------------------------------------------------- the step
    def ggml_rows(self, li: int, name: str):
        """(ggml rows as numpy, type, k) of one logical weight (unstacking the fused ones)."""
        D = self.cfg.head_dim
        qd, kvd = self.hq * D, self.hkv * D
        L = self.layers[li]
        spans = {"attn_q": (0, qd), "attn_k": (qd, qd + kvd), "attn_v": (qd + kvd, qd + 2 * kvd),
                 "ffn_gate": (0, self.ffn), "ffn_up": (self.ffn, 2 * self.ffn)}
        if name in ("attn_output", "ffn_down") or (name == "attn_v" and L["qkv_split"]):
            w = L[name]
            return w.to_ggml().cpu().numpy(), w.qtype, w.k
        key = "ffn_gate_up" if name.startswith("ffn") else ("attn_qk" if L["qkv_split"] else "attn_qkv")
        w = L[key]
        a, b = spans[name]
        return w.to_ggml().cpu().numpy()[a:b], w.qtype, w.k

    def step(self):
        """One decode token for every sequence (see _step).  With tensor parallelism the step's
        kernels are launched in plain stream order (no programmatic dependent launch): NCCL's
        collective kernels sit between them in the same stream, and a kernel that overlaps its
        predecessor's drain is only safe next to this library's own kernels."""
        if self.tp_size == 1:
            return self._step()
        lib = ops._lib.load()
        prev = lib.dcg_set_programmatic_launch(0)
        try:
            return self._step()
        finally:
            lib.dcg_set_programmatic_launch(prev)

    def _step(self):
        """One decode token for every sequence: reads self.tokens / self.ctx_lens, writes
        self.next_tokens and self.logits, appends K/V at position ctx_len-1.  Per layer: fused
        add+RMSNorm+quantize, stacked QKV matmul, fused QK-norm+RoPE+KV append, paged attention,
        quantize, O matmul, fused add+RMSNorm+quantize, stacked gate|up matmul, fused
        SwiGLU+quantize, down matmul (its output is added by the next layer's norm kernel)."""
        cfg, B = self.cfg, self.batch
        D, hq, hkv, H, ffn = cfg.head_dim, self.hq, self.hkv, cfg.hidden, self.ffn
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
            ops.add_rmsnorm_quantize(x, L["attn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wqk.qtype], act, delta)
            yqk = self._mm(("qkv", li), wqk, act, B)
            if L["qkv_split"]:
                wv = L["attn_v"]
                act_v = act
                if VEC_DOT_TYPE[wv.qtype] != VEC_DOT_TYPE[wqk.qtype]:
                    act_v = self._actbuf(("attn_v", wv.qtype), B, H, wv.qtype)
                    ops.add_rmsnorm_quantize(x, L["attn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wv.qtype], act_v)
                yv, ldv = self._mm(("v", li), wv, act_v, B), kvd
            else:
                yv, ldv = yqk[:, qd + kvd:], wqk.n
            ops.qk_norm_rope_kv_append(yqk, wqk.n, yqk[:, qd:], wqk.n, yv, ldv, B, hq, hkv, L["attn_q_norm"],
                                       L["attn_k_norm"], cfg.rms_eps, cfg.rope_theta, pos, q_rot,
                                       self.k_arena, self.v_arena, cfg.n_layer, li, self.block_tables)
            ops.paged_attn_decode(q_rot, self.k_arena, self.v_arena, cfg.n_layer, li, self.block_tables,
                                  self.ctx_lens, hkv, self.max_ctx, scale, out=attn_out, scratch=attn_scr)
            wo = L["attn_output"]
            act_o = self._actbuf(("o", wo.qtype), B, qd, wo.qtype)
            ops.quantize_act(attn_out.view(B, qd), VEC_DOT_TYPE[wo.qtype], out=act_o)
            yo = self._allreduce(self._mm(("o", li), wo, act_o, B))
            wgu = L["ffn_gate_up"]
            act_f = self._actbuf(("ffn", wgu.qtype), B, H, wgu.qtype)
            ops.add_rmsnorm_quantize(x, L["ffn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wgu.qtype], act_f, yo)
            ygu = self._mm(("gu", li), wgu, act_f, B)
            wd = L["ffn_down"]
            act_d = self._actbuf(("down", wd.qtype), B, ffn, wd.qtype)
            ops.swiglu_quantize(ygu, ygu[:, ffn:], 2 * ffn, B, ffn, VEC_DOT_TYPE[wd.qtype], act_d)
            delta = self._allreduce(self._mm(("down", li), wd, act_d, B))
        act_h = self._actbuf(("head", self.output.qtype), B, H, self.output.qtype)
        ops.add_rmsnorm_quantize(x, self.output_norm, cfg.rms_eps, VEC_DOT_TYPE[self.output.qtype], act_h, delta)
        if self.tp_size == 1:
            self.logits.copy_(self._mm(("head",), self.output, act_h, B))
        else:  # vocab-split LM head: gather the shards' columns
            import torch.distributed as dist
            self.logits_r.copy_(self._mm(("head",), self.output, act_h, B))
            dist.all_gather_into_tensor(self.gathered, self.logits_r, group=self.tp_group)
            self.logits.copy_(self.gathered.permute(1, 0, 2).reshape(B, -1))
        self.next_tokens.copy_(torch.argmax(self.logits, dim=-1))

    def prefill(self, seqs, prompts, start=None):
        """Ingest a prompt chunk for each of the sequences `seqs` (batch slots, whose block-table
        rows are already set) in one pass: every matmul runs with M = all chunk tokens, attention is
        the multi-token causal kernel.  prompts[i] are the tokens of sequence seqs[i] at positions
        start[i] .. start[i] + len - 1 (start: default 0, a whole prompt).  Their K/V are written to
        the cache; returns (next_tokens [len(seqs)] long, logits [len(seqs), vocab]) for each chunk's
        last token.  Runs eagerly (its shapes change from call to call); with tensor parallelism the
        same two all-reduces per layer and the logits all-gather run in plain stream order."""
        if self.tp_size == 1:
            return self._prefill(seqs, prompts, start)
        lib = ops._lib.load()
        prev = lib.dcg_set_programmatic_launch(0)
        try:
            return self._prefill(seqs, prompts, start)
        finally:
            lib.dcg_set_programmatic_launch(prev)

    def _prefill(self, seqs, prompts, start):
        cfg, dev = self.cfg, self.device
        D, hq, hkv, H, ffn = cfg.head_dim, self.hq, self.hkv, cfg.hidden, self.ffn
        qd, kvd = hq * D, hkv * D
        S = len(seqs)
        n_s = [len(p) for p in prompts]
        if S == 0 or min(n_s) < 1:
            raise ValueError("every sequence needs at least one token")
        start = list(start) if start is not None else [0] * S
        T = sum(n_s)
        i32 = torch.int32
        tokens = torch.tensor([t for p in prompts for t in p], dtype=torch.long, device=dev)
        local_seq = torch.tensor([i for i, n in enumerate(n_s) for _ in range(n)], dtype=i32, device=dev)
        positions = torch.tensor([start[i] + j for i, n in enumerate(n_s) for j in range(n)], dtype=i32,
                                 device=dev)
        seq_starts = torch.tensor([0] + list(np.cumsum(n_s)), dtype=i32, device=dev)
        ctx = torch.tensor([start[i] + n_s[i] for i in range(S)], dtype=i32, device=dev)
        if int(ctx.max()) > self.max_ctx:
            raise ValueError("prompt chunk runs past max_ctx")
        bt = self.block_tables[torch.tensor(list(seqs), dtype=torch.long, device=dev)].contiguous()
        scale = 1.0 / math.sqrt(D)
        x = self.tok_embd[tokens].float()
        q_rot = torch.empty((T, hq, D), device=dev)
        attn_out = torch.empty((T, hq, D), device=dev)

        def actbuf(k, wtype):
            at = VEC_DOT_TYPE[wtype]
            return torch.empty(int(ops._lib.load().dcg_act_size(at, T, k)), dtype=torch.uint8, device=dev)

        def mm(w, act, m):
            scr = torch.zeros(max(1, ops.mul_mat_q_scratch_size(w.qtype, w.n, w.k, m)), dtype=torch.uint8,
                              device=dev)
            return ops.mul_mat_q(w, act, m, scratch=scr)

        delta = None
        for li, L in enumerate(self.layers):
            wqk = L["attn_qk"] if L["qkv_split"] else L["attn_qkv"]
            act = actbuf(H, wqk.qtype)
            ops.add_rmsnorm_quantize(x, L["attn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wqk.qtype], act, delta)
            yqk = mm(wqk, act, T)
            if L["qkv_split"]:
                wv = L["attn_v"]
                act_v = act
                if VEC_DOT_TYPE[wv.qtype] != VEC_DOT_TYPE[wqk.qtype]:
                    act_v = actbuf(H, wv.qtype)
                    ops.add_rmsnorm_quantize(x, L["attn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wv.qtype], act_v)
                yv, ldv = mm(wv, act_v, T), kvd
            else:
                yv, ldv = yqk[:, qd + kvd:], wqk.n
            ops.qk_norm_rope_kv_append_tokens(yqk, wqk.n, yqk[:, qd:], wqk.n, yv, ldv, T, hq, hkv,
                                              L["attn_q_norm"], L["attn_k_norm"], cfg.rms_eps, cfg.rope_theta,
                                              local_seq, positions, q_rot, self.k_arena, self.v_arena,
                                              cfg.n_layer, li, bt)
            ops.paged_attn_prefill(q_rot, self.k_arena, self.v_arena, cfg.n_layer, li, bt, seq_starts, ctx, hkv,
                                   max(n_s), self.max_ctx, scale, out=attn_out)
            wo = L["attn_output"]
            act_o = actbuf(qd, wo.qtype)
            ops.quantize_act(attn_out.view(T, qd), VEC_DOT_TYPE[wo.qtype], out=act_o)
            yo = self._allreduce(mm(wo, act_o, T))
            wgu = L["ffn_gate_up"]
            act_f = actbuf(H, wgu.qtype)
            ops.add_rmsnorm_quantize(x, L["ffn_norm"], cfg.rms_eps, VEC_DOT_TYPE[wgu.qtype], act_f, yo)
            ygu = mm(wgu, act_f, T)
            wd = L["ffn_down"]
            act_d = actbuf(ffn, wd.qtype)
            ops.swiglu_quantize(ygu, ygu[:, ffn:], 2 * ffn, T, ffn, VEC_DOT_TYPE[wd.qtype], act_d)
            delta = self._allreduce(mm(wd, act_d, T))
        x += delta
        last = x[(seq_starts[1:] - 1).long()].contiguous()
        at = VEC_DOT_TYPE[self.output.qtype]
        act_h = torch.empty(int(ops._lib.load().dcg_act_size(at, S, H)), dtype=torch.uint8, device=dev)
        ops.add_rmsnorm_quantize(last, self.output_norm, cfg.rms_eps, at, act_h)
        logits_r = mm(self.output, act_h, S)
        if self.tp_size == 1:
            logits = logits_r
        else:
            import torch.distributed as dist
            gathered = torch.empty((self.tp_size, S, self.vocab_r), device=dev)
            dist.all_gather_into_tensor(gathered, logits_r.contiguous(), group=self.tp_group)
            logits = gathered.permute(1, 0, 2).reshape(S, -1)
        return torch.argmax(logits, dim=-1), logits

    def _allreduce(self, y):
        """Sum the K-split partial outputs of attn_output / ffn_down over the tensor-parallel group."""
        if self.tp_size > 1:
            import torch.distributed as dist
            dist.all_reduce(y, group=self.tp_group)
        return y

    def _actbuf(self, key, m, k, wtype):
        at = VEC_DOT_TYPE[wtype]
        return self._buf(("act", key, at, k), (int(ops._lib.load().dcg_act_size(at, m, k)),), torch.uint8)

    def capture(self, advance: bool = False):
        """Capture step() into a CUDA graph (buffers are static).  advance: the graph also feeds
        each sequence's next token back as its input and grows every context by one, so
        consecutive replays decode consecutive positions (greedy generation without the host)."""
        def body():
            self.step()
            if advance:
                self.tokens.copy_(self.next_tokens)
                self.ctx_lens.add_(1)
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        saved = (self.tokens.clone(), self.ctx_lens.clone())
        with torch.cuda.stream(s):
            body()  # allocates every scratch buffer outside the capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.tokens.copy_(saved[0])
        self.ctx_lens.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            body()
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
        kv = int(sum(int(c) for c in ctx_lens)) * self.cfg.n_layer * 2 * self.hkv * \
            self.cfg.head_dim * 2
        return w + kv
