"""GGUF model files: a reader for the on-disk format and the mapping of a GGUF decoder checkpoint
onto the decoder's configuration, following DenseCore's loader (core/src/model_loader.cpp):
hyper-parameters under "<general.architecture>.<key>" with a "general.<key>" fallback (:154-215),
tensor names token_embd / output_norm / output (else lm_head, else tied to the embedding) and
blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm, ffn_norm,
ffn_gate, ffn_up, ffn_down}.weight, with the ".weight" suffix optional for the QK-norms (:300-403).

File layout (GGUF v2/v3, little-endian): magic "GGUF", u32 version, u64 tensor count, u64
metadata count; metadata entries (string key, u32 value type, value); tensor infos (string name,
u32 n_dims, u64 dims[n_dims] innermost first, u32 ggml type, u64 offset); padding to
general.alignment (default 32); tensor data, each tensor at data start + offset.  A 2-D weight
has dims (K, N): N rows of K values in ggml blocks -- the row layout every dcgpu entry point takes.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

from .ggml_types import F16, F32, row_size

GGUF_MAGIC = b"GGUF"

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f",
           _BOOL: "<?", _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclasses.dataclass
class TensorInfo:
    name: str
    dims: tuple          # innermost first (ggml ne order)
    ggml_type: int
    offset: int          # from the start of the data section
    nbytes: int


def _row_bytes(ggml_type: int, k: int) -> int:
    try:
        return row_size(ggml_type, k)
    except KeyError:
        raise ValueError(f"unsupported ggml type {ggml_type}") from None


class _Reader:
    def __init__(self, f):
        self.f = f

    def take(self, fmt: str):
        n = struct.calcsize(fmt)
        b = self.f.read(n)
        if len(b) != n:
            raise ValueError("truncated GGUF file")
        return struct.unpack(fmt, b)[0]

    def string(self) -> str:
        n = self.take("<Q")
        b = self.f.read(n)
        if len(b) != n:
            raise ValueError("truncated GGUF file")
        return b.decode("utf-8")

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == _STR:
            return self.string()
        if vtype == _ARR:
            etype, count = self.take("<I"), self.take("<Q")
            if etype in _SCALAR and etype != _BOOL:
                dt = np.dtype(_SCALAR[etype])
                b = self.f.read(dt.itemsize * count)
                if len(b) != dt.itemsize * count:
                    raise ValueError("truncated GGUF file")
                return np.frombuffer(b, dtype=dt).copy()
            return [self.value(etype) for _ in range(count)]
        raise ValueError(f"unknown GGUF metadata type {vtype}")


class GGUFFile:
    """Metadata and tensor directory of a GGUF file; tensor bytes are memory-mapped."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            r = _Reader(f)
            if f.read(4) != GGUF_MAGIC:
                raise ValueError(f"{path}: not a GGUF file")
            self.version = r.take("<I")
            if self.version not in (2, 3):
                raise ValueError(f"{path}: GGUF version {self.version} is not supported")
            n_tensors, n_kv = r.take("<Q"), r.take("<Q")
            self.metadata = {}
            for _ in range(n_kv):
                key = r.string()
                self.metadata[key] = r.value(r.take("<I"))
            infos = []
            for _ in range(n_tensors):
                name = r.string()
                nd = r.take("<I")
                dims = tuple(r.take("<Q") for _ in range(nd))
                t, off = r.take("<I"), r.take("<Q")
                infos.append((name, dims, t, off))
            align = int(self.metadata.get("general.alignment", 32))
            self.data_start = (f.tell() + align - 1) // align * align
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        self.tensors = {}
        for name, dims, t, off in infos:
            rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
            nbytes = rows * _row_bytes(t, int(dims[0]))
            if self.data_start + off + nbytes > self._map.size:
                raise ValueError(f"{path}: tensor {name} runs past the end of the file")
            self.tensors[name] = TensorInfo(name, dims, t, off, nbytes)

    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's bytes as [rows, row bytes] (uint8, a view of the mapped file)."""
        ti = self.tensors[name]
        rows = int(np.prod(ti.dims[1:])) if len(ti.dims) > 1 else 1
        a = self._map[self.data_start + ti.offset: self.data_start + ti.offset + ti.nbytes]
        return a.reshape(rows, ti.nbytes // rows)

    def tensor_f32(self, name: str) -> np.ndarray:
        """An F32 / F16 tensor as float32 (norm weights), shaped innermost-last."""
        ti = self.tensors[name]
        raw = self.tensor_bytes(name).reshape(-1)
        if ti.ggml_type == F32:
            v = raw.view(np.float32)
        elif ti.ggml_type == F16:
            v = raw.view(np.float16).astype(np.float32)
        else:
            raise ValueError(f"{name}: expected an F32 / F16 tensor, got ggml type {ti.ggml_type}")
        return v.reshape(tuple(reversed(ti.dims)))

    def find(self, name: str) -> str | None:
        """The stored name of a tensor, accepting a missing ".weight" suffix."""
        if name in self.tensors:
            return name
        if name.endswith(".weight") and name[:-7] in self.tensors:
            return name[:-7]
        return None

    def hparam(self, key: str, default=None):
        """<arch>.<key>, else general.<key>, else default."""
        arch = self.metadata.get("general.architecture", "")
        for k in (f"{arch}.{key}", f"general.{key}"):
            if k in self.metadata:
                return self.metadata[k]
        return default


def shard_rows(rows: np.ndarray, r0: int, r1: int) -> np.ndarray:
    """Output rows [r0, r1) of a weight in ggml rows (rows are quantized independently)."""
    return rows[r0:r1]


def shard_cols(rows: np.ndarray, ggml_type: int, k: int, c0: int, c1: int) -> tuple[np.ndarray, int]:
    """Input columns [c0, c1) of a weight in ggml rows, for a K-split shard.  The bounds must fall on
    block boundaries; a block is then kept whole, so the shard equals quantizing the sliced matrix."""
    from .ggml_types import block_size, type_size
    bs, bb = block_size(ggml_type), type_size(ggml_type)
    if c0 % bs or c1 % bs or not 0 <= c0 < c1 <= k:
        raise ValueError(f"columns [{c0}, {c1}) do not fall on {bs}-value block boundaries of K={k}")
    return np.ascontiguousarray(rows[:, c0 // bs * bb: c1 // bs * bb]), c1 - c0


def decoder_config(g: GGUFFile):
    """DecoderConfig of a GGUF decoder checkpoint (Llama / Qwen2 / Qwen3 families)."""
    from .decoder import DecoderConfig

    arch = g.metadata.get("general.architecture", "unknown")
    emb = g.tensors.get("token_embd.weight")
    if emb is None:
        raise ValueError("no token_embd.weight tensor")
    n_layer = int(g.hparam("block_count"))
    hidden = int(g.hparam("embedding_length"))
    n_head = int(g.hparam("attention.head_count"))
    n_head_kv = int(g.hparam("attention.head_count_kv", n_head)) or n_head
    head_dim = int(g.hparam("attention.key_length", hidden // n_head))
    ffn = int(g.hparam("feed_forward_length", g.tensors["blk.0.ffn_gate.weight"].dims[1]))
    vocab = int(emb.dims[1])
    has_out = any(n in g.tensors for n in ("output.weight", "lm_head.weight"))
    qk_norm = g.find("blk.0.attn_q_norm.weight") is not None and g.find("blk.0.attn_k_norm.weight") is not None
    return DecoderConfig(
        name=str(g.metadata.get("general.name", arch)), n_layer=n_layer, hidden=hidden, n_head=n_head,
        n_head_kv=n_head_kv, head_dim=head_dim, ffn=ffn, vocab=vocab,
        rope_theta=float(g.hparam("rope.freq_base", 10000.0)),
        rms_eps=float(g.hparam("attention.layer_norm_rms_epsilon", 1e-5)),
        wtype=g.tensors["blk.0.attn_q.weight"].ggml_type, qk_norm=qk_norm, tied=not has_out,
        out_type=g.tensors[g.find("output.weight") or g.find("lm_head.weight") or "token_embd.weight"].ggml_type)


def decoder_weights(g: GGUFFile) -> dict:
    """name -> (ggml rows as uint8 [rows, row bytes], ggml type, K) for every linear weight and
    the embedding; name -> float32 vector for every norm weight.  Names are the GGUF ones."""
    cfg = decoder_config(g)
    out = {}

    def lin(name):
        ti = g.tensors[name]
        out[name] = (g.tensor_bytes(name), ti.ggml_type, int(ti.dims[0]))

    lin("token_embd.weight")
    out["output_norm.weight"] = g.tensor_f32("output_norm.weight")
    head = g.find("output.weight") or g.find("lm_head.weight")
    if head:
        ti = g.tensors[head]
        out["output.weight"] = (g.tensor_bytes(head), ti.ggml_type, int(ti.dims[0]))
    for i in range(cfg.n_layer):
        p = f"blk.{i}."
        for nm in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            lin(p + nm + ".weight")
        for nm in ("attn_norm", "ffn_norm"):
            out[p + nm + ".weight"] = g.tensor_f32(p + nm + ".weight")
        if cfg.qk_norm:
            for nm in ("attn_q_norm", "attn_k_norm"):
                out[p + nm + ".weight"] = g.tensor_f32(g.find(p + nm + ".weight"))
    return out
