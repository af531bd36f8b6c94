"""Generate the golden fixtures that pin the CPU oracle (run in the build container).

Sources of truth, none of them our own code:
  * `gguf` 0.19.0 (the GGUF Python package of the ggml project; its Q8_0 quantizer states it is
    bit-exact with ggml-quants.c's reference):  Q8_0 quantize bytes, and Q8_0 / Q4_K / Q6_K
    dequantization of random block bytes (pins the block layouts, nibble order, 6-bit scale
    packing and the Q6_K high-bit planes).
  * DenseCore's FlashAttentionGQA (core/include/flash_attention.h:239-272) compiled from the
    reference sources (oracle/_ref/libref_attn.so): decode attention outputs on a small case.

Writes tests/golden/golden.npz (a few hundred KB).  Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import gguf  # noqa: E402
from gguf import GGMLQuantizationType as T  # noqa: E402

from oracle import oracle  # noqa: E402


def random_k_blocks(rng, n_blocks, nbytes, fp16_offsets):
    """Random block bytes with sane fp16 scale fields at the given byte offsets."""
    b = rng.integers(0, 256, size=(n_blocks, nbytes), dtype=np.uint8)
    for off in fp16_offsets:
        d = (rng.uniform(1e-4, 5e-2, size=n_blocks)).astype(np.float16)
        b[:, off:off + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return b


def main():
    rng = np.random.default_rng(1234)
    out = {}

    # ---- Q8_0 quantize: seeded N(0,1) rows + edge rows (all-zero block, one-hot, ramps, huge) ----
    x = rng.standard_normal((6, 256)).astype(np.float32)
    x[1, :32] = 0.0                      # all-zero block -> d = 0, q = 0
    x[2, 32:64] = 0.0
    x[2, 40] = -3.0                      # single non-zero of negative sign
    x[3, :] = np.linspace(-1, 1, 256, dtype=np.float32)
    x[4, :] *= 1e4
    x[5, :] *= 1e-6
    out["q8_0_x"] = x
    out["q8_0_bytes"] = gguf.quants.quantize(x, T.Q8_0)

    # ---- dequantization of random block bytes ----
    n = 24
    q80 = random_k_blocks(rng, n, 34, [0])
    out["deq_q8_0_bytes"] = q80
    out["deq_q8_0_f32"] = gguf.quants.dequantize(q80.reshape(-1), T.Q8_0).reshape(-1)
    q4k = random_k_blocks(rng, n, 144, [0, 2])
    out["deq_q4_K_bytes"] = q4k
    out["deq_q4_K_f32"] = gguf.quants.dequantize(q4k.reshape(-1), T.Q4_K).reshape(-1)
    q6k = random_k_blocks(rng, n, 210, [208])
    q6k[:, 192:208] = rng.integers(-128, 128, size=(n, 16)).astype(np.int8).view(np.uint8)
    out["deq_q6_K_bytes"] = q6k
    out["deq_q6_K_f32"] = gguf.quants.dequantize(q6k.reshape(-1), T.Q6_K).reshape(-1)

    # ---- reference decode attention (DenseCore FlashAttentionGQA, causal=false) ----
    ref = oracle.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_attn.so missing: run `make -C oracle` with the "
                         "reference sources present")
    B, hq, hkv, d = 2, 16, 8, 128
    skv = 150
    Q = rng.standard_normal((B, hq, 1, d)).astype(np.float32)
    K = rng.standard_normal((B, hkv, skv, d)).astype(np.float16).astype(np.float32)
    V = rng.standard_normal((B, hkv, skv, d)).astype(np.float16).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    out["attn_q"] = Q
    out["attn_k"] = K.astype(np.float16)
    out["attn_v"] = V.astype(np.float16)
    out["attn_scale"] = np.float32(scale)
    out["attn_out_ref"] = oracle.ref_flash_attention_gqa(Q, K, V, scale, causal=False)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
