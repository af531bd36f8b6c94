"""Writes a tiny GGUF decoder checkpoint for the loader tests, with gguf-py's writer (the reference
tool chain's own writer) and oracle-quantized weights.  Test infrastructure only."""
import numpy as np

from oracle import oracle as O

TINY = dict(n_layer=2, hidden=256, n_head=4, n_head_kv=2, head_dim=128, ffn=512, vocab=512)


def write_tiny_gguf(path: str, qk_norm: bool = True, tied: bool = False, seed: int = 5,
                    wtype: int = O.Q4_K, alt_type: int = O.Q6_K, emb_type: int = O.Q4_K,
                    out_type: int = O.Q6_K) -> dict:
    """Qwen3-style checkpoint: attn_v / ffn_down of layer 0 are alt_type, the other linears
    wtype; random norm weights.  Returns {name: (ggml rows, type, k) or float32 vector}."""
    import gguf

    c = TINY
    H, D, F, V = c["hidden"], c["head_dim"], c["ffn"], c["vocab"]
    rng = np.random.default_rng(seed)
    tensors = {}

    def lin(name, n, k, t):
        rows = O.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), t)
        tensors[name] = (rows, t, k)

    def vec(name, n):
        tensors[name] = rng.uniform(0.5, 1.5, n).astype(np.float32)

    lin("token_embd.weight", V, H, emb_type)
    vec("output_norm.weight", H)
    if not tied:
        lin("output.weight", V, H, out_type)
    for i in range(c["n_layer"]):
        p = f"blk.{i}."
        alt = alt_type if i == 0 else wtype
        lin(p + "attn_q.weight", c["n_head"] * D, H, wtype)
        lin(p + "attn_k.weight", c["n_head_kv"] * D, H, wtype)
        lin(p + "attn_v.weight", c["n_head_kv"] * D, H, alt)
        lin(p + "attn_output.weight", H, c["n_head"] * D, wtype)
        lin(p + "ffn_gate.weight", F, H, wtype)
        lin(p + "ffn_up.weight", F, H, wtype)
        lin(p + "ffn_down.weight", H, F, alt)
        vec(p + "attn_norm.weight", H)
        vec(p + "ffn_norm.weight", H)
        if qk_norm:
            vec(p + "attn_q_norm.weight", D)
            vec(p + "attn_k_norm.weight", D)

    w = gguf.GGUFWriter(path, "qwen3")
    w.add_name("tiny-qwen3")
    w.add_block_count(c["n_layer"])
    w.add_embedding_length(H)
    w.add_feed_forward_length(F)
    w.add_head_count(c["n_head"])
    w.add_head_count_kv(c["n_head_kv"])
    w.add_key_length(D)
    w.add_rope_freq_base(1e6)
    w.add_layer_norm_rms_eps(1e-6)
    w.add_context_length(4096)
    for name, v in tensors.items():
        if isinstance(v, tuple):
            rows, t, k = v
            w.add_tensor(name, rows, raw_shape=rows.shape, raw_dtype=gguf.GGMLQuantizationType(t))
        else:
            w.add_tensor(name, v)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors
