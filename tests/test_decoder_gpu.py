"""End-to-end decode step of the Qwen3-architecture decoder vs a CPU reference that chains the oracle
ops (activation quantize + vec_dot mul_mat, paged attention, fp16 KV append) with float64 glue.
Bar: logits within 2e-3 relative (L2 per sequence), next tokens equal.  Cases: a tiny model, and
two-layer models at the widths and batches of the benchmarked decoders (Qwen3-0.6B: hidden 1024,
16/8 heads, Q8_0, the real 151936-row tied head, batch 64; Qwen3-4B: hidden 2560, 32/8 heads,
Q4_K_M with Q6_K alternation and a Q6_K head, batch 32), so the batched tensor-core matmuls and
split-K paths that the decode benchmark times are the ones checked."""
import numpy as np
import pytest
import torch

from chained_ref import reference_step

pytestmark = pytest.mark.gpu


def tiny(wtype, q6k_alt=()):
    from densecore_b200.decoder import DecoderConfig
    return DecoderConfig("tiny", n_layer=2, hidden=256, n_head=4, n_head_kv=2, head_dim=128, ffn=512,
                         vocab=512, wtype=wtype, q6k_alternate=q6k_alt)


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


@pytest.mark.parametrize("which", ["qwen3_0_6b", "qwen3_4b"])
def test_decode_step_at_benchmark_widths(which):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dataclasses

    from densecore_b200 import decoder as D
    if which == "qwen3_0_6b":
        cfg, batch = dataclasses.replace(D.QWEN3_0_6B, n_layer=2), 64
        ctx = np.random.default_rng(2).integers(128, 2049, batch)
    else:
        cfg, batch = dataclasses.replace(D.QWEN3_4B, n_layer=2), 32
        ctx = np.random.default_rng(3).integers(2048, 4097, batch)
    dec = D.Decoder(cfg, batch=batch, max_ctx=int(ctx.max()), seed=13)
    dec.fill_kv_random(7)
    tokens = np.random.default_rng(4).integers(0, cfg.vocab, batch)
    dec.tokens.copy_(torch.from_numpy(tokens))
    dec.ctx_lens.copy_(torch.from_numpy(ctx.astype(np.int32)))
    ref = reference_step(dec, tokens, list(ctx))
    dec.replay()
    torch.cuda.synchronize()
    got = dec.logits.cpu().numpy().astype(np.float64)
    err = np.linalg.norm(got - ref, axis=-1) / np.linalg.norm(ref, axis=-1)
    assert err.max() < 2e-3, err.max()
    assert np.array_equal(dec.next_tokens.cpu().numpy(), ref.argmax(-1))
