"""Decoder.from_gguf: a GGUF checkpoint (Q4_K_M-style mix, random norm weights, QK-norms, untied
Q6_K head or tied Q8_0 embedding) loads onto the device and its decode step matches the chained
oracle reference (logits within 2e-3 relative, same next tokens)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.gguf_fixture import write_tiny_gguf
from chained_ref import reference_step

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["q4_k_m_untied", "q8_0_tied"])
def test_gguf_decode_step(tmp_path, variant):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200.decoder import Decoder
    path = str(tmp_path / "tiny.gguf")
    if variant == "q4_k_m_untied":
        want = write_tiny_gguf(path)
    else:
        want = write_tiny_gguf(path, tied=True, wtype=O.Q8_0, alt_type=O.Q8_0, emb_type=O.Q8_0)
    dec = Decoder.from_gguf(path, batch=3, max_ctx=64)
    # the dequantized embedding equals the oracle's dequantization (fp16-rounded)
    er, et, ek = want["token_embd.weight"]
    emb = O.dequantize(er, et, ek).astype(np.float16)
    assert np.array_equal(dec.tok_embd.cpu().numpy(), emb)
    dec.fill_kv_random(5)
    tokens, ctx = [7, 300, 511], [5, 17, 33]
    dec.tokens.copy_(torch.tensor(tokens))
    dec.ctx_lens.copy_(torch.tensor(ctx, dtype=torch.int32))
    norms = {k: v for k, v in want.items() if not isinstance(v, tuple)}
    ref = reference_step(dec, tokens, ctx, norms)
    dec.replay()
    torch.cuda.synchronize()
    got = dec.logits.cpu().numpy().astype(np.float64)
    err = np.linalg.norm(got - ref, axis=-1) / np.linalg.norm(ref, axis=-1)
    assert err.max() < 2e-3, err
    assert np.array_equal(dec.next_tokens.cpu().numpy(), ref.argmax(-1))
