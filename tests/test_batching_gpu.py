"""Continuous batching on the GPU: requests with different prompt lengths join a 2-slot batch at
different steps (one waits for a free slot); every request's greedy tokens equal those of the same
request run alone.  Each sequence reads only its own KV blocks, so its output cannot depend on its
neighbours."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prefill", [True, False])
def test_batched_equals_alone(prefill):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200.batching import ContinuousBatcher
    from densecore_b200.decoder import Decoder
    from test_decoder_gpu import tiny
    from densecore_b200.ggml_types import Q4_K

    cfg = tiny(Q4_K, ("attn_v", "ffn_down"))
    prompts = [[7, 300, 11], [42], [500, 1, 2, 3, 4, 5, 6]]
    max_new = [6, 9, 4]

    def run(reqs, batch):
        dec = Decoder(cfg, batch=batch, max_ctx=32, seed=11)
        b = ContinuousBatcher(dec, prefill=prefill)
        handles = [b.submit(p, n) for p, n in reqs]
        b.run(max_steps=200)
        assert all(h.done() for h in handles) and not b.queue
        assert len(b.alloc.free) == dec.n_blocks - 1        # every request's blocks came back
        return [h.out for h in handles]

    together = run(list(zip(prompts, max_new)), batch=2)
    alone = [run([(p, n)], batch=1)[0] for p, n in zip(prompts, max_new)]
    assert together == alone
    assert [len(o) for o in together] == max_new


@pytest.mark.parametrize("layout", ["q8_0", "q4_k_m"])
def test_prefill_equals_token_by_token(layout):
    """Decoder.prefill of whole prompts (ragged, two sequences in one pass) gives the last-token
    logits of feeding the same prompts one token per decode step (2e-3, same argmax), and leaves the
    same K/V in the cache (the next decode step agrees too)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import numpy as np
    from densecore_b200.decoder import Decoder
    from densecore_b200.ggml_types import Q4_K, Q8_0
    from test_decoder_gpu import tiny
    cfg = tiny(Q8_0) if layout == "q8_0" else tiny(Q4_K, ("attn_v", "ffn_down"))
    prompts = [[7, 300, 11, 5, 9, 100, 200, 301, 4, 4, 4, 17, 18, 19, 20, 21, 22, 23], [42, 43, 44]]
    a = Decoder(cfg, batch=2, max_ctx=64, seed=11)
    b = Decoder(cfg, batch=2, max_ctx=64, seed=11)
    nxt, logits = a.prefill([0, 1], prompts)
    # token by token through the decode step (both sequences advance together; the shorter one
    # repeats its last token into a position past its prompt, which the comparison never reads)
    last = {}
    for t in range(max(len(p) for p in prompts)):
        b.tokens.copy_(torch.tensor([p[min(t, len(p) - 1)] for p in prompts]))
        b.ctx_lens.copy_(torch.tensor([min(t, len(p) - 1) + 1 for p in prompts], dtype=torch.int32))
        b.step()
        for i, p in enumerate(prompts):
            if t == len(p) - 1:
                last[i] = b.logits[i].clone()
    ref = torch.stack([last[0], last[1]]).double().cpu().numpy()
    got = logits.double().cpu().numpy()
    err = np.linalg.norm(got - ref, axis=-1) / np.linalg.norm(ref, axis=-1)
    assert err.max() < 2e-3, err
    assert np.array_equal(nxt.cpu().numpy(), ref.argmax(-1))
