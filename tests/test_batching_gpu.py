"""Continuous batching on the GPU: requests with different prompt lengths join a 2-slot batch at
different steps (one waits for a free slot); every request's greedy tokens equal those of the same
request run alone.  Each sequence reads only its own KV blocks, so its output cannot depend on its
neighbours."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_batched_equals_alone():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200.batching import ContinuousBatcher
    from densecore_b200.decoder import Decoder
    from tests.test_decoder_gpu import tiny
    from densecore_b200.ggml_types import Q4_K

    cfg = tiny(Q4_K, ("attn_v", "ffn_down"))
    prompts = [[7, 300, 11], [42], [500, 1, 2, 3, 4, 5, 6]]
    max_new = [6, 9, 4]

    def run(reqs, batch):
        dec = Decoder(cfg, batch=batch, max_ctx=32, seed=11)
        b = ContinuousBatcher(dec)
        handles = [b.submit(p, n) for p, n in reqs]
        b.run(max_steps=200)
        assert all(h.done() for h in handles) and not b.queue
        assert len(b.alloc.free) == dec.n_blocks - 1        # every request's blocks came back
        return [h.out for h in handles]

    together = run(list(zip(prompts, max_new)), batch=2)
    alone = [run([(p, n)], batch=1)[0] for p, n in zip(prompts, max_new)]
    assert together == alone
    assert [len(o) for o in together] == max_new
