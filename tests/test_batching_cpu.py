"""Host logic of continuous batching: the KV block allocator and request bookkeeping (CPU)."""
import pytest

from densecore_b200.batching import BlockAllocator, Request


def test_block_allocator():
    a = BlockAllocator(10)
    x = a.alloc(4)
    y = a.alloc(6)
    assert sorted(x + y) == list(range(10)) and a.alloc(1) is None
    a.release(x)
    z = a.alloc(3)
    assert set(z) <= set(x)
    with pytest.raises(ValueError):
        a.release([z[0], z[0]])
    with pytest.raises(ValueError):
        a.release([11])


def test_request_inputs_and_done():
    r = Request(0, [5, 6, 7], max_new=2, eos=9)
    seen = []
    for _ in range(3):
        seen.append(r.next_input())
        r.pos += 1
    assert seen == [5, 6, 7]
    r.out.append(9)
    assert r.next_input() == 9 and r.done()            # eos
    r2 = Request(1, [1], max_new=2)
    r2.out += [3, 4]
    assert r2.done() and r2.capacity == 3


class FakeDecoder:
    """Stands in for the captured decode step on CPU: each slot's next token is a function of that
    slot's own input token, position and first KV block only (what per-sequence semantics allow)."""

    def __init__(self, batch, max_ctx, n_blocks=None):
        import torch
        self.batch, self.max_ctx = batch, max_ctx
        self.blocks_per_seq = (max_ctx + 15) // 16
        self.n_blocks = n_blocks or batch * self.blocks_per_seq
        self.block_tables = torch.zeros((batch, self.blocks_per_seq), dtype=torch.int32)
        self.tokens = torch.zeros(batch, dtype=torch.long)
        self.ctx_lens = torch.ones(batch, dtype=torch.int32)
        self.next_tokens = torch.zeros(batch, dtype=torch.long)
        self.cache = {}                       # (block, slot) -> token written there
        self.steps = 0

    def _next(self, s, pos):
        hist = [self.cache[(int(self.block_tables[s, p // 16]), p % 16)] for p in range(pos + 1)]
        return (sum((i + 1) * t for i, t in enumerate(hist)) * 31 + 7) % 1000

    def replay(self):
        self.steps += 1
        for s in range(self.batch):
            pos = int(self.ctx_lens[s]) - 1
            blk = int(self.block_tables[s, pos // 16])
            self.cache[(blk, pos % 16)] = int(self.tokens[s])
            self.next_tokens[s] = self._next(s, pos)

    def prefill(self, seqs, prompts, start=None):
        import torch
        self.prefills = getattr(self, "prefills", 0) + 1
        out = []
        for i, (s, p) in enumerate(zip(seqs, prompts)):
            p0 = start[i] if start else 0
            for j, t in enumerate(p):
                pos = p0 + j
                self.cache[(int(self.block_tables[s, pos // 16]), pos % 16)] = int(t)
            out.append(self._next(s, p0 + len(p) - 1))
        return torch.tensor(out), None


@pytest.mark.parametrize("prefill", [True, False])
def test_batched_equals_alone_with_fake_decoder(prefill):
    from densecore_b200.batching import ContinuousBatcher
    reqs = [([3, 1, 4], 5), ([1], 9), ([5, 9, 2, 6, 5, 3, 5], 4), ([8, 9], 20), ([7], 1)]

    def run(batch, items, n_blocks=None):
        b = ContinuousBatcher(FakeDecoder(batch, 48, n_blocks), prefill=prefill)
        hs = [b.submit(p, n) for p, n in items]
        b.run()
        assert all(h.done() for h in hs) and not b.queue
        assert len(b.alloc.free) == b.alloc.n_blocks - 1
        return [h.out for h in hs], b.dec.steps

    alone = [run(1, [r])[0][0] for r in reqs]
    if prefill:   # prompt ingestion in one pass gives the tokens of token-by-token feeding
        b = ContinuousBatcher(FakeDecoder(1, 48), prefill=False)
        hs = [b.submit(p, n) for p, n in reqs]
        b.run()
        assert [h.out for h in hs] == alone
    together, steps = run(2, reqs)
    assert together == alone
    assert [len(o) for o in together] == [n for _, n in reqs]
    # fewer slots than requests: the later ones wait; the batch finishes in fewer steps than serially
    assert steps < sum(len(p) + n - 1 for p, n in reqs)
    # too few KV blocks for two requests at once: admission waits for blocks, results unchanged
    tight, _ = run(3, reqs, n_blocks=4)
    assert tight == alone


def test_submit_rejects_oversize_and_empty():
    from densecore_b200.batching import ContinuousBatcher
    b = ContinuousBatcher(FakeDecoder(2, 32))
    with pytest.raises(ValueError):
        b.submit([], 3)
    with pytest.raises(ValueError):
        b.submit([1] * 30, 5)
