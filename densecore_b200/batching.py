"""Continuous batching around the captured decode step: requests join and leave a fixed set of
slots between graph replays, each with its own KV blocks.  This is the host loop of DenseCore's
worker (core/src/worker.cpp:365-544: admit, build the batch, compute, sample, retire) with the
per-sequence semantics the reference's batched path lacks -- every sequence reads only its own
positions through its own block table, so its tokens do not depend on what else is in the batch.

A newly admitted request's whole prompt is ingested by one prefill pass (Decoder.prefill: every
matmul at M = prompt tokens, multi-token causal attention), batched over the requests admitted in
the same step; its last token's logits give the first generated token.  With prefill=False prompts
are instead fed one token per step through the decode graph.  Sampling is greedy.  Idle slots
point at one reserved block and run a harmless one-token step.
"""
from __future__ import annotations

import collections
import dataclasses

import torch

from .decoder import KV_BLOCK, Decoder


class BlockAllocator:
    """Free list over the KV arena's physical blocks (kv_cache.cpp's block pool)."""

    def __init__(self, n_blocks: int):
        self.free = collections.deque(range(n_blocks))
        self.n_blocks = n_blocks

    def alloc(self, n: int) -> list[int] | None:
        if n > len(self.free):
            return None
        return [self.free.popleft() for _ in range(n)]

    def release(self, blocks: list[int]):
        if len(set(blocks)) != len(blocks) or any(b < 0 or b >= self.n_blocks for b in blocks):
            raise ValueError("bad block list")
        self.free.extend(blocks)
        if len(self.free) > self.n_blocks:
            raise ValueError("block released twice")


@dataclasses.dataclass
class Request:
    rid: int
    prompt: list[int]
    max_new: int
    eos: int | None = None
    out: list[int] = dataclasses.field(default_factory=list)
    # runtime state
    slot: int = -1
    blocks: list[int] = dataclasses.field(default_factory=list)
    pos: int = 0          # tokens already written to the cache

    @property
    def capacity(self) -> int:
        return len(self.prompt) + self.max_new

    def next_input(self) -> int:
        return self.prompt[self.pos] if self.pos < len(self.prompt) else self.out[-1]

    def done(self) -> bool:
        return len(self.out) >= self.max_new or (self.eos is not None and self.out and self.out[-1] == self.eos)


class ContinuousBatcher:
    """Runs requests through `dec` (its batch size is the slot count)."""

    def __init__(self, dec: Decoder, prefill: bool = True):
        self.dec = dec
        self.use_prefill = prefill
        self.slots: list[Request | None] = [None] * dec.batch
        self.alloc = BlockAllocator(dec.n_blocks)
        self.idle_block = self.alloc.alloc(1)[0]   # where idle slots write their throw-away token
        self.queue: collections.deque[Request] = collections.deque()
        self.finished: list[Request] = []
        self._bt = torch.full((dec.batch, dec.blocks_per_seq), self.idle_block, dtype=torch.int32)
        self._tok = torch.zeros(dec.batch, dtype=torch.long)
        self._ctx = torch.ones(dec.batch, dtype=torch.int32)
        self._next_id = 0

    def submit(self, prompt: list[int], max_new: int, eos: int | None = None) -> Request:
        if not prompt or max_new < 1:
            raise ValueError("need a non-empty prompt and max_new >= 1")
        r = Request(self._next_id, list(prompt), max_new, eos)
        if r.capacity > self.dec.max_ctx:
            raise ValueError(f"request needs {r.capacity} positions, the decoder holds {self.dec.max_ctx}")
        self._next_id += 1
        self.queue.append(r)
        return r

    def _admit(self) -> list[Request]:
        new = []
        for s in range(len(self.slots)):
            if self.slots[s] is not None or not self.queue:
                continue
            r = self.queue[0]
            blocks = self.alloc.alloc((r.capacity + KV_BLOCK - 1) // KV_BLOCK)
            if blocks is None:
                break                       # wait for blocks to be released (FIFO admission)
            self.queue.popleft()
            r.slot, r.blocks = s, blocks
            self.slots[s] = r
            self._bt[s].fill_(self.idle_block)
            self._bt[s, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
            new.append(r)
        return new

    def _retire(self, s: int, r: Request):
        self.alloc.release(r.blocks)
        r.blocks, r.slot = [], -1
        self.slots[s] = None
        # the idle slot's throw-away writes must not land in blocks that now belong to others
        self._bt[s].fill_(self.idle_block)
        self.finished.append(r)

    def step(self) -> bool:
        """Admit waiting requests (prefilling their prompts), run one decode step for every slot,
        retire finished requests.  Returns False when there is nothing left to do."""
        new = self._admit()
        dec = self.dec
        dec.block_tables.copy_(self._bt, non_blocking=False)
        if new and self.use_prefill:
            nxt, _ = dec.prefill([r.slot for r in new], [r.prompt for r in new])
            for r, t in zip(new, nxt.tolist()):
                r.pos = len(r.prompt)
                r.out.append(int(t))
                if r.done():
                    self._retire(r.slot, r)
        active = [r for r in self.slots if r is not None]
        if not active:
            return bool(self.queue)
        for s, r in enumerate(self.slots):
            if r is None:
                self._tok[s], self._ctx[s] = 0, 1
            else:
                self._tok[s], self._ctx[s] = r.next_input(), r.pos + 1
        dec.tokens.copy_(self._tok)
        dec.ctx_lens.copy_(self._ctx)
        dec.replay()
        nxt = dec.next_tokens.cpu()
        for s, r in enumerate(self.slots):
            if r is None:
                continue
            r.pos += 1
            if r.pos >= len(r.prompt):      # the last prompt token and every generated one predict
                r.out.append(int(nxt[s]))
            if r.done():
                self._retire(s, r)
        return True

    def run(self, max_steps: int = 1 << 30) -> list[Request]:
        n = 0
        while n < max_steps and self.step():
            n += 1
        return self.finished
