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
