"""GPU parity of paged decode attention and KV append against the CPU oracle (which is itself
pinned to DenseCore's FlashAttentionGQA), through the C ABI.  Attention bar: 2e-3 relative
(per (sequence, head) output vector, L2); KV append: bit-exact fp16 slots."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200 import ops as _ops
    return _ops


def make_cache(rng, ctx, hkv, n_layer, d=128, extra_blocks=3):
    """Random fp16 arena with a shuffled block table per sequence (blocks shared across layers)."""
    nblk = [(c + 15) // 16 for c in ctx]
    total = sum(nblk) + extra_blocks
    mbs = max(max(nblk), 1)
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(ctx), mbs), np.int32)
    o = 0
    for s, nb in enumerate(nblk):
        bt[s, :nb] = perm[o:o + nb]
        o += nb
    ka = rng.standard_normal((total * n_layer, 16, hkv, d)).astype(np.float16)
    va = rng.standard_normal((total * n_layer, 16, hkv, d)).astype(np.float16)
    return ka, va, bt


def check(ops, ctx, hq, hkv, n_layer=2, layer=1, seed=0):
    rng = np.random.default_rng(seed)
    ka, va, bt = make_cache(rng, ctx, hkv, n_layer)
    q = rng.standard_normal((len(ctx), hq, 128)).astype(np.float32)
    scale = 1.0 / np.sqrt(128.0)
    ref = O.paged_attn_decode(q, ka, va, n_layer, layer, bt, np.array(ctx), hkv, scale, nthreads=8)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = ops.paged_attn_decode(dev(q), dev(ka), dev(va), n_layer, layer, dev(bt),
                                dev(np.array(ctx, np.int32)), hkv, max(ctx)).cpu().numpy()
    err = np.linalg.norm(out - ref, axis=-1) / (np.linalg.norm(ref, axis=-1) + 1e-30)
    assert err.max() < ATOL_REL, f"max rel err {err.max():.2e}"
    return err.max()


@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (64, 8), (8, 8)])
def test_attention_small_contexts(ops, hq, hkv):
    check(ops, [1, 15, 16, 17, 33, 100], hq, hkv)


def test_attention_config3_shapes(ops):
    """Config 3: 64 sequences, contexts U[128, 2048] from seed 2, 16 Q / 8 KV heads."""
    ctx = np.random.default_rng(2).integers(128, 2049, 64).tolist()
    check(ops, ctx, 16, 8, n_layer=1, layer=0)


def test_attention_long_single_sequence_many_splits(ops):
    check(ops, [4096], 32, 8, n_layer=1, layer=0)


def test_attention_matches_reference_flash_attention_golden(ops):
    """Dense K/V of the golden fixture (DenseCore FlashAttentionGQA output) laid into a paged
    arena; GPU output matches the reference's own CPU output."""
    G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    Q, K, V = G["attn_q"], G["attn_k"], G["attn_v"]
    B, hq, _, d = Q.shape
    hkv, skv = K.shape[1], K.shape[2]
    nblk = (skv + 15) // 16
    bt = (np.arange(B * nblk, dtype=np.int32)[::-1].reshape(B, nblk)).copy()
    ka = np.zeros((B * nblk, 16, hkv, d), np.float16)
    va = np.zeros_like(ka)
    for s in range(B):
        for t in range(skv):
            ka[bt[s, t // 16], t % 16] = K[s, :, t]
            va[bt[s, t // 16], t % 16] = V[s, :, t]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = ops.paged_attn_decode(dev(Q[:, :, 0]), dev(ka), dev(va), 1, 0, dev(bt),
                                dev(np.full(B, skv, np.int32)), hkv, skv,
                                float(G["attn_scale"])).cpu().numpy()
    ref = G["attn_out_ref"][:, :, 0]
    assert np.abs(out - ref).max() / np.abs(ref).max() < ATOL_REL


def test_kv_append_bit_exact(ops):
    rng = np.random.default_rng(4)
    hkv, d, n_layer = 8, 128, 3
    ctx = [40, 7, 1]
    ka, va, bt = make_cache(rng, ctx, hkv, n_layer)
    seq = np.array([0, 1, 2, 0], np.int32)
    pos = np.array([39, 6, 0, 17], np.int32)
    k = rng.standard_normal((4, hkv, d)).astype(np.float32) * 3
    v = rng.standard_normal((4, hkv, d)).astype(np.float32) * 3
    ka_ref, va_ref = ka.copy(), va.copy()
    O.kv_append(k, v, ka_ref, va_ref, n_layer, 2, bt, seq, pos)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    kd, vd = dev(ka), dev(va)
    ops.kv_append(dev(k), dev(v), kd, vd, n_layer, 2, dev(bt), dev(seq), dev(pos))
    assert np.array_equal(kd.cpu().numpy().view(np.uint16), ka_ref.view(np.uint16))
    assert np.array_equal(vd.cpu().numpy().view(np.uint16), va_ref.view(np.uint16))


def test_attention_ignores_slots_past_the_context(ops):
    """Arena slots past each sequence's context (the tail of its last block) may hold anything,
    NaN and Inf bit patterns included: the output must equal the oracle's, which reads only
    positions 0..ctx_len-1."""
    rng = np.random.default_rng(17)
    ctx, hq, hkv, n_layer, layer = [1, 7, 16, 21, 40], 16, 8, 2, 0
    ka, va, bt = make_cache(rng, ctx, hkv, n_layer)
    for s, c in enumerate(ctx):
        for p in range(c, ((c + 15) // 16) * 16):
            blk = bt[s, p // 16] * n_layer + layer
            ka[blk, p % 16] = np.nan
            va[blk, p % 16] = np.inf if p % 2 else np.nan
    q = rng.standard_normal((len(ctx), hq, 128)).astype(np.float32)
    scale = 1.0 / np.sqrt(128.0)
    ref = O.paged_attn_decode(q, ka, va, n_layer, layer, bt, np.array(ctx), hkv, scale, nthreads=8)
    assert np.isfinite(ref).all()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = ops.paged_attn_decode(dev(q), dev(ka), dev(va), n_layer, layer, dev(bt),
                                dev(np.array(ctx, np.int32)), hkv, max(ctx)).cpu().numpy()
    assert np.isfinite(out).all()
    err = np.linalg.norm(out - ref, axis=-1) / (np.linalg.norm(ref, axis=-1) + 1e-30)
    assert err.max() < ATOL_REL


def check_prefill(ops, ctx, ntok, hq, hkv, n_layer=2, layer=1, seed=0, nan_tail=False):
    """New tokens per sequence (ntok[s] of them, the last at position ctx[s] - 1) against the
    oracle's per-token causal attention."""
    rng = np.random.default_rng(seed)
    ka, va, bt = make_cache(rng, ctx, hkv, n_layer)
    if nan_tail:   # slots past each context hold NaN / Inf bit patterns
        for s, c in enumerate(ctx):
            if c % 16:
                blk = bt[s, c // 16]
                ka[blk * n_layer + layer, c % 16:] = np.float16(np.nan)
                va[blk * n_layer + layer, c % 16:] = np.float16(np.inf)
    starts = np.concatenate([[0], np.cumsum(ntok)]).astype(np.int32)
    q = rng.standard_normal((int(starts[-1]), hq, 128)).astype(np.float32)
    scale = 1.0 / np.sqrt(128.0)
    ref = O.paged_attn_prefill(q, ka, va, n_layer, layer, bt, starts, np.array(ctx), hkv, scale, nthreads=8)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = ops.paged_attn_prefill(dev(q), dev(ka), dev(va), n_layer, layer, dev(bt), dev(starts),
                                 dev(np.array(ctx, np.int32)), hkv, int(max(ntok)), max(ctx)).cpu().numpy()
    err = np.linalg.norm(out - ref, axis=-1) / (np.linalg.norm(ref, axis=-1) + 1e-30)
    assert np.isfinite(out).all()
    assert err.max() < ATOL_REL, f"max rel err {err.max():.2e}"


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 8), (64, 8)])
def test_prefill_ragged_sequences(ops, hq, hkv):
    """Whole prompts (ctx == ntok), prompt chunks after history (ctx > ntok), one-token rows."""
    check_prefill(ops, [1, 17, 40, 100, 300], [1, 17, 9, 100, 33], hq, hkv)


def test_prefill_ignores_slots_past_the_context(ops):
    check_prefill(ops, [5, 21, 70], [5, 3, 70], 32, 8, nan_tail=True)


def test_prefill_2048_tokens(ops):
    """Config-4 prefill shape: a 2048-token prompt, 32 Q / 8 KV heads."""
    check_prefill(ops, [2048], [2048], 32, 8, n_layer=1, layer=0)
