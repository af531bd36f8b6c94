"""Pins the CPU oracle against the golden fixtures (gguf's ggml-bit-exact Q8_0 quantizer and
Q8_0/Q4_K/Q6_K dequantizers; DenseCore's own FlashAttentionGQA) and against a float64
restatement of each vec_dot through dequantization."""
import os

import numpy as np
import pytest

from oracle import oracle as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def test_q8_0_quantize_bytes_match_gguf():
    q = O.quantize(G["q8_0_x"], O.Q8_0)
    assert np.array_equal(q, G["q8_0_bytes"])


@pytest.mark.parametrize("name,qt,blk,nb", [("q8_0", O.Q8_0, 32, 34), ("q4_K", O.Q4_K, 256, 144),
                                            ("q6_K", O.Q6_K, 256, 210)])
def test_dequantize_matches_gguf(name, qt, blk, nb):
    b = G[f"deq_{name}_bytes"]
    ref = G[f"deq_{name}_f32"]
    got = O.dequantize(b.reshape(-1), qt, b.shape[0] * blk).reshape(-1)
    assert np.array_equal(got, ref)


def _rand(rng, shape, std):
    return (rng.standard_normal(shape) * std).astype(np.float32)


@pytest.mark.parametrize("wt", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_vec_dot_equals_dequantized_dot(wt):
    rng = np.random.default_rng(7)
    k = 1024
    w = O.quantize(_rand(rng, (4, k), 0.02), wt)
    x = _rand(rng, (1, k), 1.0)
    xt = O.VEC_DOT_TYPE[wt]
    xq = O.quantize(x, xt)
    xd = O.dequantize(xq, xt, k).astype(np.float64)[0]
    for r in range(4):
        wd = O.dequantize(w[r], wt, k).astype(np.float64)[0]
        ref = float(wd @ xd)
        got = O.vec_dot(wt, k, w[r], xq[0])
        assert abs(got - ref) <= 1e-5 * float(np.abs(wd * xd).sum()) + 1e-12


@pytest.mark.parametrize("wt", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_weight_quantizer_roundtrip_error(wt):
    rng = np.random.default_rng(3)
    x = _rand(rng, (8, 512), 0.02)
    q = O.quantize(x, wt)
    xd = O.dequantize(q, wt, 512)
    rel = np.linalg.norm(xd - x) / np.linalg.norm(x)
    assert rel < {O.Q8_0: 0.01, O.Q4_K: 0.12, O.Q6_K: 0.03}[wt]


def test_q8_K_spec_properties():
    rng = np.random.default_rng(5)
    x = _rand(rng, (3, 512), 1.0)
    x[1, :256] = 0.0
    q = O.quantize(x, O.Q8_K)
    for r in range(3):
        for b in range(2):
            blk = q[r, b * 292:(b + 1) * 292]
            d = blk[:4].view(np.float32)[0]
            qs = blk[4:260].view(np.int8).astype(np.int32)
            bs = blk[260:292].view(np.int16).astype(np.int32)
            assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
            xb = x[r, b * 256:(b + 1) * 256]
            if not xb.any():
                assert d == 0 and not qs.any()
                continue
            i = int(np.argmax(np.abs(xb)))
            assert qs[i] == -127          # the max-magnitude element maps to -127
            assert np.max(np.abs(qs * d - xb)) <= abs(d) * 0.5 + 1e-6


def test_attention_oracle_matches_reference_flash_attention():
    Q, K, V = G["attn_q"], G["attn_k"], G["attn_v"]
    B, hq, _, d = Q.shape
    hkv, skv = K.shape[1], K.shape[2]
    scale = float(G["attn_scale"])
    # lay the dense K/V into a paged arena with a shuffled block table
    n_layer, layer = 3, 1
    nblk = (skv + 15) // 16
    rng = np.random.default_rng(0)
    perm = rng.permutation(B * nblk + 5)[: B * nblk].reshape(B, nblk).astype(np.int32)
    nphys = B * nblk + 5
    ka = np.zeros((nphys * n_layer, 16, hkv, d), np.float16)
    va = np.zeros_like(ka)
    for s in range(B):
        for t in range(skv):
            pb = perm[s, t // 16] * n_layer + layer
            ka[pb, t % 16] = K[s, :, t]
            va[pb, t % 16] = V[s, :, t]
    out = O.paged_attn_decode(Q[:, :, 0], ka, va, n_layer, layer, perm, np.full(B, skv), hkv,
                              scale, nthreads=4)
    ref = G["attn_out_ref"][:, :, 0]
    assert np.max(np.abs(out - ref)) / np.max(np.abs(ref)) < 2e-5


def test_kv_append_then_attention_roundtrip():
    rng = np.random.default_rng(11)
    hkv, d, n_layer = 2, 64, 2
    bt = np.array([[3, 0], [1, 2]], np.int32)
    ka = np.zeros((4 * n_layer, 16, hkv, d), np.float16)
    va = np.zeros_like(ka)
    k = rng.standard_normal((3, hkv, d)).astype(np.float32)
    v = rng.standard_normal((3, hkv, d)).astype(np.float32)
    O.kv_append(k, v, ka, va, n_layer, 1, bt, [0, 1, 0], [17, 0, 5])
    assert np.array_equal(ka[0 * n_layer + 1, 1], k[0].astype(np.float16))
    assert np.array_equal(va[1 * n_layer + 1, 0], v[1].astype(np.float16))
    assert np.array_equal(ka[3 * n_layer + 1, 5], k[2].astype(np.float16))


@pytest.mark.parametrize("isa", ["avx2", "avx512vnni"])
def test_simd_q4_K_dot_is_bit_identical(isa):
    """The AVX2 and AVX-512 VNNI restatements of vec_dot_q4_K_q8_K (the CPU baseline's compute)
    give the scalar oracle's bits, including ragged row counts and the shortest row, and extreme
    nibbles / activation bytes."""
    import numpy as np
    from oracle import oracle as O
    if isa == "avx512vnni" and O.simd_isa() != "avx512vnni":
        pytest.skip("no AVX-512 VNNI on this CPU")
    if O.simd_isa() == "scalar":
        pytest.skip("no AVX2 on this CPU")
    rng = np.random.default_rng(11)
    for n, k, m in ((64, 4096, 1), (37, 14336, 3), (5, 256, 2)):
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        x[0, :16] = 100.0   # activation bytes at +-127
        x[0, 16:32] = -100.0
        wq, xq = O.quantize(w, O.Q4_K), O.quantize(x, O.Q8_K)
        a = O.mul_mat(O.Q4_K, wq, k, xq, m, nthreads=3)
        b = O.mul_mat(O.Q4_K, wq, k, xq, m, nthreads=3, simd=isa)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_prefill_matches_reference_causal_flash_attention():
    """Prefill semantics pinned to DenseCore's own FlashAttentionGQA with causal = true
    (core/include/flash_attention.h:239-272): N new tokens from position 0 over a paged arena equal
    the reference's causal attention over the dense fp16-valued K/V (Sq = Skv = N)."""
    rng = np.random.default_rng(31)
    B, hq, hkv, N, d = 2, 8, 2, 37, 128
    Q = rng.standard_normal((B, hq, N, d)).astype(np.float32)
    K = rng.standard_normal((B, hkv, N, d)).astype(np.float16).astype(np.float32)
    V = rng.standard_normal((B, hkv, N, d)).astype(np.float16).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    ref = O.ref_flash_attention_gqa(Q, K, V, scale, causal=True)
    if ref is None:
        pytest.skip("reference FlashAttentionGQA not built here")
    nblk = (N + 15) // 16
    bt = np.arange(B * nblk, dtype=np.int32)[::-1].reshape(B, nblk).copy()
    ka = np.zeros((B * nblk, 16, hkv, d), np.float16)
    va = np.zeros_like(ka)
    for s in range(B):
        for t in range(N):
            ka[bt[s, t // 16], t % 16] = K[s, :, t].astype(np.float16)
            va[bt[s, t // 16], t % 16] = V[s, :, t].astype(np.float16)
    q = np.ascontiguousarray(Q.transpose(0, 2, 1, 3).reshape(B * N, hq, d))
    got = O.paged_attn_prefill(q, ka, va, 1, 0, bt, np.array([0, N, 2 * N]), np.array([N, N]), hkv, scale)
    want = ref.transpose(0, 2, 1, 3).reshape(B * N, hq, d)
    err = np.linalg.norm(got - want, axis=-1) / np.linalg.norm(want, axis=-1)
    assert err.max() < 1e-5, err.max()
