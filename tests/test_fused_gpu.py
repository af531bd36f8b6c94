"""GPU parity of the fused pre-matmul producers against float64 references (oracle quantizers for
the activation bytes): residual add is bit-exact; the quantized activation matches quantize(ref) in
>= 99.9% of bytes (a different fp32 reduction order may move a value across a rounding boundary) and
dequantizes to within half a quantization step (plus the fp16 rounding of the Q8_0 scale) of the reference; QK-norm + RoPE'd q within 1e-5 of
max|q| of ggml's fp32 formulas (tests/chained_ref.py); fp16 slots within one fp16 ulp."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200 import ops as _ops
    return _ops


def _align(x):
    return (x + 255) // 256 * 256


def act_to_ggml(buf: np.ndarray, at: int, m: int, k: int) -> np.ndarray:
    """SoA device activation -> ggml Q8_0 / Q8_K rows (for the oracle's dequantizer)."""
    qs = buf[: m * k].view(np.int8).reshape(m, k)
    off = _align(m * k)
    if at == O.Q8_0:
        d = buf[off: off + m * (k // 32) * 2].view(np.float16).reshape(m, k // 32)
        out = np.zeros((m, k // 32, 34), np.uint8)
        out[..., :2] = d.view(np.uint8).reshape(m, k // 32, 2)
        out[..., 2:] = qs.reshape(m, k // 32, 32).view(np.uint8)
        return out.reshape(m, -1)
    d = buf[off: off + m * (k // 256) * 4].view(np.float32).reshape(m, k // 256)
    off2 = off + _align(m * (k // 256) * 4)
    bs = buf[off2: off2 + m * (k // 16) * 2].view(np.int16).reshape(m, k // 256, 16)
    out = np.zeros((m, k // 256, 292), np.uint8)
    out[..., :4] = d.view(np.uint8).reshape(m, k // 256, 4)
    out[..., 4:260] = qs.reshape(m, k // 256, 256).view(np.uint8)
    out[..., 260:] = bs.view(np.uint8).reshape(m, k // 256, 32)
    return out.reshape(m, -1)


def check_act(buf, at, ref, m, k):
    rows = act_to_ggml(buf, at, m, k)
    want = O.quantize(ref.astype(np.float32), at)
    bb, dn, nq = (34, 2, 32) if at == O.Q8_0 else (292, 4, 256)
    g, w = rows.reshape(m, -1, bb), want.reshape(m, -1, bb)
    # quants: equal but for values that a last-ulp difference in fp32 math moves across a boundary
    assert (g[..., dn:dn + nq] == w[..., dn:dn + nq]).mean() > 0.999
    sd = np.float16 if at == O.Q8_0 else np.float32
    dg = g[..., :dn].copy().view(sd).astype(np.float64)
    dw = w[..., :dn].copy().view(sd).astype(np.float64)
    assert np.allclose(dg, dw, rtol=1e-3 if at == O.Q8_0 else 1e-6, atol=0)
    if at == O.Q8_K:   # bsums are the exact 16-value sums of the kernel's own quants
        qs = g[..., 4:260].copy().view(np.int8).astype(np.int32).reshape(m, -1, 16, 16).sum(-1)
        assert np.array_equal(g[..., 260:].copy().view(np.int16).reshape(m, -1, 16), qs)
    deq = O.dequantize(rows, at, k)
    blk = 32 if at == O.Q8_0 else 256
    step = np.abs(ref).reshape(m, -1, blk).max(-1, keepdims=True) / 127.0
    err = np.abs(deq - ref).reshape(m, -1, blk)
    # |q*d' - x| <= d/2 + 127*|d' - d|; Q8_0 stores d in fp16 (|d' - d| <= 2^-11 d), Q8_K in f32
    slack = 0.5 + (127 * 2.0 ** -11 if at == O.Q8_0 else 1e-3)
    assert np.all(err <= slack * step + 1e-6)


@pytest.mark.parametrize("at,k", [(O.Q8_0, 1024), (O.Q8_K, 2560), (O.Q8_K, 8192)])
def test_add_rmsnorm_quantize(ops, at, k):
    rng = np.random.default_rng(k)
    m, eps = 5, 1e-6
    x = rng.standard_normal((m, k)).astype(np.float32)
    dl = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, k).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    act = torch.empty(ops._lib.load().dcg_act_size(at, m, k), dtype=torch.uint8, device="cuda")
    ops.add_rmsnorm_quantize(xd, torch.from_numpy(w).cuda(), eps, at, act, torch.from_numpy(dl).cuda())
    xs = x + dl
    assert np.array_equal(xd.cpu().numpy(), xs)                      # residual add, in place
    x64 = xs.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + eps) * w
    check_act(act.cpu().numpy(), at, ref, m, k)


@pytest.mark.parametrize("at,ffn", [(O.Q8_0, 3072), (O.Q8_K, 9728)])
def test_swiglu_quantize(ops, at, ffn):
    rng = np.random.default_rng(ffn)
    m = 4
    gu = rng.standard_normal((m, 2 * ffn)).astype(np.float32)
    gd = torch.from_numpy(gu).cuda()
    act = torch.empty(ops._lib.load().dcg_act_size(at, m, ffn), dtype=torch.uint8, device="cuda")
    ops.swiglu_quantize(gd, gd[:, ffn:], 2 * ffn, m, ffn, at, act)
    g, u = gu[:, :ffn].astype(np.float64), gu[:, ffn:].astype(np.float64)
    check_act(act.cpu().numpy(), at, g / (1 + np.exp(-g)) * u, m, ffn)


@pytest.mark.parametrize("qk_norm", [True, False])
def test_qk_norm_rope_kv_append(ops, qk_norm):
    rng = np.random.default_rng(9)
    B, hq, hkv, D, n_layer, layer, theta, eps = 3, 8, 2, 128, 2, 1, 1e6, 1e-6
    n = (hq + 2 * hkv) * D
    qkv = rng.standard_normal((B, n)).astype(np.float32)
    pos = np.array([0, 17, 300], np.int32)
    mbs = 20
    bt = rng.permutation(B * mbs).astype(np.int32).reshape(B, mbs)
    ka = np.zeros((B * mbs * n_layer, 16, hkv, D), np.float16)
    va = np.zeros_like(ka)
    qw = rng.uniform(0.5, 1.5, D).astype(np.float32) if qk_norm else None
    kw = rng.uniform(0.5, 1.5, D).astype(np.float32) if qk_norm else None
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qkv_d, ka_d, va_d = dev(qkv), dev(ka), dev(va)
    q_out = torch.empty((B, hq, D), device="cuda")
    ops.qk_norm_rope_kv_append(qkv_d, n, qkv_d[:, hq * D:], n, qkv_d[:, (hq + hkv) * D:], n, B, hq, hkv,
                               dev(qw) if qk_norm else None, dev(kw) if qk_norm else None, eps, theta,
                               dev(pos), q_out, ka_d, va_d, n_layer, layer, dev(bt))

    import chained_ref as CR

    def ref(x, w):   # ggml's fp32 rms_norm and NeoX RoPE (angle recurrence theta *= powf(base, -2/D))
        if w is not None:
            x = CR.rms_norm(x, w, eps)
        return CR.rope_neox(np.asarray(x, np.float32), pos, theta)

    q = ref(qkv[:, : hq * D].reshape(B, hq, D), qw)
    k = ref(qkv[:, hq * D:(hq + hkv) * D].reshape(B, hkv, D), kw)
    v = qkv[:, (hq + hkv) * D:].reshape(B, hkv, D)
    # fp32 cosf / sinf of the GPU and of the host may differ in the last place
    assert np.abs(q_out.cpu().numpy() - q).max() <= 1e-5 * np.abs(q).max()
    kg, vg = ka_d.cpu().numpy(), va_d.cpu().numpy()
    for s in range(B):
        blk = bt[s, pos[s] // 16] * n_layer + layer
        got_k = kg[blk, pos[s] % 16]
        ulp_k = np.abs(got_k.view(np.int16).astype(np.int32) - k[s].astype(np.float16).view(np.int16).astype(np.int32))
        assert ulp_k.max() <= 1
        assert np.array_equal(vg[blk, pos[s] % 16], v[s].astype(np.float16))
