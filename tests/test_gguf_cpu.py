"""GGUF reader (densecore_b200.gguf_file) against files written by gguf-py: metadata, tensor
directory and bytes, and the decoder configuration derived from them (CPU only)."""
import numpy as np
import pytest

from densecore_b200 import gguf_file
from oracle import oracle as O
from tests.gguf_fixture import TINY, write_tiny_gguf


@pytest.mark.parametrize("tied,qk_norm", [(False, True), (True, False)])
def test_reader_and_config(tmp_path, tied, qk_norm):
    path = str(tmp_path / "tiny.gguf")
    want = write_tiny_gguf(path, qk_norm=qk_norm, tied=tied)
    g = gguf_file.GGUFFile(path)
    assert g.metadata["general.architecture"] == "qwen3"
    assert g.hparam("block_count") == TINY["n_layer"] and g.hparam("attention.key_length") == 128
    assert set(g.tensors) == set(want)
    for name, v in want.items():
        if isinstance(v, tuple):
            rows, t, k = v
            ti = g.tensors[name]
            assert ti.ggml_type == t and ti.dims == (k, rows.shape[0])
            assert np.array_equal(g.tensor_bytes(name), rows)
        else:
            assert np.array_equal(g.tensor_f32(name), v)
    cfg = gguf_file.decoder_config(g)
    assert (cfg.n_layer, cfg.hidden, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.ffn, cfg.vocab) == \
        tuple(TINY[k] for k in ("n_layer", "hidden", "n_head", "n_head_kv", "head_dim", "ffn", "vocab"))
    assert cfg.rope_theta == 1e6 and abs(cfg.rms_eps - 1e-6) < 1e-12
    assert cfg.qk_norm == qk_norm and cfg.tied == tied and cfg.wtype == O.Q4_K
    w = gguf_file.decoder_weights(g)
    assert ("output.weight" in w) == (not tied)
    assert ("blk.1.attn_q_norm.weight" in w) == qk_norm


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + bytes(20))
    with pytest.raises(ValueError, match="not a GGUF"):
        gguf_file.GGUFFile(str(p))
    good = str(tmp_path / "tiny.gguf")
    write_tiny_gguf(good)
    data = open(good, "rb").read()
    (tmp_path / "short.gguf").write_bytes(data[: len(data) // 2])
    with pytest.raises(ValueError, match="past the end|truncated"):
        gguf_file.GGUFFile(str(tmp_path / "short.gguf"))


@pytest.mark.parametrize("t", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_shards_equal_quantized_slices(t):
    """A tensor-parallel shard of file weights (whole rows, or whole blocks of columns) has the
    bytes of the quantized slice of the matrix, so sharded ranks hold exactly the unsplit model."""
    rng = np.random.default_rng(t)
    n, k = 96, 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    rows = O.quantize(w, t)
    assert np.array_equal(gguf_file.shard_rows(rows, 32, 80), O.quantize(w[32:80], t))
    sc, sk = gguf_file.shard_cols(rows, t, k, 256, 768)
    assert sk == 512 and np.array_equal(sc, O.quantize(np.ascontiguousarray(w[:, 256:768]), t))
    with pytest.raises(ValueError, match="block boundaries"):
        gguf_file.shard_cols(rows, t, k, 16 if t == O.Q8_0 else 128, 768)


def test_tp_shard_plan_on_file_weights(tmp_path):
    """The decoder's tensor-parallel plan applied to GGUF weights: every rank's shard of every
    linear weight is well formed and the shards tile the unsplit weight."""
    from densecore_b200.decoder import tp_plan
    path = str(tmp_path / "tiny.gguf")
    write_tiny_gguf(path, qk_norm=False)
    g = gguf_file.GGUFFile(path)
    cfg = gguf_file.decoder_config(g)
    w = gguf_file.decoder_weights(g)
    plans = [tp_plan(cfg, r, 2) for r in range(2)]
    r, t, k = w["blk.0.ffn_down.weight"]
    parts = [gguf_file.shard_cols(r, t, k, *p["down_cols"]) for p in plans]
    assert sum(pk for _, pk in parts) == k
    assert np.array_equal(np.concatenate([pr for pr, _ in parts], axis=1), r)
    r, t, k = w["blk.1.attn_q.weight"]
    assert np.array_equal(np.concatenate([gguf_file.shard_rows(r, *p["q_rows"]) for p in plans]), r)
