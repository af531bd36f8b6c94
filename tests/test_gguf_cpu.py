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
