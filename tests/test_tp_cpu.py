"""Tensor-parallel host logic on CPU: the shard plan covers every weight exactly once with
256-aligned K splits, and (on 2 gloo ranks) K-split partial matmuls + all_reduce and row-split
matmuls + all_gather reproduce the full quantized matmul (oracle arithmetic)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from densecore_b200.decoder import LLAMA3_70B, QWEN3_0_6B, QWEN3_4B, tp_plan
from oracle import oracle as O


def test_plan_rejects_unaligned_splits():
    """The Qwen3 configs run as replicas: their FFN does not split into 256-aligned K shards."""
    for cfg, size in ((QWEN3_4B, 8), (QWEN3_0_6B, 8), (QWEN3_4B, 4)):
        with pytest.raises(ValueError):
            tp_plan(cfg, 0, size)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_plan_partitions(size):
    cfg = LLAMA3_70B
    plans = [tp_plan(cfg, r, size) for r in range(size)]
    D = cfg.head_dim
    for key, total in (("q_rows", cfg.n_head * D), ("kv_rows", cfg.n_head_kv * D), ("o_cols", cfg.n_head * D),
                       ("ffn_rows", cfg.ffn), ("down_cols", cfg.ffn), ("vocab_rows", cfg.vocab)):
        spans = [p[key] for p in plans]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(spans[i][1] == spans[i + 1][0] for i in range(size - 1))
    for p in plans:
        assert (p["o_cols"][1] - p["o_cols"][0]) % 256 == 0
        assert (p["down_cols"][1] - p["down_cols"][0]) % 256 == 0
        # a rank's q heads use exactly its kv heads (GQA group stays local)
        assert p["hq"] // p["hkv"] == cfg.n_head // cfg.n_head_kv


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, size, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        rng = np.random.default_rng(0)  # same data on every rank
        n, k, m = 64, 1024, 3
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        wq = O.quantize(w, O.Q4_K)
        xq_full = O.quantize(x, O.Q8_K)
        full = O.mul_mat(O.Q4_K, wq, k, xq_full, m)
        # K split: columns [r*k/size, ...) of W and x; 256-aligned so blocks stay whole
        ks = k // size
        wk = O.quantize(np.ascontiguousarray(w[:, rank * ks:(rank + 1) * ks]), O.Q4_K)
        xk = O.quantize(np.ascontiguousarray(x[:, rank * ks:(rank + 1) * ks]), O.Q8_K)
        part = torch.from_numpy(O.mul_mat(O.Q4_K, wk, ks, xk, m))
        dist.all_reduce(part)
        # row split: rows [r*n/size, ...) then all_gather of the columns
        ns = n // size
        rows = torch.from_numpy(O.mul_mat(O.Q4_K, np.ascontiguousarray(wq[rank * ns:(rank + 1) * ns]), k,
                                          xq_full, m))
        gathered = [torch.empty_like(rows) for _ in range(size)]
        dist.all_gather(gathered, rows)
        cat = torch.cat(gathered, dim=1).numpy()
        bound = np.abs(O.dequantize(xq_full, O.Q8_K, k)) @ np.abs(O.dequantize(wq, O.Q4_K, k)).T
        ok_k = bool(np.all(np.abs(part.numpy() - full) <= 1e-5 * bound + 1e-12))
        ok_r = bool(np.array_equal(cat, full))
        q.put((rank, ok_k, ok_r))
    finally:
        dist.destroy_process_group()


def test_tp_split_algebra_gloo():
    size = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, size, port, q)) for r in range(size)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(size)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] for r in res), res
