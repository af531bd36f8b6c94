"""Tensor-parallel decode on 2 GPUs (NCCL): every rank's logits from the TP=2 shards equal the TP=1
model's (same seed: shards are bitwise slices of the unsplit quantized weights) within 2e-3, eager
and through a captured CUDA graph.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, size, port, q):
    import torch.distributed as dist

    from densecore_b200.decoder import Decoder, DecoderConfig
    from densecore_b200.ggml_types import Q4_K
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=size, device_id=dev)
    try:
        cfg = DecoderConfig("tiny-llama", n_layer=2, hidden=512, n_head=8, n_head_kv=4, head_dim=128, ffn=1024,
                            vocab=1024, rope_theta=5e5, rms_eps=1e-5, wtype=Q4_K, qk_norm=False, tied=False,
                            out_type=Q4_K)
        ref = Decoder(cfg, batch=3, max_ctx=64, seed=7, device=dev)
        sh = Decoder(cfg, batch=3, max_ctx=64, seed=7, device=dev, tp_rank=rank, tp_size=size,
                     tp_group=dist.group.WORLD)
        ref.fill_kv_random(3)
        h0, h1 = rank * sh.hkv, (rank + 1) * sh.hkv
        sh.k_arena.copy_(ref.k_arena[:, :, h0:h1])
        sh.v_arena.copy_(ref.v_arena[:, :, h0:h1])
        assert torch.equal(sh.block_tables, ref.block_tables)
        toks = torch.tensor([5, 700, 1023], device=dev)
        ctx = torch.tensor([9, 30, 47], dtype=torch.int32, device=dev)
        results = []
        for mode in ("eager", "graph"):
            for d in (ref, sh):
                d.tokens.copy_(toks)
                d.ctx_lens.copy_(ctx)
            ref.step()
            if mode == "eager":
                sh.step()
            else:
                sh.replay()
            torch.cuda.synchronize()
            a, b = ref.logits.double().cpu().numpy(), sh.logits.double().cpu().numpy()
            err = float((np.linalg.norm(a - b, axis=-1) / np.linalg.norm(a, axis=-1)).max())
            results.append((mode, err, bool(torch.equal(ref.next_tokens, sh.next_tokens))))
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_tp2_decode_matches_tp1():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, results in res:
        for mode, err, same in results:
            assert err < 2e-3 and same, (rank, mode, err, same)
