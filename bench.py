"""Benchmark of the quantized mat-vec hot path (Q4_K x Q8_K mul_mat at Llama-3-8B FFN shapes, M=1).

One step = the two FFN projections of one decode token (M=1): x[1,4096] . W_up^T (W 14336x4096)
and h[1,14336] . W_down^T (W 4096x14336), each the full mul_mat op (activation quantized to Q8_K
on the fly, then the Q4_K GEMV).  Weights come from an 8-slot ring of distinct seeded copies
(528 MB >> 126 MB L2) so every step streams its weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  value = weight GB/s of the whole job; e2e = the same metric
through the host-pointer C ABI (dcg_ctx_mul_mat: H2D of x, both kernels, D2H of y, per call).
--impl reference times the CPU implementation of the same op (the AVX-512 VNNI restatement of
ggml's vec_dot_q4_K_q8_K where the host has it, else AVX2; quantize_row_q8_K; all host threads)
on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "quant mat-vec weight GB/s (Q4_K x Q8_K FFN GEMV, M=1)"
UNIT = "GB/s"
SHAPES = ((14336, 4096), (4096, 14336))  # (n, k) of W_up and W_down
RING = 8
Q4_K, Q8_K = 12, 15


def q4k_bytes(n, k):
    return n * (k // 256) * 144


WEIGHT_BYTES = sum(q4k_bytes(n, k) for n, k in SHAPES)
# algorithmic bytes of one step (two launches of the M=1 kernel, which quantizes x itself):
# weights + f32 activation + f32 output
ALG_BYTES = sum(q4k_bytes(n, k) + 4 * k + 4 * n for n, k in SHAPES)


def read_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_traffic():
    """dram bytes per GEMV launch pair from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "gemv_q4_K_ffn_m1.txt")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_step:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clocks and throttle reasons during the timed region: NVML polled from a thread every
    ~0.5 ms (enough samples even for a short region), with nvidia-smi's 100 ms log as a cross-check."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.samples = []
        self._stop = None

    def _poll(self):
        import pynvml
        try:
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return
        while not self._stop.is_set():
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), float(mx), int(rs)))
            except Exception:
                break
            time.sleep(0.0005)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._th = threading.Thread(target=self._poll, daemon=True)
        self._th.start()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._th.join(timeout=2)
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [(sm, mx, [n for n, bit in self.REASONS if rs & bit]) for sm, mx, rs in self.samples]
        src = "nvml"
        if not rows:
            src = "nvidia-smi"
            names = [n for n, _ in self.REASONS]
            for line in (self.out or "").splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]),
                                 [names[i] for i, v in enumerate(parts[5:9]) if v == "Active"]))
                except ValueError:
                    continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({r for _, _, rr in rows for r in rr})
        top = max(r[0] for r in rows)
        loaded = [r[0] for r in rows if r[0] >= 0.5 * top] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(rows), "source": src}


def cpu_reference(budget_s: float, int4: bool = True):
    """The oracle's row-sliced mul_mat (ggml vec_dot_q4_K_q8_K restated, AVX-512 VNNI or AVX2 dots bit-identical
    to the scalar ones) plus quantize_row_q8_K on all host threads, on the same shapes; repeats
    whole steps until ~budget_s elapsed.  int4: also time DenseCore's own INT4 GEMV."""
    import numpy as np

    from oracle import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    mats = []
    for n, k in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
        mats.append((O.quantize(w, O.Q4_K), k, rng.standard_normal((1, k)).astype(np.float32)))
    steps = 0
    t0 = time.perf_counter()
    while True:
        for wq, k, x in mats:
            xq = O.quantize(x, O.Q8_K)
            O.mul_mat(O.Q4_K, wq, k, xq, 1, nthreads=threads, simd=True)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    isa = O.simd_isa()
    out = {"value": WEIGHT_BYTES * steps / el / 1e9, "unit": UNIT, "cores": threads,
           "kind": "port", "steps": steps, "seconds": el, "isa": isa,
           "sample": f"{steps} full steps (both FFN matmuls, M=1) of config 2 on {threads} "
                     f"host threads, {isa} restatement of ggml vec_dot_q4_K_q8_K (runtime-selected "
                     "best ISA, bit-identical to the scalar oracle)"}
    # side datapoint: DenseCore's own INT4 decode GEMV (its custom INT4 format, group 128) on the
    # same shapes -- the reference's best-ISA integer GEMV that is compiled here
    r = O.ref_int4_gemv(SHAPES, 128, threads, max(1.0, budget_s / 2)) if int4 else None
    if r is not None:
        out["reference_int4"] = {
            "value": r["weight_bytes_per_pass"] * r["passes"] / r["seconds"] / 1e9, "unit": UNIT,
            "kind": "reference", "cores": threads, "isa": r["isa"],
            "sample": f"{r['passes']} passes over W_up and W_down (M=1) with GemvInt4 "
                      f"(core/src/kernels/cpu_int4.cpp) in DenseCore's INT4 format, group 128"}
    return out


def matmul_point(qtype: int, n: int, k: int, m: int, dev, reps: int = 20) -> dict:
    """One mul_mat shape (activation quantize + matmul), CUDA-graph replays over a weight ring
    larger than L2; weight GB/s and int8 TOPS."""
    import torch

    from densecore_b200 import ops
    from densecore_b200.ggml_types import row_size
    wbytes = n * row_size(qtype, k)
    ring = max(2, -(-512 * 2**20 // wbytes))
    g = torch.Generator(device=dev)
    g.manual_seed(n + k + m)
    ws = [ops.QuantWeight.from_float(torch.randn((n, k), generator=g, device=dev) * 0.02, qtype)
          for _ in range(ring)]
    x = torch.randn((m, k), generator=g, device=dev)
    y = torch.empty((m, n), device=dev)
    scr = torch.empty(ops.mul_mat_scratch_size(qtype, n, k, m), dtype=torch.uint8, device=dev)

    def once():
        for w in ws:
            ops.mul_mat(w, x, out=y, scratch=scr)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        once()
    torch.cuda.current_stream().wait_stream(side)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        once()
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * ring)
    del ws
    torch.cuda.empty_cache()
    return {"n": n, "k": k, "m": m, "us": round(us, 2), "weight_gbs": round(wbytes / us / 1e3, 1),
            "int8_tops": round(2.0 * m * n * k / us / 1e6, 1)}


def decode_bench(which: str, steps: int, dev, warmup: int = 3):
    """Batched decode tokens/s of a random-init Qwen3-architecture decoder (Qwen3-0.6B Q8_0 at
    batch 64, contexts U[128, 2048] seed 2; Qwen3-4B Q4_K_M at batch 32, contexts U[2048, 4096]):
    KV history is seeded random fp16, and each replay of the step graph decodes the next position
    of every sequence (its greedy token fed back, contexts grow by one per step)."""
    import numpy as np
    import torch

    from densecore_b200 import decoder as D
    if which == "3":
        cfg, batch = D.QWEN3_0_6B, 64
        ctx = np.random.default_rng(2).integers(128, 2049, batch)
    else:
        cfg, batch = D.QWEN3_4B, 32
        ctx = np.random.default_rng(3).integers(2048, 4097, batch)
    max_ctx = int(ctx.max()) + warmup + steps + 2
    dec = D.Decoder(cfg, batch, max_ctx, seed=int(which), device=dev)
    dec.fill_kv_random()
    dec.tokens.copy_(torch.from_numpy(np.random.default_rng(4).integers(0, cfg.vocab, batch)))
    dec.ctx_lens.copy_(torch.from_numpy(ctx.astype(np.int32)))
    dec.capture(advance=True)
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    ctx0 = dec.ctx_lens.cpu().numpy().astype(np.int64)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec.graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # minimum bytes: weights every step + each step's KV history (contexts ctx0 .. ctx0 + steps - 1)
    kv_tok = cfg.n_layer * 2 * dec.hkv * cfg.head_dim * 2
    wbytes = dec.step_bytes(np.zeros(1, np.int64))
    nbytes = wbytes + kv_tok * int((ctx0.sum() * steps + batch * steps * (steps - 1) // 2) // steps)
    out = {"model": cfg.name + " architecture (random init)", "batch": batch,
           "weights": "Q8_0" if which == "3" else "Q4_K_M (Q6_K attn_v/ffn_down in even layers, Q6_K head)",
           "contexts": f"{int(ctx0.min())}-{int(ctx0.max())} at the first timed step, +1 per step",
           "steps": steps, "ms_per_step": round(ms, 4), "tokens_per_s": round(batch / (ms * 1e-3), 1),
           "min_bytes_per_step": nbytes, "achieved_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}
    if which == "4":
        out["prefill"] = prefill_bench(dec, cfg)
    del dec
    torch.cuda.empty_cache()
    return out


def prefill_bench(dec, cfg, n_tok: int = 2048, reps: int = 3):
    """Prefill of one 2048-token random prompt into a fresh sequence slot (time to first token)."""
    import numpy as np
    import torch
    prompt = np.random.default_rng(9).integers(0, cfg.vocab, n_tok).tolist()
    dec.ctx_lens.zero_()
    dec.prefill([0], [prompt])   # warm-up (allocations)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        dec.prefill([0], [prompt])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"prompt_tokens": n_tok, "ms": round(ms, 2), "tokens_per_s": round(n_tok / (ms * 1e-3), 1),
            "note": "eager launches (no graph); every matmul at M = 2048, causal paged attention"}


def tp70b_measure(ws: int, rank: int, dev, steps: int, layers: int = 0, warmup: int = 2):
    """Llama-3-70B architecture (random init, Q4_K), decode batch 128, contexts U[1024, 4096]
    (seed 5), tensor-parallel over the ws ranks of the default process group: QKV by kv-head group,
    gate|up by rows, attn_output and ffn_down along K with an NCCL all-reduce each, vocab-split LM
    head with an all-gather.  Each replay decodes the next position of every sequence.  Returns the
    rank-0 result (max over ranks of the device time), None on other ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from densecore_b200 import decoder as D
    batch = 128
    ctx = np.random.default_rng(5).integers(1024, 4097, batch)
    cfg = D.LLAMA3_70B if layers <= 0 else dataclasses.replace(D.LLAMA3_70B, n_layer=layers)
    grow = steps + warmup + 2
    dec = D.Decoder(cfg, batch, int(ctx.max()) + grow, seed=5, device=dev, tp_rank=rank, tp_size=ws,
                    tp_group=dist.group.WORLD if ws > 1 else None, shard_init="local", seq_tokens=ctx + grow)
    dec.fill_kv_random()
    dec.tokens.copy_(torch.from_numpy(np.random.default_rng(6).integers(0, D.LLAMA3_70B.vocab, batch)))
    dec.ctx_lens.copy_(torch.from_numpy(ctx.astype(np.int32)))
    dec.capture(advance=True)
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec.graph.replay()
    e1.record()
    torch.cuda.synchronize()
    vals = [e0.elapsed_time(e1) / steps, 0.0]
    # the step's collectives alone: 2 all-reduces per layer of the [128, 8192] fp32 partial outputs
    # and the logits all-gather, captured the same way
    if ws > 1:
        y = torch.zeros((batch, cfg.hidden), device=dev)
        lg = torch.zeros((batch, dec.vocab_r), device=dev)
        gat = torch.zeros((ws, batch, dec.vocab_r), device=dev)

        def colls():
            for _ in range(2 * cfg.n_layer):
                dist.all_reduce(y)
            dist.all_gather_into_tensor(gat, lg)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            colls()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            colls()
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        vals[1] = e0.elapsed_time(e1) / steps
        del g
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, coll_ms = t.tolist()
    per_gpu = dec.step_bytes(ctx + warmup + steps // 2)
    # captured graphs hold references to the NCCL communicator: destroying the process group while
    # the step graph is alive blocks forever, so the graph (and the model) go first
    dec.graph = None
    del dec
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"metric": "batched decode tokens/s (Llama-3-70B arch, Q4_K, tensor parallel)",
            "value": round(batch / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": ws, "steps": steps,
            "ms_per_step": round(ms, 3), "batch": batch, "n_layer": cfg.n_layer,
            "contexts": f"{int(ctx.min()) + warmup}-{int(ctx.max()) + warmup} at the first timed step, +1 per step",
            "min_bytes_per_step_per_gpu": per_gpu,
            "achieved_gbs_per_gpu": round(per_gpu / (ms * 1e-3) / 1e9, 1),
            "collectives_ms_per_step": round(coll_ms, 3) if ws > 1 else 0.0,
            "collectives_share": round(coll_ms / ms, 4) if ws > 1 else 0.0,
            "parallelism": f"tp{ws} (2 NCCL all-reduces / layer, logits all-gather)" if ws > 1 else "tp1",
            "scaling": "strong", "data": "synthetic (random-init weights, seeded random KV history)"}


def decode_70b(args):
    """--decode-70b: only the config-5 tensor-parallel decode over the torchrun ranks."""
    import torch
    import torch.distributed as dist
    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    r = tp70b_measure(ws, rank, dev, args.steps_70b, args.layers_70b)
    if r is not None:
        print(json.dumps(r), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from densecore_b200 import ops

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    # ---- resident data: RING slots x (W_up, W_down), GPU-encoded from seeded N(0, 0.02) ----
    gen = torch.Generator(device=dev)
    ring = []
    for s in range(RING):
        pair = []
        for n, k in SHAPES:
            gen.manual_seed(1 + 1000 * s + n)
            w = torch.randn((n, k), generator=gen, device=dev) * 0.02
            pair.append(ops.QuantWeight.from_float(w, Q4_K))
            del w
        ring.append(pair)
    xs = [torch.randn((1, k), generator=gen, device=dev) for _, k in SHAPES]
    ys = [torch.empty((1, n), device=dev) for n, _ in SHAPES]
    scr = [torch.empty(ops.mul_mat_scratch_size(Q4_K, n, k, 1), dtype=torch.uint8, device=dev)
           for n, k in SHAPES]
    torch.cuda.synchronize()

    def ring_pass():          # RING steps, each = 2 launches of the M=1 kernel (quantize fused)
        for s in range(RING):
            for j in range(2):
                ops.mul_mat(ring[s][j], xs[j], out=ys[j], scratch=scr[j])

    # CUDA graphs of ring passes (launch overhead off the timed path): a full pass of RING steps,
    # and the first r steps of a pass for step counts that are not a multiple of RING
    def graph_of(nsteps):
        def body():
            for i in range(nsteps):
                for j in range(2):
                    ops.mul_mat(ring[i][j], xs[j], out=ys[j], scratch=scr[j])
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            body()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        return g
    graphs = {RING: graph_of(RING)}

    def run_steps(k):    # exactly k steps (2 kernel launches each)
        for _ in range(k // RING):
            graphs[RING].replay()
        r = k % RING
        if r:
            if r not in graphs:
                graphs[r] = graph_of(r)
            graphs[r].replay()

    steps = args.steps
    for r in {steps % RING, args.warmup % RING} - {0}:   # every graph exists before the timed region
        graphs[r] = graph_of(r)
    run_steps(RING)
    run_steps(args.warmup)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record()
        run_steps(steps)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        dist.barrier()
    # a sustained run of the same steps (>= 0.5 s), with its own clock record
    sus_steps = RING * max(1, int(0.6e3 / max(ms / steps, 1e-4) / RING))
    with ClockSampler(local) as clk_s:
        e0.record()
        run_steps(sus_steps)
        e1.record()
        torch.cuda.synchronize()
    sus_ms = e0.elapsed_time(e1)

    # the step graph holds only the two M=1 kernel launches per step: the kernel time is the step time
    gemv_ms_per_step = ms / steps

    # e2e through the host-pointer ABI (weights registered once; x / y cross PCIe every call)
    ctx = ops.HostContext(local)
    hw = [[ctx.register(ring[s][j].to_ggml().cpu().numpy(), Q4_K, SHAPES[j][1]) for j in range(2)]
          for s in range(RING)]
    hx = [x.cpu().numpy() for x in xs]
    e2e_steps = min(max(steps, RING), 2048)
    for s in range(RING):
        for j in range(2):
            ctx.mul_mat(hw[s][j], hx[j])
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        s = i % RING
        for j in range(2):
            ctx.mul_mat(hw[s][j], hx[j])
    e2e_s = time.perf_counter() - t0
    ctx.close()

    # max over ranks
    vals = torch.tensor([ms, gemv_ms_per_step, e2e_s, sus_ms], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, gemv_ms_per_step, e2e_s, sus_ms = vals.tolist()
    del graphs
    torch.cuda.synchronize()
    # config 5 (the partitioned one): tensor-parallel decode over all ranks (TP = world size)
    tp = None
    if not args.no_tp70b:
        del ring
        torch.cuda.empty_cache()
        tp = tp70b_measure(ws, rank, dev, args.steps_70b, args.layers_70b)

    if rank == 0:
        peak, peak_kind = read_peak()
        achieved = ALG_BYTES / (gemv_ms_per_step * 1e-3) / 1e9
        traffic = read_traffic()
        out = {
            "metric": METRIC, "value": round(ws * WEIGHT_BYTES * steps / (ms * 1e-3) / 1e9, 2),
            "unit": UNIT, "n_gpus": ws, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(ms / steps, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights)",
            "config": {"workload": "config 2: Q4_K x Q8_K mul_mat, W_up 14336x4096 + W_down "
                                   "4096x14336, M=1, activation quantized per call",
                       "weight_bytes_per_step": WEIGHT_BYTES,
                       "l2": f"{RING}-slot weight ring, {RING * WEIGHT_BYTES / 1e6:.0f} MB > L2",
                       "parallelism": f"replicas x{ws}", "cuda_graph": True},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": traffic,
                         "kernel": "qmm_q4k_m1_kernel<true> (Q4_K, M=1, Q8_K quantize fused)",
                         "alg_bytes_per_step": ALG_BYTES,
                         "kernel_us_per_step": round(gemv_ms_per_step * 1e3, 3)},
            "e2e": {"value": round(ws * WEIGHT_BYTES * e2e_steps / e2e_s / 1e9, 2), "unit": UNIT,
                    "h2d_bytes_per_step": sum(4 * k for _, k in SHAPES),
                    "d2h_bytes_per_step": sum(4 * n for n, _ in SHAPES),
                    "steps": e2e_steps, "api": "dcg_ctx_mul_mat (host pointers)"},
            "gpu_launches": 2 * steps,
            "clocks": clk.summary(),
            "sustained": {"steps": sus_steps, "ms_per_step": round(sus_ms / sus_steps, 6),
                          "value": round(ws * WEIGHT_BYTES * sus_steps / (sus_ms * 1e-3) / 1e9, 2),
                          "clocks": clk_s.summary()},
        }
        if tp is not None:
            out["tp_decode_70b"] = tp
        if ws == 1 and not args.no_sweep:
            out["config1_q8_0"] = [matmul_point(8, 4096, 4096, m, dev) for m in (1, 8)]
            out["config2_m_sweep"] = [matmul_point(Q4_K, n, k, m, dev) for m in (16, 64, 256)
                                      for n, k in SHAPES]
        if ws == 1 and not args.no_decode:
            out["decode"] = {"config3": decode_bench("3", 20, dev)}
            if not args.quick:
                out["decode"]["config4"] = decode_bench("4", 10, dev)
        if ws == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_reference(args.cpu_seconds)
        print(json.dumps(out), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    del np


def run_reference(args):
    """The reference arm: the CPU implementation of the same op (ggml's quantize_row_q8_K +
    vec_dot_q4_K_q8_K restated with the best SIMD the host has, all host threads, rows split across
    threads as cb_gemv_custom does); one step = both FFN matmuls of one token, exactly --steps timed
    steps after --warmup untimed ones.  Rank 0 only."""
    import numpy as np

    from oracle import oracle as O
    ws, rank, _ = _dist()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    mats = []
    for n, k in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
        mats.append((O.quantize(w, O.Q4_K), k, rng.standard_normal((1, k)).astype(np.float32)))

    def step():
        for wq, k, x in mats:
            O.mul_mat(O.Q4_K, wq, k, O.quantize(x, O.Q8_K), 1, nthreads=threads, simd=True)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    total = time.perf_counter() - t0
    value = WEIGHT_BYTES * args.steps / total / 1e9
    isa = O.simd_isa()
    cb = {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port", "isa": isa,
          "sample": f"{args.steps} timed steps (both FFN matmuls of one token, M=1, activation "
                    f"quantized per call) after {args.warmup} warm-up steps on {threads} host threads; "
                    f"ggml is absent, so this is the {isa} restatement of vec_dot_q4_K_q8_K (the best "
                    "ISA the host has, selected at run time; bit-identical to the scalar oracle)"}
    side = cpu_reference(0.0, int4=True).get("reference_int4")   # timed once, not per step
    if side is not None:
        cb["reference_int4"] = side
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(total / max(args.steps, 1) * 1e3, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
           "config": {"workload": "config 2: Q4_K x Q8_K mul_mat, W_up 14336x4096 + W_down "
                                  "4096x14336, M=1", "weight_bytes_per_step": WEIGHT_BYTES},
           "cpu_baseline": cb,
           "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def profile_case(args):
    """Small eager run for ncu: one weight (a few hundred MB at most), a few launches."""
    import torch

    from densecore_b200 import ops
    torch.cuda.set_device(0)
    qtype = {"q4k": Q4_K, "q8_0": 8, "q6k": 14}[args.profile_type]
    n, k = {"up": SHAPES[0], "down": SHAPES[1], "sq": (4096, 4096)}[args.profile_shape]
    if args.profile_nk:
        n, k = (int(v) for v in args.profile_nk.split(","))
    m = args.profile_m
    w0 = ops.QuantWeight.from_float(torch.randn((n, k), device="cuda") * 0.02, qtype)
    # a ring of copies, so a launch late in the run reads its weight from DRAM, not L2
    ws = [w0] + [ops.QuantWeight(qtype, n, k, w0.packed.clone()) for _ in range(args.profile_ring - 1)]
    x = torch.randn((m, k), device="cuda")
    y = torch.empty((m, n), device="cuda")
    for i in range(args.profile_iters):
        ops.mul_mat(ws[i % len(ws)], x, out=y)
    torch.cuda.synchronize()
    print("profile case done", qtype, n, k, m)


def copy_ceiling():
    """What one launch of a plain device copy streams at the mat-vec's sizes: torch copy_ of 17.8 MB
    (the Q8_0 4096x4096 weight) and 33 MB (one Q4_K FFN matrix), back to back in a CUDA graph over a
    ring of buffers larger than L2.  GB/s counts read + written bytes, as the measured peak does."""
    import torch
    torch.cuda.set_device(0)
    out = []
    for nbytes in (17_825_792, 33_030_144):
        ring = max(4, -(-512 * 2**20 // nbytes))
        src = [torch.ones(nbytes, dtype=torch.uint8, device="cuda") for _ in range(ring)]
        dst = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(ring)]

        def once():
            for a, b in zip(src, dst):
                b.copy_(a)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            once()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            once()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * ring)
        out.append({"bytes_copied": nbytes, "us_per_launch": round(us, 2),
                    "read_plus_write_gbs": round(2 * nbytes / us / 1e3, 1)})
        del src, dst
        torch.cuda.empty_cache()
    print(json.dumps({"copy_ceiling": out}))


def attn_case(which: str, iters: int):
    """One layer of config-3/4 paged decode attention (n_layer = 1 arena), eager, for ncu."""
    import numpy as np
    import torch

    from densecore_b200 import ops
    torch.cuda.set_device(0)
    if which == "3":
        ctx, hq, hkv = np.random.default_rng(2).integers(128, 2049, 64), 16, 8
    else:
        ctx, hq, hkv = np.random.default_rng(3).integers(2048, 4097, 32), 32, 8
    B = len(ctx)
    mbs = (int(ctx.max()) + 15) // 16
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    ka = torch.randn((B * mbs, 16, hkv, 128), generator=g, device="cuda").half()
    va = torch.randn((B * mbs, 16, hkv, 128), generator=g, device="cuda").half()
    bt = torch.randperm(B * mbs, device="cuda").view(B, mbs).int()
    q = torch.randn((B, hq, 128), device="cuda")
    cl = torch.from_numpy(ctx.astype(np.int32)).cuda()
    out = torch.empty_like(q)
    scr = torch.empty(max(1, ops.paged_attn_scratch_size(B, hq, hkv, int(ctx.max()))), dtype=torch.uint8,
                      device="cuda")
    for _ in range(iters):
        ops.paged_attn_decode(q, ka, va, 1, 0, bt, cl, hkv, int(ctx.max()), out=out, scratch=scr)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        ops.paged_attn_decode(q, ka, va, 1, 0, bt, cl, hkv, int(ctx.max()), out=out, scratch=scr)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 20
    kv = int(ctx.sum()) * hkv * 128 * 2 * 2
    print(json.dumps({"attn_config": which, "us": round(us, 2), "kv_bytes": kv,
                      "gbs": round(kv / us / 1e3, 1)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=25000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-3/4 decode tokens/s")
    ap.add_argument("--quick", action="store_true", help="decode: config 3 only")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-1 / config-2 M sweep")
    ap.add_argument("--decode-70b", action="store_true",
                    help="only config 5 (Llama-3-70B arch) tensor-parallel decode over the torchrun ranks")
    ap.add_argument("--steps-70b", type=int, default=10)
    ap.add_argument("--no-tp70b", action="store_true", help="skip the config-5 tensor-parallel decode")
    ap.add_argument("--layers-70b", type=int, default=0, help="profiling only: fewer layers")
    ap.add_argument("--profile-type", default=None, choices=["q4k", "q8_0", "q6k"],
                    help="run only a small eager GEMV case (for ncu) and exit")
    ap.add_argument("--profile-shape", default="up", choices=["up", "down", "sq"])
    ap.add_argument("--profile-m", type=int, default=1)
    ap.add_argument("--profile-nk", default=None, help="profiling: weight shape n,k instead of --profile-shape")
    ap.add_argument("--profile-ring", type=int, default=1, help="profiling: distinct copies of the weight")
    ap.add_argument("--profile-iters", type=int, default=6)
    ap.add_argument("--copy-ceiling", action="store_true",
                    help="only time plain device copies at the mat-vec sizes and exit")
    ap.add_argument("--profile-attn", default=None, choices=["3", "4"],
                    help="run only one layer's paged decode attention of config 3/4 (for ncu)")
    ap.add_argument("--profile-decode", default=None, choices=["3", "4"],
                    help="run only the config-3/4 decode measurement (for ncu) and exit")
    args = ap.parse_args()
    if args.profile_type:
        profile_case(args)
        return
    if args.copy_ceiling:
        copy_ceiling()
        return
    if args.decode_70b:
        decode_70b(args)
        return
    if args.profile_attn:
        attn_case(args.profile_attn, args.profile_iters)
        return
    if args.profile_decode:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(decode_bench(args.profile_decode, args.profile_iters, torch.device("cuda", 0))))
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
