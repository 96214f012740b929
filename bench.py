#!/usr/bin/env python
"""Benchmark of the group-wise INT4 dequantizing GEMV (m = 1),
with the decode and prefill figures of BASELINE configs 1-5 beside it.

Headline step: the two Llama-style FFN pairs of BASELINE.json config 2 at
m = 1, each an up projection (K, N) in {(2048, 5632), (4096, 14336)} followed by
its down projection (5632, 2048) / (14336, 4096) fed the up projection's output
-- the four weights W [out x in] in {[5632x2048], [2048x5632], [14336x4096],
[4096x14336]}, INT4 group size 64, quantized on the device by the reference
quantizer's bit-exact kernel.  Weights ~ N(0, 0.02^2), x ~ N(0, 1), synthetic
and seeded.  On N GPUs the same four weights are split over the ranks the way a
tensor-parallel FFN splits them (strong scaling: the total work is fixed):
every up projection column-parallel, its down projection row-parallel over the
same block of the hidden width, the down projection's partial sums all-reduced
inside its GEMV over peer memory (the only exchange).

value      whole-job algorithmic HBM GB/s with the weights resident in HBM:
           bytes/step = sum over the 4 weights of K*ceil(N/2) + G*N*4 + G*N + K*4 + N*4
           (packed nibbles, fp32 scales, u8 zeros, x read, y write), divided by
           the max over ranks of the device-timed region.
e2e        the same metric through the public API with host buffers: x copied
           from page-locked host memory and y back inside the timed region
           (one GPU: MatMul.multiply_quantized on numpy arrays -> kt_qmatmul_host).
L2         each step reads a different copy of the weights, rotating over enough
           copies (> 4x the 126 MB L2 per GPU) that no step hits a weight in L2.

--impl reference times the reference algorithm on the host cores (the C
restatement of MatMul.multiplyQuantized in oracle/, all host threads) on the
same workload and metric; the Kotlin reference cannot run on this machine.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "dequant-GEMV HBM GB/s (% of peak); decode tokens/s at batch 1-256"
UNIT = "GB/s"
SHAPES = [(2048, 5632), (5632, 2048), (4096, 14336), (14336, 4096)]  # (K = in, N = out)
PAIRS = [(0, 1), (2, 3)]  # (up projection, its down projection) in SHAPES
BITS, GROUP = 4, 64
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes / algorithmic bytes of one gemv_imma_kernel launch on the
# 4096 x 14336 shape, from an `ncu --set full` capture of that kernel.
NCU_TRAFFIC_RATIO = 34011648 / 34021376
WORKLOAD = "config2-int4-ffn-gemv-m1"


def algo_bytes(k: int, n: int, m: int = 1, bits: int = BITS, g: int = GROUP) -> int:
    groups = (k + g - 1) // g
    qbytes = k * ((n + 1) // 2) if bits == 4 else k * n
    return qbytes + groups * n * 4 + (groups * n if bits == 4 else 0) + m * k * 4 + m * n * 4


STEP_BYTES = sum(algo_bytes(k, n) for k, n in SHAPES)
WEIGHT_BYTES = sum(algo_bytes(k, n) - 4 * (k + n) for k, n in SHAPES)


def headline_config(m: int = 1) -> dict:
    """The workload both arms report (identical keys, so the lines compare)."""
    return {"workload": WORKLOAD, "shapes_k_n": SHAPES, "bits": BITS, "group_size": GROUP, "m": m,
            "bytes_per_step": sum(algo_bytes(k, n, m) for k, n in SHAPES)}


def measured_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def measured_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the burst figure (a kernel timed on its own)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def pct(values, q):
    v = sorted(values)
    return v[min(len(v) - 1, max(0, int(round(q * (len(v) - 1)))))]


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU baseline

def _cpu_workload(seed: int = 4321):
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    weights, xs = [], []
    for k, n in SHAPES:
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        weights.append(O.quantize(w, BITS, GROUP))
        xs.append(rng.standard_normal((1, k), dtype=np.float32))
    return weights, xs


def _cpu_step(weights, xs, threads):
    """One headline step on the host: each up projection, then its down
    projection fed the up projection's output."""
    from oracle import oracle as O
    for u, d in PAIRS:
        y = O.multiply_quantized(xs[u], weights[u], threads=threads)
        O.multiply_quantized(y, weights[d], threads=threads)


def cpu_baseline(budget_s: float = 12.0, threads: int | None = None) -> dict:
    """The oracle's restatement of MatMul.multiplyQuantized (m = 1 work-unit
    schedule) on the host cores, over whole steps of the same workload."""
    threads = threads or (os.cpu_count() or 1)
    weights, xs = _cpu_workload()
    _cpu_step(weights, xs, threads)  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        _cpu_step(weights, xs, threads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or steps >= 200:
            break
    return {"value": round(STEP_BYTES * steps / el / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{steps} full steps (4 INT4 GEMVs, m=1) in {el:.1f} s, oracle/kt_oracle.c "
                      f"restatement of MatMul.multiplyQuantized, {threads} threads"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    weights, xs = _cpu_workload()
    for _ in range(args.warmup):
        _cpu_step(weights, xs, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_step(weights, xs, threads)
    el = time.perf_counter() - t0
    value = STEP_BYTES * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u4", "data": "synthetic",
        "config": headline_config(1),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{args.steps} full steps; the Kotlin reference cannot run here, so this is "
                                   "oracle/kt_oracle.c, the C restatement of MatMul.multiplyQuantized"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- decode

QWEN2_05B = dict(vocab=151936, dim=896, layers=24, heads=14, kv_heads=2, hidden=4864, eps=1e-6,
                 rope_theta=1000000.0, bits=4, group_size=64, tied=True, qkv_bias=True)
# Llama-3-8B-shaped INT4 (untied, Llama-3 RoPE scaling)
LLAMA3_8B = dict(vocab=128256, dim=4096, layers=32, heads=32, kv_heads=8, hidden=14336, eps=1e-5,
                 rope_theta=500000.0, rope_scaling=(8.0, 1.0, 4.0, 8192), bits=4, group_size=64, tied=False,
                 qkv_bias=False)
# a ~163M-parameter Llama-style decoder, INT8, untied embeddings,
# the reference's default RMSNorm epsilon (Transformer.kt:10)
LLAMA_163M = dict(vocab=32000, dim=768, layers=12, heads=12, kv_heads=12, hidden=2048, eps=1e-6,
                  rope_theta=10000.0, bits=8, group_size=64, tied=False, qkv_bias=False)


def decode_weights(kt, torch, seed: int, spec=None):
    """A decoder with random N(0, 0.02^2) weights quantized on the device: by
    default the Qwen2-0.5B-shaped INT4 model (tied embeddings, q/k/v biases)."""
    import numpy as np
    from types import SimpleNamespace
    from kotensor_b200 import decoder as D
    cfg = D.DecoderConfig(**(spec or QWEN2_05B))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    q = kt.Quantization(cfg.bits, cfg.group_size)

    def proj(k, n):
        w = torch.randn((k, n), generator=gen, device="cuda") * 0.02
        return kt.QuantizedTensor.quantize(w, q)

    rng = np.random.default_rng(seed)
    kv = cfg.kv_heads * cfg.head_dim
    layers = []
    for _ in range(cfg.layers):
        layers.append({
            "norm1": np.ones(cfg.dim, np.float32), "norm2": np.ones(cfg.dim, np.float32),
            "wq": proj(cfg.dim, cfg.dim), "wk": proj(cfg.dim, kv), "wv": proj(cfg.dim, kv), "wo": proj(cfg.dim, cfg.dim),
            "bq": rng.standard_normal(cfg.dim).astype(np.float32) * (0.02 if cfg.qkv_bias else 0.0),
            "bk": rng.standard_normal(kv).astype(np.float32) * (0.02 if cfg.qkv_bias else 0.0),
            "bv": rng.standard_normal(kv).astype(np.float32) * (0.02 if cfg.qkv_bias else 0.0),
            "bo": np.zeros(cfg.dim, np.float32),
            "wg": proj(cfg.dim, cfg.hidden), "wu": proj(cfg.dim, cfg.hidden), "wd": proj(cfg.hidden, cfg.dim),
            "bg": np.zeros(cfg.hidden, np.float32), "bu": np.zeros(cfg.hidden, np.float32),
            "bd": np.zeros(cfg.dim, np.float32)})
    head = proj(cfg.dim, cfg.vocab)
    embedding = None if cfg.tied else proj(cfg.vocab, cfg.dim)
    weights = SimpleNamespace(embedding=embedding, layers=layers, final_norm=np.ones(cfg.dim, np.float32), head=head,
                              head_bias=np.zeros(cfg.vocab, np.float32))
    return cfg, weights


def _max_over_ranks(torch, value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def decode_fits(torch, cfg, batch: int, max_seq: int, parts: int, block_rows: int) -> tuple[bool, str]:
    """Whether the KV cache and the prefill block buffers fit the free device memory."""
    kv = 2 * batch * cfg.layers * (cfg.kv_heads // parts) * max_seq * cfg.head_dim * 4
    row = 4 * (6 * cfg.dim + 3 * cfg.hidden // parts + 2 * cfg.kv_heads * cfg.head_dim // parts) + 2 * cfg.hidden
    need = kv + block_rows * row + (2 << 30)
    free = torch.cuda.mem_get_info()[0]
    return need < free, f"needs ~{need / 1e9:.0f} GB of {free / 1e9:.0f} GB free"


def measure_decode(kt, torch, cfg, weights, batch: int, steps: int, prompt_len: int, seed: int,
                   model: str = "qwen2-0.5b-shaped int4 g64 (random weights, tied, qkv bias)", comm=None,
                   max_seq: int | None = None, world: int = 1) -> dict:
    """Batched greedy decode: `batch` random prompts prefilled as blocks
    (Transformer.prefill, all sequences in one pass), then timed CUDA-graph decode
    steps of the whole batch (every matmul at m = batch).  Times are the max
    over ranks (one decoder per rank; tensor-parallel when `comm` is given)."""
    import numpy as np
    from kotensor_b200 import decoder as D
    rng = np.random.default_rng(seed + batch)
    max_seq = max_seq or (2 * prompt_len + steps + 8)
    dec = D.DeviceDecoder(cfg, weights, max_seq=max_seq, batch=batch, comm=comm)
    dec.max_block_rows = min(D.DeviceDecoder.max_block_rows, 16384 if batch >= 128 else 65535)
    prompts = [rng.integers(0, cfg.vocab, size=prompt_len).tolist() for _ in range(batch)]
    dec.prefill(prompts)  # warm-up prefill (module set-up, workspaces), then a timed one
    dec.reset()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    dec.prefill(prompts)
    p1.record()
    torch.cuda.synchronize()
    prefill_ms = _max_over_ranks(torch, p0.elapsed_time(p1), world)
    dec.capture()
    for _ in range(3):  # warm-up replays
        dec._graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec._graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(torch, e0.elapsed_time(e1) / steps, world)
    weight_bytes = sum(w.size_in_bytes for L in dec.layers for k, w in L.items() if k.startswith("w"))
    weight_bytes += dec.head.size_in_bytes
    out = {"model": model, "batch": batch, "prompt": prompt_len, "prefill_ms": round(prefill_ms, 3),
           "prefill_tokens_per_s": round(world * batch * prompt_len / (prefill_ms / 1e3), 1) if comm is None else
           round(batch * prompt_len / (prefill_ms / 1e3), 1),
           "steps": steps, "ms_per_step": round(ms, 4), "max_seq": max_seq,
           "weight_bytes_per_step_per_gpu": int(weight_bytes),
           "weight_gbs_per_gpu": round(weight_bytes / (ms / 1e3) / 1e9, 1),
           "context_end": prompt_len + steps + 3}
    if comm is None:
        out["tokens_per_s"] = round(world * batch * 1e3 / ms, 1)  # replicas: every rank its own batch
    else:
        out["tokens_per_s"] = round(batch * 1e3 / ms, 1)  # one batch over the tensor-parallel ranks
        out["allreduce_us_per_token"] = exchange_cost_us(torch, dec, world)
    del dec
    torch.cuda.empty_cache()
    return out


def exchange_cost_us(torch, dec, world: int) -> float:
    """Device time of one step's row-parallel products with their all-reduces
    minus the same products without the exchange (each rank's shards, local
    GEMV / GEMM only), max over ranks: the cost of the 2 x layers exchanges."""
    from kotensor_b200 import MatMul
    from kotensor_b200 import parallel as P
    m = dec.batch
    dev = dec.position.device
    xo = torch.randn((m, dec.q_width), device=dev)
    xd = torch.randn((m, dec.hidden_local), device=dev)
    out = torch.empty((m, dec.cfg.dim), device=dev)

    def with_exchange():
        for L in dec.layers:
            P.matmul_row_parallel(dec.comm, xo, L["wo"], out, m)
            P.matmul_row_parallel(dec.comm, xd, L["wd"], out, m)

    def local_only():
        for L in dec.layers:
            MatMul.multiply_quantized(xo, L["wo"], out, m, accumulate=False)
            MatMul.multiply_quantized(xd, L["wd"], out, m, accumulate=False)

    times = []
    for fn in (with_exchange, local_only):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(_max_over_ranks(torch, a.elapsed_time(b) / 10 * 1e3, world))
        del g
    return round(times[0] - times[1], 2)


# ----------------------------------------------------------------- GPU arm

def _graph_time_us(torch, fn_cycle, launches: int, reps: int = 3) -> float:
    """µs per launch of a captured cycle (fn_cycle issues `launches` matmuls)."""
    fn_cycle()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn_cycle()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (reps * launches)
    del g
    return us


def extra_points(kt, torch, weights, copies) -> dict:
    """BASELINE config 2 at M = 4, 16, 128 on the headline's rotating weights,
    and config 1 (INT8 2048 x 2048, M = 1 and 64) on its own rotating copies:
    µs per launch and the roofline of each point (HBM for M <= 64, tensor pipe
    above; arithmetic intensity of config 1 at M = 64 is ~97 flop/B, HBM-bound)."""
    from kotensor_b200 import _lib
    peak, _ = measured_peaks()
    tpeak, _ = measured_tensor_peak()
    names = {_lib.KT_PATH_GEMV: "gemv_tma (fp32)", _lib.KT_PATH_GEMV_MMA: "gemv_mma / gemv_imma (tensor core)",
             _lib.KT_PATH_TENSOR_CORE: "gemm_ts / gemm_tc (tcgen05)", _lib.KT_PATH_GENERIC: "generic"}
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2024)

    def point(ws_copies, shapes, m, bits):
        xs = [torch.randn((m, k), generator=gen, device="cuda") for k, _ in shapes]
        ys = [torch.empty((m, n), device="cuda") for _, n in shapes]

        def cycle():
            for row in ws_copies:
                for si in range(len(shapes)):
                    kt.MatMul.multiply_quantized(xs[si], row[si], ys[si], m, accumulate=False)

        us = _graph_time_us(torch, cycle, len(ws_copies) * len(shapes))
        bytes_ = sum(algo_bytes(k, n, m, bits) for k, n in shapes) / len(shapes)
        flops = sum(2.0 * m * k * n for k, n in shapes) / len(shapes)
        gbs = bytes_ / (us / 1e6) / 1e9
        tf = flops / (us / 1e6) / 1e12
        r = {"m": m, "us_per_launch": round(us, 2), "gbs": round(gbs, 1), "tflops": round(tf, 1),
             "kernel": names.get(ws_copies[0][-1].matmul_path(m), "?")}
        if m <= 64:
            r.update(bound="hbm", frac=round(gbs / peak, 4))
        else:
            r.update(bound="tensor", frac=round(tf / tpeak, 4))
        return r

    def tpoint(ws_copies, shapes, m):
        # MatMul.multiplyByQuantizedTransposed (the QLoRA / fused-loss backward):
        # dx[m x K] = dy[m x N] . deq(W)^T, the same bytes and flops as the product
        dys = [torch.randn((m, n), generator=gen, device="cuda") for _, n in shapes]
        dxs = [torch.empty((m, k), device="cuda") for k, _ in shapes]

        def cycle():
            for row in ws_copies:
                for si in range(len(shapes)):
                    kt.MatMul.multiply_by_quantized_transposed(dys[si], row[si], dxs[si], m, accumulate=False)

        us = _graph_time_us(torch, cycle, len(ws_copies) * len(shapes))
        bytes_ = sum(algo_bytes(k, n, m, 4) for k, n in shapes) / len(shapes)
        flops = sum(2.0 * m * k * n for k, n in shapes) / len(shapes)
        gbs, tf = bytes_ / (us / 1e6) / 1e9, flops / (us / 1e6) / 1e12
        r = {"m": m, "us_per_launch": round(us, 2), "gbs": round(gbs, 1), "tflops": round(tf, 1),
             "kernel": "gemm_t (tcgen05)" if ws_copies[0][-1].transposed_path(m) == _lib.KT_PATH_TENSOR_CORE
             else "matmul_t (fp32)"}
        if m <= 64:
            r.update(bound="hbm", frac=round(gbs / peak, 4))
        else:
            r.update(bound="tensor", frac=round(tf / tpeak, 4))
        return r

    out = {"config2_int4": [point(weights, SHAPES, m, 4) for m in (4, 16, 128)],
           "config2_int4_transposed": [tpoint(weights, SHAPES, m) for m in (16, 128)]}
    one = algo_bytes(2048, 2048, 1, 8) - 4 * 4096
    n8 = max(2, math.ceil(4 * L2_BYTES / one))
    c1 = []
    for c in range(n8):
        gen.manual_seed(5000 + c)
        w = torch.randn((2048, 2048), generator=gen, device="cuda") * 0.02
        c1.append([kt.QuantizedTensor.quantize(w, kt.Quantization(8, GROUP))])
        del w
    out["config1_int8"] = [point(c1, [(2048, 2048)], m, 8) for m in (1, 64)]
    del c1
    return out


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import kotensor_b200 as kt
    from kotensor_b200 import parallel as P

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        comm = P.Comm.from_process_group(ctx=kt.Context.get(local))

    def barrier():
        if world > 1:
            dist.barrier()

    m = args.m
    # ---- the headline weights: every rank quantizes the same full weights (same
    # seeds) and keeps its shards: up projections by columns, down projections by
    # the same block of rows (whole groups); one GPU keeps them whole
    blocks = [P.shard_bounds(P.ROWS, SHAPES[d][0], GROUP, world, rank) if world > 1 else (0, SHAPES[d][0])
              for _, d in PAIRS]
    per_gpu_bytes = sum(algo_bytes(k, n) - 4 * (k + n) for k, n in SHAPES) / world
    copies = max(2, math.ceil(4 * L2_BYTES / per_gpu_bytes))
    gen = torch.Generator(device="cuda")
    weights = []  # [copy][shape]: this rank's shard of each weight
    for c in range(copies):
        row = [None] * len(SHAPES)
        for (u, d), (b, e) in zip(PAIRS, blocks):
            for si in (u, d):
                k, n = SHAPES[si]
                gen.manual_seed(10 * c + si)
                w = torch.randn((k, n), generator=gen, device="cuda", dtype=torch.float32) * 0.02
                q = kt.QuantizedTensor.quantize(w, kt.Quantization(BITS, GROUP))
                del w
                if world > 1:
                    q = P.slice_weight(q, P.COLUMNS if si == u else P.ROWS, b, e)
                row[si] = q
        weights.append(row)
    gen.manual_seed(77)
    xs = {u: torch.randn((m, SHAPES[u][0]), generator=gen, device="cuda") for u, _ in PAIRS}
    ys = {u: torch.empty((m, e - b), device="cuda") for (u, _), (b, e) in zip(PAIRS, blocks)}
    ys.update({d: torch.empty((m, SHAPES[d][1]), device="cuda") for _, d in PAIRS})

    def launch_step(row) -> None:
        for u, d in PAIRS:
            kt.MatMul.multiply_quantized(xs[u], row[u], ys[u], m, accumulate=False)
            if comm is None:
                kt.MatMul.multiply_quantized(ys[u], row[d], ys[d], m, accumulate=False)
            else:
                P.matmul_row_parallel(comm, ys[u], row[d], ys[d], m)

    # warm-up outside capture over every copy (module load, attribute set-up,
    # and on N GPUs each down shard's exchange agreement, a collective), then
    # CUDA graphs: one per weight copy holding that copy's step, and one holding
    # a whole cycle over the copies (consecutive kernels chained by programmatic
    # dependent launch, as in a captured decode loop).  The timed loop replays
    # whole cycles, then single steps for the rest, so exactly --steps steps run
    # and host launch overhead stays out of the timing.
    for c in range(copies):
        launch_step(weights[c])
    for i in range(args.warmup):
        launch_step(weights[i % copies])
    torch.cuda.synchronize()
    fused = comm is None or comm.exchange_ready()
    graphs = []
    for c in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch_step(weights[c])
        graphs.append(g)
    cycle = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cycle):
        for c in range(copies):
            launch_step(weights[c])
    for i in range(args.warmup):
        graphs[i % copies].replay()
    cycle.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps // copies):
        cycle.replay()
    for i in range(args.steps % copies):
        graphs[i].replay()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    max_ms = _max_over_ranks(torch, elapsed_ms, world)
    step_bytes = sum(algo_bytes(k, n, m) for k, n in SHAPES)
    value = step_bytes * args.steps / (max_ms / 1e3) / 1e9
    # roofline of the dominant kernel (every launch of the step is the INT4
    # GEMV; on N GPUs the down projections' GEMVs carry the fused exchange):
    # this rank's algorithmic bytes per average launch / its average launch time
    launch_us = elapsed_ms * 1e3 / (args.steps * len(SHAPES))
    rank_bytes = sum(algo_bytes(k, n, m) for k, n in SHAPES) if world == 1 else \
        sum(algo_bytes(SHAPES[u][0], e - b, m) + algo_bytes(e - b, SHAPES[d][1], m)
            for (u, d), (b, e) in zip(PAIRS, blocks))
    achieved = rank_bytes / (elapsed_ms / 1e3 / args.steps) / 1e9

    # spread: per-step device times of single-copy replays (>= 200 launches)
    samples = []
    n_samples = max(64, math.ceil(200 / len(SHAPES)))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_samples)]
    barrier()
    for i, (a, b) in enumerate(evs):
        a.record(stream)
        graphs[i % copies].replay()
        b.record(stream)
    torch.cuda.synchronize()
    samples = [a.elapsed_time(b) for a, b in evs]
    stats = {"median_ms": round(statistics.median(samples), 5), "p10_ms": round(pct(samples, 0.1), 5),
             "p90_ms": round(pct(samples, 0.9), 5), "samples": len(samples), "launches": len(samples) * len(SHAPES),
             "note": "per-step device time of single-copy graph replays on this rank (rank 0 on N GPUs)"}

    # e2e through the public API with host buffers
    e2e_steps = max(1, args.steps)
    if comm is None:
        xh = {u: torch.randn((m, SHAPES[u][0])).pin_memory().numpy() for u, _ in PAIRS}
        yh = {si: torch.empty((m, SHAPES[si][1])).pin_memory().numpy() for si in range(len(SHAPES))}

        def host_step(i):
            row = weights[i % copies]
            for u, d in PAIRS:
                kt.MatMul.multiply_quantized(xh[u], row[u], yh[u], m, accumulate=False)
                kt.MatMul.multiply_quantized(yh[u], row[d], yh[d], m, accumulate=False)

        h2d = sum(m * k * 4 for k, _ in SHAPES)
        d2h = sum(m * n * 4 for _, n in SHAPES)
    else:
        xh = {u: torch.randn((m, SHAPES[u][0])).pin_memory() for u, _ in PAIRS}
        yh = {d: torch.empty((m, SHAPES[d][1])).pin_memory() for _, d in PAIRS}

        def host_step(i):
            for u, _ in PAIRS:
                xs[u].copy_(xh[u], non_blocking=True)
            launch_step(weights[i % copies])
            for _, d in PAIRS:
                yh[d].copy_(ys[d], non_blocking=True)
            torch.cuda.current_stream().synchronize()

        h2d = sum(m * SHAPES[u][0] * 4 for u, _ in PAIRS)
        d2h = sum(m * SHAPES[d][1] * 4 for _, d in PAIRS)
    for i in range(max(1, args.warmup)):
        host_step(i)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        host_step(i)
    e2e_s = _max_over_ranks(torch, time.perf_counter() - t0, world)
    e2e_value = step_bytes * e2e_steps / e2e_s / 1e9
    del cycle, graphs

    # prefill GEMM (BASELINE config 2 at M = GEMM_M): the same four weights
    # through the tcgen05 kernel (one GPU), device timed, tensor-pipe roofline
    gemm, extras = None, {}
    if world == 1 and args.gemm_m > 0:
        gm = args.gemm_m
        gxs = [torch.randn((gm, k), generator=gen, device="cuda") for k, _ in SHAPES]
        gys = [torch.empty((gm, n), device="cuda") for _, n in SHAPES]

        def gemm_cycle():
            for c in range(copies):
                for si in range(len(SHAPES)):
                    kt.MatMul.multiply_quantized(gxs[si], weights[c][si], gys[si], gm, accumulate=False)

        g_us = _graph_time_us(torch, gemm_cycle, copies * len(SHAPES))
        g_ms = g_us * len(SHAPES) / 1e3
        flops = sum(2.0 * gm * k * n for k, n in SHAPES)
        tpeak, tpeak_kind = measured_tensor_peak()
        tflops = flops / (g_ms / 1e3) / 1e12
        gemm = {"m": gm, "tflops": round(tflops, 1), "peak_tflops": tpeak, "peak_kind": tpeak_kind,
                "frac": round(tflops / tpeak, 4), "ms_per_step": round(g_ms, 4), "kernel": "gemm_tc_kernel",
                "dtype": "bf16 x bf16 -> f32 (INT4 weights dequantized)", "launches_per_step": len(SHAPES)}
        del gxs, gys
    if world == 1 and not args.no_extras:
        extras = extra_points(kt, torch, weights, copies)
    del weights
    torch.cuda.empty_cache()

    # decode tokens/s (Qwen2-0.5B-shaped INT4 at batch 1, 8, 64):
    # every rank decodes its own batch (replicas), whole-job tokens/s over the ranks
    decode_batches = []
    if args.decode_steps > 0:
        dcfg, dweights = decode_weights(kt, torch, seed=99 + rank)
        for b in [int(v) for v in args.decode_batches.split(",") if v.strip()]:
            decode_batches.append(measure_decode(kt, torch, dcfg, dweights, b, args.decode_steps, args.decode_prompt,
                                                 seed=99 + rank, world=world))
        del dweights
        torch.cuda.empty_cache()
    # Llama-3-8B-shaped INT4, 1024-token prompts, KV cache of
    # 2048 positions, tensor-parallel over the N GPUs (the same weights on every rank)
    llama = []
    if args.llama_steps > 0 and args.llama_batches.strip():
        lcfg, lweights = decode_weights(kt, torch, seed=5, spec=LLAMA3_8B)
        for b in [int(v) for v in args.llama_batches.split(",") if v.strip()]:
            ok, why = decode_fits(torch, lcfg, b, 2048, world, 16384 if b >= 128 else 65535)
            ok = _max_over_ranks(torch, 0.0 if ok else 1.0, world) == 0.0
            if not ok:
                llama.append({"batch": b, "skipped": why})
                continue
            r = measure_decode(kt, torch, lcfg, lweights, b, args.llama_steps, 1024, seed=5,
                               model="llama-3-8b-shaped int4 g64 (random weights, untied)", comm=comm,
                               max_seq=2048, world=world)
            llama.append(r)
        del lweights
        torch.cuda.empty_cache()
    # the INT8 ~163M Llama-style decoder, 128-token prompt, 256 greedy steps, batch 1
    decode_int8 = None
    if world == 1 and args.int8_decode_steps > 0:
        icfg, iweights = decode_weights(kt, torch, seed=7, spec=LLAMA_163M)
        decode_int8 = measure_decode(kt, torch, icfg, iweights, 1, args.int8_decode_steps, 128, seed=7,
                                     model="llama-style 163M int8 g64 (d768, 12 layers, vocab 32000, untied, "
                                           "random weights)")
        del iweights

    peak, peak_kind = measured_peaks()
    layout = "one GPU" if world == 1 else (f"tp{world}: up projections column-parallel, down projections "
                                           "row-parallel with the all-reduce " +
                                           ("fused into the GEMV over peer memory" if fused else "through NCCL"))
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u4", "data": "synthetic",
        "config": headline_config(m),
        "layout": layout,
        "l2": f"rotating {copies} weight copies ({copies * per_gpu_bytes / 1e6:.0f} MB per GPU > 4x L2)",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": round(NCU_TRAFFIC_RATIO * (rank_bytes // len(SHAPES))),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       f"gemv_imma_kernel launch (4096 x 14336): {NCU_TRAFFIC_RATIO:.4f} x "
                                       "its algorithmic bytes, applied to the average launch",
                     "kernel": "gemv_imma_kernel",
                     "bytes_per_launch_avg": rank_bytes // len(SHAPES), "launch_us_avg": round(launch_us, 3),
                     "per": "GPU (this rank's shards)"},
        "step_stats": stats,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (len(SHAPES) + (0 if fused else len(PAIRS))),
        "clocks": clocks,
    }
    if gemm is not None:
        line["prefill_gemm"] = gemm
    line.update(extras)
    if decode_batches:
        line["decode_qwen2_05b"] = [{k: d[k] for k in ("batch", "ms_per_step", "tokens_per_s", "prefill_tokens_per_s",
                                                       "weight_gbs_per_gpu")} for d in decode_batches]
        line["decode_qwen2_05b_layout"] = f"replicas: each of the {world} GPU(s) decodes its own batch"
    if llama:
        keys = ("batch", "prompt", "max_seq", "prefill_ms", "prefill_tokens_per_s", "ms_per_step", "tokens_per_s",
                "weight_gbs_per_gpu", "allreduce_us_per_token", "skipped")
        line["decode_llama3_8b"] = [{k: d[k] for k in keys if k in d} for d in llama]
        line["decode_llama3_8b_layout"] = "one GPU" if world == 1 else f"tensor-parallel over {world} GPUs"
    if decode_int8 is not None:
        line["decode_int8"] = {k: decode_int8[k] for k in ("model", "batch", "prompt", "prefill_ms", "steps",
                                                          "ms_per_step", "tokens_per_s", "weight_gbs_per_gpu")}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()


def profile_decode(which: str, batch: int = 1) -> None:
    """One captured decode step of a bench model (qwen: config 4, llama: config 5,
    int8: config 3; `batch` sequences) replayed once between cudaProfilerStart /
    Stop, for an `ncu --profile-from-start off` launch list of the step's kernels."""
    import numpy as np
    import torch
    import kotensor_b200 as kt
    from kotensor_b200 import decoder as D
    spec = {"qwen": QWEN2_05B, "llama": LLAMA3_8B, "int8": LLAMA_163M}[which]
    prompt = {"qwen": 512, "llama": 1024, "int8": 128}[which]
    torch.cuda.set_device(0)
    cfg, w = decode_weights(kt, torch, seed=1, spec=spec)
    dec = D.DeviceDecoder(cfg, w, max_seq=prompt + 64, batch=batch)
    rng = np.random.default_rng(0)
    dec.prefill([rng.integers(0, cfg.vocab, prompt).tolist() for _ in range(batch)])
    dec.capture()
    for _ in range(3):
        dec._graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(20):
        dec._graph.replay()
    b.record()
    torch.cuda.synchronize()
    print(json.dumps({"profile_decode": which, "batch": batch, "ms_per_step": round(a.elapsed_time(b) / 20, 4)}),
          flush=True)
    torch.cuda.profiler.start()
    dec._graph.replay()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=1, help="activation rows per GEMV (decode batch)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1 / config 2 M points")
    ap.add_argument("--decode-steps", type=int, default=128, help="timed greedy decode steps (0: skip)")
    ap.add_argument("--decode-prompt", type=int, default=512, help="prompt tokens before the timed decode")
    ap.add_argument("--decode-batches", default="1,8,64", help="decode batch sizes to time (comma-separated)")
    ap.add_argument("--llama-batches", default="1,16,64,256",
                    help="decode batch sizes of the Llama-3-8B-shaped INT4 model (BASELINE config 5; empty: skip)")
    ap.add_argument("--llama-steps", type=int, default=32, help="timed greedy steps of the Llama-3-8B-shaped model")
    ap.add_argument("--int8-decode-steps", type=int, default=256,
                    help="timed greedy steps of the INT8 163M decoder (BASELINE config 3; 0: skip)")
    ap.add_argument("--gemm-m", type=int, default=512,
                    help="also time the prefill GEMM at this M on the same weights (0: skip)")
    ap.add_argument("--profile-batch", type=int, default=1, help="batch of the --profile-decode step")
    ap.add_argument("--profile-decode", choices=["qwen", "llama", "int8"], default=None,
                    help="instead of the bench: one decode step replayed between cudaProfilerStart / Stop")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_decode:
        profile_decode(args.profile_decode, args.profile_batch)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
