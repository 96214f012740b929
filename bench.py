#!/usr/bin/env python
"""Benchmark of the INT4 group-wise dequantizing GEMV (m = 1).

One step = one decode GEMV (m = 1) over each of the four Llama-style FFN
weights of BASELINE.json config 2, W [out x in] in {[5632x2048], [2048x5632],
[14336x4096], [4096x14336]}, i.e. (K=in, N=out) in {(2048,5632), (5632,2048),
(4096,14336), (14336,4096)}, INT4 group size 64 quantized on the device by the
reference quantizer's bit-exact kernel.  Weights ~ N(0, 0.02^2), x ~ N(0, 1),
synthetic and seeded.

value      whole-job algorithmic HBM GB/s with the weights resident in HBM:
           bytes/step = sum over the 4 weights of K*ceil(N/2) + G*N*4 + G*N + K*4 + N*4
           (packed nibbles, fp32 scales, u8 zeros, x read, y write), x N ranks,
           divided by the max over ranks of the device-timed region.
e2e        the same metric through the public host-buffer entry point
           (MatMul.multiply_quantized on pinned numpy arrays -> kt_qmatmul_host):
           x copied host->device and y device->host inside the timed region.
L2         each step reads a different copy of the four weights, rotating over
           enough copies (> 4x the 126 MB L2) that no step hits a weight in L2.
N > 1      one process per GPU; every rank streams its own independent set of
           weights (different layers), no collective on the data path
           ("scaling": "weak").

--impl reference times the reference algorithm on the host cores (the C
restatement of MatMul.multiplyQuantized in oracle/, all host threads) on the
same config and metric; the Kotlin reference cannot run on this machine.
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
BITS, GROUP = 4, 64
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes / algorithmic bytes of one gemv_imma_kernel launch on the
# 4096 x 14336 shape, from `ncu --set full` (profiles/gemv_imma_int4_m1_4096x14336.md).
NCU_TRAFFIC_RATIO = 34011648 / 34021376
WORKLOAD = "config2-int4-ffn-gemv-m1"


def algo_bytes(k: int, n: int, m: int = 1, bits: int = BITS, g: int = GROUP) -> int:
    groups = (k + g - 1) // g
    qbytes = k * ((n + 1) // 2) if bits == 4 else k * n
    return qbytes + groups * n * 4 + (groups * n if bits == 4 else 0) + m * k * 4 + m * n * 4


STEP_BYTES = sum(algo_bytes(k, n) for k, n in SHAPES)
WEIGHT_BYTES = sum(algo_bytes(k, n) - 4 * (k + n) for k, n in SHAPES)


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

def cpu_baseline(budget_s: float = 12.0, threads: int | None = None) -> dict:
    """The oracle's restatement of MatMul.multiplyQuantized (m = 1 work-unit
    schedule) on the host cores, over whole steps of the same workload."""
    import numpy as np
    from oracle import oracle as O

    threads = threads or (os.cpu_count() or 1)
    rng = np.random.default_rng(4321)
    weights, xs = [], []
    for k, n in SHAPES:
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        weights.append(O.quantize(w, BITS, GROUP))
        xs.append(rng.standard_normal((1, k), dtype=np.float32))
    for t, x in zip(weights, xs):  # warm-up
        O.multiply_quantized(x, t, threads=threads)
    steps, t0 = 0, time.perf_counter()
    while True:
        for t, x in zip(weights, xs):
            O.multiply_quantized(x, t, threads=threads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or steps >= 200:
            break
    return {"value": round(STEP_BYTES * steps / el / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} full steps (4 INT4 GEMVs, m=1) in {el:.1f} s, oracle/kt_oracle.c "
                      f"restatement of MatMul.multiplyQuantized, {threads} threads"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(4321)
    weights, xs = [], []
    for k, n in SHAPES:
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        weights.append(O.quantize(w, BITS, GROUP))
        xs.append(rng.standard_normal((1, k), dtype=np.float32))
    for _ in range(args.warmup):
        for t, x in zip(weights, xs):
            O.multiply_quantized(x, t, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for t, x in zip(weights, xs):
            O.multiply_quantized(x, t, threads=threads)
    el = time.perf_counter() - t0
    value = STEP_BYTES * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes_k_n": SHAPES, "bits": BITS, "group_size": GROUP, "m": 1,
                   "bytes_per_step": STEP_BYTES},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
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
# a ~163M-parameter Llama-style decoder, INT8, untied embeddings
LLAMA_163M = dict(vocab=32000, dim=768, layers=12, heads=12, kv_heads=12, hidden=2048, eps=1e-5,
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


def measure_decode(kt, torch, cfg, weights, batch: int, steps: int, prompt_len: int, seed: int,
                   model: str = "qwen2-0.5b-shaped int4 g64 (random weights, tied, qkv bias)") -> dict:
    """Batched greedy decode: `batch` random prompts prefilled as blocks
    (Transformer.prefill, all sequences in one pass), then timed CUDA-graph decode
    steps of the whole batch (every matmul at m = batch)."""
    import numpy as np
    from kotensor_b200 import decoder as D
    rng = np.random.default_rng(seed + batch)
    dec = D.DeviceDecoder(cfg, weights, max_seq=2 * prompt_len + steps + 8, batch=batch)
    prompts = [rng.integers(0, cfg.vocab, size=prompt_len).tolist() for _ in range(batch)]
    dec.prefill(prompts)  # warm-up prefill (module set-up, workspaces), then a timed one
    dec.reset()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    dec.prefill(prompts)
    p1.record()
    torch.cuda.synchronize()
    prefill_ms = p0.elapsed_time(p1)
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
    ms = e0.elapsed_time(e1) / steps
    weight_bytes = sum(w.size_in_bytes for L in dec.layers for k, w in L.items() if k.startswith("w"))
    weight_bytes += dec.head.size_in_bytes
    out = {"model": model, "batch": batch,
           "prompt": prompt_len, "prefill_ms": round(prefill_ms, 3),
           "prefill_tokens_per_s": round(batch * prompt_len / (prefill_ms / 1e3), 1),
           "steps": steps, "ms_per_step": round(ms, 4),
           "tokens_per_s": round(batch * 1e3 / ms, 1), "weight_bytes_per_step": int(weight_bytes),
           "weight_gbs": round(weight_bytes / (ms / 1e3) / 1e9, 1),
           "context_end": prompt_len + steps + 3}
    del dec
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------- GPU arm

def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    import kotensor_b200 as kt

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    copies = max(2, math.ceil(4 * L2_BYTES / WEIGHT_BYTES))
    gen = torch.Generator(device="cuda")
    weights = []  # [copy][shape]
    for c in range(copies):
        row = []
        for si, (k, n) in enumerate(SHAPES):
            gen.manual_seed(1000 * rank + 10 * c + si)
            w = torch.randn((k, n), generator=gen, device="cuda", dtype=torch.float32) * 0.02
            row.append(kt.QuantizedTensor.quantize(w, kt.Quantization(BITS, GROUP)))
            del w
        weights.append(row)
    gen.manual_seed(77 + rank)
    xs = [torch.randn((args.m, k), generator=gen, device="cuda") for k, _ in SHAPES]
    ys = [torch.empty((args.m, n), device="cuda") for _, n in SHAPES]

    def launch_step(row) -> None:
        for si in range(len(SHAPES)):
            kt.MatMul.multiply_quantized(xs[si], row[si], ys[si], args.m, accumulate=False)

    # warm-up outside capture (module load, attribute set-up), then CUDA graphs:
    # one per weight copy holding that copy's 4 GEMV launches, and one holding a
    # whole cycle over the copies (copies x 4 launches, consecutive kernels
    # chained by programmatic dependent launch, as in a captured decode loop).
    # The timed loop replays whole cycles, then single steps for the rest, so
    # exactly --steps steps run and host launch overhead stays out of the timing.
    for i in range(args.warmup):
        launch_step(weights[i % copies])
    torch.cuda.synchronize()
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
    t = torch.tensor([elapsed_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    step_bytes = sum(algo_bytes(k, n, args.m) for k, n in SHAPES)
    value = world * step_bytes * args.steps / (max_ms / 1e3) / 1e9
    # roofline: every launch of the step is the same GEMV kernel; its average
    # launch duration is this rank's step time / 4 launches (events on the
    # launching stream, gaps between graph nodes included).
    launch_us = elapsed_ms * 1e3 / (args.steps * len(SHAPES))
    achieved = step_bytes / (elapsed_ms / 1e3 / args.steps) / 1e9

    # e2e through the host-buffer entry point (pinned host x / y)
    xh = [torch.randn((args.m, k)).pin_memory().numpy() for k, _ in SHAPES]
    yh = [torch.empty((args.m, n)).pin_memory().numpy() for _, n in SHAPES]
    e2e_steps = max(1, args.steps)

    def host_step(i):
        row = weights[i % copies]
        for si in range(len(SHAPES)):
            kt.MatMul.multiply_quantized(xh[si], row[si], yh[si], args.m, accumulate=False)

    for i in range(max(1, args.warmup)):
        host_step(i)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        host_step(i)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * step_bytes * e2e_steps / float(te.item()) / 1e9

    # prefill GEMM (BASELINE config 2 at M = GEMM_M): the same four weights
    # through the tcgen05 kernel, CUDA graphs over the rotating copies, device
    # timed; reported beside the GEMV line (tensor-pipe roofline).
    gemm = None
    if args.gemm_m > 0:
        gm = args.gemm_m
        gxs = [torch.randn((gm, k), generator=gen, device="cuda") for k, _ in SHAPES]
        gys = [torch.empty((gm, n), device="cuda") for _, n in SHAPES]

        def gemm_cycle():
            for c in range(copies):
                for si in range(len(SHAPES)):
                    kt.MatMul.multiply_quantized(gxs[si], weights[c][si], gys[si], gm, accumulate=False)

        gemm_cycle()
        torch.cuda.synchronize()
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg):
            gemm_cycle()
        gg.replay()
        torch.cuda.synchronize()
        reps = 3
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(reps):
            gg.replay()
        g1.record(stream)
        torch.cuda.synchronize()
        g_ms = g0.elapsed_time(g1) / (reps * copies)
        flops = sum(2.0 * gm * k * n for k, n in SHAPES)
        tpeak, tpeak_kind = measured_tensor_peak()
        tflops = flops / (g_ms / 1e3) / 1e12
        gemm = {"m": gm, "tflops": round(tflops, 1), "peak_tflops": tpeak, "peak_kind": tpeak_kind,
                "frac": round(tflops / tpeak, 4), "ms_per_step": round(g_ms, 4), "kernel": "gemm_tc_kernel",
                "dtype": "bf16 x bf16 -> f32 (INT4 weights dequantized)", "launches_per_step": len(SHAPES)}
        del gg

    # decode tokens/s (Qwen2-0.5B-shaped INT4 at batch 1, 8, 64):
    # the prompts prefilled as blocks, the batched decode step captured once,
    # then timed greedy steps replaying the graph (no host work between tokens).
    decode, decode_batches = None, []
    if args.decode_steps > 0:
        dcfg, dweights = decode_weights(kt, torch, seed=99 + rank)
        for b in [int(v) for v in args.decode_batches.split(",") if v.strip()]:
            decode_batches.append(measure_decode(kt, torch, dcfg, dweights, b, args.decode_steps, args.decode_prompt,
                                                 seed=99 + rank))
        decode = next((d for d in decode_batches if d["batch"] == 1), decode_batches[0] if decode_batches else None)
        del dweights
    # BASELINE config 5 on one GPU: Llama-3-8B-shaped INT4, 1024-token prompts, batches of --llama-batches
    # (batch 256 is left out: its fp32 KV cache at context 2048 alone is ~137 GB)
    llama = []
    if args.llama_steps > 0 and args.llama_batches.strip():
        lcfg, lweights = decode_weights(kt, torch, seed=5 + rank, spec=LLAMA3_8B)
        for b in [int(v) for v in args.llama_batches.split(",") if v.strip()]:
            llama.append(measure_decode(kt, torch, lcfg, lweights, b, args.llama_steps, 1024, seed=5 + rank,
                                        model="llama-3-8b-shaped int4 g64 (random weights, untied)"))
        del lweights
        torch.cuda.empty_cache()
    # the INT8 ~163M Llama-style decoder, 128-token prompt, 256 greedy steps, batch 1
    decode_int8 = None
    if args.int8_decode_steps > 0:
        icfg, iweights = decode_weights(kt, torch, seed=7 + rank, spec=LLAMA_163M)
        decode_int8 = measure_decode(kt, torch, icfg, iweights, 1, args.int8_decode_steps, 128, seed=7 + rank,
                                     model="llama-style 163M int8 g64 (d768, 12 layers, vocab 32000, untied, "
                                           "random weights)")
        del iweights

    peak, peak_kind = measured_peaks()
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u4", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes_k_n": SHAPES, "bits": BITS, "group_size": GROUP, "m": args.m,
                   "bytes_per_step_per_gpu": step_bytes, "parallelism": f"independent weights per rank x{world}",
                   "l2": f"rotating {copies} weight copies ({copies * WEIGHT_BYTES / 1e6:.0f} MB > 4x L2)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": round(NCU_TRAFFIC_RATIO * (step_bytes // len(SHAPES))),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       f"gemv_imma_kernel launch (4096 x 14336): {NCU_TRAFFIC_RATIO:.4f} x "
                                       "its algorithmic bytes, applied to the average launch",
                     "kernel": "gemv_imma_kernel",
                     "bytes_per_launch_avg": step_bytes // len(SHAPES), "launch_us_avg": round(launch_us, 3)},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": sum(args.m * k * 4 for k, _ in SHAPES),
                "d2h_bytes_per_step": sum(args.m * n * 4 for _, n in SHAPES)},
        "gpu_launches": len(SHAPES) * args.steps,
        "clocks": clocks,
    }
    if gemm is not None:
        line["prefill_gemm"] = gemm
    if decode is not None:
        line["decode"] = decode
        line["decode_batches"] = [{k: d[k] for k in ("batch", "ms_per_step", "tokens_per_s", "prefill_tokens_per_s",
                                                     "weight_gbs")} for d in decode_batches]
    if llama:
        line["decode_llama3_8b"] = [{k: d[k] for k in ("batch", "prompt", "prefill_ms", "prefill_tokens_per_s",
                                                        "ms_per_step", "tokens_per_s", "weight_gbs")} for d in llama]
    if decode_int8 is not None:
        line["decode_int8"] = {k: decode_int8[k] for k in ("model", "batch", "prompt", "prefill_ms", "steps",
                                                          "ms_per_step", "tokens_per_s", "weight_gbs")}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=1, help="activation rows per GEMV (decode batch)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-steps", type=int, default=128, help="timed greedy decode steps (0: skip)")
    ap.add_argument("--decode-prompt", type=int, default=512, help="prompt tokens before the timed decode")
    ap.add_argument("--decode-batches", default="1,8,64", help="decode batch sizes to time (comma-separated)")
    ap.add_argument("--llama-batches", default="1,16,64",
                    help="decode batch sizes of the Llama-3-8B-shaped INT4 model (BASELINE config 5; empty: skip)")
    ap.add_argument("--llama-steps", type=int, default=32, help="timed greedy steps of the Llama-3-8B-shaped model")
    ap.add_argument("--int8-decode-steps", type=int, default=256,
                    help="timed greedy steps of the INT8 163M decoder (BASELINE config 3; 0: skip)")
    ap.add_argument("--gemm-m", type=int, default=512,
                    help="also time the prefill GEMM at this M on the same weights (0: skip)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
