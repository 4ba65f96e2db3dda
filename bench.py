#!/usr/bin/env python
"""GPT-2 batch-1 greedy decode benchmark (ms/token) on B200.

Workload (default ``--config bf16``): random-init
GPT-2 124M (Linear/embedding N(0,0.02), wpe N(0,0.01), LN 1/0, biases 0;
numpy PCG64 seed 1234), BF16 weights/activations/KV, FP32 logits; a 24-token
uniform-random prompt (seed 24) is fed once, then each *step* is the 1000
greedy decode forwards at positions 24..1023 (restarting from the first
generated token).  ``--config int8|fp8|f32`` selects the other precisions
(INT8/FP8 use 8-bit KV) as the headline value.

One JSON line on rank 0.  Besides the headline value it carries
* ``precisions`` (1 GPU): INT8+KV8, FP8+KV8 and FP32 on the same workload;
* ``xl_tp`` (every N): GPT-2-XL INT8 decode, tensor parallel over all launched
  ranks (TP = N; configs[4]);
* ``gemv`` (1 GPU): the config-0 GEMVs standalone, L2 cold and warm;
* ``cpu_baseline`` (1 GPU): the reference's CPU loops on a bounded sample of
  decode positions spread over 24..1023.

``--impl reference`` times the reference's CPU decode path (its own CPU loops
compiled from source, oracle/_ref) on a bounded sample, with every host core.
``--config xl-int8`` prints the tensor-parallel GPT-2-XL line alone;
``--config fp8-long`` times configs[3] (FP8 weights + FP8 KV at positions
512..1023, attention split+merge with 8 splits against the single-CTA form).
With N > 1 GPUs (torchrun) each rank runs an independent 124M replica (the 124M
decode does not shard); the value is whole-job ms per token.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN, GEN = 24, 1000
CONFIGS = {
    "bf16": ("bf16", "floatx"),
    "int8": ("int8", "8bit"),
    "fp8": ("fp8", "8bit"),
    "f32": ("f32", "floatx"),
}
METRIC = "ms/token GPT-2 124M b=1 decode (FP32/BF16/INT8/FP8); GEMV GB/s vs HBM peak"
# GPT-2-XL INT8 weights, BF16 KV, tensor parallel over the launched ranks (TP = N)
XL_CONFIG = "xl-int8"
XL_METRIC = "ms/token GPT-2-XL INT8 b=1 decode, tensor parallel over N GPUs"
# FP8 weights + FP8 KV, positions 512..1023
LONG_CONFIG = "fp8-long"
LONG_METRIC = "ms/token GPT-2 124M FP8+FP8-KV decode at positions 512..1023; attention split+merge (S=8) vs fused_single"
LONG_FIRST = 512


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def algo_bytes_per_token(cfg, wmode, kvmode, first_pos=PROMPT_LEN, n=GEN):
    """Algorithmic HBM bytes of one decode forward, averaged over positions
    first_pos..first_pos+n-1: every weight read once (LM head over Vp rows),
    8-bit row scales, biases/LN params, one wte and one wpe row, and the KV
    rows 0..pos of every layer/head (+ 8-bit row scales)."""
    C, L, Vp, NH = cfg["C"], cfg["L"], cfg["Vp"], cfg["NH"]
    hs = C // NH
    xb = 4 if wmode == "f32" else 2
    wb = {"f32": 4, "bf16": 2, "int8": 1, "fp8": 1}[wmode]
    lin = Vp * C + L * 12 * C * C
    b = lin * wb
    if wb == 1:
        b += 4 * (Vp + L * 12 * C)  # per-row scales
    b += xb * (L * (3 * C + C + 4 * C + C) + 2 * L * C * 2 + 2 * C)  # biases + LN params
    b += xb * 2 * C  # wte row + wpe row of the embedding
    kvb = 1 if kvmode == "8bit" else xb
    mean_len = first_pos + (n - 1) / 2.0 + 1.0
    kv = L * 2 * NH * mean_len * (hs * kvb + (4 if kvmode == "8bit" else 0))
    return float(b + kv)


def spread_positions(n, first=PROMPT_LEN, last=PROMPT_LEN + GEN - 1):
    """n decode positions evenly spread over first..last; their mean is the
    workload's mean position, so a per-position cost that grows with the
    context is sampled at its average."""
    return [int(first + (last - first) * (i + 0.5) / n) for i in range(n)]


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.dev)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons, power = [], [], set(), []
        for line in open(self.path).read().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx.append(float(p[2]))
                power.append(float(p[3]))
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def quantize_image(img16, wmode):
    """The library's quantize.cu-compatible quantiser on a v5 image."""
    from cuda_gpt2_inference_b200 import check, lib
    ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
    check(lib().gpt2b_quantized_size(img16, len(img16), ctypes.byref(ob), ctypes.byref(ns)))
    out = ctypes.create_string_buffer(ob.value)
    sc = np.zeros(ns.value, np.float32)
    check(lib().gpt2b_quantize_buffer(img16, len(img16), out, sc.ctypes.data_as(ctypes.c_void_p),
                                      1 if wmode == "fp8" else 0))
    return out.raw, sc


def make_model(wmode, kvmode, seed=1234):
    """Random-init 124M image in the reference format (8-bit: quantised with the
    library's quantize.cu-compatible quantiser)."""
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.GPT2_124M
    params = weights.synth_params(cfg, seed, init="spec")
    if wmode == "f32":
        return cfg, params, weights.image(params, cfg, "f32"), None
    img16 = weights.image(params, cfg, "bf16")
    if wmode == "bf16":
        return cfg, params, img16, None
    img, sc = quantize_image(img16, wmode)
    return cfg, params, img, sc


# --------------------------------------------------------------------------------------
# standalone GEMVs
# --------------------------------------------------------------------------------------
def time_launches(fn, flush=None, reps=20, warm=5):
    """Median CUDA-event time of fn() (ms).  Before each launch the GPU is kept
    busy (an L2-sized fill for cold runs, a spin otherwise) while the host
    queues the launch, so no host launch latency lands between the events."""
    import torch
    evs = []
    for i in range(reps + warm):
        if flush is not None:
            flush.fill_(i & 0xFF)  # 512 MB > L2: the operands come from HBM
        torch.cuda._sleep(200000)  # ~0.1 ms of spinning: the host gets ahead of the GPU
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    return statistics.median(s.elapsed_time(e) for s, e in evs[warm:])


def graph_time(fn, n=20):
    """ms per launch of n back-to-back launches captured in one CUDA graph (no
    host launch latency, no other kernel in between; operands L2-warm)."""
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(n):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(200000)
    s.record()
    for _ in range(5):
        g.replay()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / (5 * n)


def gemv_table(peak):
    """Standalone decode GEMVs (config-0 shapes): GB/s of algorithmic bytes,
    L2 flushed before each launch (cold) and with the operands L2-resident
    (warm), CUDA-event median of 20 launches each."""
    import torch

    from cuda_gpt2_inference_b200 import ops
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    shapes = [(2304, 768), (768, 768), (3072, 768), (768, 3072), (50257, 768)]
    res = {}
    for dt in ("f32", "bf16", "int8"):
        for M, K in shapes:
            if dt == "int8":
                W = torch.randint(0, 255, (M, K), dtype=torch.uint8, device="cuda")
                sc = torch.rand(M, device="cuda")
                x = torch.randn(K, device="cuda").to(torch.bfloat16)
                out = torch.empty(M, device="cuda")
                fn = lambda: ops.launch_GEMV6_w8x2(out, None, W, x, sc, None, M, K, 0)  # noqa: E731
                nbytes = M * K + 2 * K + 4 * M + 4 * M
            else:
                t = torch.float32 if dt == "f32" else torch.bfloat16
                W = (torch.randn(M, K, device="cuda") * 0.02).to(t)
                x = torch.randn(K, device="cuda").to(t)
                out = torch.empty(M, device="cuda")
                fn = lambda: ops.launch_GEMV6(out, W, x, M, K)  # noqa: E731
                nbytes = (M * K + K) * W.element_size() + 4 * M
            fn()
            cold = time_launches(fn, flush)
            warm = time_launches(fn)
            graph = graph_time(fn)
            gbs = nbytes / (cold * 1e-3) / 1e9
            res[f"{dt}_{M}x{K}"] = {"us": round(cold * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3),
                                    "warm_us": round(warm * 1e3, 2),
                                    "warm_GB/s": round(nbytes / (warm * 1e-3) / 1e9, 1),
                                    "graph_us": round(graph * 1e3, 2), "bytes": nbytes}
    del flush
    return res


# --------------------------------------------------------------------------------------
# the reference's CPU decode (its own CPU loops compiled from source)
# --------------------------------------------------------------------------------------
def cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def flat_params_124m(params):
    """The 16 tensors as FP32 (the BF16-rounded values the GPU engine holds)."""
    from cuda_gpt2_inference_b200 import weights
    flat = np.concatenate([weights.bf16_to_f32(weights.bf16_bits(params[n])).ravel() for n in weights.NAMES])
    return np.ascontiguousarray(flat, np.float32)


def flat_params_cpu(cfg, fmt=None, seed=1234):
    """The 16 tensors of the benchmark model as FP32, built on the host only:
    BF16-rounded, and for ``fmt`` in {"int8", "fp8"} the five Linear groups
    quantised per row (the checker's restatement of quantize.cu) and
    dequantised (code x row scale) -- the weights the reference's CPU loops
    multiply."""
    import oracle
    from cuda_gpt2_inference_b200 import weights
    shp = weights.shapes(cfg)
    flat = np.empty(sum(int(np.prod(v)) for v in shp.values()), np.float32)
    foff = 0
    for name, a in weights.param_stream(cfg, seed, "spec"):
        a = weights.bf16_to_f32(weights.bf16_bits(a)).reshape(-1, a.shape[-1])
        n = a.size
        if fmt and name in weights.LINEAR:
            for r0 in range(0, a.shape[0], 8192):  # row blocks keep the temporaries small
                blk = a[r0:r0 + 8192]
                q, sc = oracle.quant_rows(blk, fmt)
                flat[foff + r0 * a.shape[1]: foff + r0 * a.shape[1] + blk.size] = \
                    oracle.dequant_rows(q, sc, fmt).ravel()
        else:
            flat[foff:foff + n] = a.ravel()
        foff += n
        del a
    return flat


class CpuDecoder:
    """The reference's CPU decode path over all host cores."""

    def __init__(self, flat, cfg):
        import oracle
        self.lib = oracle.ref_cpu("decode")
        # torchrun sets OMP_NUM_THREADS=1 for its ranks: the reference path gets every core
        self.threads = int(self.lib.ref_set_threads(cores()))
        self.flat = flat
        self.cfg6 = np.array([cfg["maxT"], cfg["V"], cfg["L"], cfg["NH"], cfg["C"], cfg["Vp"]], np.int32)
        self.h = self.lib.ref_decoder_create(self.cfg6.ctypes.data_as(ctypes.c_void_p),
                                             flat.ctypes.data_as(ctypes.c_void_p))

    def time_positions(self, positions):
        """ms per forward over the given positions (the timing sample; the
        attention cost of a position is the same whatever the cached rows hold)."""
        t0 = time.perf_counter()
        for p in positions:
            self.lib.ref_decoder_step(self.h, 1 + p % 97, p, None)
        return (time.perf_counter() - t0) * 1e3 / len(positions)

    def close(self):
        self.lib.ref_decoder_free(self.h)


def cpu_baseline_124m(params, cfg, budget_s=15.0):
    dec = CpuDecoder(flat_params_124m(params), cfg)  # FP32 math; only the time is used
    dec.time_positions([PROMPT_LEN])  # warm-up
    probe = dec.time_positions(spread_positions(2))
    n = int(max(4, min(64, budget_s * 1e3 / max(probe, 1e-3))))
    ms = dec.time_positions(spread_positions(n))
    dec.close()
    return {"value": round(ms, 3), "unit": "ms/token", "cores": dec.threads, "kind": "reference",
            "sample": f"{n} decode forwards of the same model by the reference CPU loops (FP32 math on the BF16 "
                      f"weights) at positions spread evenly over {PROMPT_LEN}..{PROMPT_LEN + GEN - 1} "
                      f"(mean {np.mean(spread_positions(n)):.1f})"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import oracle
    from cuda_gpt2_inference_b200 import weights
    if not oracle.ref_available("libref_cpu_decode.so"):
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU loops were not built (oracle/_ref)"}))
        return 0
    if args.config == XL_CONFIG:
        cfg = weights.GPT2_XL
        flat = flat_params_cpu(cfg, "int8")
        metric, dtype = XL_METRIC, "f32"
        wl = "gpt2-xl greedy decode (int8 weights dequantised to FP32), CPU reference loops"
        what = "FP32 math on the dequantised INT8 weights"
        par = f"reference CPU path (tp{world} on the GPU arm)"
    else:
        cfg = weights.GPT2_124M
        wmode, kvmode = CONFIGS.get(args.config, ("fp8", "8bit") if args.config == LONG_CONFIG else ("bf16", "floatx"))
        if wmode in ("int8", "fp8"):
            flat = flat_params_cpu(cfg, wmode)
            what = f"FP32 math on the dequantised {wmode.upper()} weights"
        else:
            flat = flat_params_cpu(cfg)
            what = "FP32 math on the BF16 weights"
        metric, dtype = METRIC, "f32"
        wl = "gpt2-124m greedy decode, CPU reference loops"
        par = "replicas"
    dec = CpuDecoder(flat, cfg)
    dec.time_positions([PROMPT_LEN])
    probe = dec.time_positions(spread_positions(2))
    # tokens per step sized so the whole --steps/--warmup run stays within a few minutes
    per_step = int(max(1, min(16, 8000.0 / max(probe, 1e-3) / max(1, args.steps))))
    pos = spread_positions(per_step)
    for _ in range(args.warmup):
        dec.time_positions(pos[:1])
    ms_steps = [dec.time_positions(pos) for _ in range(args.steps)]
    dec.close()
    ms = float(np.mean(ms_steps))
    sample = (f"{per_step} decode forwards per step at positions spread evenly over {PROMPT_LEN}.."
              f"{PROMPT_LEN + GEN - 1}, {what}, {per_step * args.steps} forwards timed")
    line = {
        "impl": "reference", "metric": metric, "value": round(ms, 3), "unit": "ms/token", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms * per_step, 3),
        "higher_is_better": False, "scaling": "weak" if par == "replicas" else "strong", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic",
        "config": {"workload": wl, "seq_len": cfg["maxT"], "prompt": PROMPT_LEN, "parallelism": par},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms/token", "cores": dec.threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# --------------------------------------------------------------------------------------
# the GPU engine
# --------------------------------------------------------------------------------------
def measure_engine(eng, prompt, steps, warmup, world=1, clocks=None, local_rank=0):
    """Device ms/token of `steps` decode calls of GEN tokens from position 24
    (max over ranks), then the end-to-end generate() through the C ABI with
    host buffers (wall clock, max over ranks)."""
    import torch
    import torch.distributed as dist
    first, _ = eng.generate(prompt, 0)  # prefill: 24 teacher-forced forwards
    g0 = int(first[0])
    stream = torch.cuda.ExternalStream(eng.stream)

    def step():
        eng.set_position(g0, PROMPT_LEN)
        eng.decode(GEN)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if clocks else None
    if sampler:
        sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    clk = sampler.stop() if sampler else None
    if world > 1:
        dist.barrier()
    t = torch.tensor([start.elapsed_time(end)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    decoded = eng.history(PROMPT_LEN, GEN + 1)
    e2e_tokens, _ = eng.generate(prompt, GEN)  # also warms the host API path before timing it
    deterministic = bool(np.array_equal(decoded, e2e_tokens))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        eng.generate(prompt, GEN)
    te = torch.tensor([(time.perf_counter() - t0) * 1e3], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return {"max_ms": max_ms, "ms_per_token": max_ms / (steps * GEN), "e2e_ms_per_token": float(te.item()) / (steps * GEN),
            "deterministic": deterministic, "clocks": clk}


def precision_block(wmode, kvmode, steps, warmup, peak, prompt):
    """One precision on the same workload (1 GPU, persistent kernel)."""
    from cuda_gpt2_inference_b200.engine import Engine
    cfg, _, img, sc = make_model(wmode, kvmode)
    eng = Engine.from_buffer(img, wmode, kvmode, sc)
    del img
    r = measure_engine(eng, prompt, steps, warmup)
    kps = eng.kernels_per_step()
    eng.close()
    ab = algo_bytes_per_token(cfg, wmode, kvmode)
    ach = ab / (r["ms_per_token"] * 1e-3) / 1e9
    return {"weights": wmode, "kv": "8-bit" if kvmode == "8bit" else wmode, "ms_per_token": round(r["ms_per_token"], 5),
            "e2e_ms_per_token": round(r["e2e_ms_per_token"], 5), "algorithmic_bytes_per_token": int(ab),
            "achieved_GB/s": round(ach, 1), "frac": round(ach / peak, 4), "steps": steps, "warmup": warmup,
            "deterministic": r["deterministic"],
            "kernel": "persistent cooperative kernel" if kps == 0 else f"{kps} kernels per step"}


def run_ours(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    import cuda_gpt2_inference_b200 as pkg
    from cuda_gpt2_inference_b200.engine import Engine
    wmode, kvmode = CONFIGS[args.config]
    cfg, params, img, sc = make_model(wmode, kvmode)
    eng = Engine.from_buffer(img, wmode, kvmode, sc)
    if args.path == "kernels":
        eng.set_option(pkg.OPT_PERSISTENT, 0)
    kps = eng.kernels_per_step()  # 0: persistent kernel, one launch per decode call
    prompt = np.random.default_rng(24).integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    r = measure_engine(eng, prompt, args.steps, args.warmup, world, clocks=True, local_rank=local_rank)
    max_ms = r["max_ms"]
    per_replica = r["ms_per_token"]
    value = max_ms / (args.steps * GEN * world)
    e2e_value = r["e2e_ms_per_token"] / world

    peak, peak_kind = measured_peaks()
    abytes = algo_bytes_per_token(cfg, wmode, kvmode)
    achieved = abytes / (per_replica * 1e-3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(args.config)
    except Exception:
        pass
    line = {
        "metric": METRIC, "value": round(value, 5), "unit": "ms/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": wmode if wmode != "f32" else "f32", "data": "synthetic",
        "config": {"workload": f"gpt2-124m b=1 greedy decode, {wmode} weights, {kvmode} kv, 1000 steps after a "
                               f"24-token prompt (positions 24..1023)",
                   "model": "gpt2-124m (random init)", "global_batch": world, "seq_len": cfg["maxT"],
                   "parallelism": f"replicas x{world}" if world > 1 else "single gpu",
                   "l2": "inputs larger than L2: each step streams ~1000 x %.0f MB" % (abytes / 1e6)},
        "per_replica_ms_per_token": round(per_replica, 5),
        "e2e": {"value": round(e2e_value, 5), "unit": "ms/token",
                "h2d_bytes_per_step": PROMPT_LEN * 4 + 12, "d2h_bytes_per_step": (GEN + 1) * 4,
                "includes": "24 prompt forwards + 1000 greedy forwards per call"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": ("whole decode step (%d kernels, CUDA graph + PDL)" % kps) if kps else
                               "whole decode loop (persistent cooperative kernel, 1 launch per %d steps)" % GEN,
                     "algorithmic_bytes_per_token": int(abytes), "peak_kind": peak_kind},
        "gpu_launches": kps * GEN * args.steps if kps else args.steps,
        "clocks": r["clocks"],
        "deterministic": r["deterministic"],
    }
    eng.close()
    del img
    extras = world == 1 and not args.quick
    if extras:
        # the other precisions on the same workload (a few steps each)
        line["precisions"] = {}
        for name, (wm, kv) in CONFIGS.items():
            if name == args.config:
                continue
            try:
                line["precisions"][name] = precision_block(wm, kv, min(args.steps, 5), 3, peak, prompt)
            except Exception as ex:
                line["precisions"][name] = {"error": str(ex)[:200]}
        try:
            line["gemv"] = gemv_table(peak)
        except Exception as ex:  # optional extra; never fail the bench line for it
            line["gemv"] = {"error": str(ex)[:200]}
        try:
            line["cpu_baseline"] = cpu_baseline_124m(params, cfg)
        except Exception as ex:
            line["cpu_baseline"] = {"error": str(ex)[:200]}
        try:
            line["reference_kernels_b200"] = reference_cuda_engine(*make_model(wmode, kvmode)[2:], wmode, kvmode)
        except Exception as ex:
            line["reference_kernels_b200"] = {"error": str(ex)[:200]}
    if not args.no_xl:
        # GPT-2-XL INT8 tensor parallel over every launched rank (TP = N), every N
        try:
            line["xl_tp"] = xl_tp_block(args, rank, local_rank, world, own_group=False)
        except Exception as ex:
            line["xl_tp"] = {"error": str(ex)[:300]}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def reference_cuda_engine(img, sc, wmode, kvmode):
    """The reference decode engine's own CUDA kernels built for sm_100a,
    through its stock --graph --bench loop (999 tokens from EOT, per-token host
    round trip, softmax sampling), median of 3 runs after 1 discarded."""
    import oracle
    name = {("bf16", "floatx"): "bf16", ("int8", "8bit"): "int8kv8", ("fp8", "8bit"): "fp8kv8",
            ("f32", "floatx"): "f32"}[(wmode, kvmode)]
    if not oracle.ref_available(f"libref_engine_{name}.so"):
        return {"error": "reference engine not built"}
    d = tempfile.mkdtemp()
    path = os.path.join(d, "model.bin")
    with open(path, "wb") as f:
        f.write(img)
    if sc is not None:
        with open(os.path.join(d, "model_scales.bin"), "wb") as f:
            f.write(sc.tobytes())
    lib = oracle.ref_gpu(f"engine_{name}")
    lib.ref_engine_init.argtypes = [ctypes.c_char_p, ctypes.c_int]
    lib.ref_engine_bench_graph.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p]
    if lib.ref_engine_init(path.encode(), 0 if name in ("bf16", "f32") else 1) != 0:
        return {"error": "init failed"}
    walls = np.zeros(4, np.float64)
    if lib.ref_engine_bench_graph(1000, 4, walls.ctypes.data_as(ctypes.c_void_p), d.encode()) != 0:
        return {"error": "bench failed"}
    med = float(np.median(walls[1:]))
    return {"ms_per_token": round(med / 999, 4), "runs_wall_ms": [round(x, 1) for x in walls],
            "what": "reference inference_gpt2_opt graph loop compiled for sm_100a, wall ms / 999 tokens"}


# --------------------------------------------------------------------------------------
# GPT-2-XL tensor parallel
# --------------------------------------------------------------------------------------
def xl_model(rank, world):
    """GPT-2-XL INT8 image + scales (random init, spec), generated once by rank 0
    into /dev/shm and read by every rank."""
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.GPT2_XL
    base = "/dev/shm/gpt2b_xl_int8_s1234"
    if rank == 0 and not os.path.exists(base + ".ok"):
        img16 = weights.image_stream(cfg, 1234, "spec", "bf16")
        out, sc = quantize_image(img16, "int8")
        del img16
        with open(base + ".bin", "wb") as f:
            f.write(out)
        sc.tofile(base + "_scales.bin")
        open(base + ".ok", "w").close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    with open(base + ".bin", "rb") as f:
        img = f.read()
    return cfg, img, np.fromfile(base + "_scales.bin", dtype=np.float32)


def xl_tp_block(args, rank, local_rank, world, own_group):
    """GPT-2-XL INT8 (BF16 KV), batch 1, 1000 greedy steps after a 24-token
    prompt, tensor parallel over the WORLD_SIZE ranks (one engine per GPU; the
    persistent kernel with peer stores between the ranks, or the per-kernel
    path with NCCL all-reduces for --path kernels).  Collective over the ranks;
    returns the block on every rank."""
    from cuda_gpt2_inference_b200 import tp
    from cuda_gpt2_inference_b200.engine import Engine
    cfg, img, sc = xl_model(rank, world)
    p2p = args.path == "persistent"
    if world > 1:
        eng = tp.engine(img, "int8", "floatx", sc, rank, world, tp.shared_group_id(rank), p2p=p2p)
    else:
        eng = Engine.from_buffer(img, "int8", "floatx", sc)
    del img
    kps = eng.kernels_per_step()
    steps, warmup = (args.steps, args.warmup) if own_group else (min(args.steps, 5), 3)
    prompt = np.random.default_rng(24).integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    r = measure_engine(eng, prompt, steps, warmup, world, clocks=own_group, local_rank=local_rank)
    eng.close()
    peak, peak_kind = measured_peaks()
    abytes = algo_bytes_per_token(cfg, "int8", "floatx")
    per_gpu = abytes / world / (r["ms_per_token"] * 1e-3) / 1e9  # each rank reads ~1/TP of the bytes
    exchange = ("single gpu, persistent kernel" if world == 1 and kps == 0 else
                "single gpu, per-kernel path" if world == 1 else
                "persistent kernel per rank, row-parallel partials stored into every rank's memory over NVLink"
                if kps == 0 else f"per-kernel path, NCCL all-reduce after each row-parallel GEMV ({2 * cfg['L']} "
                                 f"per token) + all-gather of the LM picks")
    return {"tp": world, "ms_per_token": round(r["ms_per_token"], 5),
            "e2e_ms_per_token": round(r["e2e_ms_per_token"], 5),
            "per_gpu_GB/s": round(per_gpu, 1), "frac": round(per_gpu / peak, 4), "peak": peak,
            "peak_kind": peak_kind, "algorithmic_bytes_per_token": int(abytes), "exchange": exchange,
            "steps": steps, "warmup": warmup, "deterministic": r["deterministic"], "clocks": r["clocks"],
            "workload": "gpt2-xl b=1 greedy decode, int8 weights, bf16 kv, 1000 steps after a 24-token prompt "
                        "(positions 24..1023)"}


def run_xl_tp(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local_rank))
    b = xl_tp_block(args, rank, local_rank, world, own_group=True)
    line = {
        "metric": XL_METRIC, "value": b["ms_per_token"], "unit": "ms/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(b["ms_per_token"] * GEN, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": b["workload"], "model": "gpt2-xl (random init)", "global_batch": 1, "seq_len": 1024,
                   "parallelism": f"tp{world}", "l2": "inputs larger than L2 (~1.7 GB per token)"},
        "e2e": {"value": b["e2e_ms_per_token"], "unit": "ms/token", "h2d_bytes_per_step": PROMPT_LEN * 4 + 12,
                "d2h_bytes_per_step": (GEN + 1) * 4},
        "roofline": {"bound": "hbm", "achieved": b["per_gpu_GB/s"], "peak": b["peak"], "unit": "GB/s",
                     "frac": b["frac"], "traffic": None, "peak_kind": b["peak_kind"], "kernel": b["exchange"],
                     "algorithmic_bytes_per_token": b["algorithmic_bytes_per_token"]},
        "gpu_launches": args.steps, "clocks": b["clocks"], "deterministic": b["deterministic"],
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))
    return 0


# --------------------------------------------------------------------------------------
# FP8 weights + FP8 KV at positions 512..1023
# --------------------------------------------------------------------------------------
def run_fp8_long(args):
    """Attention: 12 heads x 64, FP8 KV holding per-row quantised N(0,1) values,
    q N(0,1); every position 512..1023 timed with split+merge (8 splits) and
    with the single-CTA-per-head form (L2 flushed before each launch).  Whole
    model: the FP8+KV8 engine decoding positions 512..1023."""
    import torch

    import cuda_gpt2_inference_b200 as pkg
    from cuda_gpt2_inference_b200 import ops
    from cuda_gpt2_inference_b200.engine import Engine
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peaks()
    NH, hs, maxT, S = 12, 64, 1024, 8
    rng = np.random.default_rng(3)
    # the FP8 KV cache, written row by row by the library's KV append (amax/448 per row)
    cache = torch.zeros(2 * NH * maxT * hs, dtype=torch.uint8, device="cuda")
    kvsc = torch.zeros(2 * NH * maxT, device="cuda")
    qkv_all = torch.from_numpy(rng.standard_normal((maxT, 3 * NH * hs), dtype=np.float32)).to("cuda", torch.bfloat16)
    d_pos = torch.arange(maxT, dtype=torch.int32, device="cuda")
    for p in range(maxT):
        ops.kv_cache_write(cache, qkv_all[p], 1, NH, hs, maxT, d_pos[p:p + 1], kv_scale=kvsc, fmt="fp8")
    torch.cuda.synchronize()
    po = torch.empty(NH * S * hs, device="cuda")
    pl, pm = torch.empty(NH * S, device="cuda"), torch.empty(NH * S, device="cuda")
    out = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    positions = list(range(LONG_FIRST, maxT))
    res = {}
    for name in ("split8", "single"):
        total_ms = 0.0
        for p in positions:
            q, dp = qkv_all[p], d_pos[p:p + 1]
            if name == "split8":
                fn = lambda: ops.attention_forward_kv_large(out, q, cache, 1, NH, hs, maxT, dp, po, pl, pm, S,  # noqa
                                                            kv_scale=kvsc, fmt="fp8")
            else:
                fn = lambda: ops.attention_forward_kv_small(out, q, cache, 1, NH, hs, maxT, dp, kv_scale=kvsc,  # noqa
                                                            fmt="fp8")
            total_ms += time_launches(fn, flush, reps=3, warm=1)
        mean_ms = total_ms / len(positions)
        kv_bytes = float(np.mean([2 * NH * (p + 1) * (hs + 4) for p in positions]))
        gbs = kv_bytes / (mean_ms * 1e-3) / 1e9
        res[name] = {"us_per_call": round(mean_ms * 1e3, 3), "kv_bytes_mean": int(kv_bytes),
                     "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4)}
    del flush
    # whole model: FP8 weights + FP8 KV, decoding positions 512..1023
    cfg, _, img, sc = make_model("fp8", "8bit")
    eng = Engine.from_buffer(img, "fp8", "8bit", sc)
    prompt = np.random.default_rng(24).integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    first, _ = eng.generate(prompt, 0)
    eng.decode(LONG_FIRST - PROMPT_LEN)  # the cache up to position 511
    tok512 = int(eng.history(LONG_FIRST, 1)[0])
    n = maxT - LONG_FIRST
    stream = torch.cuda.ExternalStream(eng.stream)
    engines = {}
    for path in ("persistent", "kernels"):
        eng.set_option(pkg.OPT_PERSISTENT, 1 if path == "persistent" else 0)
        if path == "kernels":
            eng.set_option(pkg.OPT_SPLITS, S)

        def step():
            eng.set_position(tok512, LONG_FIRST)
            eng.decode(n)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        clocks = ClockSampler(0)
        clocks.start()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(args.steps):
            step()
        e.record(stream)
        e.synchronize()
        clk = clocks.stop()
        ms = s.elapsed_time(e) / (args.steps * n)
        ab = algo_bytes_per_token(cfg, "fp8", "8bit", first_pos=LONG_FIRST, n=n)
        engines[path] = {"ms_per_token": round(ms, 5), "achieved_GB/s": round(ab / (ms * 1e-3) / 1e9, 1),
                         "frac": round(ab / (ms * 1e-3) / 1e9 / peak, 4), "algorithmic_bytes_per_token": int(ab),
                         "clocks": clk,
                         "attention": "persistent kernel: 12 splits per head" if path == "persistent" else
                                      f"per-kernel path: {S} splits per head, merge in the projection prologue"}
    eng.close()
    line = {
        "metric": LONG_METRIC, "value": engines["persistent"]["ms_per_token"], "unit": "ms/token", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(engines["persistent"]["ms_per_token"] * n, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "fp8", "data": "synthetic",
        "config": {"workload": "gpt2-124m fp8 weights + fp8 kv, greedy decode at positions 512..1023; attention "
                               "12 heads x 64 over fp8 kv of N(0,1) values, q N(0,1)", "seq_len": maxT,
                   "l2": "attention: flushed before each launch; model: inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": engines["persistent"]["achieved_GB/s"], "peak": peak,
                     "unit": "GB/s", "frac": engines["persistent"]["frac"], "traffic": None, "peak_kind": peak_kind,
                     "kernel": "whole decode loop (persistent cooperative kernel)"},
        "engine": engines, "attention_kernels": res,
        "split8_vs_single": round(res["single"]["us_per_call"] / res["split8"]["us_per_call"], 3),
        "gpu_launches": args.steps,
    }
    print(json.dumps(line))
    return 0


def run_profile_case(args):
    """Small cases for profilers (ncu), one per --profile-case:
    decode     the 24-token prompt (tensor-core prefill), decode to position
               500, then decode(8): the persistent kernel's 2nd launch
               (-k regex:decode_persistent -s 1 -c 1) is 8 steps at 500..507;
    gemv       standalone GEMVs, per shape 2 launches after an L2 flush (cold)
               then 2 back to back (warm): bf16 50257x768, int8 50257x768,
               bf16 768x768, int8 768x768, bf16 2304x768 (20 gemv launches);
    attention  12 heads x 64 at position 1023: split+merge (8 splits) then the
               single-CTA form, BF16 KV then FP8 KV (flushed before each);
    prefill    the 24-token prompt through the tensor-core GEMMs once;
    trace      (needs the trace build: GPT2B_LIB=.../libgpt2b_trace.so) per-phase
               times of the persistent kernel from its %globaltimer stamps, at
               positions 24, 500 and 1000 (prints a JSON table)."""
    if args.profile_case == "gemv":
        return profile_gemv()
    if args.profile_case == "trace":
        return profile_trace(args)
    if args.profile_case == "attention":
        return profile_attention()
    import cuda_gpt2_inference_b200 as pkg
    from cuda_gpt2_inference_b200.engine import Engine
    if args.config == XL_CONFIG:  # one GPU
        wmode, kvmode = "int8", "floatx"
        cfg, img, sc = xl_model(0, 1)
    else:
        wmode, kvmode = CONFIGS[args.config]
        cfg, _, img, sc = make_model(wmode, kvmode)
    eng = Engine.from_buffer(img, wmode, kvmode, sc)
    if args.path == "kernels":
        eng.set_option(pkg.OPT_PERSISTENT, 0)
    prompt = np.random.default_rng(24).integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    eng.generate(prompt, 0)
    if args.profile_case == "decode":
        eng.decode(500 - PROMPT_LEN)
        eng.decode(8)
        print("profile case done:", eng.history(500, 9)[:4].tolist())
    else:
        print("profile case done:", eng.history(PROMPT_LEN, 1).tolist())
    eng.close()
    return 0


def profile_trace(args):
    """Phase times of the persistent kernel (trace build).  Thread 0 of every CTA
    stamps %globaltimer when a phase's x is ready (gather / LayerNorm done), when
    its rows are done and when its attention is done; CTA 0 stamps every stage
    (producer issue, consumer wait start / end, done).  Decodes 4 steps from each
    position and reports step 2: per-phase medians over CTAs, averaged over layers
    (us)."""
    import ctypes

    import cuda_gpt2_inference_b200 as pkg
    from cuda_gpt2_inference_b200.engine import Engine
    lib = pkg.lib()
    if not hasattr(lib, "gpt2b_persist_trace"):
        raise SystemExit("--profile-case trace needs GPT2B_LIB pointing at libgpt2b_trace.so")
    wmode, kvmode = CONFIGS[args.config]
    cfg, _, img, sc = make_model(wmode, kvmode)
    L = cfg["L"]
    eng = Engine.from_buffer(img, wmode, kvmode, sc)
    out = {}
    for pos0 in (24, 500, 1000):
        eng.set_position(7, pos0)
        eng.decode(4)
        eng.history(0, 1)
        steps, ctas, evs = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        buf = (ctypes.c_ulonglong * (4 * 160 * 640))()
        lib.gpt2b_persist_trace(buf, ctypes.byref(steps), ctypes.byref(ctas), ctypes.byref(evs))
        tr = np.frombuffer(buf, dtype=np.uint64).reshape(steps.value, ctas.value, evs.value).astype(np.int64)
        t = tr[2, :148]
        start = t[:, evs.value - 1]
        med = lambda a: float(np.median(a)) / 1000.0  # noqa: E731
        acc = {k: [] for k in ("gather_ln1", "qkv", "attn", "gather_atty", "proj", "gather_ln2", "fc", "gather_fc",
                               "fcproj")}
        for l in range(L):
            u = 4 * l
            prev = t[:, 3 * (u - 1) + 1] if l > 0 else start
            xr, rd, ad = t[:, 3 * u], t[:, 3 * u + 1], t[:, 3 * u + 2]
            attn = ad > 0
            acc["gather_ln1"].append(med(xr - prev))
            acc["qkv"].append(med(rd - xr))
            acc["attn"].append(med((ad - rd)[attn]))
            acc["gather_atty"].append(med(t[:, 3 * (u + 1)] - np.where(attn, ad, rd)))
            acc["proj"].append(med(t[:, 3 * (u + 1) + 1] - t[:, 3 * (u + 1)]))
            acc["gather_ln2"].append(med(t[:, 3 * (u + 2)] - t[:, 3 * (u + 1) + 1]))
            acc["fc"].append(med(t[:, 3 * (u + 2) + 1] - t[:, 3 * (u + 2)]))
            acc["gather_fc"].append(med(t[:, 3 * (u + 3)] - t[:, 3 * (u + 2) + 1]))
            acc["fcproj"].append(med(t[:, 3 * (u + 3) + 1] - t[:, 3 * (u + 3)]))
        row = {k: round(float(np.mean(v)), 3) for k, v in acc.items()}
        last = t[:, 3 * (4 * L - 1) + 1]
        lm0, lm1, pick = t[:, 3 * 4 * L], t[:, 3 * 4 * L + 1], t[:, 3 * 4 * L + 2]
        row.update(layer=round(med(last - start) / L, 3), lm_gather_ln=round(med(lm0 - last), 3),
                   lm_rows=round(med(lm1 - lm0), 3), lm_pick=round(med(pick - lm1), 3),
                   step=round(med(pick - start), 3))
        sbuf = (ctypes.c_ulonglong * (2048 * 8))()
        lib.gpt2b_persist_trace_stages(sbuf)
        stg = np.frombuffer(sbuf, dtype=np.uint64).reshape(2048, 8).astype(np.int64)
        ok = (stg[:, :4] > 0).all(axis=1) & (stg[:, 3] >= stg[:, 1]) & (stg[:, 1] > stg[:, 0] - 10 ** 7)
        lmr = stg[:, 4] > 0  # LM-head rounds (two stages each) carry a fifth stamp
        for name, sel in (("stage", ok & ~lmr), ("lm_round", ok & lmr)):
            v = stg[sel]
            if len(v):
                row.update({f"{name}_lead": round(med(v[:, 1] - v[:, 0]), 3),
                            f"{name}_wait": round(med(v[:, 2] - v[:, 1]), 3),
                            f"{name}_compute": round(med(v[:, 3] - v[:, 2]), 3)})
        out[pos0] = row
    eng.close()
    print(json.dumps({"config": args.config, "unit": "us", "phases": out}, indent=1))
    return 0


def profile_gemv():
    import torch

    from cuda_gpt2_inference_b200 import ops
    torch.cuda.set_device(0)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for dt, M, K in (("bf16", 50257, 768), ("int8", 50257, 768), ("bf16", 768, 768), ("int8", 768, 768),
                     ("bf16", 2304, 768)):
        out = torch.empty(M, device="cuda")
        if dt == "int8":
            W = torch.randint(0, 255, (M, K), dtype=torch.uint8, device="cuda")
            sc, x = torch.rand(M, device="cuda"), torch.randn(K, device="cuda").to(torch.bfloat16)
            fn = lambda: ops.launch_GEMV6_w8x2(out, None, W, x, sc, None, M, K, 0)  # noqa: E731
        else:
            W = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
            x = torch.randn(K, device="cuda").to(torch.bfloat16)
            fn = lambda: ops.launch_GEMV6(out, W, x, M, K)  # noqa: E731
        for _ in range(2):
            flush.fill_(1)
            fn()
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        print("gemv", dt, M, K, "done")
    return 0


def profile_attention():
    import torch

    from cuda_gpt2_inference_b200 import ops
    torch.cuda.set_device(0)
    NH, hs, maxT, S, pos = 12, 64, 1024, 8, 1023
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(5)
    d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    po = torch.empty(NH * S * hs, device="cuda")
    pl, pm = torch.empty(NH * S, device="cuda"), torch.empty(NH * S, device="cuda")
    q = torch.from_numpy(rng.standard_normal(3 * NH * hs, dtype=np.float32)).to("cuda", torch.bfloat16)
    out = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
    kvf = torch.from_numpy(rng.standard_normal(2 * NH * maxT * hs, dtype=np.float32)).to("cuda", torch.bfloat16)
    # E4M3 codes with no NaN pattern (exponent bits below 0x78), small row scales
    cache8 = torch.randint(0, 255, (2 * NH * maxT * hs,), dtype=torch.uint8, device="cuda") & 0x77
    sc8 = torch.rand(2 * NH * maxT, device="cuda") * 0.01
    for kind, cache, sc in (("bf16", kvf, None), ("fp8", cache8, sc8)):
        flush.fill_(1)
        ops.attention_forward_kv_large(out, q, cache, 1, NH, hs, maxT, d_pos, po, pl, pm, S, kv_scale=sc,
                                       fmt=None if sc is None else kind)
        flush.fill_(2)
        ops.attention_forward_kv_small(out, q, cache, 1, NH, hs, maxT, d_pos, kv_scale=sc,
                                       fmt=None if sc is None else kind)
    torch.cuda.synchronize()
    print("attention done")
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + [XL_CONFIG, LONG_CONFIG], default="bf16")
    ap.add_argument("--path", choices=["persistent", "kernels"], default="persistent",
                    help="decode step implementation (persistent falls back to kernels where unsupported)")
    ap.add_argument("--quick", action="store_true",
                    help="skip the 1-GPU extras (other precisions, GEMV table, CPU and reference bars)")
    ap.add_argument("--no-xl", action="store_true", help="skip the GPT-2-XL tensor-parallel block")
    ap.add_argument("--profile-case", nargs="?", const="decode", default=None,
                    choices=["decode", "gemv", "attention", "prefill", "trace"],
                    help="small cases for profilers (see run_profile_case); prints no bench line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    rank, local_rank, world = env_rank()
    if args.profile_case:
        return run_profile_case(args)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.config == XL_CONFIG:
        return run_xl_tp(args, rank, local_rank, world)
    if args.config == LONG_CONFIG:
        if rank != 0:
            return 0
        return run_fp8_long(args)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
