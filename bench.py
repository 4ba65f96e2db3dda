#!/usr/bin/env python
"""GPT-2 124M batch-1 greedy decode benchmark (ms/token) on B200.

Workload (default ``--config bf16``): random-init
GPT-2 124M (Linear/embedding N(0,0.02), wpe N(0,0.01), LN 1/0, biases 0;
numpy PCG64 seed 1234), BF16 weights/activations/KV, FP32 logits; a 24-token
uniform-random prompt (seed 24) is fed once, then each *step* is the 1000
greedy decode forwards at positions 24..1023 (restarting from the first
generated token).  ``--config int8|fp8|f32`` selects the other precisions
(INT8/FP8 use 8-bit KV).

One JSON line on rank 0 (see the repository's measurement notes for field
definitions).  ``--impl reference`` times the reference's CPU decode path
(its own CPU loops compiled from source, oracle/_ref) on a bounded sample.
With N > 1 GPUs (torchrun) each rank runs an independent replica (the 124M
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


def make_model(wmode, kvmode, seed=1234):
    """Random-init 124M image in the reference format (8-bit: quantised with the
    library's quantize.cu-compatible quantiser)."""
    from cuda_gpt2_inference_b200 import check, lib, weights
    cfg = weights.GPT2_124M
    params = weights.synth_params(cfg, seed, init="spec")
    if wmode == "f32":
        return cfg, params, weights.image(params, cfg, "f32"), None
    img16 = weights.image(params, cfg, "bf16")
    if wmode == "bf16":
        return cfg, params, img16, None
    ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
    check(lib().gpt2b_quantized_size(img16, len(img16), ctypes.byref(ob), ctypes.byref(ns)))
    out = ctypes.create_string_buffer(ob.value)
    sc = np.zeros(ns.value, np.float32)
    check(lib().gpt2b_quantize_buffer(img16, len(img16), out, sc.ctypes.data_as(ctypes.c_void_p),
                                      1 if wmode == "fp8" else 0))
    return cfg, params, out.raw, sc


def gemv_table(peak):
    """Standalone decode GEMVs (config-0 shapes), L2 flushed before each
    launch, CUDA-event median of 20: GB/s of algorithmic bytes."""
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
            times = []
            for i in range(25):
                flush.fill_(i & 0xFF)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                if i >= 5:
                    times.append(s.elapsed_time(e))
            ms = statistics.median(times)
            gbs = nbytes / (ms * 1e-3) / 1e9
            res[f"{dt}_{M}x{K}"] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3)}
    del flush
    return res


def cpu_reference_decode(params, cfg, tokens_per_step, steps, warmup):
    """The reference's CPU decode (its CPU loops, compiled from source)."""
    import oracle
    from cuda_gpt2_inference_b200 import weights
    lib = oracle.ref_cpu("decode")
    flat = np.concatenate([weights.bf16_to_f32(weights.bf16_bits(params[n])).ravel() for n in weights.NAMES])
    flat = np.ascontiguousarray(flat, np.float32)
    cfg6 = np.array([cfg["maxT"], cfg["V"], cfg["L"], cfg["NH"], cfg["C"], cfg["Vp"]], np.int32)
    h = lib.ref_decoder_create(cfg6.ctypes.data_as(ctypes.c_void_p), flat.ctypes.data_as(ctypes.c_void_p))
    rng = np.random.default_rng(24)
    prompt = rng.integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    tok = int(prompt[0])
    pos = 0
    for _ in range(warmup):
        tok = lib.ref_decoder_step(h, tok, pos, None)
        pos += 1
    t0 = time.perf_counter()
    n = 0
    for _ in range(steps):
        for _ in range(tokens_per_step):
            tok = lib.ref_decoder_step(h, tok, pos, None)
            pos = pos + 1 if pos + 1 < cfg["maxT"] else PROMPT_LEN
            n += 1
    dt = time.perf_counter() - t0
    lib.ref_decoder_free(h)
    return dt * 1e3 / n, n


def cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import oracle
    from cuda_gpt2_inference_b200 import weights
    if not oracle.ref_available("libref_cpu_decode.so"):
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU loops were not built (oracle/_ref)"}))
        return 0
    cfg = weights.GPT2_124M
    params = weights.synth_params(cfg, 1234, init="spec")
    # one probe token to size the sample so the whole run stays within minutes
    probe_ms, _ = cpu_reference_decode(params, cfg, 1, 1, 0)
    per_step = int(max(1, min(16, 8000.0 / max(probe_ms, 1e-3) / max(1, args.steps))))
    ms, n = cpu_reference_decode(params, cfg, per_step, args.steps, args.warmup)
    c = cores()
    sample = (f"{per_step} decode tokens per step from position 0 (prompt then greedy), "
              f"FP32 math on the BF16 weights, {n} tokens timed")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": "ms/token", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms * per_step, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "gpt2-124m greedy decode, CPU reference loops", "seq_len": cfg["maxT"],
                   "prompt": PROMPT_LEN, "parallelism": "replicas"},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms/token", "cores": c, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


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
    rng = np.random.default_rng(24)
    prompt = rng.integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    first, _ = eng.generate(prompt, 0)  # prefill: 24 teacher-forced forwards
    g0 = int(first[0])
    stream = torch.cuda.ExternalStream(eng.stream)

    def step():
        eng.set_position(g0, PROMPT_LEN)
        eng.decode(GEN)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(end)
    t = torch.tensor([total_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    per_replica = max_ms / (args.steps * GEN)
    value = max_ms / (args.steps * GEN * world)
    # determinism check: the timed device-resident decode and the host API agree
    decoded = eng.history(PROMPT_LEN, GEN + 1)
    e2e_tokens, _ = eng.generate(prompt, GEN)  # also warms the host API path before timing it
    deterministic = bool(np.array_equal(decoded, e2e_tokens))

    # end to end through the C ABI with host buffers (prompt H2D, tokens D2H)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.generate(prompt, GEN)
    e2e_ms = (time.perf_counter() - t0) * 1e3
    te = torch.tensor([e2e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = float(te.item()) / (args.steps * GEN * world)

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
        "clocks": clk,
        "deterministic": deterministic,
    }
    if rank == 0 and world == 1 and not args.quick:
        try:
            line["gemv"] = gemv_table(peak)
        except Exception as ex:  # optional extra; never fail the bench line for it
            line["gemv"] = {"error": str(ex)[:200]}
        try:
            ms, n = cpu_reference_decode(params, cfg, 2, 2, 1)
            n_tok = int(max(2, min(64, 15000.0 / max(ms, 1e-3))))
            ms, n = cpu_reference_decode(params, cfg, n_tok, 1, 0)
            line["cpu_baseline"] = {"value": round(ms, 3), "unit": "ms/token", "cores": cores(), "kind": "reference",
                                    "sample": f"{n} tokens of the same model decoded by the reference CPU loops "
                                              f"(FP32 math on the BF16 weights), from position 0"}
        except Exception as ex:
            line["cpu_baseline"] = {"error": str(ex)[:200]}
        try:
            line["reference_kernels_b200"] = reference_cuda_engine(img, sc, wmode, kvmode)
        except Exception as ex:
            line["reference_kernels_b200"] = {"error": str(ex)[:200]}
    eng.close()
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


def xl_model(rank, world):
    """GPT-2-XL INT8 image + scales (random init, spec), generated once by rank 0
    into /dev/shm and read by every rank."""
    import torch.distributed as dist

    from cuda_gpt2_inference_b200 import check, lib, weights
    cfg = weights.GPT2_XL
    base = "/dev/shm/gpt2b_xl_int8_s1234"
    if rank == 0 and not os.path.exists(base + ".ok"):
        img16 = weights.image_stream(cfg, 1234, "spec", "bf16")
        ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().gpt2b_quantized_size(img16, len(img16), ctypes.byref(ob), ctypes.byref(ns)))
        out = ctypes.create_string_buffer(ob.value)
        sc = np.zeros(ns.value, np.float32)
        check(lib().gpt2b_quantize_buffer(img16, len(img16), out, sc.ctypes.data_as(ctypes.c_void_p), 0))
        del img16
        with open(base + ".bin", "wb") as f:
            f.write(out.raw)
        sc.tofile(base + "_scales.bin")
        open(base + ".ok", "w").close()
    if world > 1:
        dist.barrier()
    with open(base + ".bin", "rb") as f:
        img = f.read()
    return cfg, img, np.fromfile(base + "_scales.bin", dtype=np.float32)


def run_xl_tp(args, rank, local_rank, world):
    """GPT-2-XL INT8 (BF16 KV), batch 1, 1000 greedy steps after a 24-token
    prompt, tensor parallel over the WORLD_SIZE ranks (one engine per GPU,
    NCCL all-reduces of the row-parallel projections)."""
    import torch
    import torch.distributed as dist

    from cuda_gpt2_inference_b200 import tp
    from cuda_gpt2_inference_b200.engine import Engine
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local_rank))
    cfg, img, sc = xl_model(rank, world)
    if world > 1:
        eng = tp.engine(img, "int8", "floatx", sc, rank, world, tp.shared_group_id(rank),
                        p2p=(args.path == "persistent"))
    else:
        eng = Engine.from_buffer(img, "int8", "floatx", sc)
    del img
    kps = eng.kernels_per_step()
    prompt = np.random.default_rng(24).integers(0, cfg["V"], PROMPT_LEN).astype(np.int32)
    first, _ = eng.generate(prompt, 0)
    g0 = int(first[0])
    stream = torch.cuda.ExternalStream(eng.stream)

    def step():
        eng.set_position(g0, PROMPT_LEN)
        eng.decode(GEN)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    end.synchronize()
    clk = clocks.stop()
    t = torch.tensor([start.elapsed_time(end)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = max_ms / (args.steps * GEN)
    decoded = eng.history(PROMPT_LEN, GEN + 1)
    e2e_tokens, _ = eng.generate(prompt, GEN)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.generate(prompt, GEN)
    te = torch.tensor([(time.perf_counter() - t0) * 1e3], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = float(te.item()) / (args.steps * GEN)
    peak, peak_kind = measured_peaks()
    abytes = algo_bytes_per_token(cfg, "int8", "floatx")
    achieved = abytes / world / (value * 1e-3) / 1e9  # per GPU: each rank reads ~1/TP of the bytes
    line = {
        "metric": XL_METRIC, "value": round(value, 5), "unit": "ms/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "gpt2-xl b=1 greedy decode, int8 weights, bf16 kv, 1000 steps after a 24-token "
                               "prompt (positions 24..1023)",
                   "model": "gpt2-xl (random init)", "global_batch": 1, "seq_len": cfg["maxT"],
                   "parallelism": f"tp{world}", "l2": "inputs larger than L2 (~1.7 GB per token)"},
        "e2e": {"value": round(e2e_value, 5), "unit": "ms/token", "h2d_bytes_per_step": PROMPT_LEN * 4 + 12,
                "d2h_bytes_per_step": (GEN + 1) * 4},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": ("whole decode step per rank (%d kernels + %d NCCL collectives)" % (
                         kps, 2 * cfg["L"] + 1 if world > 1 else 0)) if kps else
                               "persistent kernel per rank, peer stores between ranks (1 launch per %d steps)" % GEN,
                     "algorithmic_bytes_per_token": int(abytes)},
        "gpu_launches": kps * GEN * args.steps if kps else args.steps,
        "clocks": clk,
        "deterministic": bool(np.array_equal(decoded, e2e_tokens)),
    }
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))
    return 0


def run_profile_case(args):
    """Three engine launches: 24-token prefill, decode to position 500, then
    decode(8) -- the launch a profiler captures (-k <kernel> -s 2 -c 1 on the
    persistent path)."""
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
    eng.decode(500 - PROMPT_LEN)
    eng.decode(8)
    print("profile case done:", eng.history(500, 9)[:4].tolist())
    eng.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + [XL_CONFIG], default="bf16")
    ap.add_argument("--path", choices=["persistent", "kernels"], default="persistent",
                    help="decode step implementation (persistent falls back to kernels where unsupported)")
    ap.add_argument("--quick", action="store_true", help="skip the optional extras (GEMV table, CPU and reference bars)")
    ap.add_argument("--profile-case", action="store_true",
                    help="small case for profilers: prefill, decode to position 500, then one 8-step decode "
                         "(the 3rd engine launch); prints no bench line")
    args = ap.parse_args()
    rank, local_rank, world = env_rank()
    if args.profile_case:
        return run_profile_case(args)
    if args.config == XL_CONFIG and args.impl == "ours":
        return run_xl_tp(args, rank, local_rank, world)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
