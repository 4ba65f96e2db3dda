"""Tensor-parallel decode on 2, 4 and 8 GPUs (one process per GPU): the
persistent kernel with peer stores between the ranks ("p2p") and the
per-kernel path with NCCL collectives ("nccl").

* A GPT-2-XL-shaped miniature (5 heads, uneven over 2 and 4 ranks) in BF16 and
  INT8 + 8-bit KV.
* The real GPT-2-XL width (C = 1600, 25 heads: 13/12, 7/6/6/6 and 4/3x7 over
  the ranks, FC 6400) with 2 layers, INT8 weights and BF16 KV.

In both, the TP group's logits, teacher-forced on the single-GPU engine's
tokens, match the single-GPU engine (cosine >= 0.999) and the CPU oracle, and
every rank of the group decodes the same tokens.

* A group whose rank 1 is alive, built and connected but never launches its
  decode: rank 0's persistent kernel gives up within its (short) poll limit,
  reports GPT2B_DEVERR_GRID_TIMEOUT, and both ranks' contexts stay usable.

Skipped on boxes with fewer GPUs than the group.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu

MINI_XL = dict(maxT=64, V=250, L=2, NH=5, C=320, Vp=256)
XL_WIDTH = dict(maxT=128, V=500, L=2, NH=25, C=1600, Vp=512)


def _n_gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _quantize(gpt2b, img16: bytes, fmt: str):
    lib = gpt2b.lib()
    ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
    gpt2b.check(lib.gpt2b_quantized_size(img16, len(img16), ctypes.byref(ob), ctypes.byref(ns)))
    out = ctypes.create_string_buffer(ob.value)
    sc = np.zeros(ns.value, np.float32)
    gpt2b.check(lib.gpt2b_quantize_buffer(img16, len(img16), out, sc.ctypes.data_as(ctypes.c_void_p),
                                          1 if fmt == "fp8" else 0), "quantize")
    return out.raw, sc


def _rank(rank, size, port, img, wmode, kvmode, sc, gid, seq, prompt, n_gen, p2p, q):
    import os

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    torch.cuda.synchronize()
    from cuda_gpt2_inference_b200 import OPT_PERSISTENT, tp
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=size)  # host-side handle exchange only
        eng = tp.engine(img, wmode, kvmode, sc, rank, size, gid, p2p=p2p)
        eng.set_option(OPT_PERSISTENT, 1 if p2p else 0)  # fails unless the group is connected
        _, lg = eng.generate(seq, 0, want_logits=True)  # teacher-forced over seq (gathered logits)
        toks, _ = eng.generate(prompt, n_gen)           # device-resident greedy
        eng.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, toks, lg if rank == 0 else None, None))
    except Exception as ex:  # reported to the parent
        q.put((rank, None, None, repr(ex)))


@pytest.fixture(scope="module")
def mini_xl(gpt2b, cuda):
    from cuda_gpt2_inference_b200 import weights
    cfg = MINI_XL
    img16 = weights.image(weights.synth_params(cfg, 11, init="test"), cfg, "bf16")
    return cfg, {"bf16": (img16, None), "int8": _quantize(gpt2b, img16, "int8")}


def _free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def xl_width(gpt2b, cuda):
    from cuda_gpt2_inference_b200 import weights
    cfg = XL_WIDTH
    img16 = weights.image(weights.synth_params(cfg, 13, init="test"), cfg, "bf16")
    return cfg, {"int8": _quantize(gpt2b, img16, "int8")}


@pytest.mark.parametrize("path", ["p2p", "nccl"])
@pytest.mark.parametrize("size", [2, 4])  # 5 heads: a group of 8 is refused (tests/test_tp_cpu.py)
@pytest.mark.parametrize("wmode,kvmode", [("bf16", "floatx"), ("int8", "8bit")])
def test_tp_group_matches_single_gpu(mini_xl, orc, gpt2b, wmode, kvmode, size, path):
    cfg, imgs = mini_xl
    _tp_case(cfg, imgs[wmode], orc, wmode, kvmode, size, path, [7, 100, 3, 249], cfg["maxT"] - 4)


@pytest.mark.slow
@pytest.mark.parametrize("path", ["p2p", "nccl"])
@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_xl_width_matches_single_gpu(xl_width, orc, gpt2b, size, path):
    cfg, imgs = xl_width
    _tp_case(cfg, imgs["int8"], orc, "int8", "floatx", size, path, [3, 499, 17, 250, 9], 96)


def _tp_case(cfg, img_sc, orc, wmode, kvmode, size, path, prompt, n_gen):
    if _n_gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    import torch.multiprocessing as mp

    from cuda_gpt2_inference_b200 import tp
    from cuda_gpt2_inference_b200.engine import Engine
    img, sc = img_sc
    single = Engine.from_buffer(img, wmode, kvmode, sc)
    stoks, slg = single.generate(prompt, n_gen, want_logits=True)
    single.close()
    seq = list(prompt) + list(stoks[:-1])

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gid = tp.new_group_id()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, size, port, img, wmode, kvmode, sc, gid, seq, prompt, n_gen,
                                             path == "p2p", q))
             for r in range(size)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(size)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    errors = [r[3] for r in res if r[3]]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    # every rank decoded the same tokens
    for r in res[1:]:
        assert np.array_equal(r[1], res[0][1])
    tlg = res[0][2]
    cos_single = [cosine(tlg[i], slg[i]) for i in range(len(seq))]
    assert min(cos_single) >= 0.999, min(cos_single)
    m = orc.Model(img, wmode, kvmode, sc)
    cos_oracle = [cosine(tlg[i], m.step(int(t), i)) for i, t in enumerate(seq)]
    assert min(cos_oracle) >= 0.999, min(cos_oracle)


def _timeout_rank(rank, size, port, img, gid, q):
    import os
    import time

    import torch
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects in a test that aborts a rank's wait
    torch.cuda.set_device(rank)
    torch.cuda.synchronize()
    import cuda_gpt2_inference_b200 as pkg
    from cuda_gpt2_inference_b200 import OPT_PERSISTENT, OPT_POLL_LIMIT, tp
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=size)
        eng = tp.engine(img[0], "int8", "floatx", img[1], rank, size, gid, p2p=True)
        eng.set_option(OPT_PERSISTENT, 1)
        dist.barrier()  # both engines built and connected
        err, dt, after = 0, 0.0, None
        if rank == 0:
            eng.set_option(OPT_POLL_LIMIT, 1 << 16)
            eng.set_position(7, 0)
            t0 = time.perf_counter()
            eng.decode(4)          # rank 1 never runs its part: a wait on it runs out
            eng.history(0, 1)      # synchronises the engine stream (the kernel has returned)
            dt = time.perf_counter() - t0
            err = pkg.device_error()
            # the context is still usable
            x = torch.arange(1000, device="cuda", dtype=torch.float32)
            after = float(x.sum().item())
        dist.barrier()  # rank 1: alive and idle the whole time, no kernel in flight
        eng.close()
        if rank == 1:
            after = float(torch.ones(10, device="cuda").sum().item())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err, dt, after, None))
    except Exception as ex:
        q.put((rank, None, None, None, repr(ex)))


def test_tp_persistent_wait_times_out_when_a_rank_never_launches(mini_xl, gpt2b):
    """Rank 1 keeps its process, engine and mapped exchange arena alive but
    never calls decode; rank 0 decodes with a short poll limit.  Its kernel
    must return (no hang), report GPT2B_DEVERR_GRID_TIMEOUT, and leave both
    contexts usable.  No fault is injected on the GPU: the wait runs out on a
    word that nothing writes."""
    if _n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from cuda_gpt2_inference_b200 import DEVERR_GRID_TIMEOUT, tp
    cfg, imgs = mini_xl
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gid = tp.new_group_id()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_rank, args=(r, 2, port, imgs["int8"], gid, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(2)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    errors = [r[4] for r in res if r[4]]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    assert res[0][1] == DEVERR_GRID_TIMEOUT, res[0]
    assert res[0][2] < 30.0, res[0]  # 65536 polls: well under a second in practice
    assert res[0][3] == float(sum(range(1000))) and res[1][3] == 10.0
