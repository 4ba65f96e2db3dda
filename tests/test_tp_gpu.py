"""Tensor-parallel decode on 2 and 4 GPUs (one process per GPU): the
persistent kernel with peer stores between the ranks ("p2p") and the
per-kernel path with NCCL collectives ("nccl").

A GPT-2-XL-shaped miniature (5 heads, uneven over the ranks) in BF16 and
INT8 + 8-bit KV: the TP group's logits, teacher-forced on the single-GPU
engine's tokens, match the single-GPU engine (cosine >= 0.999) and the CPU
oracle; every rank of the group decodes the same tokens.  Skipped on boxes
with fewer GPUs than the group.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu

MINI_XL = dict(maxT=64, V=250, L=2, NH=5, C=320, Vp=256)


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


@pytest.mark.parametrize("path", ["p2p", "nccl"])
@pytest.mark.parametrize("size", [2, 4])
@pytest.mark.parametrize("wmode,kvmode", [("bf16", "floatx"), ("int8", "8bit")])
def test_tp_group_matches_single_gpu(mini_xl, orc, gpt2b, wmode, kvmode, size, path):
    if _n_gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    import torch.multiprocessing as mp

    from cuda_gpt2_inference_b200 import tp
    from cuda_gpt2_inference_b200.engine import Engine
    cfg, imgs = mini_xl
    img, sc = imgs[wmode]
    prompt = [7, 100, 3, 249]
    n_gen = cfg["maxT"] - len(prompt)
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
