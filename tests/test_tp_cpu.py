"""Tensor-parallel host logic on CPU: the shard plan, the weight slicing the
library performs for each rank (against numpy slicing of the same tensors),
the row/column-parallel decomposition (against the oracle's GEMV), and a
world-size-2 gloo group agreeing on the NCCL id and tiling the model."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from cuda_gpt2_inference_b200 import weights

# a GPT-2-XL-shaped miniature: 5 heads (uneven over 2 and 4 ranks), K-slices aligned
MINI_XL = dict(maxT=64, V=250, L=2, NH=5, C=320, Vp=256)


def test_plan_xl(gpt2b):
    from cuda_gpt2_inference_b200 import tp
    heads = {n: [tp.plan(weights.GPT2_XL, r, n)["heads"] for r in range(n)] for n in (1, 2, 4, 8)}
    assert heads == {1: [25], 2: [13, 12], 4: [7, 6, 6, 6], 8: [4, 3, 3, 3, 3, 3, 3, 3]}
    for n in (2, 4, 8):
        plans = [tp.plan(weights.GPT2_XL, r, n) for r in range(n)]
        assert [p["f_rows"] for p in plans] == [6400 // n] * n
        assert [p["v_rows"] for p in plans] == [50304 // n] * n
        # contiguous, disjoint, covering
        for key, cnt, total in (("h0", "heads", 25), ("f0", "f_rows", 6400), ("v0", "v_rows", 50304)):
            starts = [p[key] for p in plans]
            assert starts[0] == 0 and all(starts[i] + plans[i][cnt] == starts[i + 1] for i in range(n - 1))
            assert starts[-1] + plans[-1][cnt] == total


def test_plan_rejects_bad_groups(gpt2b):
    from cuda_gpt2_inference_b200 import tp
    for rank, size in ((0, 3), (2, 2), (-1, 2), (0, 0), (0, 32)):
        with pytest.raises(gpt2b.Gpt2bError):
            tp.plan(weights.GPT2_XL, rank, size)


def test_plan_rejects_more_ranks_than_heads(gpt2b):
    """Every rank owns at least one head: 5 heads over 8 ranks is refused (the engine
    returns GPT2B_ERR_UNSUPPORTED), 5 over 4 is planned 2/1/1/1."""
    from cuda_gpt2_inference_b200 import tp
    mini = dict(maxT=64, V=250, L=2, NH=5, C=320, Vp=256)
    with pytest.raises(gpt2b.Gpt2bError):
        tp.plan(mini, 0, 8)
    assert [tp.plan(mini, r, 4)["heads"] for r in range(4)] == [2, 1, 1, 1]


def _tensors(image: bytes, cfg: dict, w8: bool) -> dict:
    """The 16 tensors of an image as arrays (uint8 codes for 8-bit Linear groups,
    uint16 bf16 bits otherwise)."""
    out, off = {}, 1024
    for name, shp in weights.shapes(cfg).items():
        n = int(np.prod(shp))
        if w8 and name in weights.LINEAR:
            out[name] = np.frombuffer(image, np.uint8, n, off).reshape(shp)
            off += n
        else:
            out[name] = np.frombuffer(image, np.uint16, n, off).reshape(shp)
            off += 2 * n
    return out


def _expected_shard(t: dict, cfg: dict, p: dict, rank: int) -> dict:
    C, L = cfg["C"], cfg["L"]
    h0, hl, f0, fl = p["h0"] * 64, p["heads"] * 64, p["f0"], p["f_rows"]
    qrows = np.concatenate([np.arange(part * C + h0, part * C + h0 + hl) for part in range(3)])
    e = dict(t)
    e["qkvw"] = t["qkvw"][:, qrows, :]
    e["qkvb"] = t["qkvb"][:, qrows]
    e["attprojw"] = t["attprojw"][:, :, h0:h0 + hl]
    e["fcw"] = t["fcw"][:, f0:f0 + fl, :]
    e["fcb"] = t["fcb"][:, f0:f0 + fl]
    e["fcprojw"] = t["fcprojw"][:, :, f0:f0 + fl]
    if rank != 0:
        e["attprojb"] = np.zeros_like(t["attprojb"])
        e["fcprojb"] = np.zeros_like(t["fcprojb"])
    return e


def _w8_image(cfg: dict, seed: int):
    """An 8-bit mixed image with random codes and positive scales (host only)."""
    rng = np.random.default_rng(seed)
    img16 = weights.image(weights.synth_params(cfg, seed, init="test"), cfg, "bf16")
    shp = weights.shapes(cfg)
    codes = {n: rng.integers(0, 256, shp[n], dtype=np.uint8) for n in weights.LINEAR}
    nsc = cfg["Vp"] + cfg["L"] * (3 * cfg["C"] + cfg["C"] + 4 * cfg["C"] + cfg["C"])
    scales = rng.uniform(1e-4, 1e-3, nsc).astype(np.float32)
    return weights.image_w8(img16, codes, cfg), scales


@pytest.mark.parametrize("size", [2, 4])
@pytest.mark.parametrize("wmode", ["bf16", "int8"])
def test_shard_matches_numpy(gpt2b, wmode, size):
    from cuda_gpt2_inference_b200 import tp
    cfg = MINI_XL
    w8 = wmode == "int8"
    if w8:
        img, scales = _w8_image(cfg, 3)
    else:
        img, scales = weights.image(weights.synth_params(cfg, 3, init="test"), cfg, "bf16"), None
    full = _tensors(img, cfg, w8)
    C, L, Vp = cfg["C"], cfg["L"], cfg["Vp"]
    for rank in range(size):
        p = tp.plan(cfg, rank, size)
        got_b, got_sc = tp.shard_image(img, scales, wmode, rank, size)
        exp = _expected_shard(full, cfg, p, rank)
        want = b"".join(np.ascontiguousarray(exp[n]).tobytes() for n in weights.NAMES)
        assert got_b == want, rank
        if w8:
            h0, hl, f0, fl = p["h0"] * 64, p["heads"] * 64, p["f0"], p["f_rows"]
            s_wte, rest = scales[:Vp], scales[Vp:]
            s_qkv = rest[: L * 3 * C].reshape(L, 3, C)
            s_prj = rest[L * 3 * C: L * 4 * C]
            s_fc = rest[L * 4 * C: L * 8 * C].reshape(L, 4 * C)
            s_fcp = rest[L * 8 * C:]
            want_sc = np.concatenate([s_wte, s_qkv[:, :, h0:h0 + hl].ravel(), s_prj, s_fc[:, f0:f0 + fl].ravel(),
                                      s_fcp])
            assert np.array_equal(got_sc, want_sc), rank
        else:
            assert got_sc is None


def test_parallel_split_reproduces_full_products(gpt2b, orc):
    """Column-parallel QKV/FC concatenate and row-parallel projections sum to
    the full products (oracle GEMV on the library's FP32 shards)."""
    from cuda_gpt2_inference_b200 import tp
    cfg, size = MINI_XL, 2
    params = weights.synth_params(cfg, 9, init="test")
    img = weights.image(params, cfg, "f32")
    C = cfg["C"]
    rng = np.random.default_rng(1)
    x = rng.standard_normal(C).astype(np.float32)
    a = rng.standard_normal(C).astype(np.float32)       # attention output (all heads)
    g = rng.standard_normal(4 * C).astype(np.float32)   # GELU output (all FC rows)
    l = 1
    qkv_parts, fc_parts, proj_sum, fcproj_sum = [], [], 0, 0
    for rank in range(size):
        p = tp.plan(cfg, rank, size)
        b, _ = tp.shard_image(img, None, "f32", rank, size)
        loc = {}
        off = 0
        hl, fl = p["heads"] * 64, p["f_rows"]
        lshape = dict(weights.shapes(cfg), qkvw=(cfg["L"], 3 * hl, C), qkvb=(cfg["L"], 3 * hl),
                      attprojw=(cfg["L"], C, hl), fcw=(cfg["L"], fl, C), fcb=(cfg["L"], fl),
                      fcprojw=(cfg["L"], C, fl))
        for n in weights.NAMES:
            cnt = int(np.prod(lshape[n]))
            loc[n] = np.frombuffer(b, np.float32, cnt, off).reshape(lshape[n])
            off += 4 * cnt
        assert off == len(b)
        h0, f0 = p["h0"] * 64, p["f0"]
        qkv_parts.append(orc.gemv(loc["qkvw"][l], x).reshape(3, hl))
        fc_parts.append(orc.gemv(loc["fcw"][l], x))
        proj_sum = proj_sum + orc.gemv(loc["attprojw"][l], a[h0:h0 + hl])
        fcproj_sum = fcproj_sum + orc.gemv(loc["fcprojw"][l], g[f0:f0 + fl])
    full_qkv = orc.gemv(params["qkvw"][l], x).reshape(3, C)
    assert np.allclose(np.concatenate(qkv_parts, axis=1), full_qkv, rtol=1e-6, atol=1e-6)
    assert np.allclose(np.concatenate(fc_parts), orc.gemv(params["fcw"][l], x), rtol=1e-6, atol=1e-6)
    assert np.allclose(proj_sum, orc.gemv(params["attprojw"][l], a), rtol=1e-5, atol=1e-5)
    assert np.allclose(fcproj_sum, orc.gemv(params["fcprojw"][l], g), rtol=1e-5, atol=1e-5)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank: int, size: int, port: int, q):
    import torch.distributed as dist

    from cuda_gpt2_inference_b200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        gid = tp.shared_group_id(rank)
        p = tp.plan(weights.GPT2_XL, rank, size)
        q.put((rank, gid, p))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_group_agrees_on_id_and_tiles_the_model(gpt2b):
    import torch.multiprocessing as mp
    size, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, size, port, q)) for r in range(size)]
    for pr in procs:
        pr.start()
    got = sorted(q.get(timeout=120) for _ in range(size))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    ids = {g for _, g, _ in got}
    assert len(ids) == 1 and len(next(iter(ids))) == 128
    heads = sorted((p["h0"], p["heads"]) for _, _, p in got)
    assert heads == [(0, 13), (13, 12)]
    assert sum(p["v_rows"] for _, _, p in got) == 50304
