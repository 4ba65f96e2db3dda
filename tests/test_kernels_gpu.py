"""Kernel parity on the GPU, through the C ABI.

Each operator is compared with the CPU oracle on the same seeded inputs
(tolerances from the reference labs and the north-star spec), and -- where the
reference's CUDA kernels were built from source into oracle/_ref -- with the
reference kernel on the same device buffers.  Byte outputs (8-bit KV codes,
quantiser codes and scales) must match the reference kernels exactly.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(2304, 768), (768, 768), (3072, 768), (768, 3072), (50257, 768), (1, 768), (3, 16), (17, 1600),
          (2305, 768)]


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)


def host(t):
    return t.float().cpu().numpy()


def _data(M, K, seed):
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal(K, dtype=np.float32)
    b = rng.standard_normal(M, dtype=np.float32) * np.float32(0.02)
    return W, x, b


def _ref_lib(orc, name):
    return orc.ref_gpu(name) if orc.ref_available(f"libref_{name}.so") else None


# ---------------------------------------------------------------- GEMV ----
@pytest.mark.parametrize("M,K", SHAPES)
def test_gemv6_f32(cuda, orc, M, K):
    from cuda_gpt2_inference_b200 import ops
    W, x, _ = _data(M, K, M + K)
    out = torch.empty(M, device="cuda")
    ops.launch_GEMV6(out, dev(W), dev(x), M, K)
    torch.cuda.synchronize()
    assert rel_err(host(out), orc.gemv(W, x)) < 1e-4  # FP32: 1e-4 relative


@pytest.mark.parametrize("M,K", SHAPES)
@pytest.mark.parametrize("do_gelu", [0, 1])
def test_gemv6_fused_f32_and_bf16(cuda, orc, M, K, do_gelu):
    from cuda_gpt2_inference_b200 import ops
    W, x, b = _data(M, K, 3 * M + K)
    ref_out, ref_pre = orc.gemv_fused(W, x, b, do_gelu)
    out, pre = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    ops.launch_GEMV6_fused(out, pre, dev(W), dev(x), dev(b), M, K, do_gelu)
    torch.cuda.synchronize()
    assert rel_err(host(out), ref_out) < 1e-4 and rel_err(host(pre), ref_pre) < 1e-4
    # BF16 storage: the oracle sees the same bf16-rounded operands
    W16, x16, b16 = orc.bf16_round(W), orc.bf16_round(x), orc.bf16_round(b)
    r16, p16 = orc.gemv_fused(W16, x16, b16, do_gelu)
    o, p = torch.empty(M, device="cuda", dtype=torch.bfloat16), torch.empty(M, device="cuda", dtype=torch.bfloat16)
    ops.launch_GEMV6_fused(o, p, dev(W16, torch.bfloat16), dev(x16, torch.bfloat16), dev(b16, torch.bfloat16), M, K,
                           do_gelu)
    torch.cuda.synchronize()
    assert rel_err(host(o), r16) < 1e-2 and rel_err(host(p), p16) < 1e-2  # BF16: 1e-2
    # the LM-head form: bf16 weights, fp32 out, no bias
    o32 = torch.empty(M, device="cuda")
    ops.launch_GEMV6(o32, dev(W16, torch.bfloat16), dev(x16, torch.bfloat16), M, K)
    torch.cuda.synchronize()
    assert rel_err(host(o32), orc.gemv(W16, x16)) < 1e-4


@pytest.mark.parametrize("fmt", ["int8", "fp8"])
@pytest.mark.parametrize("M,K", SHAPES)
def test_gemv6_w8x2(cuda, orc, fmt, M, K):
    from cuda_gpt2_inference_b200 import ops
    W, x, b = _data(M, K, 5 * M + K)
    codes, scale = orc.quant_rows(W, fmt)
    x16, b16 = orc.bf16_round(x), orc.bf16_round(b)
    Wd, xd, sd, bd = dev(codes, torch.uint8), dev(x16, torch.bfloat16), dev(scale), dev(b16, torch.bfloat16)
    # FP32-output (LM head) form: 1e-3 relative to the FP32 dequant-GEMV
    o32 = torch.empty(M, device="cuda")
    ops.launch_GEMV6_w8x2(o32, None, Wd, xd, sd, None, M, K, 0, fmt=fmt)
    ref, _ = orc.gemv_w8(codes, fmt, x16, scale, None, 0)
    deq = orc.gemv(orc.decode_w8(codes, fmt) * scale[:, None], x16)
    torch.cuda.synchronize()
    assert rel_err(host(o32), ref) < 1e-5
    assert rel_err(host(o32), deq) < 1e-3
    # layer form: bias, GELU, pre-GELU, bf16 storage
    for do_gelu in (0, 1):
        o = torch.empty(M, device="cuda", dtype=torch.bfloat16)
        p = torch.empty(M, device="cuda", dtype=torch.bfloat16)
        ops.launch_GEMV6_w8x2(o, p, Wd, xd, sd, bd, M, K, do_gelu, fmt=fmt)
        r, rp = orc.gemv_w8(codes, fmt, x16, scale, b16, do_gelu)
        torch.cuda.synchronize()
        assert rel_err(host(o), r) < 1e-2 and rel_err(host(p), rp) < 1e-2


@pytest.mark.parametrize("fmt", ["int8", "fp8"])
@pytest.mark.parametrize("M,K", [(50257, 768), (9999, 768), (5003, 1600), (9001, 784)])
def test_gemv6_w8x2_streamed_forms(cuda, orc, fmt, M, K):
    """Streamed 8-bit GEMVs (more rows than one tile per SM): the tensor-core form
    (K a multiple of 32; 16-row tiles, ragged last tile at M = 9999 / 5003) and the
    CUDA-core form (K = 784).  Against the oracle at 1e-5; x beyond FP16's range
    (|x| ~ 1e5) and far below it (~1e-7) through the same exact power-of-two
    scaling: out(x * 2^k) == out(x) * 2^k bit for bit."""
    from cuda_gpt2_inference_b200 import ops
    W, x, _ = _data(M, K, 7 * M + K)
    codes, scale = orc.quant_rows(W, fmt)
    Wd, sd = dev(codes, torch.uint8), dev(scale)
    outs = {}
    for k in (0, 17, -23):
        x16 = orc.bf16_round(x * np.float32(2.0 ** k))
        o = torch.empty(M, device="cuda")
        ops.launch_GEMV6_w8x2(o, None, Wd, dev(x16, torch.bfloat16), sd, None, M, K, 0, fmt=fmt)
        torch.cuda.synchronize()
        outs[k] = host(o)
        ref, _ = orc.gemv_w8(codes, fmt, x16, scale, None, 0)
        assert rel_err(outs[k], ref) < 1e-5, k
    assert np.array_equal(outs[17], outs[0] * np.float32(2.0 ** 17))
    assert np.array_equal(outs[-23], outs[0] * np.float32(2.0 ** -23))


@pytest.mark.parametrize("M,K", [(2304, 768), (3072, 768), (768, 3072), (50257, 768)])
def test_gemv_against_reference_kernels(cuda, orc, M, K):
    """Our GEMVs vs the reference's GEMV6 / GEMV6_fused / GEMV6_w8x2 built for sm_100a."""
    from cuda_gpt2_inference_b200 import ops
    f32 = _ref_lib(orc, "ops_f32")
    if f32 is None:
        pytest.skip("reference kernels not built")
    W, x, b = _data(M, K, 11 * M + K)
    Wd, xd, bd = dev(W), dev(x), dev(b)
    mine, theirs = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    pm, pt = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    ops.launch_GEMV6_fused(mine, pm, Wd, xd, bd, M, K, 1)
    f32.ref_gemv6_fused(ctypes.c_void_p(theirs.data_ptr()), ctypes.c_void_p(pt.data_ptr()),
                        ctypes.c_void_p(Wd.data_ptr()), ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(bd.data_ptr()),
                        M, K, 1)
    torch.cuda.synchronize()
    assert rel_err(host(mine), host(theirs)) < 1e-5 and rel_err(host(pm), host(pt)) < 1e-5
    w8 = _ref_lib(orc, "w8_int8")
    if w8 is not None:
        codes, scale = orc.quant_rows(W, "int8")
        Cd, sd, x16 = dev(codes, torch.uint8), dev(scale), dev(x, torch.bfloat16)
        a, c = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
        ops.launch_GEMV6_w8x2(a, None, Cd, x16, sd, None, M, K, 0, fmt="int8")
        w8.ref_gemv6_w8x2_f32out(ctypes.c_void_p(c.data_ptr()), ctypes.c_void_p(Cd.data_ptr()),
                                 ctypes.c_void_p(x16.data_ptr()), ctypes.c_void_p(sd.data_ptr()), M, K)
        torch.cuda.synchronize()
        assert rel_err(host(a), host(c)) < 1e-5


def test_gemv_rejects_unaligned_and_accepts_empty(cuda, gpt2b):
    from cuda_gpt2_inference_b200 import ops
    W = torch.zeros(4, 20, device="cuda")  # 80-byte rows: fine; 20 bf16 = 40 bytes: not a multiple of 16
    with pytest.raises(gpt2b.Gpt2bError) as e:
        ops.launch_GEMV6(torch.empty(4, device="cuda"), W.to(torch.bfloat16), torch.zeros(20, device="cuda",
                         dtype=torch.bfloat16), 4, 20)
    assert e.value.status == gpt2b.ERR_ALIGNMENT
    ops.launch_GEMV6(torch.empty(1, device="cuda"), W, torch.zeros(20, device="cuda"), 0, 20)


# ----------------------------------------------------------- attention ----
def _kv_setup(kind, pos, seed, NH=12, maxT=1024, hs=64):
    rng = np.random.default_rng(seed)
    kvf = rng.standard_normal((2, NH, maxT, hs), dtype=np.float32)
    qkv = rng.standard_normal(3 * NH * hs, dtype=np.float32)
    return kvf, qkv


@pytest.mark.parametrize("kind", ["f32", "bf16", "int8", "fp8"])
@pytest.mark.parametrize("pos", [0, 1, 63, 149, 150, 511, 1023])
def test_attention_small_and_large(cuda, orc, kind, pos):
    from cuda_gpt2_inference_b200 import ops
    NH, hs, maxT = 12, 64, 1024
    kvf, qkv = _kv_setup(kind, pos, pos + 7)
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    if kind in ("f32", "bf16"):
        dt = torch.float32 if kind == "f32" else torch.bfloat16
        cache = dev(kvf.ravel(), dt)
        qd = dev(qkv, dt)
        ops.kv_cache_write(cache, qd, 1, NH, hs, maxT, dpos)
        torch.cuda.synchronize()
        ref = orc.attention_kv(host(qd), host(cache), 1, pos + 1, NH, hs, maxT)
        tol = 1e-4 if kind == "f32" else 1e-2
        out = torch.empty(NH * hs, device="cuda", dtype=dt)
        ops.attention_forward_kv_small(out, qd, cache, 1, NH, hs, maxT, dpos)
        torch.cuda.synchronize()
        err = np.abs(host(out) - ref).max() if kind == "f32" else rel_err(host(out), ref)
        assert err < tol
        for S in (1, 8, 12, 32):
            po = torch.empty(NH * S * hs, device="cuda")
            pl, pm = torch.empty(NH * S, device="cuda"), torch.empty(NH * S, device="cuda")
            out2 = torch.empty(NH * hs, device="cuda", dtype=dt)
            ops.attention_forward_kv_large(out2, qd, cache, 1, NH, hs, maxT, dpos, po, pl, pm, S)
            torch.cuda.synchronize()
            err = np.abs(host(out2) - ref).max() if kind == "f32" else rel_err(host(out2), ref)
            assert err < tol, S
    else:
        codes = np.zeros((2, NH, maxT, hs), np.uint8)
        scales = np.zeros((2, NH, maxT), np.float32)
        for kvi in range(2):
            for h in range(NH):
                for j in range(maxT):
                    codes[kvi, h, j], scales[kvi, h, j] = orc.kv_encode_row(kvf[kvi, h, j], kind)
        cache, sc = dev(codes.ravel(), torch.uint8), dev(scales.ravel())
        q16 = dev(qkv, torch.bfloat16)
        ops.kv_cache_write(cache, q16, 1, NH, hs, maxT, dpos, kv_scale=sc, fmt=kind)
        torch.cuda.synchronize()
        # the appended rows match the reference encode rule (IEEE vs fast-math division: <= 1 code apart)
        qh = host(q16)
        cc, ss = cache.cpu().numpy().reshape(2, NH, maxT, hs), sc.cpu().numpy().reshape(2, NH, maxT)
        for kvi in range(2):
            for h in range(NH):
                want_c, want_s = orc.kv_encode_row(qh[(1 + kvi) * NH * hs + h * hs:][:hs], kind)
                assert ss[kvi, h, pos] == pytest.approx(want_s, rel=1e-6)
                got = cc[kvi, h, pos]
                if kind == "int8":
                    assert np.abs(got.view(np.int8).astype(int) - want_c.view(np.int8).astype(int)).max() <= 1
        ref = orc.attention_kv_w8(qh, cc.ravel(), ss.ravel(), kind, 1, pos + 1, NH, hs, maxT)
        out = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
        ops.attention_forward_kv_small(out, q16, cache, 1, NH, hs, maxT, dpos, kv_scale=sc, fmt=kind)
        torch.cuda.synchronize()
        assert rel_err(host(out), ref) < 1e-2
        for S in (8, 13):
            po = torch.empty(NH * S * hs, device="cuda")
            pl, pm = torch.empty(NH * S, device="cuda"), torch.empty(NH * S, device="cuda")
            out2 = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
            ops.attention_forward_kv_large(out2, q16, cache, 1, NH, hs, maxT, dpos, po, pl, pm, S, kv_scale=sc,
                                           fmt=kind)
            torch.cuda.synchronize()
            assert rel_err(host(out2), ref) < 1e-2, S


@pytest.mark.parametrize("pos", [0, 150, 700, 1023])
def test_attention_against_reference_kernels(cuda, orc, pos):
    """Split partials and outputs vs the reference split/merge kernels; 8-bit KV
    append codes and scales byte-identical to kv_cache_write_kernel_w8."""
    from cuda_gpt2_inference_b200 import ops
    bf = _ref_lib(orc, "ops_bf16")
    if bf is None:
        pytest.skip("reference kernels not built")
    NH, hs, maxT, S = 12, 64, 1024, 8
    kvf, qkv = _kv_setup("bf16", pos, 99 + pos)
    cache_a = dev(kvf.ravel(), torch.bfloat16)
    cache_b = cache_a.clone()
    qd = dev(qkv, torch.bfloat16)
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    ops.kv_cache_write(cache_a, qd, 1, NH, hs, maxT, dpos)
    assert bf.ref_set_cur_len(pos) == 0
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    bf.ref_kv_cache_write(vp(cache_b), vp(qd), 1, NH, hs, maxT)
    torch.cuda.synchronize()
    assert torch.equal(cache_a, cache_b)
    outs = {}
    for who in ("mine", "ref"):
        po = torch.zeros(NH * S * hs, device="cuda")
        pl, pm = torch.zeros(NH * S, device="cuda"), torch.zeros(NH * S, device="cuda")
        out = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
        if who == "mine":
            ops.attention_forward_kv_large(out, qd, cache_a, 1, NH, hs, maxT, dpos, po, pl, pm, S)
        else:
            bf.ref_attention_split_merge(vp(out), vp(qd), vp(cache_a), 1, NH, hs, maxT, vp(po), vp(pl), vp(pm), S)
        torch.cuda.synchronize()
        outs[who] = (host(out), po.cpu().numpy(), pl.cpu().numpy(), pm.cpu().numpy())
    assert rel_err(outs["mine"][0], outs["ref"][0]) < 1e-2
    assert np.allclose(outs["mine"][3], outs["ref"][3], rtol=1e-5, atol=1e-5)  # split maxima
    assert np.allclose(outs["mine"][2], outs["ref"][2], rtol=1e-4, atol=1e-6)  # split exp-sums
    assert np.allclose(outs["mine"][1], outs["ref"][1], rtol=1e-3, atol=1e-4)  # un-normalised partials
    # 8-bit KV append: codes and scales byte-identical with kv_cache_write_kernel_w8
    # (attention_kvcache_w8.cuh:115-155) built for INT8 and for FP8 E4M3
    checked = 0
    for kind in ("int8", "fp8"):
        w8 = _ref_lib(orc, f"w8_{kind}")
        if w8 is None:
            continue
        ca = torch.zeros(2 * NH * maxT * hs, dtype=torch.uint8, device="cuda")
        cb = ca.clone()
        sa, sb = torch.zeros(2 * NH * maxT, device="cuda"), torch.zeros(2 * NH * maxT, device="cuda")
        ops.kv_cache_write(ca, qd, 1, NH, hs, maxT, dpos, kv_scale=sa, fmt=kind)
        assert w8.ref_set_cur_len(pos) == 0
        w8.ref_kv_cache_write_w8(vp(cb), vp(sb), vp(qd), 1, NH, hs, maxT)
        torch.cuda.synchronize()
        assert torch.equal(ca, cb), kind
        assert torch.equal(sa, sb), kind
        assert int(torch.count_nonzero(ca)) > 0, kind  # the row at pos was written
        checked += 1
    assert checked == 2, "reference 8-bit kernels (INT8 and FP8) not built"


@pytest.mark.parametrize("kind", ["f32", "bf16", "int8", "fp8"])
@pytest.mark.parametrize("pos,S", [(0, 8), (150, 8), (700, 13), (1023, 8)])
def test_attention_split_and_merge_halves(cuda, orc, kind, pos, S):
    """The split and merge halves on their own: bit-identical to the combined
    entry point (same kernels), and partials equal to the reference's own split
    kernel (attention_kv_split_kernel / _w8) on the same cache."""
    from cuda_gpt2_inference_b200 import ops
    NH, hs, maxT = 12, 64, 1024
    kvf, qkv = _kv_setup("bf16" if kind != "f32" else "f32", pos, 300 + pos)
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    w8 = kind in ("int8", "fp8")
    if w8:
        codes = np.zeros((2, NH, maxT, hs), np.uint8)
        scales = np.zeros((2, NH, maxT), np.float32)
        for kvi in range(2):
            for h in range(NH):
                for j in range(pos + 1):
                    codes[kvi, h, j], scales[kvi, h, j] = orc.kv_encode_row(kvf[kvi, h, j], kind)
        cache, sc = dev(codes.ravel(), torch.uint8), dev(scales.ravel())
        qd = dev(qkv, torch.bfloat16)
        odt = torch.bfloat16
    else:
        dt = torch.float32 if kind == "f32" else torch.bfloat16
        cache, sc, qd, odt = dev(kvf.ravel(), dt), None, dev(qkv, dt), dt
    parts = [torch.zeros(NH * S * hs, device="cuda"), torch.zeros(NH * S, device="cuda"),
             torch.zeros(NH * S, device="cuda")]
    ops.attention_kv_split(*parts, qd, cache, 1, NH, hs, maxT, S, dpos, kv_scale=sc, fmt=kind)
    half = torch.empty(NH * hs, device="cuda", dtype=odt)
    ops.attention_kv_merge(half, *parts, 1, NH, hs, S, w8=w8)
    whole = torch.empty(NH * hs, device="cuda", dtype=odt)
    p2 = [torch.zeros_like(t) for t in parts]
    ops.attention_forward_kv_large(whole, qd, cache, 1, NH, hs, maxT, dpos, *p2, S, kv_scale=sc, fmt=kind)
    torch.cuda.synchronize()
    assert torch.equal(half, whole)
    lib = _ref_lib(orc, {"f32": "ops_f32", "bf16": "ops_bf16", "int8": "w8_int8", "fp8": "w8_fp8"}[kind])
    if lib is None:
        pytest.skip("reference kernels not built")
    assert lib.ref_set_cur_len(pos) == 0
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rp = [torch.zeros_like(t) for t in parts]
    ro = torch.empty(NH * hs, device="cuda", dtype=odt)
    if w8:
        lib.ref_attention_split_merge_w8(vp(ro), vp(qd), vp(cache), vp(sc), 1, NH, hs, maxT, vp(rp[0]), vp(rp[1]),
                                         vp(rp[2]), S)
    else:
        lib.ref_attention_split_merge(vp(ro), vp(qd), vp(cache), 1, NH, hs, maxT, vp(rp[0]), vp(rp[1]), vp(rp[2]), S)
    torch.cuda.synchronize()
    assert np.allclose(parts[2].cpu().numpy(), rp[2].cpu().numpy(), rtol=1e-5, atol=1e-5)  # split maxima
    assert np.allclose(parts[1].cpu().numpy(), rp[1].cpu().numpy(), rtol=1e-4, atol=1e-6)  # split exp-sums
    assert np.allclose(parts[0].cpu().numpy(), rp[0].cpu().numpy(), rtol=1e-3, atol=1e-4)  # un-normalised partials
    tol = 1e-4 if kind == "f32" else 1e-2
    assert rel_err(host(half), host(ro)) < tol


# ------------------------------------------------------ LayerNorm etc. ----
@pytest.mark.parametrize("C,N", [(768, 1), (768, 5), (1600, 1), (64, 3)])
def test_layernorm_and_fused_residual(cuda, orc, C, N):
    from cuda_gpt2_inference_b200 import ops
    rng = np.random.default_rng(C + N)
    a = rng.standard_normal((N, C), dtype=np.float32)
    b = rng.standard_normal((N, C), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 5e-2)):  # fused/fused.cu:734 tolerances
        cast = (lambda v: v) if dt == torch.float32 else orc.bf16_round
        A, B_, W, Be = cast(a), cast(b), cast(w), cast(beta)
        res, out = torch.empty(N * C, device="cuda", dtype=dt), torch.empty(N * C, device="cuda", dtype=dt)
        mean, rstd = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
        ops.fused_residual_forward5(res, out, mean, rstd, dev(A, dt), dev(B_, dt), dev(W, dt), dev(Be, dt), N, C)
        ln = torch.empty(N * C, device="cuda", dtype=dt)
        ops.layernorm_forward(ln, None, None, dev(A, dt), dev(W, dt), dev(Be, dt), N, 1, C)
        torch.cuda.synchronize()
        r = cast(A + B_)
        assert np.array_equal(host(res).reshape(N, C), r)
        ref, rm, rr = orc.layernorm(r, W, Be)
        assert np.abs(host(out).reshape(N, C) - ref).max() < tol
        assert np.allclose(mean.cpu().numpy(), rm, atol=1e-5) and np.allclose(rstd.cpu().numpy(), rr, rtol=1e-4)
        ref2, _, _ = orc.layernorm(A, W, Be)
        assert np.abs(host(ln).reshape(N, C) - ref2).max() < tol


def test_encoder(cuda, orc):
    from cuda_gpt2_inference_b200 import ops
    rng = np.random.default_rng(1)
    V, maxT, C = 100, 32, 768
    wte, wpe = rng.standard_normal((V, C), dtype=np.float32), rng.standard_normal((maxT, C), dtype=np.float32)
    toks = torch.tensor([7, 99], dtype=torch.int32, device="cuda")
    for pos in (0, 31):
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        for dt in (torch.float32, torch.bfloat16):
            cast = (lambda v: v) if dt == torch.float32 else orc.bf16_round
            out = torch.empty(2 * C, device="cuda", dtype=dt)
            ops.encoder_forward_kv(out, toks, dev(cast(wte), dt), dev(cast(wpe), dt), dpos, 2, C)
            torch.cuda.synchronize()
            ref = cast(np.stack([cast(wte)[7] + cast(wpe)[pos], cast(wte)[99] + cast(wpe)[pos]]))
            assert np.array_equal(host(out).reshape(2, C), ref)


# -------------------------------------------------------------- picks ----
def test_argmax(cuda):
    from cuda_gpt2_inference_b200 import ops
    rng = np.random.default_rng(2)
    V, ld = 50257, 50304
    lg = rng.standard_normal((3, ld), dtype=np.float32)
    lg[1, 100] = lg[1, 4000] = 50.0  # a tie: the lowest index wins
    lg[2, 50300] = 1e9  # beyond V: ignored
    tok = torch.empty(3, dtype=torch.int32, device="cuda")
    ops.gpu_argmax(tok, dev(lg.ravel()), 3, V, ld)
    torch.cuda.synchronize()
    assert tok.cpu().tolist() == [int(np.argmax(lg[0, :V])), 100, int(np.argmax(lg[2, :V]))]


def test_sample_softmax_matches_reference_sampler(cuda, orc):
    from cuda_gpt2_inference_b200 import ops
    bf = _ref_lib(orc, "ops_bf16")
    if bf is None:
        pytest.skip("reference kernels not built")
    rng = np.random.default_rng(4)
    V = 50257
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    agree = 0
    for trial in range(24):
        lg = dev(rng.standard_normal(V, dtype=np.float32) * (1 + trial % 4))
        a, b = torch.empty(1, dtype=torch.int32, device="cuda"), torch.empty(1, dtype=torch.int32, device="cuda")
        ops.gpu_sample_softmax(a, lg, 1, V, 1337, trial + 1)
        bf.ref_sample_softmax(vp(b), vp(lg), 1, V, ctypes.c_ulonglong(1337), trial + 1)
        torch.cuda.synchronize()
        agree += int(a.item() == b.item())
        assert 0 <= a.item() < V
    assert agree == 24


# ---------------------------------------------------------- quantiser ----
@pytest.mark.parametrize("fmt", ["int8", "fp8"])
def test_quant_rows_bit_exact_with_reference(cuda, orc, fmt):
    from cuda_gpt2_inference_b200 import ops
    q = _ref_lib(orc, "quant")
    rng = np.random.default_rng(8)
    M, K = 3072, 768
    W = rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)
    W[5] = 0.0
    W[6] *= 1e4
    W[7] = rng.uniform(-1e-30, 1e-30, K).astype(np.float32)
    Wd = dev(W)
    c1, s1 = torch.empty(M * K, dtype=torch.uint8, device="cuda"), torch.empty(M, device="cuda")
    ops.quant_rows(Wd, c1, s1, M, K, fmt=fmt)
    torch.cuda.synchronize()
    if q is not None:
        c2, s2 = torch.empty_like(c1), torch.empty_like(s1)
        vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        assert q.ref_quant_rows(vp(Wd), vp(c2), vp(s2), M, K, 1 if fmt == "fp8" else 0) == 0
        assert torch.equal(s1, s2), "scales differ from quantize.cu"
        assert torch.equal(c1, c2), "codes differ from quantize.cu"
    # against the IEEE oracle: scales within one ulp, codes identical or one step apart
    oc, osc = orc.quant_rows(W, fmt)
    assert np.allclose(s1.cpu().numpy(), osc, rtol=2.5e-7, atol=0)
    got = c1.cpu().numpy().reshape(M, K)
    frac = (got != oc).mean()
    assert frac < 1e-3
    deq = orc.dequant_rows(got, s1.cpu().numpy(), fmt)
    back = torch.empty(M * K, dtype=torch.bfloat16, device="cuda")
    ops.dequant_wte(c1, s1, back, M, K, fmt=fmt)
    torch.cuda.synchronize()
    assert np.array_equal(host(back).reshape(M, K), deq)


def test_quantize_file_matches_reference_tool(cuda, orc, tmp_path, gpt2b):
    q = _ref_lib(orc, "quant")
    if q is None:
        pytest.skip("reference quantiser not built")
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=2, NH=2, maxT=64, V=500, Vp=512)
    src = tmp_path / "m_bf16.bin"
    src.write_bytes(weights.image(weights.synth_params(cfg, 21), cfg, "bf16"))
    q.ref_quantize_files.argtypes = [ctypes.c_char_p] * 3 + [ctypes.c_int]
    for fmt, flag in (("int8", 0), ("fp8", 1)):
        a8, as_ = tmp_path / f"mine_{fmt}.bin", tmp_path / f"mine_{fmt}_scales.bin"
        b8, bs = tmp_path / f"ref_{fmt}.bin", tmp_path / f"ref_{fmt}_scales.bin"
        gpt2b.check(gpt2b.lib().gpt2b_quantize_file(str(src).encode(), str(a8).encode(), str(as_).encode(), flag))
        assert q.ref_quantize_files(str(src).encode(), str(b8).encode(), str(bs).encode(), flag) == 0
        assert a8.read_bytes() == b8.read_bytes(), fmt
        assert as_.read_bytes() == bs.read_bytes(), fmt


# ------------------------------------------------- prompt GEMM (tcgen05) ----
MM_SHAPES = [(24, 768, 2304), (24, 3072, 768), (24, 768, 3072), (200, 768, 768), (5, 1600, 4800), (3, 776, 770),
             (1, 64, 16)]


@pytest.mark.parametrize("T,C,OC", MM_SHAPES)
@pytest.mark.parametrize("fmt", ["bf16", "int8", "fp8"])
def test_matmul_forward_tensor_cores(cuda, orc, T, C, OC, fmt):
    """The tcgen05 prompt GEMM against a torch FP32 matmul of the same
    BF16-rounded operands (8-bit: the dequantised codes x row scale): BF16
    outputs within 1e-2 relative (bias, pre-GELU and fused GELU), FP32 outputs
    within 1e-4.  Shapes cover several 128-row token tiles, N and K tails."""
    from cuda_gpt2_inference_b200 import ops
    if fmt != "bf16" and C % 16:
        pytest.skip("8-bit rows must be a multiple of 16 bytes")
    rng = np.random.default_rng(T * 7 + C + OC)
    x = torch.from_numpy(rng.standard_normal((T, C), dtype=np.float32)).to(torch.bfloat16)
    W = rng.standard_normal((OC, C), dtype=np.float32) * np.float32(0.02)
    b = torch.from_numpy(rng.standard_normal(OC, dtype=np.float32) * np.float32(0.02)).to(torch.bfloat16)
    if fmt == "bf16":
        Wd = torch.from_numpy(W).to(torch.bfloat16)
        Wref, sc = Wd.float(), None
        Wdev = Wd.cuda()
    else:
        codes, scale = orc.quant_rows(W, fmt)
        Wref = torch.from_numpy(orc.decode_w8(codes, fmt) * scale[:, None])
        Wdev, sc = dev(codes, torch.uint8), dev(scale)
    xd, bd = x.cuda(), b.cuda()
    pre = x.float() @ Wref.t() + b.float()
    out = torch.empty(T, OC, device="cuda", dtype=torch.bfloat16)
    pg = torch.empty(T, OC, device="cuda", dtype=torch.bfloat16)
    ops.matmul_forward(out, xd, Wdev, bd, 1, T, C, OC, pre_gelu=pg, scale=sc, fmt=fmt)
    plain = torch.empty(T, OC, device="cuda", dtype=torch.bfloat16)
    ops.matmul_forward(plain, xd, Wdev, bd, 1, T, C, OC, scale=sc, fmt=fmt)
    o32 = torch.empty(T, OC, device="cuda")
    ops.matmul_forward(o32, xd, Wdev, None, 1, T, C, OC, scale=sc, fmt=fmt)
    torch.cuda.synchronize()
    gelu = 0.5 * pre * (1 + torch.tanh(0.7978845608028654 * (pre + 0.044715 * pre ** 3)))
    assert rel_err(host(pg), pre.numpy()) < 1e-2
    assert rel_err(host(plain), pre.numpy()) < 1e-2
    assert rel_err(host(out), gelu.numpy()) < 1e-2
    assert rel_err(host(o32), (x.float() @ Wref.t()).numpy()) < 1e-4
