"""Pin the CPU oracle before trusting it.

1. Against the committed fixtures produced by the reference's own CPU loops
   (tests/golden/make_golden.py): these run anywhere.
2. Against the reference's CPU loops compiled from source in oracle/_ref, at
   more shapes, when those libraries are present.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err


def test_gemv_matches_reference_loop_fixture(orc, golden):
    for name in ("qkv", "fcproj", "ragged"):
        W, x, b = golden[f"gemv_{name}_W"], golden[f"gemv_{name}_x"], golden[f"gemv_{name}_b"]
        assert np.array_equal(orc.gemv(W, x), golden[f"gemv_{name}_out"]), name
        out, pre = orc.gemv_fused(W, x, b, do_gelu=True)
        assert np.array_equal(pre, golden[f"gemv_{name}_out"] + b)
        # gelu.cu writes sqrt(2/pi) as sqrtf(2.0f/M_PI); the engine epilogue as a literal
        assert rel_err(out, golden[f"gemv_{name}_gelu"]) < 1e-6


def test_attention_matches_reference_loop_fixture(orc, golden):
    qkv, kv = golden["attn_qkv"], golden["attn_kv"]
    for sl in (1, 17, 64):
        got = orc.attention_kv(qkv, kv, 1, sl, 2, 64, 64, 0.125)
        assert np.array_equal(got, golden[f"attn_out_{sl}"]), sl


def test_layernorm_residual_match_reference_loop_fixture(orc, golden):
    res = golden["ln_a"] + golden["ln_b"]
    assert np.array_equal(res, golden["ln_res"])
    out, mean, rstd = orc.layernorm(golden["ln_res"], golden["ln_w"], golden["ln_beta"])
    assert np.array_equal(out, golden["ln_out"])
    assert np.array_equal(mean, golden["ln_mean"]) and np.array_equal(rstd, golden["ln_rstd"])


def test_encoder_matches_reference_loop_fixture(orc, golden):
    wte, wpe, toks = golden["enc_wte"], golden["enc_wpe"], golden["enc_tok"][0]
    for t in range(3):
        assert np.array_equal(wte[toks[t]] + wpe[t], golden["enc_out"][0, t])


def test_whole_model_matches_reference_composed_decode(orc, golden):
    from cuda_gpt2_inference_b200 import weights
    c = golden["dec_cfg"]
    cfg = dict(maxT=int(c[0]), V=int(c[1]), L=int(c[2]), NH=int(c[3]), C=int(c[4]), Vp=int(c[5]))
    params = weights.synth_params(cfg, seed=int(golden["dec_seed"][0]), init="test")
    m = orc.Model(weights.image(params, cfg, "f32"), "f32")
    for pos, tok in enumerate(golden["dec_tokens"]):
        lg = m.step(int(tok), pos)
        assert rel_err(lg, golden["dec_logits"][pos]) < 2e-6, pos
        assert int(np.argmax(lg[: cfg["V"]])) == int(golden["dec_picks"][pos])


def test_fp8_decode_table_is_e4m3(orc):
    # spot values of the OCP E4M3 format: max normal, min normal, min subnormal, zero, sign
    d = orc.decode_w8(np.array([0x7E, 0x08, 0x01, 0x00, 0x80 | 0x7E, 0x38], np.uint8), "fp8")
    assert list(d) == [448.0, 2.0 ** -6, 2.0 ** -9, 0.0, -448.0, 1.0]
    assert list(orc.decode_w8(np.array([0x7F, 0x80, 0x01], np.uint8), "int8")) == [127.0, -128.0, 1.0]


def test_quant_rows_rule(orc):
    rng = np.random.default_rng(3)
    W = rng.standard_normal((5, 64)).astype(np.float32)
    W[2] = 0.0  # an all-zero row gets scale 1 (quantize.cu:62)
    q, s = orc.quant_rows(W, "int8")
    assert s[2] == 1.0 and not q[2].any()
    amax = np.abs(W).max(axis=1)
    assert np.allclose(s[[0, 1, 3, 4]], amax[[0, 1, 3, 4]] / 127.0, rtol=1e-7)
    deq = q.view(np.int8).astype(np.float32) * s[:, None]
    assert np.abs(deq - W).max() <= s.max() / 2 * 1.0001
    qf, sf = orc.quant_rows(W, "fp8")
    assert np.allclose(sf[[0, 1, 3, 4]], amax[[0, 1, 3, 4]] / 448.0, rtol=1e-7)
    assert np.abs(orc.decode_w8(qf, "fp8") * sf[:, None] - W).max() <= 0.07 * np.abs(W).max()


def test_kv_encode_row_rule(orc):
    x = np.linspace(-2, 2, 64).astype(np.float32)
    codes, sc = orc.kv_encode_row(x, "int8")
    assert sc == pytest.approx(2.0 / 127.0, rel=1e-7)
    assert codes.view(np.int8)[0] == -127 and codes.view(np.int8)[-1] == 127
    codes0, sc0 = orc.kv_encode_row(np.zeros(64, np.float32), "int8")  # no zero guard: scale 0, codes 0
    assert sc0 == 0.0 and not codes0.any()


# ---- live comparison with the reference CPU loops built from source ----
def _ref(orc, which):
    if not orc.ref_available(f"libref_cpu_{which}.so"):
        pytest.skip("reference CPU loops not built (no reference checkout)")
    return orc.ref_cpu(which)


@pytest.mark.parametrize("M,K", [(2304, 768), (768, 768), (3072, 768), (768, 3072), (1, 16), (5, 1600)])
def test_gemv_live_against_reference_loop(orc, M, K):
    ref = _ref(orc, "gemv")
    rng = np.random.default_rng(M * 7 + K)
    W = rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal(K, dtype=np.float32)
    out = np.zeros(M, np.float32)
    ref.ref_gemv_cpu_f32(orc.ptr(out), orc.ptr(W), orc.ptr(x), M, K)
    assert np.array_equal(orc.gemv(W, x), out)


@pytest.mark.parametrize("seq_len", [1, 2, 149, 150, 511, 1024])
def test_attention_live_against_reference_loop(orc, seq_len):
    ref = _ref(orc, "attention")
    rng = np.random.default_rng(seq_len)
    B, NH, hs, maxT = 1, 12, 64, 1024
    qkv = rng.standard_normal(3 * NH * hs).astype(np.float32)
    kv = rng.standard_normal(2 * NH * maxT * hs).astype(np.float32)
    out = np.zeros(NH * hs, np.float32)
    ref.ref_attention_kv_cpu(orc.ptr(out), orc.ptr(qkv), orc.ptr(kv), B, seq_len, NH, hs, maxT, 0.125)
    assert np.array_equal(orc.attention_kv(qkv, kv, B, seq_len, NH, hs, maxT, 0.125), out)
