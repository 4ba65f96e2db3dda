"""Generate the committed golden fixtures from the reference's own CPU loops.

The reference ships no golden vectors (its labs regenerate random data with
srand(0) at run time), so these fixtures are produced here by calling the
reference's CPU loops compiled from its sources (oracle/_ref, built by
oracle/build_oracle.py from the reference checkout) on seeded inputs:

* GEMV_cpu                (gemv/GEMV.cu:84-93)
* gelu_forward_cpu        (gelu/gelu.cu:31-37)
* attention_kv_cpu        (attention_kvcache/attention_kvcache.cu:74-103)
* layernorm_forward_cpu / residual_forward_cpu (fused/fused.cu:44-80)
* encoder_forward_cpu     (other_kernels/encoder.cu:34-48)
* a 4-step decode of a 2-layer model composed from those loops
  (oracle/ref_shims/ref_cpu_decode.cpp)

Usage: ``python tests/golden/make_golden.py`` (needs oracle/_ref built).
Output: ``tests/golden/ref_cpu_loops.npz``.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from cuda_gpt2_inference_b200 import weights  # noqa: E402

P = oracle.ptr
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_cpu_loops.npz")


def main() -> int:
    rng = np.random.default_rng(20251103)
    g = {}
    # GEMV at the decode K values, a slice of rows each
    gemv = oracle.ref_cpu("gemv")
    gelu = oracle.ref_cpu("gelu")
    for name, (M, K) in {"qkv": (24, 768), "fcproj": (8, 3072), "ragged": (7, 1600)}.items():
        W = (rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02))
        x = rng.standard_normal(K, dtype=np.float32)
        b = rng.standard_normal(M, dtype=np.float32) * np.float32(0.02)
        out = np.zeros(M, np.float32)
        gemv.ref_gemv_cpu_f32(P(out), P(W), P(x), M, K)
        pre = out + b
        act = np.zeros(M, np.float32)
        gelu.ref_gelu_cpu(P(act), P(pre), M)
        g.update({f"gemv_{name}_W": W, f"gemv_{name}_x": x, f"gemv_{name}_b": b, f"gemv_{name}_out": out,
                  f"gemv_{name}_gelu": act})
    # attention over a float cache in the reference layout
    attn = oracle.ref_cpu("attention")
    B, NH, hs, maxT = 1, 2, 64, 64
    qkv = rng.uniform(-1, 1, 3 * NH * hs).astype(np.float32)
    kv = rng.uniform(-1, 1, 2 * NH * maxT * hs).astype(np.float32)
    g["attn_qkv"], g["attn_kv"] = qkv, kv
    for sl in (1, 17, 64):
        out = np.zeros(NH * hs, np.float32)
        attn.ref_attention_kv_cpu(P(out), P(qkv), P(kv), B, sl, NH, hs, maxT, np.float32(0.125))
        g[f"attn_out_{sl}"] = out
    # residual + layernorm
    fused = oracle.ref_cpu("fused")
    C = 768
    a = rng.standard_normal((2, C), dtype=np.float32)
    bb = rng.standard_normal((2, C), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    res = np.zeros((2, C), np.float32)
    fused.ref_residual_cpu(P(res), P(a), P(bb), 2 * C)
    ln = np.zeros((2, C), np.float32)
    mean, rstd = np.zeros(2, np.float32), np.zeros(2, np.float32)
    fused.ref_layernorm_cpu(P(ln), P(mean), P(rstd), P(res), P(w), P(beta), 2, 1, C)
    g.update(dict(ln_a=a, ln_b=bb, ln_w=w, ln_beta=beta, ln_res=res, ln_out=ln, ln_mean=mean, ln_rstd=rstd))
    # encoder
    enc = oracle.ref_cpu("encoder")
    V, T, C = 20, 3, 64
    wte = rng.standard_normal((V, C), dtype=np.float32)
    wpe = rng.standard_normal((T, C), dtype=np.float32)
    toks = np.array([[3, 19, 0]], np.int32)
    eo = np.zeros((1, T, C), np.float32)
    enc.ref_encoder_cpu(P(eo), P(toks), P(wte), P(wpe), 1, T, C)
    g.update(dict(enc_wte=wte, enc_wpe=wpe, enc_tok=toks, enc_out=eo))
    # a short decode of a 2-layer model through the composed reference loops
    cfg = weights.mini_config(L=2, NH=2, maxT=64, V=500, Vp=512)
    params = weights.synth_params(cfg, seed=7, init="test")
    flat = np.concatenate([params[n].ravel() for n in weights.NAMES]).astype(np.float32)
    dec = oracle.ref_cpu("decode")
    cfg6 = np.array([cfg["maxT"], cfg["V"], cfg["L"], cfg["NH"], cfg["C"], cfg["Vp"]], np.int32)
    h = dec.ref_decoder_create(P(cfg6), P(flat))
    toks_in = [5, 17, 123, 499]
    logits = np.zeros((len(toks_in), cfg["Vp"]), np.float32)
    picks = []
    for pos, t in enumerate(toks_in):
        row = np.zeros(cfg["Vp"], np.float32)
        picks.append(dec.ref_decoder_step(h, t, pos, P(row)))
        logits[pos] = row
    dec.ref_decoder_free(h)
    g.update(dict(dec_cfg=cfg6, dec_seed=np.array([7], np.int32), dec_tokens=np.array(toks_in, np.int32),
                  dec_logits=logits, dec_picks=np.array(picks, np.int32)))
    np.savez_compressed(OUT, **g)
    print(OUT, os.path.getsize(OUT), "bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
