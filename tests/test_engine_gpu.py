"""Whole-model decode parity on the GPU.

* Small models in every precision mode against the CPU oracle, teacher-forced
  on the engine's own tokens (so a late divergence in greedy picks cannot hide
  an early numerical difference), plus FP32 greedy tokens identical.
* GPT-2 124M FP32: 24-token prompt + 128 greedy steps, tokens identical to the
  oracle and logits cosine >= 0.9999 at every step.
* GPT-2 124M BF16 / INT8+KV8 / FP8+KV8 against the reference decode engine
  compiled from source (oracle/_ref/libref_engine_*.so), teacher-forced.
* Launch modes (CUDA graph / eager, PDL on/off, device-resident decode) give
  bit-identical results.
* Both step implementations run every parity case: the persistent decode
  kernel (one cooperative launch per call) and the per-kernel path.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu

MODES = [("f32", "floatx"), ("bf16", "floatx"), ("int8", "floatx"), ("int8", "8bit"), ("fp8", "8bit"),
         ("fp8", "floatx")]
PATHS = ["persistent", "kernels"]


def _engine(img, wmode, kvmode="floatx", sc=None, path="persistent"):
    """An engine on the requested step implementation (fails if it is unavailable)."""
    from cuda_gpt2_inference_b200 import OPT_PERSISTENT
    from cuda_gpt2_inference_b200.engine import Engine
    assert path in PATHS, path
    eng = Engine.from_buffer(img, wmode, kvmode, sc)
    eng.set_option(OPT_PERSISTENT, 1 if path == "persistent" else 0)
    # a silent fallback to the other implementation fails here: the persistent
    # kernel reports 0 kernels per step (one launch per call)
    assert (eng.kernels_per_step() == 0) == (path == "persistent"), (path, eng.kernels_per_step())
    return eng


def _quantize(gpt2b, img16: bytes, fmt: str):
    lib = gpt2b.lib()
    ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
    gpt2b.check(lib.gpt2b_quantized_size(img16, len(img16), ctypes.byref(ob), ctypes.byref(ns)))
    out = ctypes.create_string_buffer(ob.value)
    sc = np.zeros(ns.value, np.float32)
    gpt2b.check(lib.gpt2b_quantize_buffer(img16, len(img16), out, sc.ctypes.data_as(ctypes.c_void_p),
                                          1 if fmt == "fp8" else 0), "quantize")
    return out.raw, sc


def _images(gpt2b, cfg, seed, init):
    from cuda_gpt2_inference_b200 import weights
    p = weights.synth_params(cfg, seed, init=init)
    imgs = {"f32": (weights.image(p, cfg, "f32"), None), "bf16": (weights.image(p, cfg, "bf16"), None)}
    for fmt in ("int8", "fp8"):
        imgs[fmt] = _quantize(gpt2b, imgs["bf16"][0], fmt)
    return imgs


@pytest.fixture(scope="module")
def mini(gpt2b, cuda):
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=2, NH=2, maxT=64, V=500, Vp=512)
    return cfg, _images(gpt2b, cfg, 31, "test")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("wmode,kvmode", MODES)
def test_mini_model_matches_oracle(mini, orc, wmode, kvmode, path):
    cfg, imgs = mini
    img, sc = imgs[wmode]
    eng = _engine(img, wmode, kvmode, sc, path)
    prompt = [5, 17, 123, 499, 0]
    n_gen = cfg["maxT"] - len(prompt)
    toks, lg = eng.generate(prompt, n_gen, want_logits=True)
    m = orc.Model(img, wmode, kvmode, sc)
    seq = list(prompt) + list(toks[:-1])
    floor = 0.99999 if wmode == "f32" else 0.999
    worst = 1.0
    for pos, t in enumerate(seq):
        ref = m.step(int(t), pos)
        worst = min(worst, cosine(lg[pos], ref))
        if wmode == "f32":
            assert int(np.argmax(ref[: cfg["V"]])) == int(np.argmax(lg[pos][: cfg["V"]])), pos
    assert worst >= floor, worst
    if wmode == "f32":
        m.reset()
        otoks, _ = m.generate(prompt, n_gen)
        assert np.array_equal(otoks, toks)
    eng.close()


def test_launch_modes_bit_identical(mini):
    from cuda_gpt2_inference_b200 import OPT_STEPS_PER_GRAPH, OPT_USE_GRAPH, OPT_USE_PDL
    cfg, imgs = mini
    img, _ = imgs["bf16"]
    prompt = [1, 2, 3]
    results = []
    for graph, pdl, spg in ((1, 1, 8), (0, 1, 8), (1, 0, 8), (0, 0, 1), (1, 1, 3)):
        eng = _engine(img, "bf16", path="kernels")
        eng.set_option(OPT_USE_GRAPH, graph)
        eng.set_option(OPT_USE_PDL, pdl)
        eng.set_option(OPT_STEPS_PER_GRAPH, spg)
        toks, lg = eng.generate(prompt, 40, want_logits=True)
        results.append((toks, lg))
        fast, _ = eng.generate(prompt, 40)  # device-resident path
        assert np.array_equal(fast, toks)
        eng.close()
    for toks, lg in results[1:]:
        assert np.array_equal(toks, results[0][0]) and np.array_equal(lg, results[0][1])


@pytest.mark.parametrize("wmode,kvmode", [("bf16", "floatx"), ("int8", "8bit"), ("f32", "floatx")])
def test_persistent_launch_splits_bit_identical(mini, wmode, kvmode):
    """One launch for the whole call, one launch per step, and a decode split
    over several calls give the same tokens (and the same last logits)."""
    cfg, imgs = mini
    img, sc = imgs[wmode]
    prompt = [7, 8, 9, 10]
    eng = _engine(img, wmode, kvmode, sc)
    per_step, lg = eng.generate(prompt, 50, want_logits=True)   # one launch per step
    one_launch, _ = eng.generate(prompt, 50)                    # one launch in total
    assert np.array_equal(per_step, one_launch)
    # the prompt teacher-forced in one call, then 50 steps in calls of 1, 7, 19, 23
    eng.generate(prompt, 0)
    for n in (1, 7, 19, 23):
        eng.decode(n)
    hist = eng.history(len(prompt), 51)
    assert np.array_equal(hist, one_launch), (hist[:12], one_launch[:12])
    # and the arithmetic of every step is independent of the call split: the last
    # step's logits are bit-identical to those of the one-launch-per-step run
    split_last = _device_logits(eng)
    assert np.array_equal(split_last, lg[-1]), float(np.abs(split_last - lg[-1]).max())
    eng.generate(prompt, 50)
    assert np.array_equal(_device_logits(eng), lg[-1])
    eng.close()


class _DevArray:
    """A raw device pointer seen by torch (CUDA array interface)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _device_logits(eng):
    import torch
    torch.cuda.synchronize()
    t = torch.as_tensor(_DevArray(eng.device_buffers()["logits"], eng.config["Vp"]), device="cuda")
    return t.cpu().numpy().copy()


def test_persistent_matches_kernel_path(mini):
    """The two step implementations agree to rounding: teacher-forced on the
    kernel path's tokens, logits cosine >= 0.9999 in BF16."""
    cfg, imgs = mini
    img, _ = imgs["bf16"]
    prompt = [3, 1, 4, 1, 5]
    ek = _engine(img, "bf16", path="kernels")
    toks, lk = ek.generate(prompt, 40, want_logits=True)
    ek.close()
    ep = _engine(img, "bf16", path="persistent")
    seq = list(prompt) + list(toks[:-1])
    _, lp = ep.generate(seq, 0, want_logits=True)
    ep.close()
    cos = [cosine(lk[i], lp[i]) for i in range(len(seq))]
    assert min(cos) >= 0.9999, min(cos)


@pytest.mark.slow
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("wmode,kvmode", [("bf16", "floatx"), ("int8", "8bit"), ("fp8", "8bit")])
def test_long_context_matches_oracle(gpt2b, orc, cuda, wmode, kvmode, path):
    """Twelve heads over the full 1024-position context: every attention split
    (up to 96 positions per CTA on the persistent path) and the merge of all of
    them, teacher-forced against the oracle."""
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=1, NH=12, maxT=1024, V=500, Vp=512)
    imgs = _images(gpt2b, cfg, 77, "test")
    img, sc = imgs[wmode]
    eng = _engine(img, wmode, kvmode, sc, path)
    prompt = [11, 22, 33]
    toks, lg = eng.generate(prompt, cfg["maxT"] - len(prompt), want_logits=True)
    eng.close()
    m = orc.Model(img, wmode, kvmode, sc)
    seq = list(prompt) + list(toks[:-1])
    cos = [cosine(lg[pos], m.step(int(t), pos)) for pos, t in enumerate(seq)]
    assert min(cos) >= 0.999, (min(cos), int(np.argmin(cos)))


@pytest.mark.slow
@pytest.mark.parametrize("wmode,kvmode", [("int8", "floatx"), ("bf16", "floatx"), ("fp8", "8bit")])
def test_wide_model_persistent_matches_kernel_path(gpt2b, orc, cuda, wmode, kvmode):
    """C = 1280 (wider than a 4-KB BF16 row), 20 heads, 7 splits of up to 160
    positions: the persistent kernel against the per-kernel path over 600
    positions and against the oracle over the first 48."""
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=2, NH=20, maxT=1024, V=500, Vp=512)
    imgs = _images(gpt2b, cfg, 5, "test")
    img, sc = imgs[wmode]
    prompt = [1, 2, 3, 4]
    ek = _engine(img, wmode, kvmode, sc, "kernels")
    toks, lk = ek.generate(prompt, 600, want_logits=True)
    ek.close()
    seq = list(prompt) + list(toks[:-1])
    ep = _engine(img, wmode, kvmode, sc, "persistent")
    _, lp = ep.generate(seq, 0, want_logits=True)
    ep.close()
    cos = [cosine(lk[i], lp[i]) for i in range(len(seq))]
    assert min(cos) >= 0.999, (min(cos), int(np.argmin(cos)))
    m = orc.Model(img, wmode, kvmode, sc)
    cos_o = [cosine(lp[i], m.step(int(t), i)) for i, t in enumerate(seq[:48])]
    assert min(cos_o) >= 0.999, min(cos_o)


@pytest.mark.slow
@pytest.mark.parametrize("wmode", ["int8", "fp8"])
def test_wide_model_extreme_activations(gpt2b, orc, cuda, wmode):
    """The wide persistent kernel feeds 8-bit weights to tensor-core stages with
    x in FP16 after a power-of-two prescale.  Layer 0's LN1 output is pushed far
    above FP16's range (gamma x 3e5) and the final LN output far below its
    normal range (gamma, beta x 1e-6, so the logits are proportional to those
    tiny values): the logits must still follow the oracle and the per-kernel
    path (FP32 CUDA-core GEMVs)."""
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=2, NH=20, maxT=128, V=500, Vp=512)
    p = weights.synth_params(cfg, 9, init="test")
    p["ln1w"][0] *= np.float32(3e5)
    p["lnfw"] *= np.float32(1e-6)
    p["lnfb"] *= np.float32(1e-6)
    img, sc = _quantize(gpt2b, weights.image(p, cfg, "bf16"), wmode)
    prompt = [9, 8, 7]
    ek = _engine(img, wmode, "floatx", sc, "kernels")
    toks, lk = ek.generate(prompt, 40, want_logits=True)
    ek.close()
    seq = list(prompt) + list(toks[:-1])
    ep = _engine(img, wmode, "floatx", sc, "persistent")
    _, lp = ep.generate(seq, 0, want_logits=True)
    ep.close()
    assert np.isfinite(lp).all()
    assert float(np.abs(lp).max()) < 1e-3  # the logits really are tiny
    cos = [cosine(lk[i], lp[i]) for i in range(len(seq))]
    assert min(cos) >= 0.999, (min(cos), int(np.argmin(cos)))
    m = orc.Model(img, wmode, "floatx", sc)
    cos_o = [cosine(lp[i], m.step(int(t), i)) for i, t in enumerate(seq)]
    assert min(cos_o) >= 0.999, min(cos_o)


@pytest.mark.parametrize("wmode,kvmode", [("int8", "8bit"), ("fp8", "floatx"), ("bf16", "floatx")])
def test_create_from_file_matches_buffer(mini, tmp_path, gpt2b, wmode, kvmode):
    """gpt2b_engine_create_from_file on files written like the reference's
    tools: the 8-bit image with its scales in "<model>_scales.bin" found
    implicitly (inference_gpt2_opt.cu:666-668), or an explicit scale path; the
    tokens and logits equal those of the engine built from the same bytes in
    memory."""
    from cuda_gpt2_inference_b200.engine import Engine
    cfg, imgs = mini
    img, sc = imgs[wmode]
    model = tmp_path / "gpt2_mini.bin"
    model.write_bytes(img)
    if sc is not None:
        (tmp_path / "gpt2_mini_scales.bin").write_bytes(sc.tobytes())
    prompt = [4, 44, 444]
    eb = _engine(img, wmode, kvmode, sc)
    want_t, want_l = eb.generate(prompt, 20, want_logits=True)
    eb.close()
    ef = Engine.from_file(str(model), wmode, kvmode)  # implicit scale file
    assert ef.config == dict(maxT=cfg["maxT"], V=cfg["V"], Vp=cfg["Vp"], L=cfg["L"], NH=cfg["NH"], C=cfg["C"])
    got_t, got_l = ef.generate(prompt, 20, want_logits=True)
    ef.close()
    assert np.array_equal(got_t, want_t) and np.array_equal(got_l, want_l)
    if sc is not None:
        other = tmp_path / "elsewhere.bin"
        other.write_bytes(sc.tobytes())
        (tmp_path / "gpt2_mini_scales.bin").unlink()
        with pytest.raises(gpt2b.Gpt2bError) as e:  # no implicit scale file any more
            Engine.from_file(str(model), wmode, kvmode)
        assert e.value.status == gpt2b.ERR_FILE
        ef = Engine.from_file(str(model), wmode, kvmode, scale_path=str(other))
        got_t, _ = ef.generate(prompt, 20)
        ef.close()
        assert np.array_equal(got_t, want_t)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("sample", [False, True])
def test_generate_dump_files(mini, tmp_path, path, sample):
    """Verification dumps (Inference_gpt2/dump_utils.h layout): step 1's
    logits, step t's logits and input prefix, and the per-step NLL of the
    appended token computed on the device, against the logits and tokens of
    gpt2b_engine_generate on the same engine and a host NLL."""
    from cuda_gpt2_inference_b200 import verify
    cfg, imgs = mini
    img, _ = imgs["bf16"]
    prompt = [50, 60, 70, 80]
    n_gen, steps, ppl_len = 30, [1, 4, 5, 17, 34], 25
    eng = _engine(img, "bf16", path=path)
    want_t, lg = eng.generate(prompt, n_gen, want_logits=True, sample=sample, seed=99)
    toks, nll = eng.generate_dump(prompt, n_gen, str(tmp_path), "opt_bf16", steps=steps, ppl_len=ppl_len,
                                  sample=sample, seed=99)
    eng.close()
    assert np.array_equal(toks, want_t)
    seq = np.array(list(prompt) + list(want_t), np.int32)  # the token at every position 0..n_prompt+n_gen
    V = cfg["V"]
    assert np.array_equal(verify.read_logits(str(tmp_path), "opt_bf16"), lg[0, :V])  # step 1
    for t in steps:
        assert np.array_equal(verify.read_logits(str(tmp_path), "opt_bf16", t), lg[t - 1, :V]), t
        assert np.array_equal(verify.read_inputs(str(tmp_path), "opt_bf16", t), seq[:t]), t
    fn, ft = verify.read_ppl(str(tmp_path), "opt_bf16")
    assert np.array_equal(fn, nll) and np.array_equal(ft, seq[1:ppl_len + 1])
    host = np.array([verify.nll(lg[t - 1, :V], int(seq[t])) for t in range(1, ppl_len + 1)], np.float32)
    assert np.allclose(nll, host, rtol=1e-5, atol=1e-5)
    assert verify.dumped_steps(str(tmp_path), "opt_bf16") == sorted(steps)


@pytest.mark.parametrize("wmode,kvmode", [("bf16", "floatx"), ("int8", "8bit"), ("fp8", "8bit"), ("int8", "floatx")])
@pytest.mark.parametrize("shape", ["mini", "long", "wide"])
def test_prefill_matches_per_step_prompt(gpt2b, orc, cuda, wmode, kvmode, shape):
    """The prompt on the tensor cores (one pass of tcgen05 GEMMs over every
    prompt position) against the same prompt fed one decode step per position:
    logits of every prompt position and of the decode steps that follow (which
    read the KV rows the prefill wrote), teacher-forced on the same tokens, and
    the first decode steps against the oracle.  "long": a 300-token prompt (three
    128-row token tiles); "wide": C = 1600, 25 heads (the GPT-2-XL width)."""
    from cuda_gpt2_inference_b200 import OPT_PREFILL, weights
    cfg = {"mini": weights.mini_config(L=2, NH=2, maxT=64, V=500, Vp=512),
           "long": weights.mini_config(L=1, NH=12, maxT=1024, V=500, Vp=512),
           "wide": weights.mini_config(L=2, NH=25, maxT=128, V=500, Vp=512)}[shape]
    n_prompt, n_gen = {"mini": (24, 30), "long": (300, 40), "wide": (24, 40)}[shape]
    imgs = _images(gpt2b, cfg, 41, "test")
    img, sc = imgs[wmode]
    prompt = np.random.default_rng(8).integers(0, cfg["V"], n_prompt).astype(np.int32)
    ep = _engine(img, wmode, kvmode, sc)
    ep.set_option(OPT_PREFILL, 1)
    toks, lp = ep.generate(prompt, n_gen, want_logits=True)
    hist = ep.history(0, n_prompt)
    ep.close()
    assert np.array_equal(hist, prompt)  # the prompt is in the device history
    seq = list(prompt) + list(toks[:-1])
    es = _engine(img, wmode, kvmode, sc)
    es.set_option(OPT_PREFILL, 0)
    _, ls = es.generate(seq, 0, want_logits=True)
    es.close()
    cos = [cosine(lp[i], ls[i]) for i in range(len(seq))]
    assert min(cos) >= 0.999, (min(cos), int(np.argmin(cos)))
    # the pick after the prompt is the greedy pick of the last prompt row
    assert int(toks[0]) == int(np.argmax(lp[n_prompt - 1][: cfg["V"]]))
    m = orc.Model(img, wmode, kvmode, sc)
    cos_o = [cosine(lp[i], m.step(int(t), i)) for i, t in enumerate(seq[: n_prompt + 4])]
    assert min(cos_o) >= 0.999, (min(cos_o), int(np.argmin(cos_o)))


def test_engine_rejects_bad_inputs(mini, gpt2b):
    cfg, imgs = mini
    eng = _engine(imgs["bf16"][0], "bf16")
    with pytest.raises(gpt2b.Gpt2bError):
        eng.forward(cfg["V"], 0)  # token out of range
    with pytest.raises(gpt2b.Gpt2bError):
        eng.forward(1, cfg["maxT"])  # position out of range
    with pytest.raises(gpt2b.Gpt2bError):
        eng.generate([1, 2], cfg["maxT"])  # prompt + generation longer than the context
    eng.forward(1, 0)
    assert gpt2b.device_error() == 0
    eng.close()


# ------------------------------------------------------------- 124M -------
@pytest.fixture(scope="module")
def m124(gpt2b, cuda):
    from cuda_gpt2_inference_b200 import weights
    return weights.GPT2_124M, _images(gpt2b, weights.GPT2_124M, 1234, "spec")


@pytest.mark.slow
@pytest.mark.parametrize("path", PATHS)
def test_124m_fp32_greedy_128_steps(m124, orc, path):
    cfg, imgs = m124
    img, _ = imgs["f32"]
    rng = np.random.default_rng(24)
    prompt = rng.integers(0, cfg["V"], 24).astype(np.int32)
    eng = _engine(img, "f32", path=path)
    toks, lg = eng.generate(prompt, 128, want_logits=True)
    eng.close()
    m = orc.Model(img, "f32")
    otoks, olg = m.generate(prompt, 128, want_logits=True)
    assert np.array_equal(toks, otoks), (toks[:20], otoks[:20])
    cos = [cosine(lg[i], olg[i]) for i in range(len(lg))]
    assert min(cos) >= 0.9999, min(cos)


def _ref_engine(orc, name, path):
    if not orc.ref_available(f"libref_engine_{name}.so"):
        pytest.skip("reference engine not built")
    lib = orc.ref_gpu(f"engine_{name}")
    lib.ref_engine_init.argtypes = [ctypes.c_char_p, ctypes.c_int]
    lib.ref_engine_step.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    assert lib.ref_engine_init(str(path).encode(), 0 if name in ("f32", "bf16") else 1) == 0
    return lib


@pytest.mark.slow
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("wmode,kvmode,refname", [("bf16", "floatx", "bf16"), ("int8", "8bit", "int8kv8"),
                                                  ("fp8", "8bit", "fp8kv8")])
def test_124m_against_reference_engine(m124, orc, tmp_path, wmode, kvmode, refname, path):
    cfg, imgs = m124
    img, sc = imgs[wmode]
    model_file = tmp_path / "model.bin"
    model_file.write_bytes(img)
    if sc is not None:
        (tmp_path / "model_scales.bin").write_bytes(sc.tobytes())
    ref = _ref_engine(orc, refname, model_file)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, cfg["V"], 24).astype(np.int32)
    n_gen = 176  # crosses the reference's 150-position switch to split+merge
    eng = _engine(img, wmode, kvmode, sc, path)
    toks, lg = eng.generate(prompt, n_gen, want_logits=True)
    eng.close()
    seq = list(prompt) + list(toks[:-1])
    row = np.zeros(cfg["Vp"], np.float32)
    cos = []
    for pos, t in enumerate(seq):
        assert ref.ref_engine_step(int(t), pos, row.ctypes.data_as(ctypes.c_void_p)) == 0
        cos.append(cosine(lg[pos], row))
    floor = 0.999 if wmode == "bf16" else 0.998
    assert min(cos) >= floor, (min(cos), int(np.argmin(cos)))
