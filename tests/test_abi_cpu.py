"""Host-side checks that need no GPU: the C-ABI library loads and exports
every declared entry point, argument validation and weight-format parsing
return the documented status codes, and the flat-bin writer round-trips."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest


def test_library_exports_every_declared_symbol(gpt2b):
    names = gpt2b.declared_functions()
    assert len(names) >= 50
    lib = gpt2b.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(gpt2b._SIGS), "ctypes table and header disagree"
    assert lib.gpt2b_version() >= 100


def test_status_strings(gpt2b):
    for code in (gpt2b.OK, gpt2b.ERR_INVALID_ARG, gpt2b.ERR_ALIGNMENT, gpt2b.ERR_UNSUPPORTED, gpt2b.ERR_FILE,
                 gpt2b.ERR_FORMAT, gpt2b.ERR_DEVICE, gpt2b.ERR_NCCL):
        assert gpt2b.status_string(code) not in ("", "unknown status")


def test_op_argument_validation_before_any_launch(gpt2b):
    lib = gpt2b.lib()
    buf = ctypes.create_string_buffer(4096 + 16)
    base = ctypes.addressof(buf)
    aligned = (base + 15) & ~15
    # negative sizes, null pointers, unaligned rows and pointers are rejected on the host
    assert lib.gpt2b_launch_GEMV6_f32(aligned, aligned, aligned, -1, 16, None) == gpt2b.ERR_INVALID_ARG
    assert lib.gpt2b_launch_GEMV6_f32(None, aligned, aligned, 4, 16, None) == gpt2b.ERR_INVALID_ARG
    assert lib.gpt2b_launch_GEMV6_bf16(aligned, aligned, aligned, 4, 12, None) == gpt2b.ERR_ALIGNMENT
    assert lib.gpt2b_launch_GEMV6_f32(aligned, aligned + 4, aligned, 4, 16, None) == gpt2b.ERR_ALIGNMENT
    assert lib.gpt2b_launch_GEMV6_w8x2_i8(aligned, None, aligned, aligned, None, None, 4, 32, 0, None) \
        == gpt2b.ERR_INVALID_ARG
    # an empty matrix is a successful no-op
    assert lib.gpt2b_launch_GEMV6_f32(aligned, aligned, aligned, 0, 16, None) == gpt2b.OK
    # attention is built for head size 64 (the reference fixes it too)
    assert lib.gpt2b_attention_forward_kv_small_bf16(aligned, aligned, aligned, 1, 12, 32, 1024, aligned,
                                                     None) == gpt2b.ERR_UNSUPPORTED
    assert lib.gpt2b_layernorm_forward_f32(aligned, None, None, aligned, aligned, aligned, 1, 1, 4096,
                                           None) == gpt2b.ERR_UNSUPPORTED
    assert lib.gpt2b_gpu_argmax(aligned, aligned, 1, 10, 5, None) == gpt2b.ERR_INVALID_ARG


def _tiny_image(dtype="bf16"):
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=1, NH=1, maxT=16, V=40, Vp=48)
    return weights.image(weights.synth_params(cfg, 1), cfg, dtype), cfg


def test_engine_rejects_malformed_images(gpt2b):
    lib = gpt2b.lib()
    img, _ = _tiny_image("bf16")
    h = ctypes.c_void_p()

    def create(buf, wmode=gpt2b.W_BF16, kv=gpt2b.KV_FLOATX, scales=None, n=0):
        b = ctypes.create_string_buffer(buf, len(buf))
        return lib.gpt2b_engine_create_from_buffer(b, len(buf), scales, n, wmode, kv, ctypes.byref(h))

    bad_magic = bytearray(img); bad_magic[0] ^= 1
    assert create(bytes(bad_magic)) == gpt2b.ERR_FORMAT
    assert create(img, wmode=gpt2b.W_F32) == gpt2b.ERR_FORMAT  # v5 image, FP32 requested
    assert create(img[:-2]) == gpt2b.ERR_FORMAT  # truncated
    assert create(img + b"\0\0") == gpt2b.ERR_FORMAT  # trailing bytes
    assert create(img[:512]) == gpt2b.ERR_FORMAT  # shorter than the header
    bad_dims = bytearray(img); bad_dims[2 * 4:3 * 4] = np.int32(32).tobytes()  # maxT 16 -> 32
    assert create(bytes(bad_dims)) == gpt2b.ERR_FORMAT  # tensor sizes no longer match the byte count
    odd_head = bytearray(img); odd_head[6 * 4:7 * 4] = np.int32(100).tobytes()  # head size 100
    assert create(bytes(odd_head)) == gpt2b.ERR_UNSUPPORTED
    assert create(img, kv=gpt2b.KV_8BIT) == gpt2b.ERR_UNSUPPORTED  # 8-bit KV needs 8-bit weights
    assert create(img, wmode=gpt2b.W_INT8) == gpt2b.ERR_FORMAT  # wrong byte count for a mixed image
    assert lib.gpt2b_engine_create_from_file(b"/nonexistent/model.bin", None, gpt2b.W_BF16, 0,
                                             ctypes.byref(h)) == gpt2b.ERR_FILE


def test_read_header(gpt2b, tmp_path):
    from cuda_gpt2_inference_b200.engine import _Config
    img, cfg = _tiny_image("f32")
    p = tmp_path / "m.bin"
    p.write_bytes(img)
    ver, c = ctypes.c_int(), _Config()
    assert gpt2b.lib().gpt2b_read_header(str(p).encode(), ctypes.byref(ver), ctypes.byref(c)) == gpt2b.OK
    assert ver.value == 3 and c.channels == cfg["C"] and c.padded_vocab_size == cfg["Vp"]
    p.write_bytes(b"\0" * 100)
    assert gpt2b.lib().gpt2b_read_header(str(p).encode(), ctypes.byref(ver), ctypes.byref(c)) == gpt2b.ERR_FORMAT
    assert gpt2b.lib().gpt2b_read_header(str(tmp_path / "missing").encode(), None, ctypes.byref(c)) \
        == gpt2b.ERR_FILE


def test_quantizer_size_query_and_rejects_fp32(gpt2b):
    lib = gpt2b.lib()
    img, cfg = _tiny_image("bf16")
    ob, ns = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.gpt2b_quantized_size(img, len(img), ctypes.byref(ob), ctypes.byref(ns)) == gpt2b.OK
    C, L, Vp = cfg["C"], cfg["L"], cfg["Vp"]
    assert ns.value == Vp + L * 3 * C + L * C + L * 4 * C + L * C
    n_lin = Vp * C + L * 12 * C * C
    assert ob.value == len(img) - n_lin
    f32, _ = _tiny_image("f32")
    assert lib.gpt2b_quantized_size(f32, len(f32), ctypes.byref(ob), ctypes.byref(ns)) == gpt2b.ERR_FORMAT


def test_weight_image_round_trip():
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=2, NH=2, maxT=32, V=100, Vp=128)
    p = weights.synth_params(cfg, 5, init="test")
    assert not p["wte"][cfg["V"]:].any()
    for dt in ("f32", "bf16"):
        img = weights.image(p, cfg, dt)
        back, cfg2 = weights.decode_image(img, dt)
        assert cfg2 == cfg
        for n in weights.NAMES:
            ref = p[n] if dt == "f32" else weights.bf16_to_f32(weights.bf16_bits(p[n]))
            assert np.array_equal(back[n], ref), n


def test_bf16_rounding_matches_cuda_host_conversion(orc):
    from cuda_gpt2_inference_b200 import weights
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3, 1e-30, 65504.0, 3.4e38], np.float32)
    mine = weights.bf16_to_f32(weights.bf16_bits(x))
    cuda = np.array([orc.orc().orc_bf16_round(float(v)) for v in x], np.float32)
    assert np.array_equal(mine, cuda)


def test_oracle_model_accepts_8bit_images(orc):
    from cuda_gpt2_inference_b200 import weights
    cfg = weights.mini_config(L=1, NH=2, maxT=16, V=60, Vp=64)
    p = weights.synth_params(cfg, 9)
    img = weights.image(p, cfg, "bf16")
    params16, _ = weights.decode_image(img, "bf16")
    codes, scales = {}, []
    for g in weights.LINEAR:
        W = params16[g].reshape(-1, params16[g].shape[-1])
        q, s = orc.quant_rows(W, "int8")
        codes[g] = q
        scales.append(s)
    img8 = weights.image_w8(img, codes, cfg)
    m = orc.Model(img8, "int8", "8bit", np.concatenate(scales))
    toks, _ = m.generate([1, 2, 3], 4)
    assert toks.shape == (5,) and (toks >= 0).all() and (toks < cfg["V"]).all()
    with pytest.raises(ValueError):
        orc.Model(img8, "int8", "8bit", np.concatenate(scales)[:-1])
