"""ctypes binding of the CPU oracle and of the reference libraries built from
source (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this package; the product (cuda_gpt2_inference_b200) never does.

* :func:`orc` -- the C++ restatement (oracle.cpp), built on demand with g++.
* :func:`ref_cpu` -- the reference's own CPU loops compiled in place
  (oracle/_ref/libref_cpu_*.so) and the CPU decode composed from them.
* :func:`ref_gpu` -- the reference's CUDA kernels / engine compiled for sm_100a
  (oracle/_ref/libref_{ops,w8,quant,engine}_*.so); usable on the GPU box only.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
_cache: dict = {}

_P, _I, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

_ORC_SIGS = {
    "orc_bf16_round": (_F, [_F]),
    "orc_w8_decode": (_F, [ctypes.c_uint8, _I]),
    "orc_gemv": (None, [_P, _P, _P, _I, _I]),
    "orc_gemv_fused": (None, [_P, _P, _P, _P, _P, _I, _I, _I]),
    "orc_gemv_w8": (None, [_P, _P, _P, _I, _P, _P, _P, _I, _I, _I]),
    "orc_dequant_rows": (None, [_P, _P, _P, _I, _I, _I]),
    "orc_quant_rows": (None, [_P, _P, _P, _I, _I, _I]),
    "orc_kv_encode_row": (None, [_P, _I, _I, _P, _P]),
    "orc_attention_kv": (None, [_P, _P, _P, _I, _I, _I, _I, _I, _F]),
    "orc_attention_kv_w8": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F]),
    "orc_layernorm": (None, [_P, _P, _P, _P, _P, _P, _I, _I]),
    "orc_residual": (None, [_P, _P, _P, _I]),
    "orc_gelu": (None, [_P, _P, _I]),
    "orc_encoder_kv": (None, [_P, _P, _P, _P, _I, _I, _I]),
    "orc_argmax": (_I, [_P, _I]),
    "orc_model_from_buffer": (_P, [_P, _SZ, _I, _P, _SZ, _I, ctypes.POINTER(ctypes.c_char_p)]),
    "orc_model_free": (None, [_P]),
    "orc_model_config": (None, [_P, _P]),
    "orc_model_reset": (None, [_P]),
    "orc_model_step": (_I, [_P, _I, _I, _P]),
    "orc_model_generate": (_I, [_P, _P, _I, _I, _P, _P]),
    "orc_model_probe": (_I, [_P, ctypes.c_char_p, _I, _P]),
}


def ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def orc() -> ctypes.CDLL:
    """The oracle library, compiled on first use."""
    if "orc" not in _cache:
        from .build_oracle import build_oracle
        lib = ctypes.CDLL(build_oracle())
        for name, (res, args) in _ORC_SIGS.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        _cache["orc"] = lib
    return _cache["orc"]


def ref_available(name: str) -> bool:
    return os.path.exists(os.path.join(REF_DIR, name))


def _load_ref(name: str) -> ctypes.CDLL:
    if name not in _cache:
        path = os.path.join(REF_DIR, name)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (python oracle/build_oracle.py with the reference present)")
        _cache[name] = ctypes.CDLL(path)
    return _cache[name]


_REF_CPU_SIGS = {
    "gemv": {"ref_gemv_cpu_f32": (None, [_P, _P, _P, _I, _I]), "ref_gemv_cpu_bf16": (None, [_P, _P, _P, _I, _I])},
    "attention": {"ref_attention_kv_cpu": (None, [_P, _P, _P, _I, _I, _I, _I, _I, _F])},
    "fused": {"ref_residual_cpu": (None, [_P, _P, _P, _I]),
              "ref_layernorm_cpu": (None, [_P, _P, _P, _P, _P, _P, _I, _I, _I])},
    "gelu": {"ref_gelu_cpu": (None, [_P, _P, _I])},
    "encoder": {"ref_encoder_cpu": (None, [_P, _P, _P, _P, _I, _I, _I])},
    "decode": {"ref_decoder_create": (_P, [_P, _P]), "ref_decoder_step": (_I, [_P, _I, _I, _P]),
               "ref_decoder_free": (None, [_P]), "ref_set_threads": (_I, [_I])},
}


def ref_cpu(which: str) -> ctypes.CDLL:
    """which in {gemv, attention, fused, gelu, encoder, decode}."""
    lib = _load_ref(f"libref_cpu_{which}.so")
    if not getattr(lib, "_typed", False):
        for name, (res, args) in _REF_CPU_SIGS[which].items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        lib._typed = True
    return lib


def ref_gpu(name: str) -> ctypes.CDLL:
    """name: e.g. 'ops_bf16', 'w8_int8', 'quant', 'engine_bf16'."""
    return _load_ref(f"libref_{name}.so")


# ---------------------------------------------------------------------------
# convenience wrappers over the oracle (float32 numpy in/out)
# ---------------------------------------------------------------------------
FMT = {"int8": 0, "fp8": 1}
WMODE = {"f32": 0, "bf16": 1, "int8": 2, "fp8": 3}
KVMODE = {"floatx": 0, "8bit": 1}


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def gemv(W, x):
    W, x = f32(W), f32(x)
    M, K = W.shape
    out = np.zeros(M, np.float32)
    orc().orc_gemv(ptr(out), ptr(W), ptr(x), M, K)
    return out


def gemv_fused(W, x, bias, do_gelu):
    W, x = f32(W), f32(x)
    M, K = W.shape
    out, pre = np.zeros(M, np.float32), np.zeros(M, np.float32)
    b = f32(bias) if bias is not None else None
    orc().orc_gemv_fused(ptr(out), ptr(pre), ptr(W), ptr(x), ptr(b) if b is not None else None, M, K, int(do_gelu))
    return out, pre


def gemv_w8(codes, fmt, x, scale, bias, do_gelu):
    codes = np.ascontiguousarray(codes, np.uint8)
    M, K = codes.shape
    x, scale = f32(x), f32(scale)
    out, pre = np.zeros(M, np.float32), np.zeros(M, np.float32)
    b = f32(bias) if bias is not None else None
    orc().orc_gemv_w8(ptr(out), ptr(pre), ptr(codes), FMT[fmt], ptr(x), ptr(scale),
                      ptr(b) if b is not None else None, M, K, int(do_gelu))
    return out, pre


def quant_rows(W, fmt):
    W = f32(W)
    M, K = W.shape
    q, s = np.zeros((M, K), np.uint8), np.zeros(M, np.float32)
    orc().orc_quant_rows(ptr(W), ptr(q), ptr(s), M, K, FMT[fmt])
    return q, s


def dequant_rows(codes, scale, fmt):
    codes = np.ascontiguousarray(codes, np.uint8)
    rows, cols = codes.shape
    out = np.zeros((rows, cols), np.float32)
    orc().orc_dequant_rows(ptr(out), ptr(codes), ptr(f32(scale)), rows, cols, FMT[fmt])
    return out


def decode_w8(codes, fmt):
    lut = np.array([orc().orc_w8_decode(i, FMT[fmt]) for i in range(256)], np.float32)
    return lut[np.asarray(codes, np.uint8)]


def kv_encode_row(x, fmt):
    x = f32(x)
    codes, sc = np.zeros(x.size, np.uint8), np.zeros(1, np.float32)
    orc().orc_kv_encode_row(ptr(x), x.size, FMT[fmt], ptr(codes), ptr(sc))
    return codes, float(sc[0])


def attention_kv(qkv, kv_cache, B, seq_len, NH, hs, maxT, scale=None):
    qkv, kv_cache = f32(qkv), f32(kv_cache)
    out = np.zeros(B * NH * hs, np.float32)
    orc().orc_attention_kv(ptr(out), ptr(qkv), ptr(kv_cache), B, seq_len, NH, hs, maxT,
                           scale if scale is not None else 1.0 / np.sqrt(hs))
    return out


def attention_kv_w8(qkv, kv_codes, kv_scale, fmt, B, seq_len, NH, hs, maxT, scale=None):
    qkv = f32(qkv)
    kv_codes = np.ascontiguousarray(kv_codes, np.uint8)
    kv_scale = f32(kv_scale)
    out = np.zeros(B * NH * hs, np.float32)
    orc().orc_attention_kv_w8(ptr(out), ptr(qkv), ptr(kv_codes), ptr(kv_scale), FMT[fmt], B, seq_len, NH, hs, maxT,
                              scale if scale is not None else 1.0 / np.sqrt(hs))
    return out


def layernorm(x, w, b):
    x = f32(x)
    N, C = x.reshape(-1, x.shape[-1]).shape
    out, mean, rstd = np.zeros_like(x), np.zeros(N, np.float32), np.zeros(N, np.float32)
    orc().orc_layernorm(ptr(out), ptr(mean), ptr(rstd), ptr(x), ptr(f32(w)), ptr(f32(b)), N, C)
    return out, mean, rstd


def bf16_round(a):
    """Round float32 values through bf16 (nearest even), vectorised."""
    from cuda_gpt2_inference_b200.weights import bf16_bits, bf16_to_f32
    return bf16_to_f32(bf16_bits(f32(a)))


class Model:
    """The whole-model CPU restatement over a flat-bin image."""

    def __init__(self, image: bytes, wmode: str, kvmode: str = "floatx", scales=None):
        self._img = ctypes.create_string_buffer(image, len(image))
        sc = f32(scales) if scales is not None else None
        self._sc = sc
        err = ctypes.c_char_p()
        h = orc().orc_model_from_buffer(self._img, len(image), WMODE[wmode], ptr(sc) if sc is not None else None,
                                        sc.size if sc is not None else 0, KVMODE[kvmode], ctypes.byref(err))
        if not h:
            raise ValueError(f"oracle rejected the image: {err.value.decode() if err.value else '?'}")
        self._h = h
        cfg = np.zeros(6, np.int32)
        orc().orc_model_config(h, ptr(cfg))
        self.config = dict(maxT=int(cfg[0]), V=int(cfg[1]), L=int(cfg[2]), NH=int(cfg[3]), C=int(cfg[4]),
                           Vp=int(cfg[5]))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            orc().orc_model_free(h)
            self._h = None

    def reset(self):
        orc().orc_model_reset(self._h)

    def step(self, token: int, pos: int):
        lg = np.zeros(self.config["Vp"], np.float32)
        rc = orc().orc_model_step(self._h, int(token), int(pos), ptr(lg))
        if rc:
            raise ValueError("oracle step rejected the token/position")
        return lg

    def generate(self, prompt, n_gen: int, want_logits: bool = False):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen + 1, np.int32)
        lg = np.zeros((len(prompt) + n_gen, self.config["Vp"]), np.float32) if want_logits else None
        rc = orc().orc_model_generate(self._h, ptr(prompt), len(prompt), n_gen, ptr(out),
                                      ptr(lg) if lg is not None else None)
        if rc:
            raise ValueError("oracle generate failed")
        return out, lg

    def probe(self, name: str, layer: int = 0):
        C = self.config["C"]
        buf = np.zeros(4 * C, np.float32)
        n = orc().orc_model_probe(self._h, name.encode(), layer, ptr(buf))
        if n < 0:
            raise KeyError(name)
        return buf[:n].copy()
