"""The reference flat-bin weight format, and a seeded synthetic writer.

Layout (Inference_gpt2/gpt2_model.h:63-87, 268-303): a 256-int32 header
``[20251103, version, maxT, V, L, NH, C, Vp, 0...]`` followed by the 16
parameter tensors in the order wte, wpe, ln1w, ln1b, qkvw, qkvb, attprojw,
attprojb, ln2w, ln2b, fcw, fcb, fcprojw, fcprojb, lnfw, lnfb; version 3 stores
FP32, version 5 BF16.  Linear weights are [out, in] row-major and wte is padded
to Vp rows with zeros (export_weights.py:57-68).  The 8-bit mixed image
(quantize.cu:190-229) keeps the header and stores wte, qkvw, attprojw, fcw,
fcprojw as 1-byte codes, with one float32 scale per row in a separate file.

The synthetic initialisation is the one the benchmark configurations name:
Linear and embedding weights N(0, 0.02), positional embeddings N(0, 0.01),
LayerNorm gamma 1 / beta 0, biases 0; drawn with numpy's PCG64 generator
(``numpy.random.default_rng(seed)``) in tensor order.  ``init="test"`` also
draws non-trivial LayerNorm parameters and biases so every code path is
exercised by the parity tests.
"""
from __future__ import annotations

import numpy as np

MAGIC = 20251103
NAMES = ["wte", "wpe", "ln1w", "ln1b", "qkvw", "qkvb", "attprojw", "attprojb",
         "ln2w", "ln2b", "fcw", "fcb", "fcprojw", "fcprojb", "lnfw", "lnfb"]
LINEAR = ("wte", "qkvw", "attprojw", "fcw", "fcprojw")  # quantised groups, in scale-file order

GPT2_124M = dict(maxT=1024, V=50257, L=12, NH=12, C=768, Vp=50304)
GPT2_XL = dict(maxT=1024, V=50257, L=48, NH=25, C=1600, Vp=50304)


def shapes(cfg: dict) -> dict:
    C, L, Vp, maxT = cfg["C"], cfg["L"], cfg["Vp"], cfg["maxT"]
    return {
        "wte": (Vp, C), "wpe": (maxT, C), "ln1w": (L, C), "ln1b": (L, C),
        "qkvw": (L, 3 * C, C), "qkvb": (L, 3 * C), "attprojw": (L, C, C), "attprojb": (L, C),
        "ln2w": (L, C), "ln2b": (L, C), "fcw": (L, 4 * C, C), "fcb": (L, 4 * C),
        "fcprojw": (L, C, 4 * C), "fcprojb": (L, C), "lnfw": (C,), "lnfb": (C,),
    }


def param_stream(cfg: dict, seed: int = 1234, init: str = "spec"):
    """Yield (name, float32 tensor) in file order, drawn one tensor at a time
    (peak host memory: one tensor), for GPT-2-XL-sized models."""
    rng = np.random.default_rng(seed)
    for name, shp in shapes(cfg).items():
        if name in LINEAR:
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif name == "wpe":
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.01)
        elif name.endswith("w"):  # LayerNorm gammas
            a = np.ones(shp, np.float32)
            if init == "test":
                a += rng.standard_normal(shp, dtype=np.float32) * np.float32(0.1)
        else:  # LayerNorm betas and Linear biases
            a = np.zeros(shp, np.float32)
            if init == "test":
                a += rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        if name == "wte":
            a[cfg["V"]:] = 0.0  # padded vocabulary rows are zero
        yield name, a


def synth_params(cfg: dict, seed: int = 1234, init: str = "spec") -> dict:
    """Seeded float32 parameters of the given architecture."""
    return dict(param_stream(cfg, seed, init))


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def header(cfg: dict, version: int) -> np.ndarray:
    h = np.zeros(256, np.int32)
    h[:8] = [MAGIC, version, cfg["maxT"], cfg["V"], cfg["L"], cfg["NH"], cfg["C"], cfg["Vp"]]
    return h


def image(params: dict, cfg: dict, dtype: str) -> bytes:
    """Serialise parameters as a v3 (``dtype="f32"``) or v5 (``"bf16"``) image."""
    if dtype not in ("f32", "bf16"):
        raise ValueError(dtype)
    parts = [header(cfg, 3 if dtype == "f32" else 5).tobytes()]
    for name in NAMES:
        a = params[name]
        parts.append(np.ascontiguousarray(a, np.float32).tobytes() if dtype == "f32" else bf16_bits(a).tobytes())
    return b"".join(parts)


def image_stream(cfg: dict, seed: int = 1234, init: str = "spec", dtype: str = "bf16") -> bytes:
    """The bytes of ``image(synth_params(cfg, seed, init), cfg, dtype)`` built one
    tensor at a time (peak host memory: the image plus one tensor), for
    GPT-2-XL-sized models."""
    if dtype not in ("f32", "bf16"):
        raise ValueError(dtype)
    eb = 4 if dtype == "f32" else 2
    shp = shapes(cfg)
    total = 1024 + sum(int(np.prod(v)) * eb for v in shp.values())
    out = np.empty(total, np.uint8)
    out[:1024] = np.frombuffer(header(cfg, 3 if dtype == "f32" else 5).tobytes(), np.uint8)
    off = 1024
    for name, a in param_stream(cfg, seed, init):
        b = (np.ascontiguousarray(a) if dtype == "f32" else bf16_bits(a)).view(np.uint8).ravel()
        out[off:off + b.size] = b
        off += b.size
        del a, b
    return out.tobytes()


def read_header(buf: bytes) -> tuple[int, dict]:
    h = np.frombuffer(buf[:1024], dtype=np.int32)
    if h[0] != MAGIC:
        raise ValueError("bad magic")
    cfg = dict(maxT=int(h[2]), V=int(h[3]), L=int(h[4]), NH=int(h[5]), C=int(h[6]), Vp=int(h[7]))
    return int(h[1]), cfg


def decode_image(buf: bytes, dtype: str) -> tuple[dict, dict]:
    """Parse a v3/v5 image back into float32 parameters (exact)."""
    version, cfg = read_header(buf)
    off = 1024
    out = {}
    for name, shp in shapes(cfg).items():
        n = int(np.prod(shp))
        if dtype == "f32":
            a = np.frombuffer(buf, np.float32, n, off).reshape(shp)
            off += 4 * n
        else:
            a = bf16_to_f32(np.frombuffer(buf, np.uint16, n, off)).reshape(shp)
            off += 2 * n
        out[name] = a
    return out, cfg


def image_w8(bf16_image: bytes, codes: dict, cfg: dict) -> bytes:
    """Assemble an 8-bit mixed image from a v5 image and per-group codes."""
    _, cfg2 = read_header(bf16_image)
    parts = [bf16_image[:1024]]
    off = 1024
    for name, shp in shapes(cfg2).items():
        n = int(np.prod(shp))
        if name in LINEAR:
            parts.append(np.ascontiguousarray(codes[name], np.uint8).tobytes())
        else:
            parts.append(bf16_image[off:off + 2 * n])
        off += 2 * n
    return b"".join(parts)


def mini_config(L: int = 2, NH: int = 2, maxT: int = 64, V: int = 1000, Vp: int = 1024) -> dict:
    """A small architecture with the 124M's head size, for fast parity tests."""
    return dict(maxT=maxT, V=V, L=L, NH=NH, C=64 * NH, Vp=Vp)
