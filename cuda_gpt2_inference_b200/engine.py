"""Python handle on the C++ decode engine (``gpt2b_engine_*`` in the C ABI).

Mirrors the reference program's flow (inference_gpt2_opt.cu main, :599-769):
build the model from a flat-bin image (``gpt2_build_from_checkpoint`` /
``gpt2_build_w8``), then generate -- with the reference's per-token host round
trip replaced by device-resident decoding.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import KV_8BIT, KV_FLOATX, W_BF16, W_F32, W_FP8, W_INT8, check, lib

WMODES = {"f32": W_F32, "bf16": W_BF16, "int8": W_INT8, "fp8": W_FP8}
KVMODES = {"floatx": KV_FLOATX, "8bit": KV_8BIT}


class _Config(ctypes.Structure):
    _fields_ = [("max_seq_len", ctypes.c_int), ("vocab_size", ctypes.c_int), ("padded_vocab_size", ctypes.c_int),
                ("num_layers", ctypes.c_int), ("num_heads", ctypes.c_int), ("channels", ctypes.c_int)]


class _DumpConfig(ctypes.Structure):
    _fields_ = [("dir", ctypes.c_char_p), ("prefix", ctypes.c_char_p), ("steps", ctypes.c_void_p),
                ("n_steps", ctypes.c_int), ("ppl_len", ctypes.c_int), ("logits_t1", ctypes.c_int)]


class Engine:
    """One decode engine on the current CUDA device."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        c = _Config()
        check(lib().gpt2b_engine_config(self._h, ctypes.byref(c)), "gpt2b_engine_config")
        self.config = dict(maxT=c.max_seq_len, V=c.vocab_size, Vp=c.padded_vocab_size, L=c.num_layers,
                           NH=c.num_heads, C=c.channels)

    # -- construction ------------------------------------------------------
    @classmethod
    def from_buffer(cls, image: bytes, wmode: str = "bf16", kvmode: str = "floatx",
                    scales: np.ndarray | None = None) -> "Engine":
        h = ctypes.c_void_p()
        img = ctypes.create_string_buffer(image, len(image))
        sc_ptr, nsc = None, 0
        if scales is not None:
            scales = np.ascontiguousarray(scales, dtype=np.float32)
            sc_ptr, nsc = scales.ctypes.data_as(ctypes.c_void_p), scales.size
        check(lib().gpt2b_engine_create_from_buffer(img, len(image), sc_ptr, nsc, WMODES[wmode], KVMODES[kvmode],
                                                    ctypes.byref(h)), "gpt2b_engine_create_from_buffer")
        return cls(h)

    @classmethod
    def from_buffer_tp(cls, image: bytes, wmode: str, kvmode: str, scales: np.ndarray | None, tp_rank: int,
                       tp_size: int, nccl_id: bytes) -> "Engine":
        """This rank's engine of a tensor-parallel group (collective: every rank
        calls it with the same image and 128-byte id, on its own device)."""
        h = ctypes.c_void_p()
        img = np.frombuffer(image, dtype=np.uint8)  # no copy: the library slices this rank's shard
        sc_ptr, nsc = None, 0
        if scales is not None:
            scales = np.ascontiguousarray(scales, dtype=np.float32)
            sc_ptr, nsc = scales.ctypes.data_as(ctypes.c_void_p), scales.size
        uid = ctypes.create_string_buffer(bytes(nccl_id), 128)
        check(lib().gpt2b_engine_create_tp_from_buffer(img.ctypes.data_as(ctypes.c_void_p), img.size, sc_ptr, nsc,
                                                       WMODES[wmode], KVMODES[kvmode], int(tp_rank), int(tp_size),
                                                       uid, ctypes.byref(h)), "gpt2b_engine_create_tp_from_buffer")
        return cls(h)

    @classmethod
    def from_file(cls, path: str, wmode: str = "bf16", kvmode: str = "floatx", scale_path: str | None = None):
        h = ctypes.c_void_p()
        check(lib().gpt2b_engine_create_from_file(path.encode(), scale_path.encode() if scale_path else None,
                                                  WMODES[wmode], KVMODES[kvmode], ctypes.byref(h)),
              "gpt2b_engine_create_from_file")
        return cls(h)

    def close(self) -> None:
        if self._h:
            check(lib().gpt2b_engine_destroy(self._h), "gpt2b_engine_destroy")
            self._h = None

    def __del__(self):  # best effort
        try:
            self.close()
        except Exception:
            pass

    # -- options / buffers ---------------------------------------------------
    def set_option(self, option: int, value: int) -> None:
        check(lib().gpt2b_engine_set_option(self._h, option, value), "gpt2b_engine_set_option")

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().gpt2b_engine_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def device_buffers(self) -> dict:
        lg, tk, ps, hi = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        check(lib().gpt2b_engine_device_buffers(self._h, ctypes.byref(lg), ctypes.byref(tk), ctypes.byref(ps),
                                                ctypes.byref(hi)))
        return dict(logits=lg.value, token=tk.value, pos=ps.value, history=hi.value)

    def kernels_per_step(self) -> int:
        n = ctypes.c_int()
        check(lib().gpt2b_engine_kernels_per_step(self._h, ctypes.byref(n)))
        return n.value

    # -- running -------------------------------------------------------------
    def forward(self, token: int, pos: int) -> None:
        check(lib().gpt2b_engine_forward(self._h, int(token), int(pos)), "gpt2b_engine_forward")

    def generate(self, prompt, n_gen: int, want_logits: bool = False, sample: bool = False,
                 seed: int = 1337):
        """Greedy (or sampled) generation through the C ABI with host buffers.
        Returns (tokens[n_gen+1], logits[(n_prompt+n_gen), Vp] or None)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen + 1, np.int32)
        logits = np.zeros((len(prompt) + n_gen, self.config["Vp"]), np.float32) if want_logits else None
        check(lib().gpt2b_engine_generate(self._h, prompt.ctypes.data_as(ctypes.c_void_p), len(prompt), n_gen,
                                          out.ctypes.data_as(ctypes.c_void_p),
                                          logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None,
                                          1 if sample else 0, seed), "gpt2b_engine_generate")
        return out, logits

    def generate_dump(self, prompt, n_gen: int, dump_dir: str | None, prefix: str = "gpt2b", steps=(),
                      ppl_len: int = 0, logits_t1: bool = True, sample: bool = False, seed: int = 1337):
        """``generate`` with the reference's verification dumps
        (Inference_gpt2/dump_utils.h file layout, written under ``dump_dir``):
        step t's logits and input prefix for t in ``steps``, step 1's logits,
        and the NLL of each appended token for steps 1..``ppl_len``
        (computed on the device).  Returns (tokens[n_gen+1], nll[ppl_len])."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen + 1, np.int32)
        nll = np.zeros(max(ppl_len, 1), np.float32)
        st = np.ascontiguousarray(list(steps), dtype=np.int32)
        cfg = _DumpConfig(dump_dir.encode() if dump_dir else None, prefix.encode(),
                          st.ctypes.data if st.size else None, int(st.size), int(ppl_len), int(bool(logits_t1)))
        check(lib().gpt2b_engine_generate_dump(self._h, prompt.ctypes.data_as(ctypes.c_void_p), len(prompt), n_gen,
                                               out.ctypes.data_as(ctypes.c_void_p), 1 if sample else 0, seed,
                                               ctypes.byref(cfg), nll.ctypes.data_as(ctypes.c_void_p)),
              "gpt2b_engine_generate_dump")
        return out, nll[:ppl_len]

    def set_position(self, token: int, pos: int) -> None:
        check(lib().gpt2b_engine_set_position(self._h, int(token), int(pos)), "gpt2b_engine_set_position")

    def history(self, first: int, count: int) -> np.ndarray:
        """Tokens at positions first..first+count-1 of the device history."""
        out = np.zeros(count, np.int32)
        check(lib().gpt2b_engine_history(self._h, out.ctypes.data_as(ctypes.c_void_p), first, count),
              "gpt2b_engine_history")
        return out

    def decode(self, n_steps: int) -> None:
        """Asynchronous device-resident greedy decode on the engine stream."""
        check(lib().gpt2b_engine_decode(self._h, int(n_steps)), "gpt2b_engine_decode")
