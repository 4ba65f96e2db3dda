"""B200-native GPT-2 batch-1 decode engine (host side).

The compute lives in ``libgpt2b.so`` (hand-written sm_100a CUDA kernels behind
the C ABI declared in ``include/gpt2_b200.h``).  This package only binds that
ABI with ctypes and mirrors the reference operator surface for Python callers:

* :mod:`.ops`     -- one function per reference launcher (``launch_GEMV6``,
                     ``attention_forward_kv_small``, ...), on torch CUDA tensors;
* :mod:`.engine`  -- the whole-model decode engine;
* :mod:`.weights` -- the reference flat-bin weight format (synthetic writer).

There is no CPU fallback: every op raises if the library is missing.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
# GPT2B_LIB selects another build of the library (the trace build of the build script)
LIB_PATH = os.environ.get("GPT2B_LIB") or os.path.join(_HERE, "libgpt2b.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "gpt2_b200.h")

# status codes (include/gpt2_b200.h)
OK = 0
ERR_INVALID_ARG = 1001
ERR_ALIGNMENT = 1002
ERR_UNSUPPORTED = 1003
ERR_FILE = 1004
ERR_FORMAT = 1005
ERR_DEVICE = 1006
ERR_NCCL = 1007
ERR_CUDA = 2000
# weight / KV modes
W_F32, W_BF16, W_INT8, W_FP8 = 0, 1, 2, 3
KV_FLOATX, KV_8BIT = 0, 1
OPT_USE_GRAPH, OPT_USE_PDL, OPT_SPLITS, OPT_STEPS_PER_GRAPH, OPT_PERSISTENT, OPT_POLL_LIMIT, OPT_PREFILL = \
    1, 2, 3, 4, 5, 6, 7
# device error codes (gpt2b_device_error)
DEVERR_GRID_TIMEOUT = 5

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_U64 = ctypes.c_ulonglong
_SZ = ctypes.c_size_t
_S = ctypes.c_char_p

# argument signatures of every exported function (pointers as void*)
_SIGS = {
    "gpt2b_status_string": (_S, [_I]),
    "gpt2b_device_error": (_I, [_P]),
    "gpt2b_version": (_I, []),
    "gpt2b_launch_GEMV6_f32": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_launch_GEMV6_bf16": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_launch_GEMV6_fused_f32": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_launch_GEMV6_fused_bf16": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_launch_GEMV6_w8x2_i8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_launch_GEMV6_w8x2_fp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_launch_GEMV6_w8x2_i8_f32out": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_launch_GEMV6_w8x2_fp8_f32out": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_dequant_wte_i8": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_dequant_wte_fp8": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_quant_rows_i8": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_quant_rows_fp8": (_I, [_P, _P, _P, _I, _I, _P]),
    "gpt2b_quantize_file": (_I, [_S, _S, _S, _I]),
    "gpt2b_quantized_size": (_I, [_P, _SZ, _P, _P]),
    "gpt2b_quantize_buffer": (_I, [_P, _SZ, _P, _P, _I]),
    "gpt2b_kv_cache_write_f32": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_kv_cache_write_bf16": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_kv_cache_write_w8_i8": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_kv_cache_write_w8_fp8": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_forward_kv_small_f32": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_forward_kv_small_bf16": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_forward_kv_small_w8_i8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_forward_kv_small_w8_fp8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_forward_kv_large_f32": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I]),
    "gpt2b_attention_forward_kv_large_bf16": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I]),
    "gpt2b_attention_forward_kv_large_w8_i8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I]),
    "gpt2b_attention_forward_kv_large_w8_fp8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I]),
    "gpt2b_attention_kv_split_bf16": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_kv_merge_bf16": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_attention_kv_merge_f32": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_attention_kv_split_f32": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_kv_split_w8_i8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_kv_split_w8_fp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "gpt2b_attention_kv_merge_w8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_attention_forward_kv_large_bf16_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _P]),
    "gpt2b_layernorm_forward_f32": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_layernorm_forward_bf16": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "gpt2b_fused_residual_forward5_f32": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_fused_residual_forward5_bf16": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_encoder_forward_kv_f32": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_encoder_forward_kv_bf16": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "gpt2b_gpu_sample_softmax": (_I, [_P, _P, _I, _I, _U64, _I, _P]),
    "gpt2b_gpu_argmax": (_I, [_P, _P, _I, _I, _I, _P]),
    "gpt2b_logits_nll": (_I, [_P, _P, _I, _P, _P]),
    "gpt2b_engine_generate_dump": (_I, [_P, _P, _I, _I, _P, _I, _U64, _P, _P]),
    "gpt2b_matmul_forward_bf16": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_matmul_forward_f32out_bf16": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_matmul_forward_w8_i8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_matmul_forward_w8_fp8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "gpt2b_matmul_forward_w8_i8_f32out": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_matmul_forward_w8_fp8_f32out": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "gpt2b_read_header": (_I, [_S, _P, _P]),
    "gpt2b_engine_create_from_file": (_I, [_S, _S, _I, _I, _P]),
    "gpt2b_engine_create_from_buffer": (_I, [_P, _SZ, _P, _SZ, _I, _I, _P]),
    "gpt2b_engine_destroy": (_I, [_P]),
    "gpt2b_engine_config": (_I, [_P, _P]),
    "gpt2b_engine_set_option": (_I, [_P, _I, _I]),
    "gpt2b_engine_stream": (_I, [_P, _P]),
    "gpt2b_engine_device_buffers": (_I, [_P, _P, _P, _P, _P]),
    "gpt2b_engine_forward": (_I, [_P, _I, _I]),
    "gpt2b_engine_generate": (_I, [_P, _P, _I, _I, _P, _P, _I, _U64]),
    "gpt2b_engine_decode": (_I, [_P, _I]),
    "gpt2b_engine_set_position": (_I, [_P, _I, _I]),
    "gpt2b_engine_history": (_I, [_P, _P, _I, _I]),
    "gpt2b_engine_kernels_per_step": (_I, [_P, _P]),
    "gpt2b_nccl_unique_id": (_I, [_P]),
    "gpt2b_tp_plan": (_I, [_P, _I, _I, _P]),
    "gpt2b_tp_shard_image": (_I, [_P, _SZ, _P, _SZ, _I, _I, _I, _P, _P, _P, _P]),
    "gpt2b_engine_create_tp_from_buffer": (_I, [_P, _SZ, _P, _SZ, _I, _I, _I, _I, _P, _P]),
    "gpt2b_engine_tp_ipc_handle": (_I, [_P, _P]),
    "gpt2b_engine_tp_connect": (_I, [_P, _P, _I]),
}
# only in the trace build
_TRACE_SIGS = {
    "gpt2b_persist_trace": (_I, [_P, _P, _P, _P]),
    "gpt2b_persist_trace_stages": (_I, [_P]),
}

_lib = None


class Gpt2bError(RuntimeError):
    """A library call returned a non-zero status."""

    def __init__(self, status: int, where: str = ""):
        self.status = status
        super().__init__(f"{where}: status {status} ({status_string(status)})" if where else
                         f"status {status} ({status_string(status)})")


def lib() -> ctypes.CDLL:
    """The loaded libgpt2b.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m cuda_gpt2_inference_b200.build`")
        dll = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(dll, name)
            fn.restype = res
            fn.argtypes = args
        for name, (res, args) in _TRACE_SIGS.items():
            if hasattr(dll, name):
                getattr(dll, name).restype = res
                getattr(dll, name).argtypes = args
        _lib = dll
    return _lib


def status_string(status: int) -> str:
    try:
        return lib().gpt2b_status_string(int(status)).decode()
    except Exception:
        return "?"


def check(status: int, where: str = "") -> None:
    if status != OK:
        raise Gpt2bError(status, where)


def device_error() -> int:
    """Read and clear the device error word of the current device."""
    v = ctypes.c_int(0)
    check(lib().gpt2b_device_error(ctypes.byref(v)), "gpt2b_device_error")
    return v.value


def declared_functions(header: str = HEADER_PATH) -> list[str]:
    """Names of every function declared in include/gpt2_b200.h."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gpt2b_[A-Za-z0-9_]+)\s*\(", text)))
