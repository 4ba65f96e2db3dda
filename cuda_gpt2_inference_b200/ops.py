"""The reference operator surface on torch CUDA tensors.

One function per reference launcher, same argument order and meaning
(Inference_gpt2/GEMV.cuh, GEMV_w8.cuh, attention_kvcache(_w8).cuh,
layernorm.cuh, encoder.cuh, sampler_gpu.cuh); the storage type is taken from
the tensors and the current length is a device tensor (``d_pos``) instead of
the reference's ``g_cur_len`` symbol.  Every call goes to libgpt2b.so and
raises :class:`Gpt2bError` on a non-zero status; torch only supplies device
memory and the current stream.
"""
from __future__ import annotations

import torch

from . import check, lib


def _p(t):
    return None if t is None else t.data_ptr()


def _s(stream):
    return (stream if stream is not None else torch.cuda.current_stream()).cuda_stream


def _sfx(t):
    return {torch.float32: "f32", torch.bfloat16: "bf16"}[t.dtype]


def launch_GEMV6(out, W, x, M, K, stream=None):
    """out[M] (fp32) = W[M,K] . x  (GEMV.cuh:112)."""
    fn = getattr(lib(), f"gpt2b_launch_GEMV6_{_sfx(W)}")
    check(fn(_p(out), _p(W), _p(x), M, K, _s(stream)), "launch_GEMV6")


def launch_GEMV6_fused(out, pre_gelu, W, x, bias, M, K, do_gelu, stream=None):
    """out = gelu?(W.x + b), pre_gelu <- W.x + b  (GEMV.cuh:204)."""
    fn = getattr(lib(), f"gpt2b_launch_GEMV6_fused_{_sfx(W)}")
    check(fn(_p(out), _p(pre_gelu), _p(W), _p(x), _p(bias), M, K, int(bool(do_gelu)), _s(stream)),
          "launch_GEMV6_fused")


def launch_GEMV6_w8x2(out, pre_gelu, W, x, scale, bias, M, K, do_gelu, fmt="int8", stream=None):
    """8-bit weight-only GEMV (GEMV_w8.cuh:162); fp32 `out` selects the LM-head form."""
    sfx = "i8" if fmt == "int8" else "fp8"
    if out.dtype == torch.float32:
        fn = getattr(lib(), f"gpt2b_launch_GEMV6_w8x2_{sfx}_f32out")
        check(fn(_p(out), _p(W), _p(x), _p(scale), M, K, _s(stream)), "launch_GEMV6_w8x2")
    else:
        fn = getattr(lib(), f"gpt2b_launch_GEMV6_w8x2_{sfx}")
        check(fn(_p(out), _p(pre_gelu), _p(W), _p(x), _p(scale), _p(bias), M, K, int(bool(do_gelu)), _s(stream)),
              "launch_GEMV6_w8x2")


def dequant_wte(w8, scale, out, Vp, C, fmt="int8", stream=None):
    fn = getattr(lib(), "gpt2b_dequant_wte_" + ("i8" if fmt == "int8" else "fp8"))
    check(fn(_p(w8), _p(scale), _p(out), Vp, C, _s(stream)), "dequant_wte")


def quant_rows(W, W8, scale, M, K, fmt="int8", stream=None):
    fn = getattr(lib(), "gpt2b_quant_rows_" + ("i8" if fmt == "int8" else "fp8"))
    check(fn(_p(W), _p(W8), _p(scale), M, K, _s(stream)), "quant_rows")


def kv_cache_write(kv_cache, qkv, B, NH, hs, maxT, d_pos, kv_scale=None, fmt=None, stream=None):
    if kv_cache.dtype == torch.uint8:
        fn = getattr(lib(), "gpt2b_kv_cache_write_w8_" + ("i8" if fmt == "int8" else "fp8"))
        check(fn(_p(kv_cache), _p(kv_scale), _p(qkv), B, NH, hs, maxT, _p(d_pos), _s(stream)), "kv_cache_write_w8")
    else:
        fn = getattr(lib(), f"gpt2b_kv_cache_write_{_sfx(kv_cache)}")
        check(fn(_p(kv_cache), _p(qkv), B, NH, hs, maxT, _p(d_pos), _s(stream)), "kv_cache_write")


def attention_forward_kv_small(out, qkv, kv_cache, B, NH, hs, maxT, d_pos, kv_scale=None, fmt=None, stream=None):
    if kv_cache.dtype == torch.uint8:
        fn = getattr(lib(), "gpt2b_attention_forward_kv_small_w8_" + ("i8" if fmt == "int8" else "fp8"))
        check(fn(_p(out), _p(qkv), _p(kv_cache), _p(kv_scale), B, NH, hs, maxT, _p(d_pos), _s(stream)),
              "attention_forward_kv_small_w8")
    else:
        fn = getattr(lib(), f"gpt2b_attention_forward_kv_small_{_sfx(kv_cache)}")
        check(fn(_p(out), _p(qkv), _p(kv_cache), B, NH, hs, maxT, _p(d_pos), _s(stream)),
              "attention_forward_kv_small")


def attention_forward_kv_large(out, qkv, kv_cache, B, NH, hs, maxT, d_pos, part_out, part_lse, part_max, S,
                               kv_scale=None, fmt=None, stream=None):
    if kv_cache.dtype == torch.uint8:
        fn = getattr(lib(), "gpt2b_attention_forward_kv_large_w8_" + ("i8" if fmt == "int8" else "fp8"))
        check(fn(_p(out), _p(qkv), _p(kv_cache), _p(kv_scale), B, NH, hs, maxT, _p(d_pos), _s(stream),
                 _p(part_out), _p(part_lse), _p(part_max), S), "attention_forward_kv_large_w8")
    else:
        fn = getattr(lib(), f"gpt2b_attention_forward_kv_large_{_sfx(kv_cache)}")
        check(fn(_p(out), _p(qkv), _p(kv_cache), B, NH, hs, maxT, _p(d_pos), _s(stream), _p(part_out),
                 _p(part_lse), _p(part_max), S), "attention_forward_kv_large")


def attention_kv_split(part_out, part_lse, part_max, qkv, kv_cache, B, NH, hs, maxT, S, d_pos, kv_scale=None,
                       fmt=None, stream=None):
    """The split half alone (attention_kv_split_kernel(_w8), attention_kvcache.cuh:185, _w8.cuh:260)."""
    if kv_cache.dtype == torch.uint8:
        fn = getattr(lib(), "gpt2b_attention_kv_split_w8_" + ("i8" if fmt == "int8" else "fp8"))
        check(fn(_p(part_out), _p(part_lse), _p(part_max), _p(qkv), _p(kv_cache), _p(kv_scale), B, NH, hs, maxT, S,
                 _p(d_pos), _s(stream)), "attention_kv_split_w8")
    else:
        fn = getattr(lib(), f"gpt2b_attention_kv_split_{_sfx(kv_cache)}")
        check(fn(_p(part_out), _p(part_lse), _p(part_max), _p(qkv), _p(kv_cache), B, NH, hs, maxT, S, _p(d_pos),
                 _s(stream)), "attention_kv_split")


def attention_kv_merge(out, part_out, part_lse, part_max, B, NH, hs, S, w8=False, stream=None):
    """The merge half alone (attention_kv_merge_kernel(_w8), attention_kvcache.cuh:298, _w8.cuh:374)."""
    name = "gpt2b_attention_kv_merge_w8" if w8 else f"gpt2b_attention_kv_merge_{_sfx(out)}"
    check(getattr(lib(), name)(_p(out), _p(part_out), _p(part_lse), _p(part_max), B, NH, hs, S, _s(stream)),
          "attention_kv_merge")


def matmul_forward(out, inp, weight, bias, B, T, C, OC, pre_gelu=None, scale=None, fmt=None, stream=None):
    """out[B*T, OC] = inp . weight^T (+ bias), on the tensor cores
    (matmul_forward_cublaslt, matmul.cuh:141).  BF16 inp; weight BF16 or 8-bit
    codes (uint8 + per-row ``scale``, ``fmt`` "int8"/"fp8"); FP32 ``out``
    selects the LM-head form (no bias); ``pre_gelu`` fuses tanh-GELU."""
    w8 = weight.dtype == torch.uint8
    sfx = ("i8" if fmt == "int8" else "fp8") if w8 else None
    if out.dtype == torch.float32:
        if w8:
            rc = getattr(lib(), f"gpt2b_matmul_forward_w8_{sfx}_f32out")(_p(out), _p(inp), _p(weight), _p(scale), B, T,
                                                                          C, OC, _s(stream))
        else:
            rc = lib().gpt2b_matmul_forward_f32out_bf16(_p(out), _p(inp), _p(weight), B, T, C, OC, _s(stream))
    elif w8:
        rc = getattr(lib(), f"gpt2b_matmul_forward_w8_{sfx}")(_p(out), _p(inp), _p(weight), _p(scale), _p(bias), B, T,
                                                               C, OC, _p(pre_gelu), _s(stream))
    else:
        rc = lib().gpt2b_matmul_forward_bf16(_p(out), _p(inp), _p(weight), _p(bias), B, T, C, OC, _p(pre_gelu),
                                             _s(stream))
    check(rc, "matmul_forward")


def layernorm_forward(out, mean, rstd, inp, weight, bias, B, T, C, stream=None):
    fn = getattr(lib(), f"gpt2b_layernorm_forward_{_sfx(inp)}")
    check(fn(_p(out), _p(mean), _p(rstd), _p(inp), _p(weight), _p(bias), B, T, C, _s(stream)), "layernorm_forward")


def fused_residual_forward5(residual, normed, mean, rstd, inp1, inp2, weight, bias, N, C, stream=None):
    fn = getattr(lib(), f"gpt2b_fused_residual_forward5_{_sfx(inp1)}")
    check(fn(_p(residual), _p(normed), _p(mean), _p(rstd), _p(inp1), _p(inp2), _p(weight), _p(bias), N, C,
             _s(stream)), "fused_residual_forward5")


def encoder_forward_kv(out, inp, wte, wpe, d_pos, B, C, stream=None):
    fn = getattr(lib(), f"gpt2b_encoder_forward_kv_{_sfx(wte)}")
    check(fn(_p(out), _p(inp), _p(wte), _p(wpe), _p(d_pos), B, C, _s(stream)), "encoder_forward_kv")


def gpu_sample_softmax(d_token, logits, B, V, seed, step, stream=None):
    check(lib().gpt2b_gpu_sample_softmax(_p(d_token), _p(logits), B, V, seed, step, _s(stream)),
          "gpu_sample_softmax")


def gpu_argmax(d_token, logits, B, V, ld=None, stream=None):
    check(lib().gpt2b_gpu_argmax(_p(d_token), _p(logits), B, V, ld or V, _s(stream)), "gpu_argmax")
