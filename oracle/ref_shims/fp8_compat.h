/* The reference's FP8 decode (Inference_gpt2/GEMV_w8.cuh:40,
 * Inference_gpt2/attention_kvcache_w8.cuh:74) calls __nv_cvt_fp8_to_bf16raw,
 * which the CUDA 12.9 headers here do not declare.  Every E4M3 value is exact
 * in half and in bf16, so this stand-in (through the toolkit's half
 * converter) yields the same bf16 the reference expects.  TEST INFRASTRUCTURE. */
#pragma once
#include <cuda_fp8.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#if defined(USE_FP8)
static __host__ __device__ inline __nv_bfloat16_raw __nv_cvt_fp8_to_bf16raw(__nv_fp8_storage_t x,
                                                                             __nv_fp8_interpretation_t fmt) {
    __half_raw hr = __nv_cvt_fp8_to_halfraw(x, fmt);
    __half h(hr);
    __nv_bfloat16 b = __float2bfloat16(__half2float(h));
    return (__nv_bfloat16_raw)b;
}
#endif
