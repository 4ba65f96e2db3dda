/* The reference's own 8-bit CUDA kernels (GEMV_w8.cuh, attention_kvcache_w8.cuh),
 * compiled in place for sm_100a with the flags of Makefile:80-105
 * (-DENABLE_BF16 -DUSE_W8 -DUSE_KV_W8 and -DUSE_INT8 or -DUSE_FP8).
 * TEST INFRASTRUCTURE. */
#include "ref_api.h"
#include "fp8_compat.h"
#include "Inference_gpt2/common.h"
#include "Inference_gpt2/GEMV_w8.cuh"
#include "Inference_gpt2/attention_kvcache_w8.cuh"

REFAPI int ref_set_cur_len(int v) { return (int)cudaMemcpyToSymbol(g_cur_len, &v, sizeof(int)); }
REFAPI int ref_sync() { return (int)cudaDeviceSynchronize(); }

/* launch_GEMV6_w8x2<floatX, floatX> (layers, GEMV_w8.cuh:162) */
REFAPI void ref_gemv6_w8x2(void* out, void* pre_gelu, const uint8_t* W, const void* x,
                           const float* scale, const void* bias, int M, int K, int do_gelu) {
    launch_GEMV6_w8x2<floatX, floatX>((floatX*)out, (floatX*)pre_gelu, W, (const __nv_bfloat16*)x, scale,
                                      (const floatX*)bias, M, K, do_gelu != 0, 0);
}
/* launch_GEMV6_w8x2<float, floatX> (LM head, inference_gpt2_opt.cu:394) */
REFAPI void ref_gemv6_w8x2_f32out(float* out, const uint8_t* W, const void* x, const float* scale,
                                  int M, int K) {
    launch_GEMV6_w8x2<float, floatX>(out, (float*)nullptr, W, (const __nv_bfloat16*)x, scale,
                                     (const floatX*)nullptr, M, K, false, 0);
}
REFAPI void ref_dequant_wte(const uint8_t* w8, const float* scale, void* out, int Vp, int C) {
    dequant_wte_kernel<<<Vp, 256>>>(w8, scale, (floatX*)out, Vp, C);
}
REFAPI void ref_kv_cache_write_w8(uint8_t* kv, float* kv_scale, const void* qkv, int B, int NH, int hs,
                                  int maxT) {
    kv_cache_write_kernel_w8<<<B * NH * 2, 256>>>(kv, kv_scale, (const floatX*)qkv, B, NH, hs, maxT);
}
REFAPI void ref_attention_small_w8(void* out, const void* qkv, uint8_t* kv, const float* kv_scale,
                                   int B, int NH, int hs, int maxT) {
    attention_forward_kv_small_w8((floatX*)out, (const floatX*)qkv, kv, kv_scale, B, NH, hs, maxT, 0);
}
REFAPI void ref_attention_split_merge_w8(void* out, const void* qkv, const uint8_t* kv,
                                         const float* kv_scale, int B, int NH, int hs, int maxT,
                                         float* part_out, float* part_lse, float* part_max, int S) {
    attention_kv_split_kernel_w8<<<B * NH * S, 256>>>(part_out, part_lse, part_max, (const floatX*)qkv,
                                                     kv, kv_scale, B, NH, hs, maxT, S, 1.f / sqrtf(hs));
    attention_kv_merge_kernel_w8<<<B * NH, 64>>>((floatX*)out, part_out, part_lse, part_max, NH, hs, S);
}
