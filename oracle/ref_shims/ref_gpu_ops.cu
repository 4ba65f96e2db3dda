/* The reference's own CUDA kernels for the floatX path (FP32 or BF16, chosen
 * by -DENABLE_FP32 / -DENABLE_BF16 as in Makefile:78-85), compiled from the
 * reference headers in place for sm_100a.  Used on the GPU box as a second
 * oracle and as the "reference kernels on the same box" timing bar.
 * TEST INFRASTRUCTURE: only tests/ and bench.py load it.
 * Device pointers are passed as void*; cur_len is set through the reference's
 * own g_cur_len symbol (attention_kvcache.cuh:39). */
#include "ref_api.h"
#include "Inference_gpt2/common.h"
#include "Inference_gpt2/GEMV.cuh"
#include "Inference_gpt2/attention_kvcache.cuh"
#include "Inference_gpt2/layernorm.cuh"
#include "Inference_gpt2/encoder.cuh"
#include "Inference_gpt2/sampler_gpu.cuh"

REFAPI int ref_floatx_bytes() { return (int)sizeof(floatX); }
REFAPI int ref_set_cur_len(int v) { return (int)cudaMemcpyToSymbol(g_cur_len, &v, sizeof(int)); }
REFAPI int ref_cur_len_ptr(void** p) { return (int)cudaGetSymbolAddress(p, g_cur_len); }
REFAPI int ref_sync() { return (int)cudaDeviceSynchronize(); }

/* launch_GEMV6<floatX> (GEMV.cuh:112): default stream, float output */
REFAPI void ref_gemv6(void* out, const void* W, const void* x, int M, int K) {
    launch_GEMV6<floatX>((float*)out, (const floatX*)W, (const floatX*)x, M, K);
}
/* launch_GEMV6_fused<floatX> (GEMV.cuh:204) as matmul_forward uses it (opt.cu:111) */
REFAPI void ref_gemv6_fused(void* out, void* pre_gelu, const void* W, const void* x,
                            const void* bias, int M, int K, int do_gelu) {
    launch_GEMV6_fused<floatX>((floatX*)out, (floatX*)pre_gelu, (const floatX*)W, (const floatX*)x,
                               (const floatX*)bias, M, K, do_gelu != 0, 0);
}
REFAPI void ref_kv_cache_write(void* kv_cache, const void* qkv, int B, int NH, int hs, int maxT) {
    kv_cache_write_kernel<<<CEIL_DIV(B * NH * hs, 256), 256>>>((floatX*)kv_cache, (const floatX*)qkv,
                                                               B, NH, hs, maxT);
}
REFAPI void ref_attention_small(void* out, const void* qkv, void* kv_cache, int B, int NH, int hs,
                                int maxT) {
    attention_forward_kv_small((floatX*)out, (const floatX*)qkv, (floatX*)kv_cache, B, NH, hs, maxT, 0);
}
/* split + merge, the graph-capturable large path (inference_gpt2_opt.cu:336-341) */
REFAPI void ref_attention_split_merge(void* out, const void* qkv, void* kv_cache, int B, int NH,
                                      int hs, int maxT, float* part_out, float* part_lse,
                                      float* part_max, int S) {
    attention_kv_split_kernel<<<B * NH * S, 256>>>(part_out, part_lse, part_max, (const floatX*)qkv,
                                                  (const floatX*)kv_cache, B, NH, hs, maxT, S,
                                                  1.f / sqrtf(hs));
    attention_kv_merge_kernel<<<B * NH, 64>>>((floatX*)out, part_out, part_lse, part_max, NH, hs, S);
}
REFAPI void ref_layernorm(void* out, float* mean, float* rstd, void* inp, const void* w,
                          const void* b, int B, int T, int C) {
    layernorm_forward((floatX*)out, mean, rstd, (floatX*)inp, (const floatX*)w, (const floatX*)b, B, T,
                      C, 0);
}
REFAPI void ref_fused_residual(void* residual, void* normed, float* mean, float* rstd,
                               const void* in1, const void* in2, const void* w, const void* b,
                               int N, int C) {
    fused_residual_forward5((floatX*)residual, (floatX*)normed, mean, rstd, (const floatX*)in1,
                            (const floatX*)in2, (const floatX*)w, (const floatX*)b, N, C, 0);
}
REFAPI void ref_encoder_kv(void* out, const int* inp, const void* wte, const void* wpe,
                           const int* cur_len_ptr, int B, int C) {
    encoder_forward_kv((floatX*)out, inp, (const floatX*)wte, (const floatX*)wpe, cur_len_ptr, B, C, 0);
}
REFAPI void ref_sample_softmax(int* d_token, const float* logits, int B, int V,
                               unsigned long long seed, int step) {
    gpu_sample_softmax(d_token, logits, B, V, seed, step, 0);
}
