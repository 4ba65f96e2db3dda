/*
 * gpt2_b200.h -- C ABI of the B200-native GPT-2 batch-1 decode library.
 *
 * This is the drop-in boundary for the decode hot path of the
 * CUDA_GPT2_Inference reference (inference_gpt2_opt.cu and the
 * Inference_gpt2/ operator headers).  The reference exposes header-only C++
 * templates selected by compile-time precision macros; this library exports
 * one plain C function per (operator, storage type) instead, with the same
 * argument order and meaning, plus:
 *   - an explicit `const int* d_pos` (device pointer to the current length)
 *     where the reference reads its hidden `__device__ int g_cur_len`
 *     (Inference_gpt2/attention_kvcache.cuh:39, encoder.cuh:71), so every call
 *     is CUDA-graph safe without cudaMemcpyToSymbol;
 *   - an explicit stream on every call (the reference defaults some to 0);
 *   - an int status return (0 = success) where the reference prints and calls
 *     exit(1) (GEMV.cuh:27-30, GEMV_w8.cuh:169-170, common.h:123-130).
 * No function allocates device memory except the engine constructors; the
 * caller owns every pointer it passes in.
 *
 * Type suffixes: _f32 (FP32 storage), _bf16 (BF16 storage), _i8 (INT8 weight
 * or KV codes), _fp8 (FP8 E4M3 codes).  bf16 arguments are passed as
 * `uint16_t*` (raw bits), FP8/INT8 codes as `uint8_t*`.
 */
#ifndef GPT2_B200_H
#define GPT2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gpt2b_stream_t; /* == cudaStream_t */

/* ---- status codes ------------------------------------------------------- */
enum {
    GPT2B_OK = 0,
    GPT2B_ERR_INVALID_ARG = 1001,  /* a size, pointer or option is out of range */
    GPT2B_ERR_ALIGNMENT = 1002,    /* a pointer or row pitch is not 16-byte aligned */
    GPT2B_ERR_UNSUPPORTED = 1003,  /* shape/mode combination not implemented */
    GPT2B_ERR_FILE = 1004,         /* weight/scale file missing or unreadable */
    GPT2B_ERR_FORMAT = 1005,       /* bad magic/version/header/size in a weight image */
    GPT2B_ERR_DEVICE = 1006,       /* a kernel reported an error word (see gpt2b_device_error) */
    GPT2B_ERR_NCCL = 1007,         /* a collective call failed or timed out */
    GPT2B_ERR_CUDA = 2000          /* GPT2B_ERR_CUDA + cudaError_t */
};
/* device error words (gpt2b_device_error) */
enum {
    GPT2B_DEVERR_MBAR_TIMEOUT = 1, /* a bulk copy never completed within its bound */
    GPT2B_DEVERR_BAD_TOKEN = 2,    /* token id outside [0, vocab) */
    GPT2B_DEVERR_BAD_POS = 3,      /* position outside [0, maxT) */
    GPT2B_DEVERR_PEER_TIMEOUT = 4, /* a cross-GPU flag wait hit its bound */
    GPT2B_DEVERR_GRID_TIMEOUT = 5  /* a wait on another CTA of the persistent decode kernel hit its bound */
};

const char* gpt2b_status_string(int status);
/* Reads and clears the device error word of the current device (0 = none). */
int gpt2b_device_error(int* code);
int gpt2b_version(void);

/* ======================================================================== */
/* Decode GEMVs                                                              */
/* ======================================================================== */
/* out[m] = sum_k W[m,k] x[k], FP32 output, no bias.
 * Replaces launch_GEMV6<T> (Inference_gpt2/GEMV.cuh:112; lab twin gemv/GEMV.cu:419).
 * W row-major M x K; K*sizeof(T) must be a multiple of 16 and W 16-byte aligned.
 * Also the FP32/BF16 LM head: replaces matmul_forward_cublaslt_f32
 * (Inference_gpt2/matmul.cuh:158, called at inference_gpt2_opt.cu:399) with
 * M = Vp, W = wte. */
int gpt2b_launch_GEMV6_f32(float* out, const float* W, const float* x, int M, int K, gpt2b_stream_t stream);
int gpt2b_launch_GEMV6_bf16(float* out, const uint16_t* W, const uint16_t* x, int M, int K,
                            gpt2b_stream_t stream);

/* pre = W.x + bias (bias may be NULL); pre_gelu[m] <- pre when pre_gelu != NULL;
 * out = do_gelu ? gelu_tanh(pre) : pre, stored in the storage type.
 * Replaces launch_GEMV6_fused<T,OT,BT> (Inference_gpt2/GEMV.cuh:204) as used by
 * matmul_forward (inference_gpt2_opt.cu:106-116). */
int gpt2b_launch_GEMV6_fused_f32(float* out, float* pre_gelu, const float* W, const float* x, const float* bias,
                                 int M, int K, int do_gelu, gpt2b_stream_t stream);
int gpt2b_launch_GEMV6_fused_bf16(uint16_t* out, uint16_t* pre_gelu, const uint16_t* W, const uint16_t* x,
                                  const uint16_t* bias, int M, int K, int do_gelu, gpt2b_stream_t stream);

/* 8-bit weight-only GEMV: pre = scale[m] * sum_k decode(W[m,k]) x[k] + bias[m];
 * epilogue as above.  x, bias, out, pre_gelu are BF16.  K % 16 == 0.
 * Replaces launch_GEMV6_w8x2<floatX,floatX> (Inference_gpt2/GEMV_w8.cuh:162)
 * as used by matmul_forward_w8 (inference_gpt2_opt.cu:121-131). */
int gpt2b_launch_GEMV6_w8x2_i8(uint16_t* out, uint16_t* pre_gelu, const uint8_t* W, const uint16_t* x,
                               const float* scale, const uint16_t* bias, int M, int K, int do_gelu,
                               gpt2b_stream_t stream);
int gpt2b_launch_GEMV6_w8x2_fp8(uint16_t* out, uint16_t* pre_gelu, const uint8_t* W, const uint16_t* x,
                                const float* scale, const uint16_t* bias, int M, int K, int do_gelu,
                                gpt2b_stream_t stream);
/* FP32-output form used for the 8-bit LM head, bias NULL, M = Vp: replaces
 * launch_GEMV6_w8x2<float,floatX> (inference_gpt2_opt.cu:394). */
int gpt2b_launch_GEMV6_w8x2_i8_f32out(float* out, const uint8_t* W, const uint16_t* x, const float* scale,
                                      int M, int K, gpt2b_stream_t stream);
int gpt2b_launch_GEMV6_w8x2_fp8_f32out(float* out, const uint8_t* W, const uint16_t* x, const float* scale,
                                       int M, int K, gpt2b_stream_t stream);

/* out[r,c] = bf16(decode(w8[r,c]) * scale[r]).  Replaces dequant_wte_kernel
 * (Inference_gpt2/GEMV_w8.cuh:179, launched at inference_gpt2_opt.cu:214). */
int gpt2b_dequant_wte_i8(const uint8_t* w8, const float* scale, uint16_t* out, int Vp, int C,
                         gpt2b_stream_t stream);
int gpt2b_dequant_wte_fp8(const uint8_t* w8, const float* scale, uint16_t* out, int Vp, int C,
                          gpt2b_stream_t stream);

/* Per-row symmetric quantiser: s = amax/127 (INT8) or amax/448 (FP8), s = 1 for
 * an all-zero row, codes = encode(W/s).  Bit-exact with quant_rows
 * (quantize.cu:41-81) built with the reference's --use_fast_math. */
int gpt2b_quant_rows_i8(const float* W, uint8_t* W8, float* scale, int M, int K, gpt2b_stream_t stream);
int gpt2b_quant_rows_fp8(const float* W, uint8_t* W8, float* scale, int M, int K, gpt2b_stream_t stream);
/* Whole-file quantiser: BF16 v5 image in, 8-bit mixed image + float32 per-row
 * scales out (the 5 Linear groups wte, qkvw, attprojw, fcw, fcprojw as codes,
 * the other 11 tensors unchanged, header unchanged), byte-compatible with the
 * quantize tool (quantize.cu:83-233).  fp8 = 0: INT8, 1: FP8 E4M3.  Runs on the
 * current device.  The buffer form writes into caller memory: out8 must hold
 * gpt2b_quantized_size() bytes and scales gpt2b_quantized_scale_count() floats. */
int gpt2b_quantize_file(const char* in_bf16_path, const char* out8_path, const char* scale_path, int fp8);
int gpt2b_quantized_size(const void* bf16_image, size_t nbytes, size_t* out8_bytes, size_t* scale_count);
int gpt2b_quantize_buffer(const void* bf16_image, size_t nbytes, void* out8, float* scales, int fp8);

/* ======================================================================== */
/* KV cache and decode attention                                             */
/* ======================================================================== */
/* Layout (attention_kvcache.cuh:8-13): one layer's cache is [K | V], each
 * B*NH*maxT*hs elements; element (b,h,j,d) at ((b*NH+h)*maxT + j)*hs + d.
 * 8-bit scales: [K | V], each B*NH*maxT floats, index (b*NH+h)*maxT + j
 * (attention_kvcache_w8.cuh:129-131).  qkv is [Q(NH*hs) | K | V] per batch row.
 * hs must be 64 (the reference's thread mapping fixes it); *d_pos < maxT. */

/* Append K,V of the current token at position *d_pos.  Replaces
 * kv_cache_write_kernel (attention_kvcache.cuh:46) / kv_cache_write_kernel_w8
 * (attention_kvcache_w8.cuh:115). */
int gpt2b_kv_cache_write_f32(float* kv_cache, const float* qkv, int B, int NH, int hs, int maxT,
                             const int* d_pos, gpt2b_stream_t stream);
int gpt2b_kv_cache_write_bf16(uint16_t* kv_cache, const uint16_t* qkv, int B, int NH, int hs, int maxT,
                              const int* d_pos, gpt2b_stream_t stream);
int gpt2b_kv_cache_write_w8_i8(uint8_t* kv_cache, float* kv_scale, const uint16_t* qkv, int B, int NH, int hs,
                               int maxT, const int* d_pos, gpt2b_stream_t stream);
int gpt2b_kv_cache_write_w8_fp8(uint8_t* kv_cache, float* kv_scale, const uint16_t* qkv, int B, int NH, int hs,
                                int maxT, const int* d_pos, gpt2b_stream_t stream);

/* out = softmax(q.K^T / sqrt(hs)) V over positions [0, *d_pos], one pass per
 * head.  Replaces attention_forward_kv_small (attention_kvcache.cuh:453) and
 * attention_forward_kv_small_w8 (attention_kvcache_w8.cuh:529). */
int gpt2b_attention_forward_kv_small_f32(float* out, const float* qkv, const float* kv_cache, int B, int NH,
                                         int hs, int maxT, const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_forward_kv_small_bf16(uint16_t* out, const uint16_t* qkv, const uint16_t* kv_cache, int B,
                                          int NH, int hs, int maxT, const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_forward_kv_small_w8_i8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                           const float* kv_scale, int B, int NH, int hs, int maxT,
                                           const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_forward_kv_small_w8_fp8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                            const float* kv_scale, int B, int NH, int hs, int maxT,
                                            const int* d_pos, gpt2b_stream_t stream);

/* Flash-decoding: split [0, *d_pos] into S chunks of ceil((pos+1)/S), write
 * per-split partials (part_out un-normalised [B*NH*S*hs], part_max, part_lse
 * [B*NH*S]; an empty split writes max=-FLT_MAX, lse=0, out=0), then merge.
 * Graph-capturable.  Replaces attention_forward_kv_large(_w8)
 * (attention_kvcache.cuh:464, attention_kvcache_w8.cuh:541) and the raw
 * split+merge launches of inference_gpt2_opt.cu:310-314,338-341. */
int gpt2b_attention_forward_kv_large_f32(float* out, const float* qkv, const float* kv_cache, int B, int NH,
                                         int hs, int maxT, const int* d_pos, gpt2b_stream_t stream,
                                         float* part_out, float* part_lse, float* part_max, int S);
int gpt2b_attention_forward_kv_large_bf16(uint16_t* out, const uint16_t* qkv, const uint16_t* kv_cache, int B,
                                          int NH, int hs, int maxT, const int* d_pos, gpt2b_stream_t stream,
                                          float* part_out, float* part_lse, float* part_max, int S);
int gpt2b_attention_forward_kv_large_w8_i8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                           const float* kv_scale, int B, int NH, int hs, int maxT,
                                           const int* d_pos, gpt2b_stream_t stream, float* part_out,
                                           float* part_lse, float* part_max, int S);
int gpt2b_attention_forward_kv_large_w8_fp8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                            const float* kv_scale, int B, int NH, int hs, int maxT,
                                            const int* d_pos, gpt2b_stream_t stream, float* part_out,
                                            float* part_lse, float* part_max, int S);
/* The two halves on their own: attention_kv_split_kernel(_w8)
 * (attention_kvcache.cuh:185, _w8.cuh:260) and attention_kv_merge_kernel(_w8)
 * (attention_kvcache.cuh:298, _w8.cuh:374). */
int gpt2b_attention_kv_split_bf16(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                  const uint16_t* kv_cache, int B, int NH, int hs, int maxT, int S,
                                  const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_kv_merge_bf16(uint16_t* out, const float* part_out, const float* part_lse,
                                  const float* part_max, int B, int NH, int hs, int S, gpt2b_stream_t stream);
int gpt2b_attention_kv_merge_f32(float* out, const float* part_out, const float* part_lse, const float* part_max,
                                 int B, int NH, int hs, int S, gpt2b_stream_t stream);
/* FP32 split (attention_kvcache.cuh:185 in an FP32 build) and the 8-bit-KV
 * halves launched raw by inference_gpt2_opt.cu:310-314:
 * attention_kv_split_kernel_w8 (attention_kvcache_w8.cuh:260; codes x row scale,
 * kv_scale as written by gpt2b_kv_cache_write_w8_*) and
 * attention_kv_merge_kernel_w8 (attention_kvcache_w8.cuh:374; BF16 output, the
 * same merge as gpt2b_attention_kv_merge_bf16). */
int gpt2b_attention_kv_split_f32(float* part_out, float* part_lse, float* part_max, const float* qkv,
                                 const float* kv_cache, int B, int NH, int hs, int maxT, int S, const int* d_pos,
                                 gpt2b_stream_t stream);
int gpt2b_attention_kv_split_w8_i8(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                   const uint8_t* kv_cache, const float* kv_scale, int B, int NH, int hs, int maxT,
                                   int S, const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_kv_split_w8_fp8(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                    const uint8_t* kv_cache, const float* kv_scale, int B, int NH, int hs, int maxT,
                                    int S, const int* d_pos, gpt2b_stream_t stream);
int gpt2b_attention_kv_merge_w8(uint16_t* out, const float* part_out, const float* part_lse, const float* part_max,
                                int B, int NH, int hs, int S, gpt2b_stream_t stream);
/* No counterpart in the reference.  gpt2b_attention_forward_kv_large_bf16
 * without the three caller-provided partial buffers, for callers that cannot
 * allocate device memory (a host whose memory pool owns the whole device, or a
 * hot path that must not pay cudaMalloc's implicit synchronisation).  The split
 * partials live in a fixed array inside the library (about 0.5 MB per GPU,
 * held until the process exits): B*NH*S must not exceed 2048, else
 * GPT2B_ERR_INVALID_ARG.  Allocates nothing.  The first call on a device looks
 * up that array's device address (cudaGetSymbolAddress), so make that first
 * call before any stream capture.  That address is kept per device ordinal for
 * the life of the process; after cudaDeviceReset on a device it is stale, so do
 * not call this entry point on a device that was reset.  All calls share the
 * one array: calls that can overlap on the GPU (different streams, or different
 * host threads on the same device) race and must be serialised by the caller. */
int gpt2b_attention_forward_kv_large_bf16_noalloc(uint16_t* out, const uint16_t* qkv, const uint16_t* kv_cache, int B,
                                                  int NH, int hs, int maxT, const int* d_pos, int S,
                                                  gpt2b_stream_t stream);

/* ======================================================================== */
/* LayerNorm, residual, embedding                                            */
/* ======================================================================== */
/* out = (x-mean)*rstd*w + b per row of C; mean/rstd (float, may be NULL).
 * Replaces layernorm_forward (Inference_gpt2/layernorm.cuh:282). N = B*T rows. */
int gpt2b_layernorm_forward_f32(float* out, float* mean, float* rstd, const float* inp, const float* weight,
                                const float* bias, int B, int T, int C, gpt2b_stream_t stream);
int gpt2b_layernorm_forward_bf16(uint16_t* out, float* mean, float* rstd, const uint16_t* inp,
                                 const uint16_t* weight, const uint16_t* bias, int B, int T, int C,
                                 gpt2b_stream_t stream);
/* residual = inp1 + inp2 (stored), normed = LN(residual).  Replaces
 * fused_residual_forward5 (Inference_gpt2/layernorm.cuh:336). */
int gpt2b_fused_residual_forward5_f32(float* residual, float* normed, float* mean, float* rstd, const float* inp1,
                                      const float* inp2, const float* weight, const float* bias, int N, int C,
                                      gpt2b_stream_t stream);
int gpt2b_fused_residual_forward5_bf16(uint16_t* residual, uint16_t* normed, float* mean, float* rstd,
                                       const uint16_t* inp1, const uint16_t* inp2, const uint16_t* weight,
                                       const uint16_t* bias, int N, int C, gpt2b_stream_t stream);
/* out[b] = wte[inp[b]] + wpe[*d_pos].  Replaces encoder_forward_kv
 * (Inference_gpt2/encoder.cuh:87). */
int gpt2b_encoder_forward_kv_f32(float* out, const int* inp, const float* wte, const float* wpe, const int* d_pos,
                                 int B, int C, gpt2b_stream_t stream);
int gpt2b_encoder_forward_kv_bf16(uint16_t* out, const int* inp, const uint16_t* wte, const uint16_t* wpe,
                                  const int* d_pos, int B, int C, gpt2b_stream_t stream);

/* ======================================================================== */
/* Token selection                                                           */
/* ======================================================================== */
/* Softmax sampling with Philox(seed, subsequence=b, offset=step) uniform draws
 * (curand), one token per batch row.  Replaces gpu_sample_softmax
 * (Inference_gpt2/sampler_gpu.cuh:94); same ordering of the cumulative sum. */
int gpt2b_gpu_sample_softmax(int* d_token, const float* logits, int B, int V, unsigned long long seed, int step,
                             gpt2b_stream_t stream);
/* Greedy pick: index of the largest logit among the first V, lowest index on
 * ties.  No counterpart in the reference (it only samples); the greedy decode
 * configurations need it. */
int gpt2b_gpu_argmax(int* d_token, const float* logits, int B, int V, int ld, gpt2b_stream_t stream);
/* *d_nll = log(sum_i exp(logits[i])) - logits[*d_token] over the first V
 * logits (max-shifted, sum in double): the negative log-likelihood the
 * reference's ppl_record_nll computes on the host after copying the logits
 * back (Inference_gpt2/dump_utils.h:63-79), here on the device. */
int gpt2b_logits_nll(float* d_nll, const float* logits, int V, const int* d_token, gpt2b_stream_t stream);

/* ======================================================================== */
/* Prompt GEMM on the tensor cores (tcgen05)                                */
/* ======================================================================== */
/* out[B*T x OC] = inp[B*T x C] . weight[OC x C]^T + bias, BF16 in and out,
 * FP32 accumulation in tensor memory.  pre_gelu non-NULL: pre_gelu receives
 * the pre-activation and out = gelu_tanh(pre).  Replaces
 * matmul_forward_cublaslt (Inference_gpt2/matmul.cuh:141; the fused-GELU
 * form, gelu_fusion >= 1).  inp and weight 16-byte aligned, C a multiple of 8. */
int gpt2b_matmul_forward_bf16(uint16_t* out, const uint16_t* inp, const uint16_t* weight, const uint16_t* bias,
                              int B, int T, int C, int OC, uint16_t* pre_gelu, gpt2b_stream_t stream);
/* FP32 output, no bias (the LM head).  Replaces matmul_forward_cublaslt_f32
 * (Inference_gpt2/matmul.cuh:158). */
int gpt2b_matmul_forward_f32out_bf16(float* out, const uint16_t* inp, const uint16_t* weight, int B, int T, int C,
                                     int OC, gpt2b_stream_t stream);
/* 8-bit weight-only forms: weight = INT8 / E4M3 codes [OC x C] with one FP32
 * scale per output row (quantize.cu format); out = gelu?(scale * (inp .
 * codes^T) + bias).  No counterpart in the reference (its prompt path keeps
 * BF16 weights); they run the prompt of the 8-bit engines.  C a multiple of 16. */
int gpt2b_matmul_forward_w8_i8(uint16_t* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                               const uint16_t* bias, int B, int T, int C, int OC, uint16_t* pre_gelu,
                               gpt2b_stream_t stream);
int gpt2b_matmul_forward_w8_fp8(uint16_t* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                const uint16_t* bias, int B, int T, int C, int OC, uint16_t* pre_gelu,
                                gpt2b_stream_t stream);
int gpt2b_matmul_forward_w8_i8_f32out(float* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                      int B, int T, int C, int OC, gpt2b_stream_t stream);
int gpt2b_matmul_forward_w8_fp8_f32out(float* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                       int B, int T, int C, int OC, gpt2b_stream_t stream);

/* ======================================================================== */
/* Whole-model decode engine (replaces forward_kv_graph_ready,               */
/* graph_capture_all and run_generation_once_graph, inference_gpt2_opt.cu)   */
/* ======================================================================== */
/* Weight storage modes (the reference's PRECISION switch, Makefile:62-85). */
enum { GPT2B_W_F32 = 0, GPT2B_W_BF16 = 1, GPT2B_W_INT8 = 2, GPT2B_W_FP8 = 3 };
/* KV-cache modes: the activation type, or 8-bit codes in the weights' format
 * with one float scale per (K/V, layer, head, position) (Makefile:96-105). */
enum { GPT2B_KV_FLOATX = 0, GPT2B_KV_8BIT = 1 };
/* Engine options (gpt2b_engine_set_option). */
enum {
    GPT2B_OPT_USE_GRAPH = 1,  /* 1 (default): replay the captured step graph; 0: launch kernels */
    GPT2B_OPT_USE_PDL = 2,    /* 1 (default): programmatic dependent launch between kernels */
    GPT2B_OPT_SPLITS = 3,     /* attention splits per head for long contexts (default: fills the SMs) */
    GPT2B_OPT_STEPS_PER_GRAPH = 4, /* decode steps captured into one graph (default 8) */
    GPT2B_OPT_PERSISTENT = 5, /* 1 (default where the shape allows): the whole decode loop runs in one
                                 cooperative kernel; 0: per-kernel steps (GEMV / attention launches) */
    GPT2B_OPT_POLL_LIMIT = 6, /* persistent kernel: polls of one wait on another CTA (or another rank of a
                                 tensor-parallel group) before it gives up, records
                                 GPT2B_DEVERR_GRID_TIMEOUT and makes every CTA of the group leave
                                 (default 4194304, a few seconds; at least 1024).  After a timeout in a
                                 tensor-parallel group the exchange words of the aborted call are
                                 stale: destroy and rebuild the group's engines. */
    GPT2B_OPT_PREFILL = 7     /* 1 (default where the model allows: BF16 / 8-bit weights, single GPU): the
                                 prompt of gpt2b_engine_generate (two tokens or more) runs as tensor-core
                                 GEMMs over all its positions at once; 0: one decode step per position */
};

/* GPT2Config field order (Inference_gpt2/gpt2_model.h:28-35). */
typedef struct {
    int max_seq_len;
    int vocab_size;
    int padded_vocab_size;
    int num_layers;
    int num_heads;
    int channels;
} gpt2b_config;

typedef struct gpt2b_engine gpt2b_engine;

/* Reads the 256-int header of a flat-bin weight file (gpt2_model.h:268-296).
 * Host only.  version: 3 = FP32, 5 = BF16 or 8-bit mixed. */
int gpt2b_read_header(const char* path, int* version, gpt2b_config* cfg);

/* Builds an engine on the current device from a weight image in the
 * reference format: v3 FP32 / v5 BF16 (gpt2_build_from_checkpoint,
 * gpt2_model.h:268-303) or the 8-bit mixed file of quantize.cu:190-229 with
 * its per-row scales (gpt2_build_w8, inference_gpt2_opt.cu:143-219).
 * One device arena holds all parameters; another the activations; the KV
 * cache is a third.  scale_path may be NULL: then "<model minus .bin>_scales.bin"
 * is used as in inference_gpt2_opt.cu:666-668. */
int gpt2b_engine_create_from_file(const char* model_path, const char* scale_path, int wmode, int kvmode,
                                  gpt2b_engine** out);
int gpt2b_engine_create_from_buffer(const void* image, size_t nbytes, const float* scales, size_t nscales,
                                    int wmode, int kvmode, gpt2b_engine** out);
int gpt2b_engine_destroy(gpt2b_engine* e);
int gpt2b_engine_config(const gpt2b_engine* e, gpt2b_config* cfg);
int gpt2b_engine_set_option(gpt2b_engine* e, int option, int value);
int gpt2b_engine_stream(const gpt2b_engine* e, gpt2b_stream_t* stream);
/* Device pointers owned by the engine: logits (Vp floats), the current token
 * and position (int), and the token history (maxT+1 ints). */
int gpt2b_engine_device_buffers(const gpt2b_engine* e, float** logits, int** token, int** pos, int** history);

/* One forward of `token` at position `pos` on the engine stream (host
 * values; copied to the engine's device slots).  Logits land in the engine's
 * logits buffer.  The equivalent of gpt2_forward_kv (inference_gpt2_opt.cu:403). */
int gpt2b_engine_forward(gpt2b_engine* e, int token, int pos);
/* Teacher-forced prompt at positions 0..n_prompt-1 then n_gen greedy steps;
 * out_tokens (host) receives n_gen+1 tokens (the pick after the prompt and
 * after each step).  logits_host (optional) receives (n_prompt+n_gen) x Vp
 * floats.  Host buffers; copies included.  sample != 0 uses
 * gpt2b_gpu_sample_softmax(seed, step) instead of greedy. */
int gpt2b_engine_generate(gpt2b_engine* e, const int* prompt, int n_prompt, int n_gen, int* out_tokens,
                          float* logits_host, int sample, unsigned long long seed);
/* Verification dumps (Inference_gpt2/dump_utils.h; the --dump-steps,
 * --dump-prefix and --ppl options of inference_gpt2_opt.cu:634-651).  Step t
 * (t = 1 .. n_prompt + n_gen) is the forward at position t - 1; its "appended
 * token" is the one at position t (teacher-forced from the prompt, then the
 * greedy or sampled pick).  Files, in the reference's layout, under `dir`
 * (created if missing):
 *   <prefix>_logits_t1.bin            step 1's logits, V floats (logits_t1 != 0)
 *   <prefix>_logits_step<t>.bin       step t's logits, V floats (t in steps[])
 *   <prefix>_inputs_step<t>.bin       the tokens at positions 0..t-1, t ints
 *   ppl_<prefix>_nll.bin              the NLL of each step's appended token, steps
 *                                     1..ppl_len, floats (computed on the device)
 *   ppl_<prefix>_tokens.bin           those tokens, ints
 * dir NULL writes no files (nll_out still receives the NLLs). */
typedef struct {
    const char* dir;
    const char* prefix;
    const int* steps;
    int n_steps;
    int ppl_len;   /* 0: no NLL record */
    int logits_t1;
} gpt2b_dump_config;
/* gpt2b_engine_generate (host buffers, one launch per step) with the dumps of
 * `dump`.  nll_out (optional, host): ppl_len floats. */
int gpt2b_engine_generate_dump(gpt2b_engine* e, const int* prompt, int n_prompt, int n_gen, int* out_tokens,
                               int sample, unsigned long long seed, const gpt2b_dump_config* dump, float* nll_out);
/* Device-resident decode: starting from the token and position already in the
 * engine's device slots, run n_steps greedy forwards without host round trips
 * (token and position advance on the device; picks are appended to the
 * device history).  Asynchronous on the engine stream. */
int gpt2b_engine_decode(gpt2b_engine* e, int n_steps);
/* Sets the device token/position slots (asynchronous copy on the engine
 * stream) so gpt2b_engine_decode continues from (token, pos); the KV cache
 * below pos is kept. */
int gpt2b_engine_set_position(gpt2b_engine* e, int token, int pos);
/* Waits for the engine stream and copies history[first .. first+count) (the
 * token at each position; history[p+1] is the pick after position p) to host. */
int gpt2b_engine_history(gpt2b_engine* e, int* out_host, int first, int count);
/* ------------------------------------------------------------------------ */
/* Tensor parallelism (no counterpart in the reference, which is single-GPU). */
/* GPT-2-XL-style sharding for decode: QKV and FC column-parallel (this rank's */
/* heads / FC rows), attention projection and FC projection row-parallel     */
/* (FP32 partial sums all-reduced with NCCL), LM head vocab-parallel with an  */
/* all-gather of (best logit, index) pairs; residual and LayerNorms replicated.*/
/* Heads split unevenly (25 heads: 13/12, 7/6/6/6, 4/3x7); 4C and Vp must be  */
/* divisible by 16*tp_size and tp_size.                                       */
/* ------------------------------------------------------------------------ */
/* 128-byte NCCL unique id for a new group (rank 0 creates it, the host       */
/* distributes it).  GPT2B_ERR_UNSUPPORTED when built without NCCL.           */
int gpt2b_nccl_unique_id(void* id_out);
/* This rank's shard: out6 = {first head, heads, first FC row, FC rows, first */
/* vocab row, vocab rows}.  Host only.                                        */
int gpt2b_tp_plan(const gpt2b_config* cfg, int tp_rank, int tp_size, int* out6);
/* This rank's parameter tensors (file order, element sizes as stored, sliced */
/* per the plan; row-parallel biases only on rank 0, zeros elsewhere) and its */
/* scale arrays.  With out_params NULL only the sizes are returned.  Host only.*/
int gpt2b_tp_shard_image(const void* image, size_t nbytes, const float* scales, size_t nscales, int wmode,
                         int tp_rank, int tp_size, void* out_params, size_t* out_bytes, float* out_scales,
                         size_t* out_nscales);
/* Collective over the tp_size ranks (one process per GPU, each on its own   */
/* current device, all passing the same image and id): builds this rank's    */
/* engine.  Its generate/decode/forward calls are collectives too; logits    */
/* returned to the host are the full gathered Vp.  Per-kernel path only.     */
int gpt2b_engine_create_tp_from_buffer(const void* image, size_t nbytes, const float* scales, size_t nscales,
                                       int wmode, int kvmode, int tp_rank, int tp_size, const void* nccl_id,
                                       gpt2b_engine** out);

/* Persistent kernel across the group: the row-parallel partial sums and the  */
/* LM-head picks go straight into every rank's exchange arena (peer stores   */
/* over NVLink, tagged words, no NCCL).  Each rank exports the IPC handle of */
/* its arena (64 bytes); the host gathers the tp_size handles in rank order  */
/* and every rank connects; the engine then uses the persistent kernel.      */
int gpt2b_engine_tp_ipc_handle(gpt2b_engine* e, void* handle_out);
int gpt2b_engine_tp_connect(gpt2b_engine* e, const void* handles, int n);

/* Kernel launches one step issues (for launch accounting); 0 when the
 * persistent kernel runs: it issues one launch per decode/generate call for
 * all of that call's steps. */
int gpt2b_engine_kernels_per_step(const gpt2b_engine* e, int* n);

#ifdef __cplusplus
}
#endif
#endif /* GPT2_B200_H */
