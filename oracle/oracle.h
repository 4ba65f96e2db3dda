/*
 * oracle.h -- CPU restatement of the reference GPT-2 batch-1 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library under
 * cuda_gpt2_inference_b200/) links, loads or calls this code.  It is used by
 * tests/ as the checker, by __graft_entry__.smoke() as the checker, and by
 * bench.py's cpu_baseline leg.
 *
 * Every routine cites the reference file:line whose behaviour it restates
 * (paths are relative to the reference project root).  The per-op loops follow
 * the reference's own CPU loops; the whole-model step follows the kernel order
 * of forward_kv_graph_ready (inference_gpt2_opt.cu:235-400), including the
 * points where the reference stores activations in its storage type
 * ("floatX": BF16 in the BF16/INT8/FP8 builds, FP32 in the FP32 build).
 *
 * Pinning: tests/test_oracle_pin.py checks these routines against the
 * reference's CPU loops compiled from source (oracle/_ref, built by
 * oracle/build_oracle.py) and against the committed fixtures in tests/golden/
 * that were produced from those compiled loops.
 *
 * Floating-point notes: the reference builds with --use_fast_math
 * (Makefile:137), so its GPU division and expf are approximate.  This oracle
 * uses IEEE float arithmetic; integer/byte results that depend on a division
 * (quantiser codes) are therefore pinned bit-exactly against the reference
 * CUDA kernel on the GPU, and against this oracle only up to rare one-code
 * differences at rounding boundaries.
 */
#ifndef GPT2B_ORACLE_H
#define GPT2B_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight storage modes (the reference's PRECISION build switch, Makefile:62-85). */
enum { ORC_W_F32 = 0, ORC_W_BF16 = 1, ORC_W_INT8 = 2, ORC_W_FP8 = 3 };
/* KV-cache modes: floatX (the activation type) or 8-bit codes + per-row scale
 * (the reference's KV_W8 switch, Makefile:96-105; format follows the weights). */
enum { ORC_KV_FLOATX = 0, ORC_KV_8BIT = 1 };
/* 8-bit code formats (quantize.cu:29-33). */
enum { ORC_FMT_INT8 = 0, ORC_FMT_FP8 = 1 };

/* ---- scalar format helpers ---------------------------------------------- */
float orc_bf16_round(float x);                 /* float -> bf16 (RNE) -> float */
uint16_t orc_f32_to_bf16_bits(float x);
float orc_bf16_bits_to_f32(uint16_t b);
float orc_w8_decode(uint8_t code, int fmt);    /* GEMV_w8.cuh:37-48 */
void orc_bf16_to_f32(float* out, const uint16_t* in, size_t n);
void orc_f32_to_bf16(uint16_t* out, const float* in, size_t n);

/* ---- per-op loops --------------------------------------------------------- */
/* out[m] = sum_k W[m,k] x[k]  (gemv/GEMV.cu:84-93, GEMV_cpu) */
void orc_gemv(float* out, const float* W, const float* x, int M, int K);
/* GEMV6_fused epilogue (Inference_gpt2/GEMV.cuh:190-200) over GEMV_cpu sums:
 * pre = W.x + b; pre_gelu <- pre (if non-null); out = do_gelu ? gelu(pre) : pre */
void orc_gemv_fused(float* out, float* pre_gelu, const float* W, const float* x,
                    const float* bias, int M, int K, int do_gelu);
/* GEMV6_w8x2 (Inference_gpt2/GEMV_w8.cuh:64-160): pre = scale[m] * sum_k
 * decode(code[m,k]) x[k] + b[m]; then the same epilogue as above. */
void orc_gemv_w8(float* out, float* pre_gelu, const uint8_t* W8, int fmt,
                 const float* x, const float* scale, const float* bias,
                 int M, int K, int do_gelu);
/* dequant_wte_kernel (GEMV_w8.cuh:179-190): out = bf16(decode(code) * s[row]) */
void orc_dequant_rows(float* out, const uint8_t* W8, const float* scale, int rows, int cols,
                      int fmt);
/* quant_rows (quantize.cu:41-81), IEEE division. */
void orc_quant_rows(const float* W, uint8_t* W8, float* scale, int M, int K, int fmt);
/* kv_cache_write_kernel_w8 row encoder (attention_kvcache_w8.cuh:115-155). */
void orc_kv_encode_row(const float* x, int hs, int fmt, uint8_t* codes, float* scale);
/* attention_kv_cpu (attention_kvcache/attention_kvcache.cu:74-103); float cache in
 * the reference layout [K: B*NH*maxT*hs][V: same]; seq_len = cur_len + 1. */
void orc_attention_kv(float* out, const float* qkv, const float* kv_cache,
                      int B, int seq_len, int NH, int hs, int maxT, float scale);
/* Same computation over an 8-bit cache with per-row scales (the reference's
 * _w8 kernels: kv_dot16 applies the K scale per row after the code dot,
 * attention_kvcache_w8.cuh:91-100, V is decoded times its row scale, :235). */
void orc_attention_kv_w8(float* out, const float* qkv, const uint8_t* kv_cache,
                         const float* kv_scale, int fmt, int B, int seq_len, int NH,
                         int hs, int maxT, float scale);
/* layernorm_forward_cpu (fused/fused.cu:50-80; layernorm/layernorm.cu:35) */
void orc_layernorm(float* out, float* mean, float* rstd, const float* inp,
                   const float* weight, const float* bias, int N, int C);
/* residual_forward_cpu (fused/fused.cu:44-48) */
void orc_residual(float* out, const float* a, const float* b, int N);
/* gelu_forward_cpu (gelu/gelu.cu:31-37) */
void orc_gelu(float* out, const float* inp, int N);
/* encoder (other_kernels/encoder.cu:34; decode form encoder.cuh:67-85):
 * out[b] = wte[tok[b]] + wpe[pos] */
void orc_encoder_kv(float* out, const int* tokens, const float* wte, const float* wpe,
                    int pos, int B, int C);
/* Greedy pick: index of the largest logit, lowest index on ties (new; the
 * reference only samples). */
int orc_argmax(const float* logits, int V);

/* ---- whole model ----------------------------------------------------------- */
typedef struct orc_model orc_model;

/* Parse a reference flat-bin image (gpt2_model.h:268-303 for v3/v5; the 8-bit
 * mixed layout of quantize.cu:190-229 when wmode is INT8/FP8, together with the
 * concatenated per-row scales of quantize.cu:226-229).  Returns NULL on a
 * malformed image; *err receives a short reason. */
orc_model* orc_model_from_buffer(const void* image, size_t nbytes, int wmode,
                                 const float* scales, size_t nscales, int kvmode,
                                 const char** err);
void orc_model_free(orc_model* m);
void orc_model_config(const orc_model* m, int cfg[6]); /* maxT,V,L,NH,C,Vp */
void orc_model_reset(orc_model* m);                  /* clears the KV cache */
/* One decode forward of `token` at position `pos` (forward_kv_graph_ready).
 * logits (Vp floats) may be NULL.  Returns 0 on success. */
int orc_model_step(orc_model* m, int token, int pos, float* logits);
/* Teacher-forced prompt at positions 0..n_prompt-1, then n_gen greedy forwards
 * at positions n_prompt..n_prompt+n_gen-1.  out_tokens receives n_gen+1 tokens:
 * the greedy pick after the last prompt position and after each decode step.
 * logits_out (optional) receives (n_prompt+n_gen) x Vp floats. */
int orc_model_generate(orc_model* m, const int* prompt, int n_prompt, int n_gen,
                       int* out_tokens, float* logits_out);
/* Activation probe of the last step: name in {"encoded","ln1","qkv","atty",
 * "residual2","ln2","fch","fch_gelu","residual3","lnf"}; layer-indexed ones take
 * `layer`.  Copies C (or 3C / 4C) floats; returns count or -1. */
int orc_model_probe(const orc_model* m, const char* name, int layer, float* out);

#ifdef __cplusplus
}
#endif
#endif
