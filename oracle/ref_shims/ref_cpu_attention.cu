/* Reference CPU loop attention_kv_cpu (attention_kvcache/attention_kvcache.cu:74-103).
 * TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_attn_lab_main
#include "attention_kvcache/attention_kvcache.cu"
#undef main
REFAPI void ref_attention_kv_cpu(float* out, const float* qkv, const float* kv_cache, int B,
                                 int seq_len, int NH, int hs, int maxT, float scale) {
    attention_kv_cpu(out, qkv, kv_cache, B, seq_len, NH, hs, maxT, scale);
}
