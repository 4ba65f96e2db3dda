/* Reference CPU loops residual_forward_cpu / layernorm_forward_cpu
 * (fused/fused.cu:44-80).  TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_fused_lab_main
#include "fused/fused.cu"
#undef main
REFAPI void ref_residual_cpu(float* out, const float* a, const float* b, int N) {
    residual_forward_cpu(out, a, b, N);
}
REFAPI void ref_layernorm_cpu(float* out, float* mean, float* rstd, const float* inp,
                              const float* weight, const float* bias, int B, int T, int C) {
    layernorm_forward_cpu(out, mean, rstd, inp, weight, bias, B, T, C);
}
