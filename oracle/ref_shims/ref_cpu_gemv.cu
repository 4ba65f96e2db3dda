/* Reference CPU loop GEMV_cpu (gemv/GEMV.cu:84-93), compiled from the
 * reference source in place.  TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_gemv_lab_main
#include "gemv/GEMV.cu"
#undef main
REFAPI void ref_gemv_cpu_f32(float* out, const float* W, const float* x, int M, int K) {
    GEMV_cpu<float>(out, W, x, M, K);
}
REFAPI void ref_gemv_cpu_bf16(float* out, const void* W, const void* x, int M, int K) {
    GEMV_cpu<__nv_bfloat16>(out, (const __nv_bfloat16*)W, (const __nv_bfloat16*)x, M, K);
}
