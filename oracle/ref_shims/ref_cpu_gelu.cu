/* Reference CPU loop gelu_forward_cpu (gelu/gelu.cu:31-37).  TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_gelu_lab_main
#include "gelu/gelu.cu"
#undef main
REFAPI void ref_gelu_cpu(float* out, const float* inp, int N) { gelu_forward_cpu(out, inp, N); }
