/* Reference CPU loop encoder_forward_cpu (other_kernels/encoder.cu:34-48).
 * TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_encoder_lab_main
#include "other_kernels/encoder.cu"
#undef main
REFAPI void ref_encoder_cpu(float* out, const int* inp, const float* wte, const float* wpe, int B,
                            int T, int C) {
    encoder_forward_cpu(out, inp, wte, wpe, B, T, C);
}
