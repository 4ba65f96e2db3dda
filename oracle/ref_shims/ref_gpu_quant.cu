/* The reference quantiser (quantize.cu) compiled in place with the reference's
 * build flags (Makefile:137,187-188: --use_fast_math).  Exposes its kernel and
 * its whole file-to-file main for bit-exact comparison on the GPU box.
 * TEST INFRASTRUCTURE. */
#include "ref_api.h"
#define main ref_quantize_main
#include "quantize.cu"
#undef main
REFAPI int ref_quantize_files(const char* in_path, const char* out8_path, const char* scale_path,
                              int fp8) {
    const char* argv[] = {"quantize", in_path, out8_path, scale_path, "--format", fp8 ? "fp8" : "int8"};
    return ref_quantize_main(6, (char**)argv);
}
REFAPI int ref_quant_rows(const float* d_W, uint8_t* d_W8, float* d_scale, int M, int K, int fp8) {
    quant_rows<<<M, 256>>>(d_W, d_W8, d_scale, M, K, fp8 ? QFMT_FP8 : QFMT_INT8);
    return (int)cudaDeviceSynchronize();
}
