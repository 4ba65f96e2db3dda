// quant.cu -- per-row symmetric 8-bit weight quantisation and dequantisation.
//
// The quantiser must reproduce quantize.cu's codes and scales byte for byte.
// That tool is built with --use_fast_math (Makefile:137,187-188), so its
// divisions are the approximate fast-math form; this file is built with the
// same flag and evaluates the same expressions per element -- amax over the
// row, s = amax / 127 (or / 448), s = 1 when amax == 0, code = encode(w / s)
// (quantize.cu:41-81) -- with one block per row and a strided loop, so the
// compiler sees the same division pattern.  It runs once at load time; the
// layout is chosen for exactness, not speed.
#include "common.cuh"
#include "internal.h"

#include <stdio.h>
#include <string.h>
#include <algorithm>
#include <vector>

namespace gpt2b {

constexpr int kQThreads = 256;

template <bool FP8>
__global__ void __launch_bounds__(kQThreads) quant_rows_kernel(const float* W, uint8_t* W8, float* scale, int M, int K) {
    const int row = blockIdx.x;
    if (row >= M) return;
    const int tid = threadIdx.x;
    __shared__ float red[kQThreads];
    float local = 0.0f;
    for (int i = tid; i < K; i += kQThreads) local = fmaxf(local, fabsf(W[(size_t)row * K + i]));
    red[tid] = local;
    __syncthreads();
    for (int off = kQThreads / 2; off > 0; off >>= 1) {
        if (tid < off) red[tid] = fmaxf(red[tid], red[tid + off]);
        __syncthreads();
    }
    const float full = FP8 ? 448.0f : 127.0f;
    const float s = (red[0] == 0.0f) ? 1.0f : (red[0] / full);
    if (tid == 0) scale[row] = s;
    for (int i = tid; i < K; i += kQThreads) {
        const float v = W[(size_t)row * K + i] / s;
        if (FP8) {
            W8[(size_t)row * K + i] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
        } else {
            int q = __float2int_rn(v);
            q = min(max(q, -127), 127);
            W8[(size_t)row * K + i] = (uint8_t)(int8_t)q;
        }
    }
}

// out = bf16(decode(code) * scale[row])  (dequant_wte_kernel, GEMV_w8.cuh:388-397)
template <bool FP8>
__global__ void dequant_rows_kernel(const uint8_t* w8, const float* scale, __nv_bfloat16* out, int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t code = w8[i];
        const float v = FP8 ? e4m3_to_f(code, 0) : (float)(int8_t)code;
        out[i] = __float2bfloat16_rn(v * scale[i / cols]);
    }
}

__global__ void widen_bf16_kernel(const uint16_t* in, float* out, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __uint_as_float((uint32_t)in[i] << 16);
}

// Layout of a v5 image: element counts (gpt2_model.h:63-87) and whether each
// tensor is one of the 5 quantised Linear groups (quantize.cu:190-196).
struct ImageLayout {
    size_t n[16];
    int M[5], K[5];
    int maxT, L, C, Vp;
};
static const int kGroupOfTensor[16] = {0, -1, -1, -1, 1, -1, 2, -1, -1, -1, 3, -1, 4, -1, -1, -1};

static int parse_v5(const void* image, size_t nbytes, ImageLayout& lay) {
    if (!image || nbytes < 1024) return GPT2B_ERR_FORMAT;
    const int* h = static_cast<const int*>(image);
    if (h[0] != 20251103 || h[1] != 5) return GPT2B_ERR_FORMAT;  // quantize.cu:115
    lay.maxT = h[2]; lay.L = h[4]; lay.C = h[6]; lay.Vp = h[7];
    if (lay.maxT <= 0 || lay.L <= 0 || lay.C <= 0 || lay.Vp <= 0) return GPT2B_ERR_FORMAT;
    const size_t C = lay.C, L = lay.L, Vp = lay.Vp, maxT = lay.maxT;
    const size_t n[16] = {Vp * C, maxT * C, L * C, L * C, L * 3 * C * C, L * 3 * C, L * C * C, L * C,
                          L * C, L * C, L * 4 * C * C, L * 4 * C, L * C * 4 * C, L * C, C, C};
    size_t total = 0;
    for (int i = 0; i < 16; i++) { lay.n[i] = n[i]; total += n[i]; }
    if (nbytes != 1024 + total * 2) return GPT2B_ERR_FORMAT;
    const int M[5] = {lay.Vp, lay.L * 3 * lay.C, lay.L * lay.C, lay.L * 4 * lay.C, lay.L * lay.C};
    const int K[5] = {lay.C, lay.C, lay.C, lay.C, 4 * lay.C};
    for (int g = 0; g < 5; g++) { lay.M[g] = M[g]; lay.K[g] = K[g]; }
    return GPT2B_OK;
}

}  // namespace gpt2b

using namespace gpt2b;

extern "C" {

int gpt2b_quantized_size(const void* bf16_image, size_t nbytes, size_t* out8_bytes, size_t* scale_count) {
    ImageLayout lay;
    int rc = parse_v5(bf16_image, nbytes, lay);
    if (rc) return rc;
    size_t b = 1024, s = 0;
    for (int i = 0; i < 16; i++) b += lay.n[i] * (kGroupOfTensor[i] >= 0 ? 1 : 2);
    for (int g = 0; g < 5; g++) s += (size_t)lay.M[g];
    if (out8_bytes) *out8_bytes = b;
    if (scale_count) *scale_count = s;
    return GPT2B_OK;
}

int gpt2b_quantize_buffer(const void* bf16_image, size_t nbytes, void* out8, float* scales, int fp8) {
    ImageLayout lay;
    int rc = parse_v5(bf16_image, nbytes, lay);
    if (rc) return rc;
    if (!out8 || !scales) return GPT2B_ERR_INVALID_ARG;
    size_t maxn = 0;
    for (int g = 0; g < 5; g++) maxn = std::max(maxn, (size_t)lay.M[g] * lay.K[g]);
    uint16_t* d_in = nullptr;
    float* d_f = nullptr;
    float* d_s = nullptr;
    uint8_t* d_q = nullptr;
    cudaError_t err = cudaMalloc(&d_in, maxn * 2);
    if (err == cudaSuccess) err = cudaMalloc(&d_f, maxn * 4);
    if (err == cudaSuccess) err = cudaMalloc(&d_q, maxn);
    if (err == cudaSuccess) err = cudaMalloc(&d_s, (size_t)lay.Vp * 4 + (size_t)lay.L * 4 * lay.C * 4);
    const unsigned char* src = static_cast<const unsigned char*>(bf16_image) + 1024;
    unsigned char* dst = static_cast<unsigned char*>(out8);
    memcpy(dst, bf16_image, 1024);  // header unchanged (quantize.cu:199)
    dst += 1024;
    size_t sc_off[5], acc = 0;
    for (int g = 0; g < 5; g++) { sc_off[g] = acc; acc += (size_t)lay.M[g]; }
    for (int i = 0; i < 16 && err == cudaSuccess; i++) {
        const int g = kGroupOfTensor[i];
        if (g < 0) {  // non-Linear tensors stay BF16 (truncating the widened value is the identity)
            memcpy(dst, src, lay.n[i] * 2);
            dst += lay.n[i] * 2;
            src += lay.n[i] * 2;
            continue;
        }
        const size_t n = lay.n[i];
        err = cudaMemcpy(d_in, src, n * 2, cudaMemcpyHostToDevice);
        if (err != cudaSuccess) break;
        err = launch_k(widen_bf16_kernel, dim3(4 * sm_count()), dim3(256), 0, (cudaStream_t)0, false,
                       (const uint16_t*)d_in, d_f, n);
        if (err == cudaSuccess)
            err = fp8 ? launch_k(quant_rows_kernel<true>, dim3(lay.M[g]), dim3(kQThreads), 0, (cudaStream_t)0, false,
                                 (const float*)d_f, d_q, d_s, lay.M[g], lay.K[g])
                      : launch_k(quant_rows_kernel<false>, dim3(lay.M[g]), dim3(kQThreads), 0, (cudaStream_t)0, false,
                                 (const float*)d_f, d_q, d_s, lay.M[g], lay.K[g]);
        if (err == cudaSuccess) err = cudaMemcpy(dst, d_q, n, cudaMemcpyDeviceToHost);
        if (err == cudaSuccess) err = cudaMemcpy(scales + sc_off[g], d_s, (size_t)lay.M[g] * 4, cudaMemcpyDeviceToHost);
        dst += n;
        src += n * 2;
    }
    cudaFree(d_in);
    cudaFree(d_f);
    cudaFree(d_q);
    cudaFree(d_s);
    return status_from(err);
}

int gpt2b_quantize_file(const char* in_bf16_path, const char* out8_path, const char* scale_path, int fp8) {
    if (!in_bf16_path || !out8_path || !scale_path) return GPT2B_ERR_INVALID_ARG;
    FILE* f = fopen(in_bf16_path, "rb");
    if (!f) return GPT2B_ERR_FILE;
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz <= 0) { fclose(f); return GPT2B_ERR_FORMAT; }
    std::vector<unsigned char> img((size_t)sz);
    const size_t got = fread(img.data(), 1, (size_t)sz, f);
    fclose(f);
    if (got != (size_t)sz) return GPT2B_ERR_FILE;
    size_t ob = 0, ns = 0;
    int rc = gpt2b_quantized_size(img.data(), img.size(), &ob, &ns);
    if (rc) return rc;
    std::vector<unsigned char> out(ob);
    std::vector<float> sc(ns);
    rc = gpt2b_quantize_buffer(img.data(), img.size(), out.data(), sc.data(), fp8);
    if (rc) return rc;
    FILE* fo = fopen(out8_path, "wb");
    if (!fo) return GPT2B_ERR_FILE;
    const bool ok1 = fwrite(out.data(), 1, out.size(), fo) == out.size();
    fclose(fo);
    FILE* fs = fopen(scale_path, "wb");
    if (!fs) return GPT2B_ERR_FILE;
    const bool ok2 = fwrite(sc.data(), 4, sc.size(), fs) == sc.size();
    fclose(fs);
    return (ok1 && ok2) ? GPT2B_OK : GPT2B_ERR_FILE;
}

int gpt2b_quant_rows_i8(const float* W, uint8_t* W8, float* scale, int M, int K, gpt2b_stream_t stream) {
    if (M < 0 || K <= 0 || !W || !W8 || !scale) return GPT2B_ERR_INVALID_ARG;
    if (M == 0) return GPT2B_OK;
    return status_from(launch_k(quant_rows_kernel<false>, dim3(M), dim3(kQThreads), 0, (cudaStream_t)stream, false, W,
                                W8, scale, M, K));
}
int gpt2b_quant_rows_fp8(const float* W, uint8_t* W8, float* scale, int M, int K, gpt2b_stream_t stream) {
    if (M < 0 || K <= 0 || !W || !W8 || !scale) return GPT2B_ERR_INVALID_ARG;
    if (M == 0) return GPT2B_OK;
    return status_from(launch_k(quant_rows_kernel<true>, dim3(M), dim3(kQThreads), 0, (cudaStream_t)stream, false, W, W8, scale, M, K));
}
int gpt2b_dequant_wte_i8(const uint8_t* w8, const float* scale, uint16_t* out, int Vp, int C, gpt2b_stream_t stream) {
    if (Vp <= 0 || C <= 0 || !w8 || !scale || !out) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_k(dequant_rows_kernel<false>, dim3(4 * sm_count()), dim3(256), 0, (cudaStream_t)stream, false, w8, scale, (__nv_bfloat16*)out, Vp, C));
}
int gpt2b_dequant_wte_fp8(const uint8_t* w8, const float* scale, uint16_t* out, int Vp, int C,
                          gpt2b_stream_t stream) {
    if (Vp <= 0 || C <= 0 || !w8 || !scale || !out) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_k(dequant_rows_kernel<true>, dim3(4 * sm_count()), dim3(256), 0, (cudaStream_t)stream, false, w8, scale, (__nv_bfloat16*)out, Vp, C));
}

}  // extern "C"
