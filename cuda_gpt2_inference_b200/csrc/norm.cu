// norm.cu -- LayerNorm, fused residual + LayerNorm, and the decode embedding.
//
// Decode rows are single tokens (N = B*T rows of C channels), so these are
// latency kernels: one warp per row holds the row in registers (C <= 2048),
// two shuffle all-reduces give mean and variance, no shared memory and no
// block barrier.  The engine folds the same math into the GEMV prologues; these
// kernels are the standalone operator surface.
#include "common.cuh"
#include "internal.h"

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(norm_device_error)

constexpr int kNormWarps = 4;
constexpr int kNormMaxPer = 64;  // C <= 64 * 32

// residual (optional) + LayerNorm of one row per warp.  With inp2 == nullptr
// this is layernorm_forward (layernorm.cuh:94-159); otherwise
// fused_residual_forward_kernel5 (layernorm.cuh:171-241): the sum is stored in
// the storage type and the LayerNorm reads the stored (rounded) values.
template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32)
    ln_rows_kernel(T* residual, T* normed, float* mean, float* rstd, const T* inp1, const T* inp2,
                   const T* weight, const T* bias, int N, int C) {
    const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    const T* a = inp1 + (size_t)row * C;
    const T* b = inp2 ? inp2 + (size_t)row * C : nullptr;
    float v[kNormMaxPer];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kNormMaxPer; i++) {
        const int c = lane + 32 * i;
        float x = 0.0f;
        if (c < C) {
            x = to_f<T>(a[c]);
            if (b) {
                x = round_to<T>(x + to_f<T>(b[c]));
                residual[(size_t)row * C + c] = from_f<T>(x);
            }
            sum += x;
        }
        v[i] = x;
    }
    const float m = warp_sum(sum) / (float)C;
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < kNormMaxPer; i++) {
        const int c = lane + 32 * i;
        if (c < C) { const float d = v[i] - m; sq += d * d; }
    }
    const float s = rsqrtf(warp_sum(sq) / (float)C + 1e-5f);
#pragma unroll
    for (int i = 0; i < kNormMaxPer; i++) {
        const int c = lane + 32 * i;
        if (c < C) normed[(size_t)row * C + c] = from_f<T>((s * (v[i] - m)) * to_f<T>(weight[c]) + to_f<T>(bias[c]));
    }
    if (lane == 0) {
        if (mean) mean[row] = m;
        if (rstd) rstd[row] = s;
    }
}

// out[b] = wte[inp[b]] + wpe[*d_pos]   (encoder.cuh:67-85)
template <typename T>
__global__ void encoder_kv_kernel(T* out, const int* inp, const T* wte, const T* wpe, const int* d_pos, int B, int C,
                                  int V, int maxT) {
    const int b = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B || c >= C) return;
    int pos = *d_pos, tok = inp[b];
    if (pos < 0 || pos >= maxT) { if (c == 0) report_device_error(GPT2B_DEVERR_BAD_POS); return; }
    if (V > 0 && (tok < 0 || tok >= V)) { if (c == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN); return; }
    out[(size_t)b * C + c] = from_f<T>(to_f<T>(wte[(size_t)tok * C + c]) + to_f<T>(wpe[(size_t)pos * C + c]));
}

template <typename T>
static int ln_entry(T* residual, T* normed, float* mean, float* rstd, const T* in1, const T* in2, const T* w,
                    const T* b, int N, int C, cudaStream_t st) {
    if (N < 0 || C <= 0 || !normed || !in1 || !w || !b || (in2 && !residual)) return GPT2B_ERR_INVALID_ARG;
    if (C > kNormMaxPer * 32) return GPT2B_ERR_UNSUPPORTED;
    if (N == 0) return GPT2B_OK;
    return status_from(launch_k(ln_rows_kernel<T>, dim3((N + kNormWarps - 1) / kNormWarps), dim3(kNormWarps * 32), 0, st, false, residual, normed, mean, rstd,
                                                                                    in1, in2, w, b, N, C));
}

template <typename T>
static int enc_entry(T* out, const int* inp, const T* wte, const T* wpe, const int* d_pos, int B, int C,
                     cudaStream_t st) {
    if (B <= 0 || C <= 0 || !out || !inp || !wte || !wpe || !d_pos) return GPT2B_ERR_INVALID_ARG;
    dim3 grid((C + 255) / 256, B);
    return status_from(launch_k(encoder_kv_kernel<T>, dim3(grid), dim3(256), 0, st, false, out, inp, wte, wpe, d_pos, B, C, 0, 1 << 30));
}

}  // namespace gpt2b

using namespace gpt2b;
typedef __nv_bfloat16 bf16_t;

extern "C" {

int gpt2b_layernorm_forward_f32(float* out, float* mean, float* rstd, const float* inp, const float* weight,
                                const float* bias, int B, int T, int C, gpt2b_stream_t stream) {
    return ln_entry<float>(nullptr, out, mean, rstd, inp, nullptr, weight, bias, B * T, C, (cudaStream_t)stream);
}
int gpt2b_layernorm_forward_bf16(uint16_t* out, float* mean, float* rstd, const uint16_t* inp, const uint16_t* weight,
                                 const uint16_t* bias, int B, int T, int C, gpt2b_stream_t stream) {
    return ln_entry<bf16_t>(nullptr, (bf16_t*)out, mean, rstd, (const bf16_t*)inp, nullptr, (const bf16_t*)weight,
                            (const bf16_t*)bias, B * T, C, (cudaStream_t)stream);
}
int gpt2b_fused_residual_forward5_f32(float* residual, float* normed, float* mean, float* rstd, const float* inp1,
                                      const float* inp2, const float* weight, const float* bias, int N, int C,
                                      gpt2b_stream_t stream) {
    if (!inp2) return GPT2B_ERR_INVALID_ARG;
    return ln_entry<float>(residual, normed, mean, rstd, inp1, inp2, weight, bias, N, C, (cudaStream_t)stream);
}
int gpt2b_fused_residual_forward5_bf16(uint16_t* residual, uint16_t* normed, float* mean, float* rstd,
                                       const uint16_t* inp1, const uint16_t* inp2, const uint16_t* weight,
                                       const uint16_t* bias, int N, int C, gpt2b_stream_t stream) {
    if (!inp2) return GPT2B_ERR_INVALID_ARG;
    return ln_entry<bf16_t>((bf16_t*)residual, (bf16_t*)normed, mean, rstd, (const bf16_t*)inp1, (const bf16_t*)inp2,
                            (const bf16_t*)weight, (const bf16_t*)bias, N, C, (cudaStream_t)stream);
}
int gpt2b_encoder_forward_kv_f32(float* out, const int* inp, const float* wte, const float* wpe, const int* d_pos,
                                 int B, int C, gpt2b_stream_t stream) {
    return enc_entry<float>(out, inp, wte, wpe, d_pos, B, C, (cudaStream_t)stream);
}
int gpt2b_encoder_forward_kv_bf16(uint16_t* out, const int* inp, const uint16_t* wte, const uint16_t* wpe,
                                  const int* d_pos, int B, int C, gpt2b_stream_t stream) {
    return enc_entry<bf16_t>((bf16_t*)out, inp, (const bf16_t*)wte, (const bf16_t*)wpe, d_pos, B, C,
                             (cudaStream_t)stream);
}

}  // extern "C"
