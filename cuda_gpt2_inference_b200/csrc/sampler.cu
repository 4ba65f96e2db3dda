// sampler.cu -- token selection over float logits.
//
// gpu_sample_softmax keeps the reference's sampling definition
// (Inference_gpt2/sampler_gpu.cuh:10-87) so a given (seed, step) picks the same
// token: the cumulative distribution is ordered by thread segment (thread t of
// 256 owns indices t, t+256, ...), segment sums are formed in that order, the
// total is the same two-level butterfly sum, and the uniform draw is curand's
// Philox4_32_10 with (seed, subsequence = row, offset = step).  The float
// operation order has to match for the picks to match, so the steps are alike.
//
// gpu_argmax is new (the reference has no greedy pick): largest logit, lowest
// index on ties, 1024 threads per row.
#include "common.cuh"
#include "internal.h"

#include <curand_kernel.h>
#include <float.h>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(sampler_device_error)

constexpr int kSampThreads = 256;

__global__ void __launch_bounds__(kSampThreads)
    sample_softmax_kernel(int* out_token, const float* logits, int B, int V, unsigned long long seed, int step) {
    const int b = blockIdx.x;
    if (b >= B) return;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    __shared__ float seg[kSampThreads];
    __shared__ float wbuf[kSampThreads / 32];
    __shared__ float s_max, s_sum, s_u;
    __shared__ int s_pick;
    const float* row = logits + (size_t)b * V;

    float mx = -FLT_MAX;
    for (int i = tid; i < V; i += kSampThreads) mx = fmaxf(mx, row[i]);
    mx = warp_max(mx);
    if (lane == 0) wbuf[w] = mx;
    __syncthreads();
    if (tid < 8) {
        float v = wbuf[tid];
        for (int o = 4; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffu, v, o));
        if (tid == 0) s_max = v;
    }
    __syncthreads();
    const float m = s_max;

    float mine = 0.0f;
    for (int i = tid; i < V; i += kSampThreads) mine += expf(row[i] - m);
    seg[tid] = mine;
    float ws = warp_sum(mine);
    if (lane == 0) wbuf[w] = ws;
    __syncthreads();
    if (tid < 8) {
        float v = wbuf[tid];
        for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffu, v, o);
        if (tid == 0) { s_sum = v; s_pick = V - 1; }
    }
    __syncthreads();
    if (tid == 0) {
        curandStatePhilox4_32_10_t rng;
        curand_init(seed, (unsigned long long)b, (unsigned long long)step, &rng);
        s_u = curand_uniform(&rng) * s_sum;
        float run = 0.0f;  // exclusive prefix over the thread segments
        for (int j = 0; j < kSampThreads; j++) {
            const float v = seg[j];
            seg[j] = run;
            run += v;
        }
    }
    __syncthreads();
    const float lo = seg[tid], hi = lo + mine, u = s_u;
    if (u >= lo && u < hi) {
        float run = lo;
        for (int i = tid; i < V; i += kSampThreads) {
            run += expf(row[i] - m);
            if (run >= u) { s_pick = i; break; }
        }
    }
    __syncthreads();
    if (tid == 0) out_token[b] = s_pick;
}

constexpr int kArgThreads = 1024;

__global__ void __launch_bounds__(kArgThreads) argmax_kernel(int* out_token, const float* logits, int V, int ld) {
    const float* row = logits + (size_t)blockIdx.x * ld;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += kArgThreads) {
        const float v = row[i];
        if (v > bv) { bv = v; bi = i; }  // increasing i per thread: keeps the lowest index on ties
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        bv = sv[lane];
        bi = si[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) out_token[blockIdx.x] = (bi == 0x7fffffff) ? 0 : bi;
    }
}

constexpr int kNllThreads = 1024;

// Negative log-likelihood of one token under softmax(logits[0..V)): the
// reference's ppl_record_nll (Inference_gpt2/dump_utils.h:63-79) on the
// device, with no logits copy to the host.  The maximum, the sum of
// exp(l - max) accumulated in double, nll = max + log(sum) - l[token].
// The token is *tok (hist null; result in out[0]) or hist[p], the token the
// engine appended at position p (result in out[p - 1]), with p = *pos, or
// fixed_pos when pos is null.
__global__ void __launch_bounds__(kNllThreads)
    nll_kernel(float* out, const float* logits, int V, const int* tok, const int* hist, const int* pos, int fixed_pos) {
    __shared__ float smx[32];
    __shared__ double ssum[32];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float mx = -FLT_MAX;
    for (int i = tid; i < V; i += kNllThreads) mx = fmaxf(mx, logits[i]);
    mx = warp_max(mx);
    if (lane == 0) smx[w] = mx;
    __syncthreads();
    mx = smx[0];
    for (int k = 1; k < kNllThreads / 32; k++) mx = fmaxf(mx, smx[k]);
    double s = 0.0;
    for (int i = tid; i < V; i += kNllThreads) s += exp((double)logits[i] - (double)mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) ssum[w] = s;
    __syncthreads();
    if (tid == 0) {
        double total = 0.0;
        for (int k = 0; k < kNllThreads / 32; k++) total += ssum[k];
        const int p = pos ? *pos : fixed_pos;
        const int t = hist ? hist[p] : *tok;
        if (t < 0 || t >= V || (hist && p < 1)) {
            report_device_error(GPT2B_DEVERR_BAD_TOKEN);
            return;
        }
        out[hist ? p - 1 : 0] = (float)((double)mx + log(total) - (double)logits[t]);
    }
}

cudaError_t launch_nll(float* out, const float* logits, int V, const int* tok, const int* hist, const int* pos,
                       int fixed_pos, cudaStream_t st) {
    return launch_k(nll_kernel, dim3(1), dim3(kNllThreads), 0, st, false, out, logits, V, tok, hist, pos, fixed_pos);
}

}  // namespace gpt2b

using namespace gpt2b;

extern "C" {

int gpt2b_gpu_sample_softmax(int* d_token, const float* logits, int B, int V, unsigned long long seed, int step,
                             gpt2b_stream_t stream) {
    if (B <= 0 || V <= 0 || !d_token || !logits) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_k(sample_softmax_kernel, dim3(B), dim3(kSampThreads), 0, (cudaStream_t)stream, false, d_token, logits, B, V, seed, step));
}

int gpt2b_logits_nll(float* d_nll, const float* logits, int V, const int* d_token, gpt2b_stream_t stream) {
    if (V <= 0 || !d_nll || !logits || !d_token) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_nll(d_nll, logits, V, d_token, nullptr, nullptr, 0, (cudaStream_t)stream));
}

int gpt2b_gpu_argmax(int* d_token, const float* logits, int B, int V, int ld, gpt2b_stream_t stream) {
    if (B <= 0 || V <= 0 || ld < V || !d_token || !logits) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_k(argmax_kernel, dim3(B), dim3(kArgThreads), 0, (cudaStream_t)stream, false, d_token, logits, V, ld));
}

}  // extern "C"
