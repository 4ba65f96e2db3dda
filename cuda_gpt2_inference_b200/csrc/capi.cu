// capi.cu -- library-wide C entry points: status strings, device error word,
// device queries shared by the launchers.
#include "common.cuh"
#include "internal.h"

#include <mutex>

namespace gpt2b {

int sm_count() {
    static int cache[64] = {0};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int max_dyn_smem() {
    static int cache[64] = {0};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 227 * 1024;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || n <= 0)
            n = 227 * 1024;
        cache[dev] = n;
    }
    return cache[dev];
}

int status_from(cudaError_t e) { return e == cudaSuccess ? GPT2B_OK : GPT2B_ERR_CUDA + (int)e; }

}  // namespace gpt2b

using namespace gpt2b;

extern "C" {

int gpt2b_version(void) { return 100; }

const char* gpt2b_status_string(int s) {
    switch (s) {
        case GPT2B_OK: return "ok";
        case GPT2B_ERR_INVALID_ARG: return "invalid argument";
        case GPT2B_ERR_ALIGNMENT: return "pointer or row pitch not 16-byte aligned";
        case GPT2B_ERR_UNSUPPORTED: return "unsupported shape or mode";
        case GPT2B_ERR_FILE: return "file missing or unreadable";
        case GPT2B_ERR_FORMAT: return "malformed weight image (magic, version, header or size)";
        case GPT2B_ERR_DEVICE: return "a kernel reported a device error word";
        case GPT2B_ERR_NCCL: return "collective failed or timed out";
    }
    if (s > GPT2B_ERR_CUDA) return cudaGetErrorString((cudaError_t)(s - GPT2B_ERR_CUDA));
    return "unknown status";
}

int gpt2b_device_error(int* code) {
    if (!code) return GPT2B_ERR_INVALID_ARG;
    const int v[5] = {gemv_device_error(), attention_device_error(), norm_device_error(), sampler_device_error(),
                      persistent_device_error()};
    *code = 0;
    for (int x : v) {
        if (x < 0) return GPT2B_ERR_CUDA;
        if (x && !*code) *code = x;
    }
    return GPT2B_OK;
}

}  // extern "C"
