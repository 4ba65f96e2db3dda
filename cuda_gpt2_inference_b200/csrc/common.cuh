// common.cuh -- device and launch helpers shared by every kernel of the library.
//
// B200 (sm_100a) building blocks used throughout:
//   * 1-D bulk async copies global -> shared (cp.async.bulk) completing on an
//     mbarrier: one elected thread moves a whole contiguous weight tile, so the
//     copy engine, not 256 threads, carries the bytes and the copy can be issued
//     before the kernel waits on its predecessor;
//   * programmatic dependent launch (griddepcontrol): a kernel issues its
//     weight copies, then waits for the previous kernel's outputs;
//   * every spin-wait is bounded and reports through a device error word.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/gpt2_b200.h"

namespace gpt2b {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// error reporting from device code
// ---------------------------------------------------------------------------
// One error word per translation unit (no relocatable device code needed);
// gpt2b_device_error() reads and clears all of them.
static __device__ int g_device_error = 0;

__device__ __forceinline__ void report_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// Host side: read-and-clear this translation unit's error word.
#define GPT2B_DEFINE_ERROR_READER(fn)                                      \
    int fn() {                                                              \
        int v = 0, z = 0;                                                   \
        if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1; \
        if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));         \
        return v;                                                           \
    }

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------
// Blocks until every grid this one depends on has completed and its memory
// is visible.  A no-op when the launch carried no programmatic dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream start launching.  Called right after
// pdl_wait so at most two kernels of a stream overlap: the running one and
// the next one staging its weights.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (PTX ISA: mbarrier.*, cp.async.bulk)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on an mbarrier phase.  Returns false (and records
// GPT2B_DEVERR_MBAR_TIMEOUT) when the phase does not complete within about
// two seconds (a try_wait may suspend the thread for a while, so the bound is
// taken on %globaltimer, with an iteration cap behind it).
constexpr uint32_t kMbarSpinLimit = 1u << 24;
constexpr uint64_t kMbarTimeoutNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && global_ns() - t0 > kMbarTimeoutNs) break;
    }
    report_device_error(GPT2B_DEVERR_MBAR_TIMEOUT);
    return false;
}
// 1-D bulk copy global -> this CTA's shared memory; completes `bytes` of
// transaction count on `bar`.  Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// The same with an L2 cache policy (from createpolicy) on the read lines.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
// L2 policy: lines read under it are evicted after evict_normal lines of the same set.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Hint: pull a global range into L2 ahead of use (no completion tracking).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// number formats
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f_to_bf16(float v) { return __float2bfloat16_rn(v); }

// Storage-type conversions used by templates over the activation type.
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
// Round a float through the storage type (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float v) { return to_f<T>(from_f<T>(v)); }

// INT8 code (two's complement) of byte j of a 32-bit word -> exact float.
// The byte, sign-flipped, becomes the low mantissa bits of 2^23; subtracting
// 2^23 + 128 recovers the signed value.  One byte-permute and one add.
__device__ __forceinline__ float i8_to_f(uint32_t word_xor80, int j) {
    const uint32_t sel = 0x7540u + (uint32_t)j;
    return __uint_as_float(__byte_perm(word_xor80, 0x4B000000u, sel)) - 8388736.0f;
}
// E4M3 code (byte j of a word) -> exact float.  The 7 magnitude bits are
// placed so that the float exponent field reads e and the mantissa reads m,
// then a multiply by 2^120 rebases the exponent (bias 127 -> 7).  The multiply
// is written without .ftz so subnormal E4M3 codes (e == 0) stay exact under
// --use_fast_math.
__device__ __forceinline__ float e4m3_to_f(uint32_t word, int j) {
    const uint32_t b = (word >> (8 * j)) & 0xffu;
    const uint32_t bits = ((b & 0x7fu) << 20) | ((b & 0x80u) << 24);
    float r;
    asm("mul.rn.f32 %0, %1, 0f7B800000;" : "=f"(r) : "f"(__uint_as_float(bits)));
    return r;
}

// ---------------------------------------------------------------------------
// legacy tensor-core tiles (mma.sync m16n8k16, FP32 accumulation) for the
// 8-bit weight streams: ldmatrix of 16 code rows, codes -> exact FP16 pairs
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Two codes of a 32-bit word (bytes 0-1 for hi = false, 2-3 for hi = true) as an
// exact FP16 pair.  INT8: the sign-flipped byte under the FP16 exponent of 1024
// reads 1024 + code + 128; subtracting 1152 leaves the code.  E4M3: the 7
// magnitude bits placed as FP16 exponent/mantissa read 2^(e-15) x 1.m (or the
// FP16 subnormal for e = 0); a multiply by 2^8 rebases the exponent.
template <bool kFp8>
__device__ __forceinline__ uint32_t code2_to_f16x2(uint32_t word, bool hi) {
    uint32_t r;
    if constexpr (!kFp8) {
        const uint32_t h = __byte_perm(word ^ 0x80808080u, 0x64646464u, hi ? 0x4342u : 0x4140u);
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
    } else {
        const uint32_t w = __byte_perm(word, 0u, hi ? 0x3424u : 0x1404u);  // bytes -> bits 8..15 / 24..31
        const uint32_t f = (w & 0x80008000u) | ((w & 0x7f007f00u) >> 1);
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(f), "r"(0x5c005c00u));
    }
    return r;
}

// GPT-2 tanh GELU, the expression of the reference epilogue.
__device__ __forceinline__ float gelu_tanh(float x) {
    float cube = 0.044715f * x * x * x;
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + cube)));
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// All-reduce over the whole block through `scratch` (>= 32 floats).  Every
// thread returns the total.  Ends with a barrier so scratch can be reused.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    if (lane == 0) scratch[w] = v;
    __syncthreads();
    float t = (lane < nw) ? scratch[lane] : 0.0f;
    t = warp_sum(t);
    __syncthreads();
    return t;
}

}  // namespace gpt2b

// ---------------------------------------------------------------------------
// host-side launch helpers
// ---------------------------------------------------------------------------
namespace gpt2b {

// Launch with (optionally) the programmatic-stream-serialization attribute.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

int sm_count();                   // SMs of the current device (cached per device)
int max_dyn_smem();               // opt-in dynamic shared memory per block (cached per device)
int status_from(cudaError_t e);   // 0 or GPT2B_ERR_CUDA + code

// Raise a kernel's dynamic shared-memory limit to the device maximum (minus
// the kernel's static shared memory), once per device (bit d of *mask).  A
// single maximal setting keeps every launch and every captured graph node
// valid whatever size it requests.
template <typename Kernel>
inline cudaError_t ensure_smem_limit(Kernel k, unsigned long long* mask) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (*mask & bit) return cudaSuccess;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_dyn_smem() - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) *mask |= bit;
    return e;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace gpt2b
