// prefill.cu -- the prompt as dense GEMMs on the 5th-generation tensor cores.
//
// The reference feeds a prompt through matmul_forward_cublaslt
// (Inference_gpt2/matmul.cuh:141-165; inference_gpt2.cu:431-458): for T
// prompt tokens every Linear layer is a [T x K] x [K x N] product.  Here that
// product is tc_gemm_kernel:
//   * a TMA producer warp streams 64-wide K slices of the activations (A,
//     T rows padded to the 128-row tile by the copy engine's zero fill) and of
//     the weights (B, BN rows) into a ring of shared-memory stages, both in the
//     128-byte-swizzled K-major layout the tensor core reads;
//   * one thread issues tcgen05.mma (kind::f16, BF16 x BF16 -> FP32, M = 128,
//     N = BN, K = 16 per instruction) into an accumulator in tensor memory, and
//     tcgen05.commit releases each stage when its products are done;
//   * 8-bit weights (INT8 / E4M3 codes) arrive as plain byte tiles and four
//     warps convert them to BF16 (exactly: every code is a BF16 value) into the
//     swizzled B stage before the MMA reads it; the row scale is applied in the
//     epilogue, as in the decode GEMVs;
//   * the same four warps then read the accumulator (tcgen05.ld, one TMEM lane
//     per token row) and apply scale, bias and tanh-GELU, rounding to BF16 (or
//     writing FP32 logits for the LM head).
// The GEMMs are weight-bandwidth bound at prompt lengths like 24 (each weight
// is read once and used T times), so tiles are narrow (BN = 16) to spread the
// weight rows of even the smallest matrix over many SMs.
//
// Around the GEMMs, small row kernels rebuild the decode path's arithmetic for
// all prompt positions at once: embedding + LayerNorm, residual + LayerNorm,
// the KV-cache append of every position (8-bit: the per-row amax/127|448 code
// of kv_cache_write_kernel_w8), and causal attention over the cached rows.
#include "common.cuh"
#include "internal.h"

#include <cudaTypedefs.h>
#include <float.h>

#include <mutex>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(prefill_device_error)

namespace {

constexpr int kTcM = 128;                  // token rows of one accumulator tile
constexpr int kTcK = 64;                   // K per stage: one 128-byte swizzle span of BF16
constexpr int kTcThreads = 192;            // warp 0: TMA; warp 1: MMA + TMEM; warps 2-5: convert + epilogue
constexpr int kTcABytes = kTcM * kTcK * 2; // 16 KB A tile per stage
constexpr int kRowThreads = 256;           // row kernels
constexpr int kRowMaxC = 2048;             // channels a row kernel holds in registers (8 per thread)

// ---------------------------------------------------------------------------
// tcgen05 / TMA building blocks (PTX ISA 8.7, sm_100a)
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor of a 1024-byte-aligned tile in the canonical
// K-major 128-byte-swizzle layout: rows 128 bytes apart, 8-row groups 1024
// bytes apart (stride byte offset), version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: FP32 accumulator, BF16 A and B, both K-major, N, M.
__host__ __device__ constexpr uint32_t bf16_idesc(int n, int m) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrives once on `bar` when every tcgen05.mma issued so far by this thread is complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
// 16 consecutive FP32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Eight 8-bit codes -> eight BF16 values (exact for every INT8 and E4M3 code).
template <int WK>
__device__ __forceinline__ uint4 codes8_to_bf16(uint2 w) {
    const uint32_t cw[2] = {w.x, w.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float a, b;
        const uint32_t word = cw[i >> 1];
        const int j = (i & 1) * 2;
        if constexpr (WK == WK_I8) {
            a = (float)(int8_t)((word >> (8 * j)) & 0xffu);
            b = (float)(int8_t)((word >> (8 * (j + 1))) & 0xffu);
        } else {
            a = e4m3_to_f(word, j);
            b = e4m3_to_f(word, j + 1);
        }
        const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
        o[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int WK, int BN, bool OUTF32>
struct TcCfg {
    static constexpr bool kW8 = WK != WK_BF16;
    static constexpr int kBBytes = BN * 128;                          // swizzled BF16 B tile
    static constexpr int kCBytes = kW8 ? ((BN * 64 + 1023) & ~1023) : 0;  // 8-bit code tile
    static constexpr int kStage = kTcABytes + kBBytes + kCBytes;      // multiple of 1024
    static constexpr int kNS = (BN >= 128) ? 3 : 4;                   // ring stages
    static constexpr uint32_t kCols = BN <= 32 ? 32u : (uint32_t)BN;  // TMEM columns (power of two >= 32)
    static constexpr int kSmem = kNS * kStage + 1024 /*alignment*/ + 256 /*barriers*/;
};

}  // namespace

// out[T x N] = epilogue(A[T x K] . W[N x K]^T): see the file comment.  Grid
// (ceil(N / BN), ceil(T / 128)).
template <int WK, int BN, bool OUTF32>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcGemmArgs g) {
    using Cfg = TcCfg<WK, BN, OUTF32>;
    constexpr int NS = Cfg::kNS;
    extern __shared__ unsigned char smraw[];
    // 1024-byte aligned base (the swizzle pattern is taken from address bits 4-9)
    const uint32_t raw = smem_addr(smraw);
    unsigned char* sm = smraw + (((raw + 1023u) & ~1023u) - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + NS * Cfg::kStage);
    uint64_t* empty = full + NS;
    uint64_t* conv = empty + NS;
    uint64_t* done = conv + NS;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kTcM;
    const int nk = (g.K + kTcK - 1) / kTcK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&conv[s], 128);
        }
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tslot, Cfg::kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int k = 0;
            for (; k < nk; k++) {
                const int s = k % NS;
                if (k >= NS && !mbar_wait(&empty[s], (uint32_t)((k / NS - 1) & 1))) break;
                unsigned char* st = sm + s * Cfg::kStage;
                mbar_arrive_expect_tx(&full[s], (uint32_t)(kTcABytes + (Cfg::kW8 ? BN * 64 : Cfg::kBBytes)));
                tma_load_2d(st, &tmA, k * kTcK, m0, &full[s]);
                tma_load_2d(st + kTcABytes + (Cfg::kW8 ? Cfg::kBBytes : 0), &tmB, k * kTcK, n0, &full[s]);
            }
            // leave with none of this thread's copies in flight
            for (int j = (k > NS ? k - NS : 0); j < k; j++) mbar_wait(&full[j % NS], (uint32_t)((j / NS) & 1));
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = bf16_idesc(BN, kTcM);
            for (int k = 0; k < nk; k++) {
                const int s = k % NS;
                if (!mbar_wait(Cfg::kW8 ? &conv[s] : &full[s], (uint32_t)((k / NS) & 1))) break;
                tc_fence_after();
                const uint32_t a = smem_addr(sm + s * Cfg::kStage);
                const uint64_t da = sw128_desc(a), db = sw128_desc(a + kTcABytes);
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; kk++)  // +32 bytes of K per instruction
                    tc_mma(tmem, da + 2 * kk, db + 2 * kk, idesc, (uint32_t)(k | kk));
                tc_commit(&empty[s]);
            }
            tc_commit(done);  // every product issued above is complete
        }
    } else {
        // ---------------- warps 2-5: 8-bit conversion, then the epilogue ----------------
        const int t = threadIdx.x - 64;
        if constexpr (Cfg::kW8) {
            for (int k = 0; k < nk; k++) {
                const int s = k % NS;
                mbar_wait(&full[s], (uint32_t)((k / NS) & 1));
                unsigned char* bt = sm + s * Cfg::kStage + kTcABytes;
                const unsigned char* codes = bt + Cfg::kBBytes;
                for (int id = t; id < BN * 8; id += 128) {  // row r, 16-byte chunk c of the BF16 row
                    const int r = id >> 3, c = id & 7;
                    const uint2 w = *reinterpret_cast<const uint2*>(codes + r * 64 + c * 8);
                    *reinterpret_cast<uint4*>(bt + r * 128 + ((c ^ (r & 7)) << 4)) = codes8_to_bf16<WK>(w);
                }
                // the tensor core reads shared memory through the async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive1(&conv[s]);
            }
        }
        mbar_wait(done, 0u);
        tc_fence_after();
        const int q = warp & 3;  // TMEM lanes 32q..32q+31 belong to this warp
        const int row = m0 + 32 * q + lane;
#pragma unroll 1
        for (int cb = 0; cb < BN / 16; cb++) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(cb * 16), v);
            if (row >= g.T) continue;
            const int nb = n0 + cb * 16;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int n = nb + j;
                if (n >= g.N) break;
                float x = v[j];
                if constexpr (Cfg::kW8) x *= g.scale[n];
                if constexpr (OUTF32) {
                    reinterpret_cast<float*>(g.out)[(size_t)row * g.ldo + n] = x;
                } else {
                    if (g.bias) x += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g.bias)[n]);
                    if (g.pre_gelu) reinterpret_cast<__nv_bfloat16*>(g.pre_gelu)[(size_t)row * g.ldo + n] = __float2bfloat16_rn(x);
                    if (g.do_gelu) x = gelu_tanh(x);
                    reinterpret_cast<__nv_bfloat16*>(g.out)[(size_t)row * g.ldo + n] = __float2bfloat16_rn(x);
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kCols);
    }
}

// ---------------------------------------------------------------------------
// row kernels of the prompt (one CTA per token row)
// ---------------------------------------------------------------------------
namespace {

// LayerNorm of the row r[] held by the block (two-pass, as layernorm_forward_kernel6), rounded to BF16.
__device__ __forceinline__ void block_ln(const float* r, int n, int C, const __nv_bfloat16* w,
                                         const __nv_bfloat16* b, __nv_bfloat16* out, float* scratch) {
    float s = 0.0f;
    for (int j = 0; j < n; j++) s += r[j];
    const float mean = block_sum(s, scratch) / (float)C;
    float q = 0.0f;
    for (int j = 0; j < n; j++) { const float d = r[j] - mean; q += d * d; }
    const float rstd = rsqrtf(block_sum(q, scratch) / (float)C + 1e-5f);
    for (int j = 0; j < n; j++) {
        const int c = threadIdx.x + j * kRowThreads;
        out[c] = __float2bfloat16_rn((rstd * (r[j] - mean)) * __bfloat162float(w[c]) + __bfloat162float(b[c]));
    }
}

}  // namespace

// res[t] = round(wte[tok_t] + wpe[t]) (encoder_forward_kv), x[t] = LN1 of layer 0.
template <int WK>
__global__ void __launch_bounds__(kRowThreads)
    prefill_embed_ln_kernel(__nv_bfloat16* res, __nv_bfloat16* x, const int* tokens, int V, const void* wte,
                            const float* wte_scale, const __nv_bfloat16* wpe, const __nv_bfloat16* lnw,
                            const __nv_bfloat16* lnb, int C) {
    __shared__ float scratch[32];
    const int t = blockIdx.x, tok = tokens[t];
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN);
        return;
    }
    float r[kRowMaxC / kRowThreads];
    int n = 0;
    for (int c = threadIdx.x; c < C; c += kRowThreads, n++) {
        float e;
        if constexpr (WK == WK_BF16) {
            e = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(wte)[(size_t)tok * C + c]);
        } else {
            const uint32_t code = reinterpret_cast<const uint8_t*>(wte)[(size_t)tok * C + c];
            const float v = (WK == WK_I8) ? (float)(int8_t)code : e4m3_to_f(code, 0);
            e = round_to<__nv_bfloat16>(v * wte_scale[tok]);
        }
        r[n] = round_to<__nv_bfloat16>(e + __bfloat162float(wpe[(size_t)t * C + c]));
        res[(size_t)t * C + c] = __float2bfloat16_rn(r[n]);
    }
    block_ln(r, n, C, lnw, lnb, x + (size_t)t * C, scratch);
}

// res[t] = round(res[t] + delta[t]) (fused_residual_forward5), x[t] = LN(res[t]).
__global__ void __launch_bounds__(kRowThreads)
    prefill_res_ln_kernel(__nv_bfloat16* res, const __nv_bfloat16* delta, __nv_bfloat16* x, const __nv_bfloat16* lnw,
                          const __nv_bfloat16* lnb, int C) {
    __shared__ float scratch[32];
    const int t = blockIdx.x;
    float r[kRowMaxC / kRowThreads];
    int n = 0;
    for (int c = threadIdx.x; c < C; c += kRowThreads, n++) {
        const size_t i = (size_t)t * C + c;
        r[n] = round_to<__nv_bfloat16>(__bfloat162float(res[i]) + __bfloat162float(delta[i]));
        res[i] = __float2bfloat16_rn(r[n]);
    }
    block_ln(r, n, C, lnw, lnb, x + (size_t)t * C, scratch);
}

// K and V of every prompt position into the cache (kv_cache_write_kernel(_w8)):
// grid (T, NH, 2), one warp per row of 64.
template <int KV>
__global__ void prefill_kv_append_kernel(const __nv_bfloat16* qkv, unsigned char* kv, float* kv_scale, int NH, int maxT) {
    const int t = blockIdx.x, h = blockIdx.y, which = blockIdx.z, lane = threadIdx.x;
    const int C = NH * 64;
    const __nv_bfloat16* src = qkv + (size_t)t * 3 * C + (size_t)(1 + which) * C + (size_t)h * 64;
    const size_t row = (size_t)which * NH * maxT + (size_t)h * maxT + t;
    const float v0 = __bfloat162float(src[lane]), v1 = __bfloat162float(src[lane + 32]);
    if constexpr (KV == KV_BF16) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(kv) + row * 64;
        dst[lane] = src[lane];
        dst[lane + 32] = src[lane + 32];
    } else {
        const float mx = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
        const float sc = mx / (KV == KV_FP8 ? 448.0f : 127.0f);
        uint8_t c0 = 0, c1 = 0;
        if (sc > 0.0f) {
            if constexpr (KV == KV_FP8) {
                c0 = (uint8_t)__nv_cvt_float_to_fp8(v0 / sc, __NV_SATFINITE, __NV_E4M3);
                c1 = (uint8_t)__nv_cvt_float_to_fp8(v1 / sc, __NV_SATFINITE, __NV_E4M3);
            } else {
                int q0 = __float2int_rn(v0 / sc), q1 = __float2int_rn(v1 / sc);
                c0 = (uint8_t)(int8_t)max(-127, min(127, q0));
                c1 = (uint8_t)(int8_t)max(-127, min(127, q1));
            }
        }
        kv[row * 64 + lane] = c0;
        kv[row * 64 + lane + 32] = c1;
        if (lane == 0) kv_scale[row] = sc;
    }
}

// Causal attention of prompt token t, head h over cached positions 0..t:
// grid (T, NH), 128 threads; scores and weights in shared memory (t + 1 floats).
template <int KV>
__global__ void __launch_bounds__(128)
    prefill_attention_kernel(const __nv_bfloat16* qkv, const unsigned char* kv, const float* kv_scale,
                             __nv_bfloat16* atty, int NH, int maxT, float attn_scale) {
    extern __shared__ float p[];
    __shared__ float qs[64], red[8];
    const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int C = NH * 64, n = t + 1;
    if (tid < 64) qs[tid] = __bfloat162float(qkv[(size_t)t * 3 * C + (size_t)h * 64 + tid]);
    __syncthreads();
    const size_t kbase = (size_t)h * maxT, vbase = (size_t)NH * maxT + (size_t)h * maxT;
    auto elem = [&](size_t row, int d) -> float {
        if constexpr (KV == KV_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(kv)[row * 64 + d]);
        else if constexpr (KV == KV_FP8) return e4m3_to_f((uint32_t)kv[row * 64 + d], 0);
        else return (float)(int8_t)kv[row * 64 + d];
    };
    for (int j = w; j < n; j += 4) {
        float d = qs[lane] * elem(kbase + j, lane) + qs[lane + 32] * elem(kbase + j, lane + 32);
        d = warp_sum(d);
        if (lane == 0) {
            if constexpr (KV != KV_BF16) d *= kv_scale[kbase + j];
            p[j] = d * attn_scale;
        }
    }
    __syncthreads();
    float mx = -FLT_MAX;
    for (int j = tid; j < n; j += 128) mx = fmaxf(mx, p[j]);
    mx = warp_max(mx);
    if (lane == 0) red[w] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float s = 0.0f;
    for (int j = tid; j < n; j += 128) {
        const float e = __expf(p[j] - mx);
        p[j] = e;
        s += e;
    }
    s = warp_sum(s);
    __syncthreads();
    if (lane == 0) red[4 + w] = s;
    __syncthreads();
    const float l = (red[4] + red[5]) + (red[6] + red[7]);
    if (tid < 64) {
        float o = 0.0f;
        for (int j = 0; j < n; j++) {
            float pv = p[j];
            if constexpr (KV != KV_BF16) pv *= kv_scale[vbase + j];
            o += pv * elem(vbase + j, tid);
        }
        atty[(size_t)t * C + (size_t)h * 64 + tid] = __float2bfloat16_rn(o / l);
    }
}

// The token after the prompt: greedy pick over row T-1 of the prompt logits,
// the engine's device state advanced as after T decode forwards (the history
// holds the prompt at positions 0..T-1 and the pick at T).
__global__ void __launch_bounds__(1024)
    prefill_pick_kernel(const float* logits_rows, int T, int V, int Vp, float* logits_last, int* d_token, int* d_pos,
                        int* history, const int* tokens) {
    for (int i = threadIdx.x; i < T; i += 1024) history[i] = tokens[i];
    const float* row = logits_rows + (size_t)(T - 1) * Vp;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < Vp; i += 1024) {
        const float v = row[i];
        logits_last[i] = v;
        if (i < V && v > bv) { bv = v; bi = i; }
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
        if (lane == 0) {
            if (bi < 0 || bi >= V) {  // no finite logit
                report_device_error(GPT2B_DEVERR_BAD_TOKEN);
                bi = 0;
            }
            *d_token = bi;
            *d_pos = T;
            history[T] = bi;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int WK, int BN, bool OUTF32>
cudaError_t launch_tc_t(const CUtensorMap& a, const CUtensorMap& b, const TcGemmArgs& g, cudaStream_t st) {
    using Cfg = TcCfg<WK, BN, OUTF32>;
    auto k = tc_gemm_kernel<WK, BN, OUTF32>;
    static unsigned long long mask = 0;
    cudaError_t e = ensure_smem_limit(k, &mask);
    if (e != cudaSuccess) return e;
    const dim3 grid((g.N + BN - 1) / BN, (g.T + kTcM - 1) / kTcM);
    return launch_k(k, grid, dim3(kTcThreads), (size_t)Cfg::kSmem, st, false, a, b, g);
}

}  // namespace

// A K-major 2-D tensor map (rows x cols, row pitch cols * esize) with a box of
// box_rows x box_cols; swizzled (128 B) for the BF16 operands, plain for 8-bit
// code tiles.  Rows and columns outside the tensor read as zero.
bool make_tensor_map(CUtensorMap* m, const void* base, int esize, uint64_t rows, uint64_t cols, uint32_t box_rows,
                     uint32_t box_cols, bool swizzle) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn || !aligned16(base) || (cols * esize) % 16 != 0) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (cuuint64_t)esize};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r =
        fn(m, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int tc_block_n(bool out_f32) { return out_f32 ? 128 : 16; }

// Maps of one GEMM: A = activations [rows x K] (BF16), B = weights [N x K].
bool tc_maps(CUtensorMap* a, CUtensorMap* b, int wk, const void* act, int act_rows, const void* W, int N, int K,
             bool out_f32) {
    const int bn = tc_block_n(out_f32);
    if (act && !make_tensor_map(a, act, 2, (uint64_t)act_rows, (uint64_t)K, kTcM, kTcK, true)) return false;
    if (W) {
        if (wk == WK_BF16) return make_tensor_map(b, W, 2, (uint64_t)N, (uint64_t)K, bn, kTcK, true);
        return make_tensor_map(b, W, 1, (uint64_t)N, (uint64_t)K, bn, kTcK, false);
    }
    return true;
}

cudaError_t launch_tc_gemm(int wk, const CUtensorMap& a, const CUtensorMap& b, const TcGemmArgs& g, bool out_f32,
                           cudaStream_t st) {
    if (g.T <= 0 || g.N <= 0) return cudaSuccess;
    if (out_f32) {
        if (wk == WK_BF16) return launch_tc_t<WK_BF16, 128, true>(a, b, g, st);
        if (wk == WK_I8) return launch_tc_t<WK_I8, 128, true>(a, b, g, st);
        if (wk == WK_FP8) return launch_tc_t<WK_FP8, 128, true>(a, b, g, st);
    } else {
        if (wk == WK_BF16) return launch_tc_t<WK_BF16, 16, false>(a, b, g, st);
        if (wk == WK_I8) return launch_tc_t<WK_I8, 16, false>(a, b, g, st);
        if (wk == WK_FP8) return launch_tc_t<WK_FP8, 16, false>(a, b, g, st);
    }
    return cudaErrorInvalidValue;
}

bool prefill_supported(int wk, int kvk, int C, int NH, int maxT) {
    return (wk == WK_BF16 || wk == WK_I8 || wk == WK_FP8) && kvk != KV_F32 && C == NH * 64 && C % 64 == 0 &&
           C <= kRowMaxC && maxT <= 4096 && encode_fn() != nullptr;
}

cudaError_t run_prefill(const PrefillPlan& P, int T, cudaStream_t st) {
    const int C = P.C, NH = P.NH;
    using BF = __nv_bfloat16;
    BF* res = reinterpret_cast<BF*>(P.res);
    BF* x = reinterpret_cast<BF*>(P.x);
    BF* qkv = reinterpret_cast<BF*>(P.qkv);
    BF* atty = reinterpret_cast<BF*>(P.atty);
    BF* proj = reinterpret_cast<BF*>(P.proj);
    BF* f = reinterpret_cast<BF*>(P.f);
    cudaError_t e;
    const dim3 rows(T);
    switch (P.wk) {
        case WK_BF16:
            e = launch_k(prefill_embed_ln_kernel<WK_BF16>, rows, dim3(kRowThreads), 0, st, false, res, x, P.tokens, P.V,
                         P.wte, P.wte_scale, (const BF*)P.wpe, (const BF*)P.layers[0].ln1w, (const BF*)P.layers[0].ln1b, C);
            break;
        case WK_I8:
            e = launch_k(prefill_embed_ln_kernel<WK_I8>, rows, dim3(kRowThreads), 0, st, false, res, x, P.tokens, P.V,
                         P.wte, P.wte_scale, (const BF*)P.wpe, (const BF*)P.layers[0].ln1w, (const BF*)P.layers[0].ln1b, C);
            break;
        default:
            e = launch_k(prefill_embed_ln_kernel<WK_FP8>, rows, dim3(kRowThreads), 0, st, false, res, x, P.tokens, P.V,
                         P.wte, P.wte_scale, (const BF*)P.wpe, (const BF*)P.layers[0].ln1w, (const BF*)P.layers[0].ln1b, C);
    }
    if (e != cudaSuccess) return e;
    const size_t attn_smem = (size_t)T * sizeof(float);
    for (int l = 0; l < P.L && e == cudaSuccess; l++) {
        const PrefillLayer& Ly = P.layers[l];
        TcGemmArgs g{};
        g.T = T;
        g.ldo = 3 * C;
        g.N = 3 * C;
        g.K = C;
        g.bias = Ly.qkvb;
        g.scale = Ly.s_qkv;
        g.out = qkv;
        if ((e = launch_tc_gemm(P.wk, P.a_x, Ly.w_qkv, g, false, st)) != cudaSuccess) break;
        const dim3 kvgrid(T, NH, 2), agrid(T, NH);
        if (P.kvk == KV_BF16) {
            e = launch_k(prefill_kv_append_kernel<KV_BF16>, kvgrid, dim3(32), 0, st, false, (const BF*)qkv, Ly.kv,
                         Ly.kv_scale, NH, P.maxT);
            if (e == cudaSuccess)
                e = launch_k(prefill_attention_kernel<KV_BF16>, agrid, dim3(128), attn_smem, st, false, (const BF*)qkv,
                             (const unsigned char*)Ly.kv, (const float*)Ly.kv_scale, atty, NH, P.maxT, P.attn_scale);
        } else if (P.kvk == KV_I8) {
            e = launch_k(prefill_kv_append_kernel<KV_I8>, kvgrid, dim3(32), 0, st, false, (const BF*)qkv, Ly.kv,
                         Ly.kv_scale, NH, P.maxT);
            if (e == cudaSuccess)
                e = launch_k(prefill_attention_kernel<KV_I8>, agrid, dim3(128), attn_smem, st, false, (const BF*)qkv,
                             (const unsigned char*)Ly.kv, (const float*)Ly.kv_scale, atty, NH, P.maxT, P.attn_scale);
        } else {
            e = launch_k(prefill_kv_append_kernel<KV_FP8>, kvgrid, dim3(32), 0, st, false, (const BF*)qkv, Ly.kv,
                         Ly.kv_scale, NH, P.maxT);
            if (e == cudaSuccess)
                e = launch_k(prefill_attention_kernel<KV_FP8>, agrid, dim3(128), attn_smem, st, false, (const BF*)qkv,
                             (const unsigned char*)Ly.kv, (const float*)Ly.kv_scale, atty, NH, P.maxT, P.attn_scale);
        }
        if (e != cudaSuccess) break;
        g.ldo = g.N = C;
        g.K = C;
        g.bias = Ly.projb;
        g.scale = Ly.s_proj;
        g.out = proj;
        if ((e = launch_tc_gemm(P.wk, P.a_atty, Ly.w_proj, g, false, st)) != cudaSuccess) break;
        e = launch_k(prefill_res_ln_kernel, rows, dim3(kRowThreads), 0, st, false, res, (const BF*)proj, x,
                     (const BF*)Ly.ln2w, (const BF*)Ly.ln2b, C);
        if (e != cudaSuccess) break;
        g.ldo = g.N = 4 * C;
        g.K = C;
        g.bias = Ly.fcb;
        g.scale = Ly.s_fc;
        g.out = f;
        g.do_gelu = 1;
        if ((e = launch_tc_gemm(P.wk, P.a_x, Ly.w_fc, g, false, st)) != cudaSuccess) break;
        g.do_gelu = 0;
        g.ldo = g.N = C;
        g.K = 4 * C;
        g.bias = Ly.fcprojb;
        g.scale = Ly.s_fcproj;
        g.out = proj;
        if ((e = launch_tc_gemm(P.wk, P.a_f, Ly.w_fcproj, g, false, st)) != cudaSuccess) break;
        const bool last = (l + 1 == P.L);
        e = launch_k(prefill_res_ln_kernel, rows, dim3(kRowThreads), 0, st, false, res, (const BF*)proj, x,
                     (const BF*)(last ? P.lnfw : P.layers[l + 1].ln1w), (const BF*)(last ? P.lnfb : P.layers[l + 1].ln1b),
                     C);
    }
    if (e != cudaSuccess) return e;
    // LM head over every prompt row (FP32 logits), then the pick after the prompt
    TcGemmArgs g{};
    g.T = T;
    g.N = P.Vp;
    g.K = C;
    g.ldo = P.Vp;
    g.scale = P.s_lm;
    g.out = P.logits_rows;
    if ((e = launch_tc_gemm(P.wk, P.a_x, P.w_lm, g, true, st)) != cudaSuccess) return e;
    return launch_k(prefill_pick_kernel, dim3(1), dim3(1024), 0, st, false, (const float*)P.logits_rows, T, P.V, P.Vp,
                    P.logits_last, P.d_token, P.d_pos, P.history, P.tokens);
}

}  // namespace gpt2b

using namespace gpt2b;

// ---------------------------------------------------------------------------
// C ABI: the prompt GEMM on its own (matmul_forward_cublaslt, matmul.cuh:141)
// ---------------------------------------------------------------------------
namespace {

int matmul_forward(int wk, void* out, const uint16_t* inp, const void* weight, const float* scale,
                   const uint16_t* bias, int B, int T, int C, int OC, uint16_t* pre_gelu, bool out_f32,
                   gpt2b_stream_t stream) {
    if (B <= 0 || T <= 0 || C <= 0 || OC <= 0 || !out || !inp || !weight) return GPT2B_ERR_INVALID_ARG;
    if (wk != WK_BF16 && !scale) return GPT2B_ERR_INVALID_ARG;
    if (!aligned16(inp) || !aligned16(weight) || (C * 2) % 16 != 0 || (wk != WK_BF16 && C % 16 != 0))
        return GPT2B_ERR_ALIGNMENT;
    CUtensorMap a, b;
    if (!tc_maps(&a, &b, wk, inp, B * T, weight, OC, C, out_f32)) return GPT2B_ERR_UNSUPPORTED;
    TcGemmArgs g{};
    g.T = B * T;
    g.N = OC;
    g.K = C;
    g.ldo = OC;
    g.bias = out_f32 ? nullptr : bias;
    g.scale = scale;
    g.out = out;
    g.pre_gelu = out_f32 ? nullptr : pre_gelu;
    g.do_gelu = (!out_f32 && pre_gelu) ? 1 : 0;
    return status_from(launch_tc_gemm(wk, a, b, g, out_f32, (cudaStream_t)stream));
}

}  // namespace

extern "C" {

int gpt2b_matmul_forward_bf16(uint16_t* out, const uint16_t* inp, const uint16_t* weight, const uint16_t* bias, int B,
                              int T, int C, int OC, uint16_t* pre_gelu, gpt2b_stream_t stream) {
    return matmul_forward(WK_BF16, out, inp, weight, nullptr, bias, B, T, C, OC, pre_gelu, false, stream);
}
int gpt2b_matmul_forward_f32out_bf16(float* out, const uint16_t* inp, const uint16_t* weight, int B, int T, int C,
                                     int OC, gpt2b_stream_t stream) {
    return matmul_forward(WK_BF16, out, inp, weight, nullptr, nullptr, B, T, C, OC, nullptr, true, stream);
}
int gpt2b_matmul_forward_w8_i8(uint16_t* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                               const uint16_t* bias, int B, int T, int C, int OC, uint16_t* pre_gelu,
                               gpt2b_stream_t stream) {
    return matmul_forward(WK_I8, out, inp, weight, scale, bias, B, T, C, OC, pre_gelu, false, stream);
}
int gpt2b_matmul_forward_w8_fp8(uint16_t* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                const uint16_t* bias, int B, int T, int C, int OC, uint16_t* pre_gelu,
                                gpt2b_stream_t stream) {
    return matmul_forward(WK_FP8, out, inp, weight, scale, bias, B, T, C, OC, pre_gelu, false, stream);
}
int gpt2b_matmul_forward_w8_i8_f32out(float* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                      int B, int T, int C, int OC, gpt2b_stream_t stream) {
    return matmul_forward(WK_I8, out, inp, weight, scale, nullptr, B, T, C, OC, nullptr, true, stream);
}
int gpt2b_matmul_forward_w8_fp8_f32out(float* out, const uint16_t* inp, const uint8_t* weight, const float* scale,
                                       int B, int T, int C, int OC, gpt2b_stream_t stream) {
    return matmul_forward(WK_FP8, out, inp, weight, scale, nullptr, B, T, C, OC, nullptr, true, stream);
}

}  // extern "C"
