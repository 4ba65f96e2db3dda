// attention.cu -- KV-cache append and flash-decoding attention (B200).
//
// KV layout is the reference's (attention_kvcache.cuh:8-13): per layer
// [K | V], each B*NH*maxT*hs, element (b,h,j,d) at ((b*NH+h)*maxT + j)*hs + d;
// 8-bit scales per (K/V, b, h, j) (attention_kvcache_w8.cuh:129-131).
//
// One kernel template serves every mode.  A CTA owns a contiguous position
// range of one head.  K rows (and V rows, and 8-bit row scales) of that range
// are contiguous in memory, so a single thread stages a sub-chunk of up to CH
// positions with cp.async.bulk into shared memory (two-stage ring), and the
// CTA runs an online softmax over its sub-chunks:
//   scores: LP lanes per K row (one 16-byte slice each), shuffle-reduced;
//   V:      the same 16-byte slices, each thread accumulating its dims over a
//           strided set of rows, reduced across row groups at the end.
// Modes:
//   SINGLE  one CTA per head covers [0, pos]           (attention_forward_kv_small)
//   SPLIT   reference chunking, partials to the caller  (split kernel of _large)
//   ENGINE  the decode engine: K/V staging issued before griddepcontrol.wait
//           (rows < pos were written by earlier tokens), the CTA that owns
//           position pos appends the current token's K/V (quantising for 8-bit
//           KV) to global memory and to its staged copy, and every CTA writes
//           its split partials; the projection GEMV that follows merges them in
//           its prologue, so no merge launch, atomic or fence is needed here.
#include "common.cuh"
#include "internal.h"

#include <float.h>
#include <mutex>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(attention_device_error)

constexpr int kAttnThreads = 256;
constexpr int kHS = 64;  // head size the kernels are built for (the reference fixes it too)

enum AttnMode { AM_SINGLE = 0, AM_SPLIT = 1, AM_ENGINE = 2 };

template <int KV> struct KvT;
template <> struct KvT<KV_F32> { using XT = float; static constexpr int kB = 4; static constexpr int kCH = 64; };
template <> struct KvT<KV_BF16> { using XT = __nv_bfloat16; static constexpr int kB = 2; static constexpr int kCH = 128; };
template <> struct KvT<KV_I8> { using XT = __nv_bfloat16; static constexpr int kB = 1; static constexpr int kCH = 128; };
template <> struct KvT<KV_FP8> { using XT = __nv_bfloat16; static constexpr int kB = 1; static constexpr int kCH = 128; };

// ---------------------------------------------------------------------------
// 8-bit KV encode: the expressions of attention_kvcache_w8.cuh:56-65,147-154
// under the same --use_fast_math build, so codes match the reference kernel.
// ---------------------------------------------------------------------------
template <int KV>
__device__ __forceinline__ uint8_t kv8_encode(float x, float scale) {
    if constexpr (KV == KV_FP8) {
        return (uint8_t)__nv_cvt_float_to_fp8(x / scale, __NV_SATFINITE, __NV_E4M3);
    } else {
        int q = __float2int_rn(x / scale);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        return (uint8_t)(int8_t)q;
    }
}
template <int KV> __device__ __forceinline__ float kv8_limit() { return KV == KV_FP8 ? 448.0f : 127.0f; }
template <int KV> __device__ __forceinline__ float kv8_decode(uint32_t word, int j) {
    if constexpr (KV == KV_FP8) return e4m3_to_f(word, j);
    else return (float)(int8_t)((word >> (8 * j)) & 0xffu);
}

// ---------------------------------------------------------------------------
// KV append (boundary kernels)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void kv_write_kernel(T* kv, const T* qkv, int B, int NH, int hs, int maxT, const int* d_pos) {
    const int pos = *d_pos;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * NH * hs) return;
    if (pos < 0 || pos >= maxT) { if (idx == 0) report_device_error(GPT2B_DEVERR_BAD_POS); return; }
    const int b = idx / (NH * hs), rest = idx % (NH * hs), h = rest / hs, d = rest % hs;
    const size_t src = (size_t)b * 3 * NH * hs + (size_t)h * hs + d;
    const size_t dst = ((size_t)b * NH + h) * maxT * hs + (size_t)pos * hs + d;
    kv[dst] = qkv[src + (size_t)NH * hs];
    kv[(size_t)B * NH * maxT * hs + dst] = qkv[src + 2 * (size_t)NH * hs];
}

// One warp per (K|V, b, h) row: amax over hs bf16 values, scale = amax/LIMIT,
// codes (zero when the scale is 0).
template <int KV>
__global__ void kv_write_w8_kernel(uint8_t* kv, float* kv_scale, const __nv_bfloat16* qkv, int B, int NH, int hs,
                                   int maxT, const int* d_pos) {
    const int pos = *d_pos;
    const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= B * NH * 2) return;
    if (pos < 0 || pos >= maxT) { if (row == 0 && lane == 0) report_device_error(GPT2B_DEVERR_BAD_POS); return; }
    const bool is_v = row >= B * NH;
    const int kh = row - (is_v ? B * NH : 0), b = kh / NH, h = kh % NH;
    const __nv_bfloat16* src = qkv + (size_t)b * 3 * NH * hs + (size_t)h * hs + (is_v ? 2 : 1) * (size_t)NH * hs;
    float mx = 0.0f;
    for (int d = lane; d < hs; d += 32) mx = fmaxf(mx, fabsf(__bfloat162float(src[d])));
    mx = warp_max(mx);
    const float scale = mx / kv8_limit<KV>();
    uint8_t* dst = kv + (is_v ? (size_t)B * NH * maxT * hs : 0) + (size_t)kh * maxT * hs + (size_t)pos * hs;
    if (lane == 0) kv_scale[(is_v ? (size_t)B * NH * maxT : 0) + (size_t)kh * maxT + pos] = scale;
    for (int d = lane; d < hs; d += 32)
        dst[d] = (scale > 0.0f) ? kv8_encode<KV>(__bfloat162float(src[d]), scale) : (uint8_t)0;
}

// ---------------------------------------------------------------------------
// attention core
// ---------------------------------------------------------------------------
template <int KV>
struct AttnSmem {
    static constexpr int kRowB = kHS * KvT<KV>::kB;  // bytes per K or V row
    static constexpr int kCH = KvT<KV>::kCH;         // positions per staged sub-chunk
    static constexpr int kLP = kRowB / 16;           // lanes per row
    static constexpr int kRPP = kAttnThreads / kLP;  // rows per pass
    static constexpr int kE = 16 / KvT<KV>::kB;      // elements per 16-byte slice
    static constexpr bool k8 = (KV == KV_I8 || KV == KV_FP8);
    // stage: K rows | V rows | K scales | V scales.  Scale copies start at the
    // 16-byte boundary below the first position, so each scale array holds up
    // to kCH + 8 floats and is indexed from (first position & 3).
    static constexpr int kScaleSlots = kCH + 8;
    static constexpr int kStageBytes = 2 * kCH * kRowB + (k8 ? 2 * kScaleSlots * 4 : 0);
    static constexpr int kAccBytes = kRPP * kHS * 4;
    static constexpr int kBytes = 2 * kStageBytes + kAccBytes + kHS * 4 /*q*/ + kCH * 4 /*p*/ + 64 /*red*/ +
                                  32 /*bars*/;
};

struct AttnArgs {
    void* out;              // SINGLE: B*NH*hs activations; ENGINE: atty (NH*hs)
    float* part_out;        // SPLIT / ENGINE partials
    float* part_max;
    float* part_lse;
    const void* qkv;
    void* kv;               // cache (layer base)
    float* kv_scale;        // 8-bit scales (layer base)
    const int* d_pos;
    int B, NH, maxT, S;     // S: splits (SPLIT: caller's; ENGINE: grid splits per head)
    float scale;            // 1/sqrt(hs)
};

// Stage n positions starting at cache rows krow (K) / vrow (V); for 8-bit KV
// also their scales at ksi (K) / vsi (V).  Scale indices are rounded down to a
// multiple of 4 (16 bytes) and the count up; rows past the range stay inside
// the head's maxT slots because maxT % 4 == 0.
template <int KV>
__device__ __forceinline__ void stage_issue(unsigned char* stage, uint64_t* bar, const AttnArgs& a, size_t krow,
                                            size_t vrow, size_t ksi, size_t vsi, int n) {
    using S = AttnSmem<KV>;
    const unsigned char* kv = reinterpret_cast<const unsigned char*>(a.kv);
    const uint32_t rb = (uint32_t)(n * S::kRowB);
    uint32_t tx = 2 * rb;
    uint32_t sb = 0;
    size_t k0 = 0, v0 = 0;
    if constexpr (S::k8) {
        k0 = ksi & ~(size_t)3;
        v0 = vsi & ~(size_t)3;
        sb = (uint32_t)((((ksi + n + 3) & ~(size_t)3) - k0) * 4);
        tx += 2 * sb;
    }
    mbar_arrive_expect_tx(bar, tx);
    bulk_g2s(stage, kv + krow * S::kRowB, rb, bar);
    bulk_g2s(stage + S::kCH * S::kRowB, kv + vrow * S::kRowB, rb, bar);
    if constexpr (S::k8) {
        bulk_g2s(stage + 2 * S::kCH * S::kRowB, a.kv_scale + k0, sb, bar);
        bulk_g2s(stage + 2 * S::kCH * S::kRowB + S::kScaleSlots * 4, a.kv_scale + v0, sb, bar);
    }
}

__device__ __forceinline__ float block_max_256(float v, float* red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = (lane < 8) ? red[lane] : -FLT_MAX;
    t = warp_max(t);
    __syncthreads();
    return t;
}

template <int KV, int MODE>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
    using S = AttnSmem<KV>;
    using XT = typename KvT<KV>::XT;
    extern __shared__ __align__(16) unsigned char sm[];
    unsigned char* stage0 = sm;
    float* accbuf = reinterpret_cast<float*>(sm + 2 * S::kStageBytes);
    float* q_s = accbuf + S::kRPP * kHS;
    float* p_s = q_s + kHS;
    float* red = p_s + S::kCH;
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 16);

    const int tid = threadIdx.x;
    const int NH = a.NH, maxT = a.maxT;
    int b, h, s, nsplit;
    if (MODE == AM_SINGLE) { b = blockIdx.x / NH; h = blockIdx.x % NH; s = 0; nsplit = 1; }
    else { b = blockIdx.x / (NH * a.S); h = (blockIdx.x / a.S) % NH; s = blockIdx.x % a.S; nsplit = a.S; }

    // Position: in ENGINE mode it was written by an earlier step (two or more
    // kernels back), so it is safe to read before griddepcontrol.wait.
    int pos = *a.d_pos;
    if (pos < 0 || pos >= maxT) {
        if (tid == 0 && blockIdx.x == 0) report_device_error(GPT2B_DEVERR_BAD_POS);
        pdl_wait();
        pdl_trigger();
        return;
    }
    const int total = pos + 1;
    int j0, j1;
    if (MODE == AM_SINGLE) { j0 = 0; j1 = total; }
    else if (MODE == AM_SPLIT) {
        const int chunk = (total + nsplit - 1) / nsplit;  // attention_kvcache.cuh:197-199
        j0 = s * chunk; j1 = min(j0 + chunk, total);
    } else {
        // engine chunking: multiples of 16 positions, at most CH per CTA; the
        // merging GEMV prologue derives the same split count from the position
        const int chunk = engine_attn_chunk(total, nsplit);
        j0 = s * chunk; j1 = min(j0 + chunk, total);
    }
    const int n_local = j1 - j0;
    const size_t bh = (size_t)b * NH + h;
    const size_t krow0 = bh * maxT;                         // row index of (b,h,0) in K
    const size_t vrow0 = (size_t)a.B * NH * maxT + krow0;  // and in V
    const size_t vs0 = (size_t)a.B * NH * maxT;

    if (n_local <= 0) {
        pdl_wait();
        pdl_trigger();
        if (MODE == AM_SPLIT) {  // neutral partials (attention_kvcache.cuh:202-206)
            const size_t slot = bh * a.S + s;
            if (tid == 0) { a.part_max[slot] = -FLT_MAX; a.part_lse[slot] = 0.0f; }
            if (tid < kHS) a.part_out[slot * kHS + tid] = 0.0f;
        }
        return;
    }

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    const int nsub = (n_local + S::kCH - 1) / S::kCH;
    if (tid == 0) {
        for (int c = 0; c < 2 && c < nsub; c++) {
            const int js = j0 + c * S::kCH, n = min(S::kCH, j1 - js);
            stage_issue<KV>(stage0 + c * S::kStageBytes, &bars[c], a, krow0 + js, vrow0 + js, krow0 + js,
                            vs0 + krow0 + js, n);
        }
    }
    pdl_wait();
    pdl_trigger();

    // q (and the current token's K/V in ENGINE mode) come from this step's QKV
    const XT* qkv = reinterpret_cast<const XT*>(a.qkv) + (size_t)b * 3 * NH * kHS;
    if (tid < kHS) q_s[tid] = to_f<XT>(qkv[(size_t)h * kHS + tid]);
    const bool owns_pos = (MODE == AM_ENGINE) && (pos >= j0 && pos < j1);
    if (owns_pos) {
        // append K/V of the current token to the cache (the reference's
        // kv_cache_write_kernel(_w8) folded into the attention launch)
        if constexpr (S::k8) {
            if (tid < 64) {
                const int which = tid >> 5, lane = tid & 31;  // warp 0: K, warp 1: V
                const XT* src = qkv + (size_t)(1 + which) * NH * kHS + (size_t)h * kHS;
                const float v0 = to_f<XT>(src[lane]), v1 = to_f<XT>(src[lane + 32]);
                const float mx = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
                const float sc = mx / kv8_limit<KV>();
                const uint8_t c0 = sc > 0.0f ? kv8_encode<KV>(v0, sc) : (uint8_t)0;
                const uint8_t c1 = sc > 0.0f ? kv8_encode<KV>(v1, sc) : (uint8_t)0;
                uint8_t* dst = reinterpret_cast<uint8_t*>(a.kv) + ((which ? vrow0 : krow0) + pos) * kHS;
                dst[lane] = c0;
                dst[lane + 32] = c1;
                if (lane == 0) a.kv_scale[(which ? vs0 : 0) + krow0 + pos] = sc;
                // keep the codes for the staged copy (patched after the copy lands)
                reinterpret_cast<uint8_t*>(accbuf)[which * 64 + lane] = c0;
                reinterpret_cast<uint8_t*>(accbuf)[which * 64 + lane + 32] = c1;
                if (lane == 0) red[8 + which] = sc;
            }
        } else {
            if (tid < 2 * kHS) {
                const int which = tid / kHS, d = tid % kHS;
                const XT v = qkv[(size_t)(1 + which) * NH * kHS + (size_t)h * kHS + d];
                XT* dst = reinterpret_cast<XT*>(a.kv) + ((which ? vrow0 : krow0) + pos) * kHS;
                dst[d] = v;
            }
        }
    }
    __syncthreads();

    // online softmax state (uniform across the block)
    float m_run = -FLT_MAX, l_run = 0.0f;
    float acc[S::kE];
#pragma unroll
    for (int e = 0; e < S::kE; e++) acc[e] = 0.0f;
    const int lp = tid % S::kLP, rg = tid / S::kLP;

    for (int c = 0; c < nsub; c++) {
        const int st = c & 1;
        unsigned char* stage = stage0 + st * S::kStageBytes;
        const int js = j0 + c * S::kCH, n = min(S::kCH, j1 - js);
        if (!mbar_wait(&bars[st], (uint32_t)((c >> 1) & 1))) return;
        const int soff = (int)((krow0 + js) & 3);  // scale slot of position js
        if (owns_pos && pos >= js && pos < js + n) {
            // overwrite the stale cache row of `pos` in the staged copy
            const int r = pos - js;
            if constexpr (S::k8) {
                if (tid < 128) stage[(tid >> 6) * S::kCH * S::kRowB + r * S::kRowB + (tid & 63)] =
                    reinterpret_cast<uint8_t*>(accbuf)[tid];
                if (tid < 2)
                    reinterpret_cast<float*>(stage + 2 * S::kCH * S::kRowB)[tid * S::kScaleSlots + soff + r] =
                        red[8 + tid];
            } else {
                if (tid < 2 * kHS) {
                    const int which = tid / kHS, d = tid % kHS;
                    reinterpret_cast<XT*>(stage + which * S::kCH * S::kRowB + r * S::kRowB)[d] =
                        qkv[(size_t)(1 + which) * NH * kHS + (size_t)h * kHS + d];
                }
            }
            __syncthreads();
        }
        const unsigned char* Kst = stage;
        const unsigned char* Vst = stage + S::kCH * S::kRowB;
        const float* ksc = reinterpret_cast<const float*>(stage + 2 * S::kCH * S::kRowB) + soff;
        const float* vsc = ksc + S::kScaleSlots;

        // scores: the loop bound is warp-uniform so the LP-lane shuffles below
        // always run with the whole warp; rows past n contribute nothing.
        for (int rbase = 0; rbase < n; rbase += S::kRPP) {
            const int r = rbase + rg;
            const bool valid = r < n;
            const uint4 w = valid ? *reinterpret_cast<const uint4*>(Kst + r * S::kRowB + lp * 16)
                                  : make_uint4(0u, 0u, 0u, 0u);
            const float* q = q_s + lp * S::kE;
            float d = 0.0f;
            if constexpr (KV == KV_F32) {
                d = __uint_as_float(w.x) * q[0] + __uint_as_float(w.y) * q[1] + __uint_as_float(w.z) * q[2] +
                    __uint_as_float(w.w) * q[3];
            } else if constexpr (KV == KV_BF16) {
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; i++) d += bf16lo(ww[i]) * q[2 * i] + bf16hi(ww[i]) * q[2 * i + 1];
            } else {
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) d += kv8_decode<KV>(ww[i], j) * q[4 * i + j];
            }
#pragma unroll
            for (int o = S::kLP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            if (lp == 0 && valid) {
                if constexpr (S::k8) d *= ksc[r];
                p_s[r] = d * a.scale;
            }
        }
        __syncthreads();
        const float smax = block_max_256(tid < n ? p_s[tid] : -FLT_MAX, red);
        const float m_new = fmaxf(m_run, smax);
        const float alpha = __expf(m_run - m_new);
        float ev = 0.0f;
        if (tid < n) { ev = __expf(p_s[tid] - m_new); p_s[tid] = ev; }
        const float lsum = block_sum(ev, red);  // ends with a barrier: p_s is complete
        l_run = l_run * alpha + lsum;
        m_run = m_new;
#pragma unroll
        for (int e = 0; e < S::kE; e++) acc[e] *= alpha;
        for (int r = rg; r < n; r += S::kRPP) {
            const uint4 w = *reinterpret_cast<const uint4*>(Vst + r * S::kRowB + lp * 16);
            const float p = p_s[r];
            if constexpr (KV == KV_F32) {
                acc[0] += p * __uint_as_float(w.x); acc[1] += p * __uint_as_float(w.y);
                acc[2] += p * __uint_as_float(w.z); acc[3] += p * __uint_as_float(w.w);
            } else if constexpr (KV == KV_BF16) {
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; i++) { acc[2 * i] += p * bf16lo(ww[i]); acc[2 * i + 1] += p * bf16hi(ww[i]); }
            } else {
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                const float pv = p * vsc[r];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[4 * i + j] += pv * kv8_decode<KV>(ww[i], j);
            }
        }
        __syncthreads();  // stage and p_s fully consumed
        if (tid == 0 && c + 2 < nsub) {
            const int jn = j0 + (c + 2) * S::kCH, nn = min(S::kCH, j1 - jn);
            stage_issue<KV>(stage, &bars[st], a, krow0 + jn, vrow0 + jn, krow0 + jn, vs0 + krow0 + jn, nn);
        }
    }

    // reduce the row groups: o[d] = sum over rg of acc
#pragma unroll
    for (int e = 0; e < S::kE; e++) accbuf[rg * kHS + lp * S::kE + e] = acc[e];
    __syncthreads();
    float o = 0.0f;
    if (tid < kHS)
        for (int g = 0; g < S::kRPP; g++) o += accbuf[g * kHS + tid];

    if (MODE == AM_SINGLE) {
        if (tid < kHS) reinterpret_cast<XT*>(a.out)[bh * kHS + tid] = from_f<XT>(o / l_run);
        return;
    }
    // SPLIT and ENGINE: per-split partials (the engine's projection GEMV merges
    // them in its prologue, PRO_ATTN_MERGE)
    const size_t slot = bh * a.S + s;
    if (tid < kHS) a.part_out[slot * kHS + tid] = o;
    if (tid == 0) { a.part_max[slot] = m_run; a.part_lse[slot] = l_run; }
}

// LSE merge of S partials (attention_kvcache.cuh:298-318).
template <typename OT>
__global__ void attn_merge_kernel(OT* out, const float* part_out, const float* part_lse, const float* part_max,
                                  int NH, int hs, int S) {
    const int bh = blockIdx.x, tid = threadIdx.x;
    if (tid >= hs) return;
    float mg = -FLT_MAX;
    for (int s = 0; s < S; s++) mg = fmaxf(mg, part_max[bh * S + s]);
    float of = 0.0f, lf = 0.0f;
    for (int s = 0; s < S; s++) {
        const float rs = __expf(part_max[bh * S + s] - mg);
        of += rs * part_out[((size_t)bh * S + s) * hs + tid];
        lf += rs * part_lse[bh * S + s];
    }
    out[(size_t)bh * hs + tid] = from_f<OT>(of / lf);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int KV, int MODE>
static cudaError_t launch_attn(const AttnArgs& a, int grid, cudaStream_t st, bool pdl) {
    auto k = attn_kernel<KV, MODE>;
    static unsigned long long smem_set = 0;
    const int smem = AttnSmem<KV>::kBytes;
    cudaError_t e = ensure_smem_limit(k, &smem_set);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(grid), dim3(kAttnThreads), (size_t)smem, st, pdl, a);
}

template <int MODE>
static cudaError_t launch_attn_kind(int kv, const AttnArgs& a, int grid, cudaStream_t st, bool pdl) {
    switch (kv) {
        case KV_F32: return launch_attn<KV_F32, MODE>(a, grid, st, pdl);
        case KV_BF16: return launch_attn<KV_BF16, MODE>(a, grid, st, pdl);
        case KV_I8: return launch_attn<KV_I8, MODE>(a, grid, st, pdl);
        case KV_FP8: return launch_attn<KV_FP8, MODE>(a, grid, st, pdl);
    }
    return cudaErrorInvalidValue;
}

int attn_engine_max_chunk(int kv) { return kv == KV_F32 ? KvT<KV_F32>::kCH : KvT<KV_BF16>::kCH; }

cudaError_t launch_attention_engine(int kv, const void* qkv, void* kv_layer, float* kv_scale_layer, const int* d_pos,
                                    int NH, int maxT, int splits, float* part_out, float* part_max, float* part_lse,
                                    cudaStream_t st, bool pdl) {
    AttnArgs a{};
    a.part_out = part_out; a.part_max = part_max; a.part_lse = part_lse;
    a.qkv = qkv; a.kv = kv_layer; a.kv_scale = kv_scale_layer; a.d_pos = d_pos;
    a.B = 1; a.NH = NH; a.maxT = maxT; a.S = splits; a.scale = 1.0f / sqrtf((float)kHS);
    return launch_attn_kind<AM_ENGINE>(kv, a, NH * splits, st, pdl);
}

}  // namespace gpt2b

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace gpt2b;

static int attn_check(int B, int NH, int hs, int maxT, const void* kv, const int* d_pos) {
    if (B <= 0 || NH <= 0 || maxT <= 0 || !kv || !d_pos) return GPT2B_ERR_INVALID_ARG;
    if (hs != kHS) return GPT2B_ERR_UNSUPPORTED;
    if (!aligned16(kv) || (maxT % 4) != 0) return GPT2B_ERR_ALIGNMENT;
    return GPT2B_OK;
}

static int attn_small(int kv, void* out, const void* qkv, const void* cache, const float* sc, int B, int NH, int hs,
                      int maxT, const int* d_pos, cudaStream_t st) {
    int rc = attn_check(B, NH, hs, maxT, cache, d_pos);
    if (rc) return rc;
    if ((kv == KV_I8 || kv == KV_FP8) && (!sc || !aligned16(sc))) return GPT2B_ERR_ALIGNMENT;
    AttnArgs a{};
    a.out = out; a.qkv = qkv; a.kv = const_cast<void*>(cache); a.kv_scale = const_cast<float*>(sc); a.d_pos = d_pos;
    a.B = B; a.NH = NH; a.maxT = maxT; a.S = 1; a.scale = 1.0f / sqrtf((float)hs);
    return status_from(launch_attn_kind<AM_SINGLE>(kv, a, B * NH, st, false));
}

static int attn_split(int kv, float* po, float* pl, float* pm, const void* qkv, const void* cache, const float* sc,
                      int B, int NH, int hs, int maxT, int S, const int* d_pos, cudaStream_t st) {
    int rc = attn_check(B, NH, hs, maxT, cache, d_pos);
    if (rc) return rc;
    if (S <= 0 || !po || !pl || !pm) return GPT2B_ERR_INVALID_ARG;
    if ((kv == KV_I8 || kv == KV_FP8) && (!sc || !aligned16(sc))) return GPT2B_ERR_ALIGNMENT;
    AttnArgs a{};
    a.part_out = po; a.part_lse = pl; a.part_max = pm; a.qkv = qkv; a.kv = const_cast<void*>(cache);
    a.kv_scale = const_cast<float*>(sc); a.d_pos = d_pos;
    a.B = B; a.NH = NH; a.maxT = maxT; a.S = S; a.scale = 1.0f / sqrtf((float)hs);
    return status_from(launch_attn_kind<AM_SPLIT>(kv, a, B * NH * S, st, false));
}

template <typename OT>
static int attn_merge(OT* out, const float* po, const float* pl, const float* pm, int B, int NH, int hs, int S,
                      cudaStream_t st) {
    if (B <= 0 || NH <= 0 || hs <= 0 || hs > 1024 || S <= 0 || !out) return GPT2B_ERR_INVALID_ARG;
    return status_from(launch_k(attn_merge_kernel<OT>, dim3(B * NH), dim3(((hs + 31) / 32) * 32), 0, st, false, out, po, pl, pm, NH, hs, S));
}

extern "C" {

int gpt2b_kv_cache_write_f32(float* kv_cache, const float* qkv, int B, int NH, int hs, int maxT, const int* d_pos,
                             gpt2b_stream_t stream) {
    if (B <= 0 || NH <= 0 || hs <= 0 || maxT <= 0 || !kv_cache || !qkv || !d_pos) return GPT2B_ERR_INVALID_ARG;
    const int n = B * NH * hs;
    return status_from(launch_k(kv_write_kernel<float>, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t)stream, false, kv_cache, qkv, B, NH, hs, maxT, d_pos));
}
int gpt2b_kv_cache_write_bf16(uint16_t* kv_cache, const uint16_t* qkv, int B, int NH, int hs, int maxT,
                              const int* d_pos, gpt2b_stream_t stream) {
    if (B <= 0 || NH <= 0 || hs <= 0 || maxT <= 0 || !kv_cache || !qkv || !d_pos) return GPT2B_ERR_INVALID_ARG;
    const int n = B * NH * hs;
    return status_from(launch_k(kv_write_kernel<__nv_bfloat16>, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t)stream, false, 
        (__nv_bfloat16*)kv_cache, (const __nv_bfloat16*)qkv, B, NH, hs, maxT, d_pos));
}
int gpt2b_kv_cache_write_w8_i8(uint8_t* kv_cache, float* kv_scale, const uint16_t* qkv, int B, int NH, int hs,
                               int maxT, const int* d_pos, gpt2b_stream_t stream) {
    if (B <= 0 || NH <= 0 || hs <= 0 || maxT <= 0 || !kv_cache || !kv_scale || !qkv || !d_pos)
        return GPT2B_ERR_INVALID_ARG;
    const int rows = B * NH * 2;
    return status_from(launch_k(kv_write_w8_kernel<KV_I8>, dim3((rows + 7) / 8), dim3(256), 0, (cudaStream_t)stream, false, 
        kv_cache, kv_scale, (const __nv_bfloat16*)qkv, B, NH, hs, maxT, d_pos));
}
int gpt2b_kv_cache_write_w8_fp8(uint8_t* kv_cache, float* kv_scale, const uint16_t* qkv, int B, int NH, int hs,
                                int maxT, const int* d_pos, gpt2b_stream_t stream) {
    if (B <= 0 || NH <= 0 || hs <= 0 || maxT <= 0 || !kv_cache || !kv_scale || !qkv || !d_pos)
        return GPT2B_ERR_INVALID_ARG;
    const int rows = B * NH * 2;
    return status_from(launch_k(kv_write_w8_kernel<KV_FP8>, dim3((rows + 7) / 8), dim3(256), 0, (cudaStream_t)stream, false, 
        kv_cache, kv_scale, (const __nv_bfloat16*)qkv, B, NH, hs, maxT, d_pos));
}

int gpt2b_attention_forward_kv_small_f32(float* out, const float* qkv, const float* kv_cache, int B, int NH, int hs,
                                         int maxT, const int* d_pos, gpt2b_stream_t stream) {
    return attn_small(KV_F32, out, qkv, kv_cache, nullptr, B, NH, hs, maxT, d_pos, (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_small_bf16(uint16_t* out, const uint16_t* qkv, const uint16_t* kv_cache, int B, int NH,
                                          int hs, int maxT, const int* d_pos, gpt2b_stream_t stream) {
    return attn_small(KV_BF16, out, qkv, kv_cache, nullptr, B, NH, hs, maxT, d_pos, (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_small_w8_i8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                           const float* kv_scale, int B, int NH, int hs, int maxT, const int* d_pos,
                                           gpt2b_stream_t stream) {
    return attn_small(KV_I8, out, qkv, kv_cache, kv_scale, B, NH, hs, maxT, d_pos, (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_small_w8_fp8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                            const float* kv_scale, int B, int NH, int hs, int maxT,
                                            const int* d_pos, gpt2b_stream_t stream) {
    return attn_small(KV_FP8, out, qkv, kv_cache, kv_scale, B, NH, hs, maxT, d_pos, (cudaStream_t)stream);
}

int gpt2b_attention_forward_kv_large_f32(float* out, const float* qkv, const float* kv_cache, int B, int NH, int hs,
                                         int maxT, const int* d_pos, gpt2b_stream_t stream, float* part_out,
                                         float* part_lse, float* part_max, int S) {
    int rc = attn_split(KV_F32, part_out, part_lse, part_max, qkv, kv_cache, nullptr, B, NH, hs, maxT, S, d_pos,
                        (cudaStream_t)stream);
    return rc ? rc : attn_merge<float>(out, part_out, part_lse, part_max, B, NH, hs, S, (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_large_bf16(uint16_t* out, const uint16_t* qkv, const uint16_t* kv_cache, int B, int NH,
                                          int hs, int maxT, const int* d_pos, gpt2b_stream_t stream, float* part_out,
                                          float* part_lse, float* part_max, int S) {
    int rc = attn_split(KV_BF16, part_out, part_lse, part_max, qkv, kv_cache, nullptr, B, NH, hs, maxT, S, d_pos,
                        (cudaStream_t)stream);
    return rc ? rc
              : attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                          (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_large_w8_i8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                           const float* kv_scale, int B, int NH, int hs, int maxT, const int* d_pos,
                                           gpt2b_stream_t stream, float* part_out, float* part_lse, float* part_max,
                                           int S) {
    int rc = attn_split(KV_I8, part_out, part_lse, part_max, qkv, kv_cache, kv_scale, B, NH, hs, maxT, S, d_pos,
                        (cudaStream_t)stream);
    return rc ? rc
              : attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                          (cudaStream_t)stream);
}
int gpt2b_attention_forward_kv_large_w8_fp8(uint16_t* out, const uint16_t* qkv, const uint8_t* kv_cache,
                                            const float* kv_scale, int B, int NH, int hs, int maxT,
                                            const int* d_pos, gpt2b_stream_t stream, float* part_out,
                                            float* part_lse, float* part_max, int S) {
    int rc = attn_split(KV_FP8, part_out, part_lse, part_max, qkv, kv_cache, kv_scale, B, NH, hs, maxT, S, d_pos,
                        (cudaStream_t)stream);
    return rc ? rc
              : attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                          (cudaStream_t)stream);
}
int gpt2b_attention_kv_split_bf16(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                  const uint16_t* kv_cache, int B, int NH, int hs, int maxT, int S, const int* d_pos,
                                  gpt2b_stream_t stream) {
    return attn_split(KV_BF16, part_out, part_lse, part_max, qkv, kv_cache, nullptr, B, NH, hs, maxT, S, d_pos,
                      (cudaStream_t)stream);
}
int gpt2b_attention_kv_split_f32(float* part_out, float* part_lse, float* part_max, const float* qkv,
                                 const float* kv_cache, int B, int NH, int hs, int maxT, int S, const int* d_pos,
                                 gpt2b_stream_t stream) {
    return attn_split(KV_F32, part_out, part_lse, part_max, qkv, kv_cache, nullptr, B, NH, hs, maxT, S, d_pos,
                      (cudaStream_t)stream);
}
int gpt2b_attention_kv_split_w8_i8(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                   const uint8_t* kv_cache, const float* kv_scale, int B, int NH, int hs, int maxT,
                                   int S, const int* d_pos, gpt2b_stream_t stream) {
    if (!kv_scale) return GPT2B_ERR_INVALID_ARG;
    return attn_split(KV_I8, part_out, part_lse, part_max, qkv, kv_cache, kv_scale, B, NH, hs, maxT, S, d_pos,
                      (cudaStream_t)stream);
}
int gpt2b_attention_kv_split_w8_fp8(float* part_out, float* part_lse, float* part_max, const uint16_t* qkv,
                                    const uint8_t* kv_cache, const float* kv_scale, int B, int NH, int hs, int maxT,
                                    int S, const int* d_pos, gpt2b_stream_t stream) {
    if (!kv_scale) return GPT2B_ERR_INVALID_ARG;
    return attn_split(KV_FP8, part_out, part_lse, part_max, qkv, kv_cache, kv_scale, B, NH, hs, maxT, S, d_pos,
                      (cudaStream_t)stream);
}
int gpt2b_attention_kv_merge_w8(uint16_t* out, const float* part_out, const float* part_lse, const float* part_max,
                                int B, int NH, int hs, int S, gpt2b_stream_t stream) {
    return attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                     (cudaStream_t)stream);
}
int gpt2b_attention_kv_merge_bf16(uint16_t* out, const float* part_out, const float* part_lse, const float* part_max,
                                  int B, int NH, int hs, int S, gpt2b_stream_t stream) {
    return attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                     (cudaStream_t)stream);
}
int gpt2b_attention_kv_merge_f32(float* out, const float* part_out, const float* part_lse, const float* part_max,
                                 int B, int NH, int hs, int S, gpt2b_stream_t stream) {
    return attn_merge<float>(out, part_out, part_lse, part_max, B, NH, hs, S, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free split+merge attention (BF16 KV)
// ---------------------------------------------------------------------------
// Some callers cannot hand this library a scratch buffer: a host that owns
// every byte of device memory through its own pool and forbids side
// allocations, or code on a latency-critical path where cudaMalloc's implicit
// device synchronisation is not acceptable.  For them the split partials of
// the flash-decoding attention live in a fixed array inside this library
// instead of caller memory.  The array is sized for kNoAllocMaxSlots
// (batch x heads x splits) partial rows; every GPU that loads the library
// keeps it (about 0.5 MB) until the process exits.
namespace gpt2b {

constexpr int kNoAllocMaxSlots = 2048;  // B * NH * S limit of the allocation-free entry point

// [part_out: kNoAllocMaxSlots * 64 floats][part_max: kNoAllocMaxSlots][part_lse: kNoAllocMaxSlots]
static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxSlots * (kHS + 2)];

// Host code must not pass &g_noalloc_partials to a kernel: on the host that
// name is only a stand-in, not the device address.  The device address is
// looked up once per device with that device current and cached here.
static float* g_noalloc_dev_ptr[64] = {nullptr};
static std::mutex g_noalloc_mu;

static int noalloc_partials_ptr(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return status_from(e);
    if (dev < 0 || dev >= 64) return GPT2B_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_dev_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess) return status_from(e);
        g_noalloc_dev_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_dev_ptr[dev];
    return GPT2B_OK;
}

}  // namespace gpt2b

extern "C" int gpt2b_attention_forward_kv_large_bf16_noalloc(uint16_t* out, const uint16_t* qkv,
                                                             const uint16_t* kv_cache, int B, int NH, int hs,
                                                             int maxT, const int* d_pos, int S,
                                                             gpt2b_stream_t stream) {
    if (B <= 0 || NH <= 0 || S <= 0) return GPT2B_ERR_INVALID_ARG;
    if ((long long)B * NH * S > kNoAllocMaxSlots) return GPT2B_ERR_INVALID_ARG;  // beyond the built-in scratch
    float* base = nullptr;
    int rc = noalloc_partials_ptr(&base);
    if (rc) return rc;
    // Every partial slot the merge reads is written by the split kernel of the
    // same call (empty splits write neutral values), so nothing is cleared.
    float* part_out = base;
    float* part_max = base + (size_t)kNoAllocMaxSlots * kHS;
    float* part_lse = part_max + kNoAllocMaxSlots;
    rc = attn_split(KV_BF16, part_out, part_lse, part_max, qkv, kv_cache, nullptr, B, NH, hs, maxT, S, d_pos,
                    (cudaStream_t)stream);
    return rc ? rc
              : attn_merge<__nv_bfloat16>((__nv_bfloat16*)out, part_out, part_lse, part_max, B, NH, hs, S,
                                          (cudaStream_t)stream);
}
