// persistent.cu -- the whole greedy decode loop in one cooperative launch.
//
// One CTA per SM, resident for all steps of a call.  A decode step is a chain
// of phases; per layer:
//   QKV     rows of W_qkv . LN1(residual)              -> qkv words
//   ATTN    CTA (head h, split s): KV append + flash-decoding over its
//           position range (rows staged one layer ahead); split 0 of each head
//           merges the partials of its head (attention_kvcache.cuh:298-318)
//                                                       -> atty words
//   PROJ    rows of W_proj . atty                       -> proj words
//   FC      rows of gelu(W_fc . LN2(residual + proj))   -> fc words
//   FCPROJ  rows of W_fcproj . fc                       -> fcproj words
// then LM: logits = wte . LNf(residual) with a per-CTA argmax and an
// all-gather of the per-CTA (value, index) pairs, so every CTA knows the next
// token and carries on with the next step: no launch, no host round trip.
// The arithmetic of each phase is the per-kernel path's (gemv.cu,
// attention.cu): the same roundings to the activation type at the same points.
//
// Exchange between phases uses 64-bit words holding a 32-bit step tag and a
// 32-bit value, written with one relaxed store: a consumer's poll returns data
// and readiness in one L2 round trip, with no fence and no grid barrier on the
// data path.  The residual stream and every LayerNorm are recomputed in each
// CTA from the exchanged phase outputs, so the residual is never exchanged.
// Tags are a per-call epoch plus the step, so words of an earlier step or call
// never match.  A buffer is rewritten only one step later, after every CTA has
// passed the LM all-gather of the step that read it.  Every poll is bounded; a
// CTA whose wait runs out records GPT2B_DEVERR_GRID_TIMEOUT and raises an
// abort flag that makes every other CTA leave at its next poll.  A CTA leaves
// only when none of its bulk copies is still in flight.
//
// Weights: CTA b owns rows [b*M/G, (b+1)*M/G) of every matrix.  A producer
// warp streams them, in consumption order across phases, layers and steps,
// through a ring of stages of 16 row-units of C elements (16 rows of K = C, or
// 8 half-rows of K = 4C), with the rows' bias and scale values in the stage
// tail; so the ring runs ahead while the consumers wait for their inputs.
// Consumer warp w takes rows w and w + 8 of a stage (one row for K = 4C), two
// independent dot products sharing each x chunk and one shuffle reduction.
//
// Shapes: head size 64, C <= 2048, heads x splits <= CTAs, at most 256
// positions per attention CTA (persist_supported); the engine uses the
// per-kernel path otherwise.
#include "common.cuh"
#include "internal.h"

#include <float.h>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(persistent_device_error)

namespace {

constexpr int kCW = 8;                // consumer warps
constexpr int kCT = kCW * 32;         // consumer threads
constexpr int kThreads = kCT + 32;    // + the producer warp
constexpr int kStageUnits = 16;       // row-units of C elements per stage
constexpr int kTailSlot = 96;         // a 16-byte aligned window of 16 bias (or scale) values
constexpr int kTail = 2 * kTailSlot;  // stage tail: bias window + scale window
constexpr int kMaxNs = 24;            // ring stages (upper bound)
constexpr int kMaxKvRows = 256;       // positions per attention CTA (one per consumer thread in the softmax)
constexpr int kMaxCtas = 160;         // CTAs of the grid (one per SM)
constexpr int kMaxC = 2048;           // channels
constexpr int kNarrowC = 1024;        // kernels for C <= 1024 keep per-thread arrays small
constexpr int kNarrowKvRows = 96;     // and stage at most 96 positions per attention CTA
constexpr int kHSz = 64;              // head size
constexpr int kMaxSplits = 32;        // attention splits per head
constexpr int kMiscFloats = 128;      // reduction scratch, new-row codes and scales, stop flag
constexpr int kXmaxSlot = 104;        // misc[104..111]: per-warp max |x| of a phase (8-bit tensor-core stages)
constexpr int kMaxLayers = 127;       // layers of the persistent kernel (LayerNorm exponents in shared memory)
constexpr int kGatherJ = 32;          // exchange words per consumer thread and gather (4C <= 8192)
constexpr int kGatherJs = 16;         // the short gather (n <= 4096 words)
enum { kPhQkv = 0, kPhProj = 1, kPhFc = 2, kPhFcproj = 3, kPhLm = 4 };

// Phase timeline for profiling builds (-DGPT2B_PERSIST_TRACE): consumer
// thread 0 of every CTA stamps %globaltimer at phase boundaries of the first
// kTraceSteps steps.  Off in the library build.
#ifdef GPT2B_PERSIST_TRACE
constexpr int kTraceSteps = 4, kTraceCtas = 160, kTraceEv = 640;
__device__ unsigned long long g_trace[kTraceSteps * kTraceCtas * kTraceEv];
#define PTRACE(ev)                                                                            \
    do {                                                                                      \
        if (tid == 0 && step < kTraceSteps && (ev) < kTraceEv && b < kTraceCtas) {            \
            unsigned long long t_;                                                            \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                            \
            g_trace[((size_t)step * kTraceCtas + b) * kTraceEv + (ev)] = t_;                  \
        }                                                                                     \
    } while (0)
// per-stage stamps of CTA 0: producer issue time, consumer warp 0 wait start / wait end / done
constexpr int kTraceStages = 2048;
__device__ unsigned long long g_trace_stage[kTraceStages * 8];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define PTRACE_STAGE(k, idx)                                                         \
    do {                                                                             \
        if (b == 0 && (idx) < kTraceStages) g_trace_stage[(idx) * 8 + (k)] = gtimer(); \
    } while (0)
#else
#define PTRACE(ev) \
    do {           \
    } while (0)
#define PTRACE_STAGE(k, idx) \
    do {                     \
    } while (0)
#endif

// ---------------------------------------------------------------------------
// exchange words
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ll_store(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Words written by other GPUs of the group (system scope).
__device__ __forceinline__ unsigned long long ll_load_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ bool aborted(const int* flag) { return *(volatile const int*)flag != 0; }

// The exchange arenas of a tensor-parallel group, copied out of the kernel
// parameters (helpers take this, never the parameter block: indexing the
// parameters at run time would make the compiler copy all of them to local
// memory).
struct PeerSet {
    unsigned char* x[8];
    int n, rank;
    size_t off_abort;
};
__device__ __forceinline__ void ll_store_sys(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// A word of a cross-GPU part to every rank of the group (own copy included);
// own: this rank's arena (single GPU), ps: the group's arenas.
template <bool TPG>
__device__ __forceinline__ void ll_store_group(unsigned char* own, const PeerSet* ps, size_t xoff, size_t word,
                                               float v, uint32_t tag) {
    if constexpr (!TPG) {
        ll_store(reinterpret_cast<unsigned long long*>(own + xoff) + word, v, tag);
    } else {
        for (int r = 0; r < ps->n; r++)
            ll_store_sys(reinterpret_cast<unsigned long long*>(ps->x[r] + xoff) + word, v, tag);
    }
}
__device__ __noinline__ void give_up(int* flag, const PeerSet* ps) {
    report_device_error(GPT2B_DEVERR_GRID_TIMEOUT);
    atomicExch(flag, 1);
    if (ps)
        for (int r = 0; r < ps->n; r++)  // the other ranks leave too
            if (r != ps->rank)
                asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(ps->x[r] + ps->off_abort), "r"(1) : "memory");
}

// Polls spin without a sleep: every iteration is already an L2 round trip, and a
// __nanosleep(32) between polls measured 0.7 % (GPT-2 124M) to 3.3 % (GPT-2-XL)
// slower per token.  The poll limit counts iterations (2^22 by default: seconds).
//
// Words i = tid + j*kCT (i < n, j < J) of src into out[j]; all loads of a
// round are in flight together.  False on timeout (recorded) or abort.
template <int J, bool SYS>
__device__ __noinline__ bool ll_gather_j(int* abort_flag, const PeerSet* ps, uint32_t plim, const unsigned long long* src, int n,
                                         uint32_t tag,
                                         float* out) {
    const int tid = threadIdx.x;
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < J; j++)
        if (tid + j * kCT < n) pending |= 1u << j;
    for (uint32_t it = 0; pending; ++it) {
        unsigned long long w[J];
#pragma unroll
        for (int j = 0; j < J; j++)
            if (pending & (1u << j)) w[j] = SYS ? ll_load_sys(src + tid + j * kCT) : ll_load(src + tid + j * kCT);
#pragma unroll
        for (int j = 0; j < J; j++)
            if ((pending & (1u << j)) && (uint32_t)(w[j] >> 32) == tag) {
                out[j] = __uint_as_float((uint32_t)w[j]);
                pending &= ~(1u << j);
            }
        if (!pending) break;
        if (it > plim) { give_up(abort_flag, ps); return false; }
        if ((it & 15) == 15 && aborted(abort_flag)) return false;
    }
    return true;
}
// Words 2q and 2q + 1 for q = tid + j*kCT (j < J2) of src into out[2j], out[2j + 1]: one
// 16-byte poll per pair (half the requests of word polls; src 16-byte aligned).  False on
// timeout (recorded) or abort.
template <int J2, bool SYS>
__device__ __noinline__ bool ll_gather2_j(int* abort_flag, const PeerSet* ps, uint32_t plim, const unsigned long long* src, int n,
                                          uint32_t tag, float* out) {
    const int tid = threadIdx.x;
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < J2; j++)
        if (2 * (tid + j * kCT) < n) pending |= 1u << j;
    for (uint32_t it = 0; pending; ++it) {
        unsigned long long a[J2], c[J2];
#pragma unroll
        for (int j = 0; j < J2; j++) {
            if (!(pending & (1u << j))) continue;
            const unsigned long long* p = src + 2 * (tid + j * kCT);
            if (2 * (tid + j * kCT) + 1 < n) {
                if (SYS)
                    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a[j]), "=l"(c[j]) : "l"(p) : "memory");
                else
                    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a[j]), "=l"(c[j]) : "l"(p) : "memory");
            } else {  // an odd count's last word alone
                a[j] = SYS ? ll_load_sys(p) : ll_load(p);
                c[j] = (unsigned long long)tag << 32;
            }
        }
#pragma unroll
        for (int j = 0; j < J2; j++)
            if ((pending & (1u << j)) && (uint32_t)(a[j] >> 32) == tag && (uint32_t)(c[j] >> 32) == tag) {
                out[2 * j] = __uint_as_float((uint32_t)a[j]);
                out[2 * j + 1] = __uint_as_float((uint32_t)c[j]);
                pending &= ~(1u << j);
            }
        if (!pending) break;
        if (it > plim) { give_up(abort_flag, ps); return false; }
        if ((it & 15) == 15 && aborted(abort_flag)) return false;
    }
    return true;
}
template <bool WIDE>
__device__ __forceinline__ bool ll_gather2(int* abort_flag, const PeerSet* ps, uint32_t plim, const unsigned long long* src, int n,
                                           uint32_t tag, float* out) {
    if constexpr (!WIDE) return ll_gather2_j<kGatherJs / 2, false>(abort_flag, ps, plim, src, n, tag, out);
    return n <= kGatherJs * kCT ? ll_gather2_j<kGatherJs / 2, false>(abort_flag, ps, plim, src, n, tag, out)
                                : ll_gather2_j<kGatherJ / 2, false>(abort_flag, ps, plim, src, n, tag, out);
}
// Word index of slot j of this thread in a pair gather (and the channel a thread owns in
// the residual / LayerNorm passes, which follow the same order).
__device__ __forceinline__ int pair_slot(int tid, int j) { return 2 * (tid + (j >> 1) * kCT) + (j & 1); }

// The LM-head pick: pair k = (value, index bits) at words k * kPersistLmStride + {0, 1},
// one 16-byte poll per pair, into vals[k] / idx[k] (shared memory).
template <bool SYS>
__device__ __noinline__ bool ll_gather_pairs(int* abort_flag, const PeerSet* ps, uint32_t plim, const unsigned long long* src,
                                             int npairs, uint32_t tag, float* vals, int* idx) {
    constexpr int J = kMaxCtas * 8 / kCT + 1;  // pairs per thread (8 ranks of kMaxCtas CTAs)
    const int tid = threadIdx.x;
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < J; j++)
        if (tid + j * kCT < npairs) pending |= 1u << j;
    for (uint32_t it = 0; pending; ++it) {
#pragma unroll
        for (int j = 0; j < J; j++) {
            if (!(pending & (1u << j))) continue;
            const int k = tid + j * kCT;
            const unsigned long long* p = src + (size_t)k * kPersistLmStride;
            unsigned long long a, c;
            if (SYS)
                asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(c) : "l"(p) : "memory");
            else
                asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(c) : "l"(p) : "memory");
            if ((uint32_t)(a >> 32) == tag && (uint32_t)(c >> 32) == tag) {
                vals[k] = __uint_as_float((uint32_t)a);
                idx[k] = (int)(uint32_t)c;
                pending &= ~(1u << j);
            }
        }
        if (!pending) break;
        if (it > plim) { give_up(abort_flag, ps); return false; }
        if ((it & 15) == 15 && aborted(abort_flag)) return false;
    }
    return true;
}
// Words written by the ranks of a tensor-parallel group (system scope, 32-word rounds).
__device__ __forceinline__ bool ll_gather_group(int* abort_flag, const PeerSet* ps, uint32_t plim, const unsigned long long* src,
                                                int n, uint32_t tag, float* out) {
    return ll_gather_j<kGatherJ, true>(abort_flag, ps, plim, src, n, tag, out);
}

// consumer-only barriers (named barrier 1, the 256 consumer threads)
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool cta_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 256, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void best_merge(float& bv, int& bi, float ov, int oi) {
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

// ---------------------------------------------------------------------------
// phases
// ---------------------------------------------------------------------------
template <int WK> struct PTraits;
template <> struct PTraits<WK_F32> { using XT = float; static constexpr int kWB = 4; };
template <> struct PTraits<WK_BF16> { using XT = __nv_bfloat16; static constexpr int kWB = 2; };
template <> struct PTraits<WK_I8> { using XT = __nv_bfloat16; static constexpr int kWB = 1; };
template <> struct PTraits<WK_FP8> { using XT = __nv_bfloat16; static constexpr int kWB = 1; };

// Rows, columns, stage geometry and this CTA's row range of phase `ph` (this
// rank's shard).  Tensor-core stages (MMA): 16 rows (one tile), rows wider
// than C in K-parts of C.  CUDA-core stages: 16 rows of K <= C, wider rows 8
// per stage in K-parts of at most 2C.
struct PhaseRows {
    int M, K, kparts, part, rs, c0, c1;  // rows, columns, K-parts, columns per part, rows per stage, CTA range
    int pad;
};
template <bool MMA>
__device__ __forceinline__ PhaseRows phase_rows(const PersistParams& P, int ph, int b) {
    PhaseRows r;
    const int C = P.C;
    r.M = (ph == kPhQkv) ? P.qkv_rows : (ph == kPhFc) ? P.fc_rows : (ph == kPhLm) ? P.v_rows : C;
    r.K = (ph == kPhProj) ? P.proj_k : (ph == kPhFcproj) ? P.fcproj_k : C;
    if (MMA || r.K <= C) {
        r.rs = kStageUnits;
        r.kparts = (r.K + C - 1) / C;
    } else {
        r.rs = kStageUnits / 2;
        r.kparts = (r.K + 2 * C - 1) / (2 * C);
    }
    r.part = r.K / r.kparts;
    r.c0 = b * r.M / P.G;
    r.c1 = (b + 1) * r.M / P.G;
    return r;
}
// Rows of tensor-core stages whose byte length is a multiple of 128 would put
// the 8 rows of an ldmatrix tile in one bank group: they get 16 bytes of
// padding.  Other stages keep their rows contiguous (one bulk copy per stage).
__host__ __device__ __forceinline__ int row_stride(int part_bytes, bool mma) {
    return (mma && (part_bytes & 127) == 0) ? part_bytes + 16 : part_bytes;
}
__device__ __forceinline__ int phase_widx(int ph) { return ph == kPhLm ? 0 : ph + 1; }

// One 16-byte weight chunk (chunk index c of the x vector) against x in shared memory.
template <int WK>
__device__ __forceinline__ float chunk_dot(const uint4& w, const unsigned char* xs, int c) {
    float a = 0.0f, b = 0.0f;
    if constexpr (WK == WK_F32) {
        const float4 x = *reinterpret_cast<const float4*>(xs + (size_t)c * 16);
        a = fmaf(__uint_as_float(w.x), x.x, a); b = fmaf(__uint_as_float(w.y), x.y, b);
        a = fmaf(__uint_as_float(w.z), x.z, a); b = fmaf(__uint_as_float(w.w), x.w, b);
    } else if constexpr (WK == WK_BF16) {
        const uint4 x = *reinterpret_cast<const uint4*>(xs + (size_t)c * 16);
        const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            a = fmaf(bf16lo(ww[i]), bf16lo(xw[i]), a);
            b = fmaf(bf16hi(ww[i]), bf16hi(xw[i]), b);
        }
    } else {
        const uint4 xa = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32 + 16);
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float x0 = bf16lo(xw[2 * i]), x1 = bf16hi(xw[2 * i]);
            const float x2 = bf16lo(xw[2 * i + 1]), x3 = bf16hi(xw[2 * i + 1]);
            if constexpr (WK == WK_I8) {
                const uint32_t p = ww[i] ^ 0x80808080u;
                a = fmaf(i8_to_f(p, 0), x0, a); b = fmaf(i8_to_f(p, 1), x1, b);
                a = fmaf(i8_to_f(p, 2), x2, a); b = fmaf(i8_to_f(p, 3), x3, b);
            } else {
                a = fmaf(e4m3_to_f(ww[i], 0), x0, a); b = fmaf(e4m3_to_f(ww[i], 1), x1, b);
                a = fmaf(e4m3_to_f(ww[i], 2), x2, a); b = fmaf(e4m3_to_f(ww[i], 3), x3, b);
            }
        }
    }
    return a + b;
}

// Two rows' 16-byte chunks against the same x chunk (loaded once).
template <int WK>
__device__ __forceinline__ void chunk_dot2(const uint4& w0, const uint4& w1, const unsigned char* xs, int c, float& a0,
                                           float& a1) {
    if constexpr (WK == WK_F32) {
        const float4 x = *reinterpret_cast<const float4*>(xs + (size_t)c * 16);
        a0 = fmaf(__uint_as_float(w0.x), x.x, a0); a1 = fmaf(__uint_as_float(w1.x), x.x, a1);
        a0 = fmaf(__uint_as_float(w0.y), x.y, a0); a1 = fmaf(__uint_as_float(w1.y), x.y, a1);
        a0 = fmaf(__uint_as_float(w0.z), x.z, a0); a1 = fmaf(__uint_as_float(w1.z), x.z, a1);
        a0 = fmaf(__uint_as_float(w0.w), x.w, a0); a1 = fmaf(__uint_as_float(w1.w), x.w, a1);
    } else if constexpr (WK == WK_BF16) {
        const uint4 x = *reinterpret_cast<const uint4*>(xs + (size_t)c * 16);
        const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, u0[4] = {w0.x, w0.y, w0.z, w0.w}, u1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float xl = bf16lo(xw[i]), xh = bf16hi(xw[i]);
            a0 = fmaf(bf16lo(u0[i]), xl, a0); a1 = fmaf(bf16lo(u1[i]), xl, a1);
            a0 = fmaf(bf16hi(u0[i]), xh, a0); a1 = fmaf(bf16hi(u1[i]), xh, a1);
        }
    } else {
        const uint4 xa = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32 + 16);
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const uint32_t u0[4] = {w0.x, w0.y, w0.z, w0.w}, u1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float x[4] = {bf16lo(xw[2 * i]), bf16hi(xw[2 * i]), bf16lo(xw[2 * i + 1]), bf16hi(xw[2 * i + 1])};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if constexpr (WK == WK_I8) {
                    a0 = fmaf(i8_to_f(u0[i] ^ 0x80808080u, j), x[j], a0);
                    a1 = fmaf(i8_to_f(u1[i] ^ 0x80808080u, j), x[j], a1);
                } else {
                    a0 = fmaf(e4m3_to_f(u0[i], j), x[j], a0);
                    a1 = fmaf(e4m3_to_f(u1[i], j), x[j], a1);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// tensor-core stage products (mma.sync m16n8k16, FP32 accumulation): A = the
// stage's 16 rows, B = x in column 0 (the other 7 columns zero)
// ---------------------------------------------------------------------------
// Two codes of a 32-bit word as an exact FP16 pair (common.cuh: code2_to_f16x2).
template <int WK>
__device__ __forceinline__ uint32_t code2_f16x2(uint32_t word, bool hi) {
    return code2_to_f16x2<WK == WK_FP8>(word, hi);
}
// This warp's share of a stage: 16-column blocks kb = warp, warp + 8, ...
// (BF16) or 32-column units (8-bit: two MMAs per ldmatrix, the codes of an
// FP16 pair taken 4 apart, with x loaded in the same order).  Returns, for
// lanes with (lane & 3) == 0, the partial sums of rows lane/4 (s0) and
// lane/4 + 8 (s1).
template <int WK>
__device__ __forceinline__ void stage_mma(uint32_t a_base, const unsigned char* xb, int part, int warp, int lane,
                                          float& s0, float& s1) {
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int g = lane >> 2, t = lane & 3;
    if constexpr (WK == WK_BF16) {
        const int nkb = part >> 4;
        for (int kb = warp; kb < nkb; kb += kCW) {
            uint32_t a0, a1, a2, a3, b0 = 0u, b1 = 0u;
            ldsm_x4(a_base + (uint32_t)kb * 32u, a0, a1, a2, a3);
            if (g == 0) {
                const uint32_t* xw = reinterpret_cast<const uint32_t*>(xb + (size_t)kb * 32);
                b0 = xw[t];
                b1 = xw[4 + t];
            }
            mma_bf16(d, a0, a1, a2, a3, b0, b1);
        }
    } else {
        const int nku = part >> 5;
        for (int ku = warp; ku < nku; ku += kCW) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4(a_base + (uint32_t)ku * 32u, r0, r1, r2, r3);
            uint2 x0 = make_uint2(0u, 0u), x1 = make_uint2(0u, 0u);
            if (g == 0) {
                const uint2* xw = reinterpret_cast<const uint2*>(xb + (size_t)ku * 64);  // 32 FP16 values
                x0 = xw[t];
                x1 = xw[4 + t];
            }
            mma_f16(d, code2_f16x2<WK>(r0, false), code2_f16x2<WK>(r1, false), code2_f16x2<WK>(r0, true),
                    code2_f16x2<WK>(r1, true), x0.x, x0.y);
            mma_f16(d, code2_f16x2<WK>(r2, false), code2_f16x2<WK>(r3, false), code2_f16x2<WK>(r2, true),
                    code2_f16x2<WK>(r3, true), x1.x, x1.y);
        }
    }
    s0 = d[0];
    s1 = d[2];
}

// One LM-head stage by one warp on the tensor cores (narrow kernels): 16 rows stored as
// row pairs (rows 2p, 2p + 1 adjacent at pitch 2 x row + 16 bytes, so the 8 rows of every
// ldmatrix fall in distinct banks; ldmatrix rows 0-7 are the even rows, 8-15 the odd
// ones) times x over all K columns, two accumulator chains.  BF16 rows take x as BF16;
// 8-bit codes become exact FP16 pairs against x as FP16 (xb = the scaled copy).  Returns,
// for lanes with (lane & 3) == 0, the sums of stage rows 2(lane/4) (s0) and 2(lane/4) + 1 (s1).
template <int WK>
__device__ __forceinline__ void lm_stage_mma(uint32_t a, const unsigned char* xb, int K, int lane, float& s0,
                                             float& s1) {
    float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if constexpr (WK == WK_BF16) {
        float d2[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d3[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(xb) + (lane & 3);
        const int nkb = K >> 4;  // 16-column blocks (K a multiple of 64: whole groups of 4)
        for (int kb = 0; kb < nkb; kb += 4) {
            uint32_t a0, a1, a2, a3, c0, c1, c2, c3, e0, e1, e2, e3, f0, f1, f2, f3;
            ldsm_x4(a + (uint32_t)kb * 32u, a0, a1, a2, a3);
            ldsm_x4(a + (uint32_t)kb * 32u + 32u, c0, c1, c2, c3);
            ldsm_x4(a + (uint32_t)kb * 32u + 64u, e0, e1, e2, e3);
            ldsm_x4(a + (uint32_t)kb * 32u + 96u, f0, f1, f2, f3);
            mma_bf16(d0, a0, a1, a2, a3, xw[kb * 8], xw[kb * 8 + 4]);
            mma_bf16(d1, c0, c1, c2, c3, xw[kb * 8 + 8], xw[kb * 8 + 12]);
            mma_bf16(d2, e0, e1, e2, e3, xw[kb * 8 + 16], xw[kb * 8 + 20]);
            mma_bf16(d3, f0, f1, f2, f3, xw[kb * 8 + 24], xw[kb * 8 + 28]);
        }
        d0[0] += d2[0]; d0[2] += d2[2];
        d1[0] += d3[0]; d1[2] += d3[2];
    } else {
        const uint2* xw = reinterpret_cast<const uint2*>(xb) + (lane & 3);
        const int nku = K >> 5;  // 32-code units
#pragma unroll 2
        for (int ku = 0; ku < nku; ku++) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4(a + (uint32_t)ku * 32u, r0, r1, r2, r3);
            const uint2 x0 = xw[ku * 8], x1 = xw[ku * 8 + 4];
            mma_f16(d0, code2_f16x2<WK>(r0, false), code2_f16x2<WK>(r1, false), code2_f16x2<WK>(r0, true),
                    code2_f16x2<WK>(r1, true), x0.x, x0.y);
            mma_f16(d1, code2_f16x2<WK>(r2, false), code2_f16x2<WK>(r3, false), code2_f16x2<WK>(r2, true),
                    code2_f16x2<WK>(r3, true), x1.x, x1.y);
        }
    }
    s0 = d0[0] + d1[0];
    s1 = d0[2] + d1[2];
}

// x (activation type) -> FP16 scaled by 2^-e, e chosen so max |x| = am lands in [2^14, 2^15);
// each thread rewrites its own channel pairs (2t, 2t+1) + 512j.  Returns 2^e.  Out of line:
// rarely taken, and the per-layer code of the kernel is instruction-cache bound.
template <typename XT>
__device__ __noinline__ float rescale_x_fp16(const XT* xv, unsigned char* xh, int n, float am) {
    const int e = am <= FLT_MAX ? ((__float_as_int(am) >> 23) & 0xff) - 127 - 14 : 100;
    const int ec = max(-100, min(100, e));
    const float x_down = __int_as_float((127 - ec) << 23);
    for (int w = 2 * (int)threadIdx.x; w < n; w += 2 * kCT)
        for (int k = 0; k < 2 && w + k < n; k++)
            reinterpret_cast<__half*>(xh)[w + k] = __float2half_rn(to_f<XT>(xv[w + k]) * x_down);
    return __int_as_float((127 + ec) << 23);
}

template <int KV>
__device__ __forceinline__ float kv_code(uint32_t word, int j) {
    if constexpr (KV == KV_FP8) return e4m3_to_f(word, j);
    else return (float)(int8_t)((word >> (8 * j)) & 0xffu);
}
// 8-bit KV code of x at row scale `scale` (the per-kernel KV write's expression).
template <int KV>
__device__ __forceinline__ uint8_t kv_encode(float x, float scale) {
    if constexpr (KV == KV_FP8) {
        return (uint8_t)__nv_cvt_float_to_fp8(x / scale, __NV_SATFINITE, __NV_E4M3);
    } else {
        int q = __float2int_rn(x / scale);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        return (uint8_t)(int8_t)q;
    }
}

// ---------------------------------------------------------------------------
// shared memory layout
// ---------------------------------------------------------------------------
struct PSmem {
    int stage_bytes, ring, kvbuf, uni, res, lnp, red, xh, lnx, mred, misc, geo, bars, total;
};

template <int WK, int KV>
__host__ __device__ inline PSmem persist_layout(int C, int ns, int kv_rows, int tp) {
    const int xb = (WK == WK_F32) ? 4 : 2;
    const int wb = PTraits<WK>::kWB;
    const int kvb = (KV == KV_F32) ? 4 : (KV == KV_BF16 ? 2 : 1);
    const bool k8 = (KV == KV_I8 || KV == KV_FP8);
    const int rpp = kCT / (kHSz * kvb / 16);
    PSmem s;
    s.stage_bytes = kStageUnits * (C * wb + 16) + kTail;
    int off = 0;
    s.ring = off; off += ns * s.stage_bytes;
    s.kvbuf = off; off += 2 * kv_rows * kHSz * kvb + (k8 ? 2 * (kv_rows + 8) * 4 : 0);
    off = (off + 15) & ~15;
    s.uni = off;  // x vector of the current phase, or the attention scratch
    int xs_bytes = 4 * C * xb;
    if (tp * kMaxCtas * 8 > xs_bytes) xs_bytes = tp * kMaxCtas * 8;  // the LM pairs of every CTA of every rank
    const int attn_bytes = (rpp * kHSz + 3 * kHSz + kv_rows + (kMaxSplits - 1) * (kHSz + 2)) * 4;
    off += ((xs_bytes > attn_bytes ? xs_bytes : attn_bytes) + 15) & ~15;
    s.res = off; off += C * 4;
    s.lnp = off; off += ((2 * C * xb) + 15) & ~15;  // LayerNorm gamma | beta of the current phase
    s.red = off; off += (tp > 1) ? tp * C * 4 : 0;  // every rank's projection partials
    s.xh = off; off += (wb == 1) ? 4 * C * 2 : 0;   // x as FP16, the B operand of 8-bit weights
    s.lnx = off; off += (wb == 1) ? (2 * kMaxLayers + 2) * 4 : 0;  // LayerNorm exponents of 8-bit weights
    s.mred = off; off += 2 * kCW * 16 * 4;           // per-warp row sums of a stage, double-buffered
    s.misc = off; off += kMiscFloats * 4;
    s.geo = off; off += 5 * (int)sizeof(PhaseRows) + 4 * 8;  // this CTA's phase geometry, output bases
    s.bars = off; off += (2 * kMaxNs + 3) * 8;
    s.total = off;
    return s;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// MODE 0 (narrow): C <= 1024, at most 96 positions per attention CTA,
// LayerNorm parameters in registers, short gathers.  MODE 1 (wide): C up to
// 2048 and attention chunks up to 256 positions (GPT-2-XL).  MODE 2: wide,
// as one rank of a tensor-parallel group.
template <int WK, int KV, int MODE>
__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const PersistParams P) {
    constexpr bool WIDE = MODE >= 1;
    constexpr bool TPG = MODE == 2;
    // tensor-core stage products for the wide kernels (8-bit / BF16 weights); CUDA cores otherwise
    constexpr bool MMA = WIDE && (WK != WK_F32);
    using XT = typename PTraits<WK>::XT;
    constexpr int kWB = PTraits<WK>::kWB;
    constexpr int kXB = (int)sizeof(XT);
    constexpr bool w8 = (WK == WK_I8 || WK == WK_FP8);
    constexpr bool k8 = (KV == KV_I8 || KV == KV_FP8);
    constexpr int kvb = (KV == KV_F32) ? 4 : (KV == KV_BF16 ? 2 : 1);
    constexpr int kRowB = kHSz * kvb;  // bytes of one K or V row
    constexpr int kLP = kRowB / 16;    // lanes per row in the attention loops
    constexpr int kRPP = kCT / kLP;    // rows per pass
    constexpr int kE = 16 / kvb;       // elements per 16-byte slice
    using KT = typename PTraits<(KV == KV_F32) ? WK_F32 : WK_BF16>::XT;  // KV element type (float kinds)
    extern __shared__ __align__(16) unsigned char sm[];
    const PSmem lay = persist_layout<WK, KV>(P.C, P.nsw, WIDE ? P.kv_rows : kNarrowKvRows, P.tp_size);
    const int kKvRows = WIDE ? P.kv_rows : kNarrowKvRows;  // staged positions per attention CTA
    constexpr int kCPT = (WIDE ? kMaxC : kNarrowC) / kCT;  // channels per consumer thread
    unsigned char* ring = sm + lay.ring;
    unsigned char* kvbuf = sm + lay.kvbuf;
    unsigned char* xs = sm + lay.uni;
    float* res = reinterpret_cast<float*>(sm + lay.res);
    float* red = reinterpret_cast<float*>(sm + lay.red);
    unsigned char* xh = sm + lay.xh;                      // x as FP16 (8-bit weights)
    float* mred = reinterpret_cast<float*>(sm + lay.mred);
    float* misc = reinterpret_cast<float*>(sm + lay.misc);
    int* misc_i = reinterpret_cast<int*>(misc);
    volatile int* stop = misc_i + (kMiscFloats - 1);  // consumers left early: the producer stops
    volatile int* lm_done = misc_i + (kMiscFloats - 2);  // steps whose LM head all consumers finished
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + lay.bars);
    uint64_t* empty = full + kMaxNs;
    uint64_t* kv_bar = empty + kMaxNs;
    uint64_t* ln_bar = kv_bar + 1;
    const XT* lnp = reinterpret_cast<const XT*>(sm + lay.lnp);
    // attention scratch (aliases xs: never live at the same time)
    float* accbuf = reinterpret_cast<float*>(xs);
    float* q_s = accbuf + kRPP * kHSz;
    float* kcur = q_s + kHSz;
    float* vcur = kcur + kHSz;
    float* p_s = vcur + kHSz;
    float* mrg = p_s + kKvRows;  // (splits - 1) x (64 + 2) partials of the head
    uint8_t* cur8 = reinterpret_cast<uint8_t*>(misc + 64);  // 8-bit codes of the new K | V rows
    float* cur_sc = misc + 96;                              // and their scales

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int C = P.C, L = P.L, NH = P.NH, maxT = P.maxT, S = P.splits, G = P.G, NS = P.nsw;
    const int LA = max(2, min(NS, P.lookahead));
    PeerSet peers;  // tensor parallel only (constant indices into the parameters)
    const PeerSet* pgp = nullptr;
    if constexpr (TPG) {
#pragma unroll
        for (int r = 0; r < 8; r++) peers.x[r] = P.peer_x[r];
        peers.n = P.tp_size;
        peers.rank = P.tp_rank;
        peers.off_abort = P.xoff_abort;
        pgp = &peers;
    }
    const int b = blockIdx.x;
    const int unit_bytes = C * kWB;  // one row-unit: a row of K = C, half a K-half of K = 4C
    const uint32_t plim = P.poll_limit;  // polls of one exchange wait before it gives up
    const uint32_t epoch0 = *P.d_epoch;
    const int pos0 = *P.d_pos;
    int tok = *P.d_token;
    // the same checks in every CTA, so all of them leave together
    if (pos0 < 0 || pos0 + P.n_steps > maxT) {
        if (b == 0 && tid == 0) report_device_error(GPT2B_DEVERR_BAD_POS);
        return;
    }
    if (tok < 0 || tok >= P.V) {
        if (b == 0 && tid == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN);
        return;
    }
    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kCW);
        }
        mbar_init(kv_bar, 1);
        mbar_init(ln_bar, 1);
        *stop = 0;
        *lm_done = 0;
        mbar_fence_init();
    }
    // the row geometry of every phase and the exchange bases, computed once: the per-phase
    // paths read them from shared memory (no divisions or parameter loads there)
    PhaseRows* geo = reinterpret_cast<PhaseRows*>(sm + lay.geo);
    unsigned long long** obase = reinterpret_cast<unsigned long long**>(sm + lay.geo + 5 * sizeof(PhaseRows));
    if constexpr (w8)  // the LayerNorm exponents, read once: global memory is far on the per-phase path
        for (int i = tid; i <= 2 * L; i += kThreads) reinterpret_cast<int*>(sm + lay.lnx)[i] = P.ln_exp[i];
    if (tid < 5) {
        geo[tid] = phase_rows<MMA>(P, tid, b);
    } else if (tid < 9) {
        const int k = tid - 5;
        obase[k] = k == kPhQkv ? P.ll_qkv : (k == kPhProj ? P.ll_proj : (k == kPhFc ? P.ll_fc : P.ll_fcproj));
    }
    __syncthreads();  // the last block-wide barrier: producer and consumers part here

    // =====================================================================
    // producer warp: every weight stage of every phase, layer and step
    // =====================================================================
    if (warp == kCW) {
        if (lane != 0) return;
        const uint64_t pol_lm = l2_evict_last_policy(), pol_layer = l2_evict_first_policy();
        int issued = 0, st = 0;
        int skip_lo = 0, skip_hi = 0;  // the latest block of stages the LM head's warps issue
        int lm_gate = -1;              // step of that block: wait for its LM head before the next issue
        for (int step = 0; step < P.n_steps; step++) {
            for (int u = 0; u <= 4 * L; u++) {
                const int l = (u == 4 * L) ? 0 : (u >> 2);
                const int ph = (u == 4 * L) ? kPhLm : (u & 3);
                const PhaseRows pr = geo[ph];
                const int widx = phase_widx(ph);
                const int part_bytes = pr.part * kWB;  // per row and stage
                const size_t row_bytes = (size_t)pr.K * kWB;
                const unsigned char* wl = P.W[widx] + (ph == kPhLm ? (size_t)P.v0 * row_bytes
                                                                   : (size_t)l * pr.M * row_bytes);
                const unsigned char* bias = nullptr;
                if (ph == kPhQkv) bias = reinterpret_cast<const unsigned char*>(P.qkvb);
                else if (ph == kPhProj) bias = reinterpret_cast<const unsigned char*>(P.attprojb);
                else if (ph == kPhFc) bias = reinterpret_cast<const unsigned char*>(P.fcb);
                else if (ph == kPhFcproj) bias = reinterpret_cast<const unsigned char*>(P.fcprojb);
                if (bias) bias += (size_t)l * pr.M * kXB;
                const float* scl = w8 ? P.S[widx] + (ph == kPhLm ? (size_t)P.v0 : (size_t)l * pr.M) : nullptr;
                // look-ahead: the whole ring for the LM head, P.lookahead stages in the layers
                const int ahead = ph == kPhLm ? NS : LA;
                // the narrow tensor-core LM head issues its own stages from NS on: the producer
                // only counts them, and before its next issue waits until the consumers have
                // finished the whole LM head (the warps advance the slots' barriers by several
                // phases meanwhile; after that point every LM phase has completed, so its
                // parity waits see each barrier at most one phase behind again)
                const bool lm_self = !MMA && WK != WK_F32 && ph == kPhLm;
                for (int r0 = pr.c0; r0 < pr.c1; r0 += pr.rs) {
                    const int nr = min(pr.rs, pr.c1 - r0);
                    const bool skip = lm_self && r0 - pr.c0 >= NS * pr.rs;
                    for (int kq = 0; kq < pr.kparts; kq++) {
                        if (skip) {
                            if (skip_hi != issued) skip_lo = issued;  // a new block of skipped stages
                            skip_hi = ++issued;
                            lm_gate = step;
                            if (++st == NS) st = 0;
                            continue;
                        }
                        if (lm_gate >= 0) {
                            bool ok = false;
                            for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
                                if (*lm_done > lm_gate) { ok = true; break; }
                                if (*stop) break;
                                __nanosleep(64);
                            }
                            if (!ok) goto producer_drain;
                            __threadfence_block();
                            lm_gate = -1;
                        }
                        // wait until (a) the slot's previous use, stage issued - NS, and (b) the
                        // look-ahead bound, stage issued - ahead, were released.  (a) is needed
                        // on its own: the LM head's warps release their stages out of order, so
                        // a later stage's release does not free an earlier stage's slot.  Every
                        // earlier issue waited for its own (a), so neither barrier can be two
                        // phases behind the parity waited for
                        for (int q = 0; q < 2; q++) {
                            const int j = issued - (q == 0 ? NS : ahead);
                            if (j < 0 || (q == 1 && ahead == NS)) continue;
                            const uint32_t par = (uint32_t)((j / NS) & 1);
                            bool ok = false;
                            for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
                                if (mbar_try_wait(&empty[j % NS], par)) { ok = true; break; }
                                if (*stop) break;
                            }
                            if (!ok) goto producer_drain;
                        }
                        unsigned char* sd = ring + (size_t)st * lay.stage_bytes;
                        unsigned char* tail = sd + kStageUnits * (unit_bytes + 16);
                        const bool last = (kq == pr.kparts - 1);
                        uint32_t bb = 0, sb = 0;
                        size_t ba = 0, sa = 0;
                        if (last && bias) {
                            ba = ((size_t)r0 * kXB) & ~(size_t)15;
                            bb = (uint32_t)((((size_t)(r0 + nr) * kXB + 15) & ~(size_t)15) - ba);
                        }
                        if (last && w8) {
                            sa = ((size_t)r0 * 4) & ~(size_t)15;
                            sb = (uint32_t)((((size_t)(r0 + nr) * 4 + 15) & ~(size_t)15) - sa);
                        }
                        PTRACE_STAGE(0, issued);
                        mbar_arrive_expect_tx(&full[st], (uint32_t)(nr * part_bytes) + bb + sb);
                        const int rstride = row_stride(part_bytes, MMA);
                        // L2 policy: the LM head's rows under evict_last, the layers' weights under
                        // evict_first, so the LM head (77 MB BF16, 39 MB INT8) stays in L2 across the
                        // tokens of a call while the layers stream through (-1.8 % BF16, -4.3 % INT8
                        // per token; evict_last alone -0.3 %)
                        const uint64_t pol = ph == kPhLm ? pol_lm : pol_layer;
                        if (!MMA && WK != WK_F32 && ph == kPhLm) {  // row pairs for the LM head's tensor cores
                            for (int i = 0; 2 * i < nr; i++)
                                bulk_g2s_hint(sd + (size_t)i * (2 * part_bytes + 16), wl + (size_t)(r0 + 2 * i) * row_bytes,
                                              (uint32_t)(min(2, nr - 2 * i) * part_bytes), &full[st], pol);
                        } else if (rstride == part_bytes && pr.kparts == 1) {  // contiguous rows: one copy
                            bulk_g2s_hint(sd, wl + (size_t)r0 * row_bytes, (uint32_t)(nr * part_bytes), &full[st], pol);
                        } else {
                            for (int i = 0; i < nr; i++)
                                bulk_g2s_hint(sd + (size_t)i * rstride,
                                              wl + (size_t)(r0 + i) * row_bytes + (size_t)kq * part_bytes,
                                              (uint32_t)part_bytes, &full[st], pol);
                        }
                        if (bb) bulk_g2s(tail, bias + ba, bb, &full[st]);
                        if (sb)
                            bulk_g2s(tail + kTailSlot, reinterpret_cast<const unsigned char*>(scl) + sa, sb, &full[st]);
                        issued++;
                        if (++st == NS) st = 0;
                    }
                }
            }
        }
    producer_drain:
        // leave with none of this warp's copies in flight: the stages before an LM head's own
        // block landed once its consumers finished it; the LM head's warps wait for their own
        if (lm_gate >= 0)
            for (uint32_t i = 0; i < kMbarSpinLimit && *lm_done <= lm_gate && !*stop; ++i) __nanosleep(64);
        for (int k = issued > NS ? issued - NS : 0; k < issued; k++)
            if (k < skip_lo || k >= skip_hi) mbar_wait(&full[k % NS], (uint32_t)((k / NS) & 1));
        return;
    }

    // =====================================================================
    // consumers (256 threads)
    // =====================================================================
    const bool attn_cta = b < NH * S;
    const int ah = attn_cta ? b / S : 0, as = attn_cta ? b % S : 0;
    const size_t NHmT = (size_t)NH * maxT;
    bool bad = false;
    int cst = 0;            // ring position of the next stage
    uint32_t cpar = 0;      // and its full-barrier parity
    int kv_issued = 0, kv_uses = 0;
    uint32_t ln_par = 0;    // phase parity of the LayerNorm parameter barrier
    bool ln_pending = false;  // thread 0: a parameter copy is in flight
    uint32_t consumed_stages = 0;  // selects the mred buffer of a stage
#ifdef GPT2B_PERSIST_TRACE
    int consumed_n = 0;
#endif

    // ---- KV staging of an attention CTA: one buffer; the next layer's rows
    //      are staged as soon as this layer's attention is done ----
    auto kv_issue = [&](int step, int l) {  // tid 0 only
        const int pos = pos0 + step, total = pos + 1;
        const int chunk = engine_attn_chunk(total, S);
        const int j0 = as * chunk, j1 = min(j0 + chunk, total);
        if (j1 <= j0) return;
        if (step > 0) {
            // rows below pos were appended during earlier steps of this call:
            // acquire the release of step - 1, whose tag is epoch0 + step (rows
            // written by earlier launches are ordered by the kernel boundary)
            const uint32_t need = epoch0 + (uint32_t)step;
            const unsigned* flag = P.kv_flag + l * NH + ah;
            for (uint32_t it = 0;; ++it) {
                unsigned f;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
                if ((int)(f - need) >= 0) break;
                if (it > plim) { give_up(P.abort_flag, pgp); bad = true; return; }
                if ((it & 15) == 15 && aborted(P.abort_flag)) { bad = true; return; }
                __nanosleep(64);
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        const size_t lk = (size_t)l * 2 * NHmT;  // layer offset in rows
        const size_t krow = (size_t)ah * maxT + j0;
        const int n = j1 - j0;
        const uint32_t rb = (uint32_t)(n * kRowB);
        uint32_t tx = 2 * rb, sb = 0;
        size_t k0 = 0;
        if constexpr (k8) {  // scale copies start at the 16-byte boundary below the first row
            k0 = krow & ~(size_t)3;
            sb = (uint32_t)((((krow + n + 3) & ~(size_t)3) - k0) * 4);
            tx += 2 * sb;
        }
        mbar_arrive_expect_tx(kv_bar, tx);
        bulk_g2s(kvbuf, P.kv + (lk + krow) * kRowB, rb, kv_bar);
        bulk_g2s(kvbuf + kKvRows * kRowB, P.kv + (lk + NHmT + krow) * kRowB, rb, kv_bar);
        if constexpr (k8) {
            const float* sc = P.kv_scale + lk;
            bulk_g2s(kvbuf + 2 * kKvRows * kRowB, sc + k0, sb, kv_bar);
            bulk_g2s(kvbuf + 2 * kKvRows * kRowB + (kKvRows + 8) * 4, sc + NHmT + k0, sb, kv_bar);
        }
        kv_issued++;
    };
    if (attn_cta && tid == 0) kv_issue(0, 0);
    if (cta_any(bad)) goto consumer_abort;

    {
        const XT* wpe = reinterpret_cast<const XT*>(P.wpe);
        float gv[(WIDE || TPG) ? kGatherJ : kGatherJs];
        for (int step = 0; step < P.n_steps; step++) {
            // the last LayerNorm's mean within this step (the same in every consumer thread);
            // zero at each step's first LayerNorm, so a step's arithmetic does not depend on
            // how the steps are split into calls
            float ln_shift = 0.0f;
            const uint32_t tag = epoch0 + (uint32_t)step + 1u;
            const int pos = pos0 + step;
            PTRACE(kTraceEv - 1);
            float best_v = -FLT_MAX;
            int best_i = 0x7fffffff;
#pragma unroll 1
            for (int u = 0; u <= 4 * L; u++) {
                const bool lm = (u == 4 * L);
                const int l = lm ? 0 : (u >> 2);
                const int ph = lm ? kPhLm : (u & 3);
                XT* xv = reinterpret_cast<XT*>(xs);
                // 8-bit tensor-core stages take x as FP16 scaled by 2^-e, and the row sums are
                // multiplied back by 2^e (exact): no overflow for large activations, full precision
                // for small ones.  LayerNorm phases take e from a bound of |x| fixed by the LayerNorm
                // parameters (P.ln_exp); the gather phases from the CTA's max |x| (xmax: this
                // thread's part), combined on the barrier that follows the gather.
                float xmax = 0.0f, x_up = 1.0f, x_down = 1.0f;

                // ---------- x of this phase ----------
                if (ph == kPhQkv || ph == kPhFc || lm) {
                    int ln_e = 0;
                    if constexpr (w8)
                        ln_e = reinterpret_cast<const int*>(sm + lay.lnx)[lm ? 2 * L : 2 * l + (ph == kPhFc ? 1 : 0)];
                    // residual update (fcproj of the previous layer, or proj), then LayerNorm;
                    // gamma and beta are loaded (narrow: into registers; wide: bulk-copied into
                    // shared memory) while the inputs are awaited
                    float lw[WIDE ? 1 : kCPT], lb[WIDE ? 1 : kCPT];
                    if constexpr (!WIDE) {
                        const XT* lnw = reinterpret_cast<const XT*>(lm ? P.lnfw : (ph == kPhQkv ? P.ln1w : P.ln2w));
                        const XT* lnb = reinterpret_cast<const XT*>(lm ? P.lnfb : (ph == kPhQkv ? P.ln1b : P.ln2b));
                        const size_t lo = lm ? 0 : (size_t)l * C;
#pragma unroll
                        for (int j = 0; j < kCPT; j++) {
                            const int c = pair_slot(tid, j);
                            lw[j] = c < C ? to_f<XT>(lnw[lo + c]) : 0.0f;
                            lb[j] = c < C ? to_f<XT>(lnb[lo + c]) : 0.0f;
                        }
                    } else if (tid == 0) {
                        const void* lnw = lm ? P.lnfw : (ph == kPhQkv ? P.ln1w : P.ln2w);
                        const void* lnb = lm ? P.lnfb : (ph == kPhQkv ? P.ln1b : P.ln2b);
                        const size_t lo = lm ? 0 : (size_t)l * C;
                        const uint32_t nb = (uint32_t)(C * sizeof(XT));
                        mbar_arrive_expect_tx(ln_bar, 2 * nb);
                        bulk_g2s(sm + lay.lnp, reinterpret_cast<const XT*>(lnw) + lo, nb, ln_bar);
                        bulk_g2s(sm + lay.lnp + nb, reinterpret_cast<const XT*>(lnb) + lo, nb, ln_bar);
                        ln_pending = true;
                    }
                    if (u == 0) {  // embedding: res = round(wte[tok] + wpe[pos]) (encoder_forward_kv)
#pragma unroll 1
                        for (int j = 0; j < kCPT; j++) {
                            const int c = pair_slot(tid, j);
                            if (c < C) {
                                float e;
                                if constexpr (w8) {
                                    const uint8_t code = P.W[0][(size_t)tok * C + c];
                                    const float v = (WK == WK_I8) ? (float)(int8_t)code : e4m3_to_f((uint32_t)code, 0);
                                    e = round_to<__nv_bfloat16>(v * P.S[0][tok]);
                                } else {
                                    e = to_f<XT>(reinterpret_cast<const XT*>(P.W[0])[(size_t)tok * C + c]);
                                }
                                res[c] = round_to<XT>(e + to_f<XT>(wpe[(size_t)pos * C + c]));
                            }
                        }
                    } else {
                        const int TP = TPG ? P.tp_size : 1;
                        const size_t lsrc = (ph == kPhFc) ? (size_t)l : (size_t)(lm ? L - 1 : l - 1);
                        const unsigned long long* src = ((ph == kPhFc) ? P.ll_proj : P.ll_fcproj) + lsrc * TP * C;
                        bool ok = true;
                        if constexpr (!TPG) {
                            ok = ll_gather2<WIDE>(P.abort_flag, pgp, plim, src, C, tag, gv);
#pragma unroll
                            for (int j = 0; j < kCPT; j++) {
                                const int c = pair_slot(tid, j);
                                if (c < C) res[c] = round_to<XT>(res[c] + gv[j]);
                            }
                        } else {
                            // every rank's FP32 partial [TP][C] into red, then the sum in rank
                            // order (the same on every rank), rounded as the single-GPU store
                            const int n = TP * C;
                            for (int base = 0; base < n && ok; base += kGatherJ * kCT) {
                                ok = ll_gather_group(P.abort_flag, pgp, plim, src + base, min(n - base, kGatherJ * kCT), tag, gv);
#pragma unroll
                                for (int j = 0; j < kGatherJ; j++)
                                    if (base + tid + j * kCT < n) red[base + tid + j * kCT] = gv[j];
                            }
                            cta_sync();
#pragma unroll
                            for (int j = 0; j < kCPT; j++) {
                                const int c = pair_slot(tid, j);
                                if (c < C) {
                                    float v = 0.0f;
                                    for (int r = 0; r < TP; r++) v += red[r * C + c];
                                    res[c] = round_to<XT>(res[c] + round_to<XT>(v));
                                }
                            }
                        }
                        if (cta_any(!ok)) goto consumer_abort;
                    }
                    // LayerNorm (layernorm.cuh:171-241) statistics in one pass: sum and sum of
                    // squares of the rounded residual, warp totals in misc[0..15], one barrier
                    // (the two-pass form costs a second barrier and measured 2 % slower per
                    // token).  The sums are taken about the previous LayerNorm's mean, so the
                    // variance E[(x-k)^2] - E[x-k]^2 does not cancel when a row's mean is large
                    // against its spread
                    float s = 0.0f, q = 0.0f;
#pragma unroll
                    for (int j = 0; j < kCPT; j++)
                        if (pair_slot(tid, j) < C) {
                            const float v = res[pair_slot(tid, j)] - ln_shift;
                            s += v;
                            q += v * v;
                        }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        s += __shfl_xor_sync(0xffffffffu, s, o);
                        q += __shfl_xor_sync(0xffffffffu, q, o);
                    }
                    if (lane == 0) { misc[warp] = s; misc[kCW + warp] = q; }
                    cta_sync();
                    s = 0.0f;
                    q = 0.0f;
#pragma unroll
                    for (int w = 0; w < kCW; w++) { s += misc[w]; q += misc[kCW + w]; }
                    const float ms = s / (float)C;
                    const float mean = ln_shift + ms;
                    const float rstd = rsqrtf(fmaxf(q / (float)C - ms * ms, 0.0f) + 1e-5f);
                    ln_shift = mean;
                    if constexpr (WIDE) {
                        if (!mbar_wait(ln_bar, ln_par)) bad = true;
                        ln_par ^= 1u;
                        ln_pending = false;
                    }
                    if constexpr (w8) {  // tensor-core stages: every phase (wide), the LM head (narrow)
                        x_down = __int_as_float((127 - ln_e) << 23);
                        x_up = __int_as_float((127 + ln_e) << 23);
                    }
#pragma unroll
                    for (int j = 0; j < kCPT; j++) {
                        const int c = pair_slot(tid, j);
                        if (c < C) {
                            const float g = WIDE ? to_f<XT>(lnp[c]) : lw[j];
                            const float bb = WIDE ? to_f<XT>(lnp[C + c]) : lb[j];
                            const XT xvv = from_f<XT>((rstd * (res[c] - mean)) * g + bb);
                            xv[c] = xvv;
                            if constexpr (w8)
                                if (MMA || lm) reinterpret_cast<__half*>(xh)[c] = __float2half_rn(to_f<XT>(xvv) * x_down);
                        }
                    }
                } else {
                    // PROJ: x = atty of this rank's heads; FCPROJ: x = gelu(fc) of this rank's FC rows
                    const int n = (ph == kPhProj) ? P.proj_k : P.fcproj_k;
                    const unsigned long long* src = (ph == kPhProj) ? P.ll_atty + (size_t)l * n : P.ll_fc + (size_t)l * n;
                    const bool ok = ll_gather2<WIDE>(P.abort_flag, pgp, plim, src, n, tag, gv);
#pragma unroll
                    for (int j = 0; j < (WIDE ? kGatherJ : kGatherJs); j++) {
                        const int w = pair_slot(tid, j);
                        if (w < n) {
                            const XT xvv = from_f<XT>(gv[j]);
                            xv[w] = xvv;
                            if constexpr (MMA && w8) {  // FP16 as is: exact for |x| in [2^-14, 65504]
                                xmax = fmaxf(xmax, fabsf(to_f<XT>(xvv)));
                                reinterpret_cast<__half*>(xh)[w] = __float2half_rn(to_f<XT>(xvv));
                            }
                        }
                    }
                    if constexpr (MMA && w8) {
                        xmax = warp_max(xmax);
                        if (lane == 0) misc[kXmaxSlot + warp] = xmax;
                    }
                    if (cta_any(!ok)) goto consumer_abort;
                    if constexpr (MMA && w8) {
                        // the CTA's max |x| (NaN entries are skipped by fmaxf and stay NaN): outside
                        // [2^-4, 2^15] the FP16 copy is redone with x scaled into [2^14, 2^15) (rare;
                        // kept compact, the per-layer code is instruction-cache bound)
                        float am = misc[kXmaxSlot];
#pragma unroll
                        for (int w = 1; w < kCW; w++) am = fmaxf(am, misc[kXmaxSlot + w]);
                        if (am > 32768.0f || (am > 0.0f && am < 0.0625f)) x_up = rescale_x_fp16(xv, xh, n, am);
                    }
                }
                cta_sync();
                PTRACE(u * 3 + 0);

                // ---------- the matrix rows of this CTA ----------
                {
                    const PhaseRows pr = geo[ph];
                    unsigned long long* out = lm ? nullptr : obase[ph] + (size_t)l * pr.M;
                    const bool has_bias = !lm;
                    const int part_bytes = pr.part * kWB;
                    const int rstride = row_stride(part_bytes, MMA);
                    const int pc = part_bytes / 16;  // chunks per row and stage
                    // emit one finished row (bias, scale, GELU / partial store / logits)
                    auto emit = [&](const unsigned char* sd, int r0, int rl, float v) {
                        const unsigned char* tail = sd + kStageUnits * (unit_bytes + 16);
                        const int row = r0 + rl;
                        if constexpr (w8) v *= reinterpret_cast<const float*>(tail + kTailSlot + ((r0 * 4) & 15))[rl];
                        if (has_bias) v += to_f<XT>(reinterpret_cast<const XT*>(tail + ((r0 * kXB) & 15))[rl]);
                        if (lm) {
                            P.logits[row] = v;
                            if (P.v0 + row < P.V) best_merge(best_v, best_i, v, P.v0 + row);
                        } else if (TPG && (ph == kPhProj || ph == kPhFcproj)) {  // FP32 partials to every rank
                            ll_store_group<TPG>(P.peer_x[0], pgp, ph == kPhProj ? P.xoff_proj : P.xoff_fcproj,
                                                ((size_t)l * P.tp_size + P.tp_rank) * C + row, v, tag);
                        } else {
                            ll_store(out + row, round_to<XT>(ph == kPhFc ? gelu_tanh(v) : v), tag);
                        }
                    };
                    if (!MMA && WK != WK_F32 && lm) {
                        // the LM head on the tensor cores, one warp per stage: stage k of this CTA
                        // goes to warp k mod nw, which multiplies its 16 rows by x over all of K and
                        // emits them, then releases the stage with the 8 arrivals its barrier counts.
                        // nw divides the ring depth, so every ring slot is used by one warp only and
                        // a warp never waits for a slot's phase more than one ahead of the last it
                        // consumed there (a parity wait cannot tell phases two apart)
                        // The producer issues the first NS stages; every later stage k is issued by
                        // its own warp into the slot it has just read (stage k - NS, the same warp
                        // and slot), so a slot is refilled as soon as its warp is done with it.
                        int nw = kCW;
                        while (NS % nw) nw--;
                        const int lmrs = 2 * part_bytes + 16;
                        const int nst = (pr.c1 - pr.c0 + pr.rs - 1) / pr.rs;
                        const unsigned char* wlm = P.W[0] + (size_t)P.v0 * part_bytes;
                        const unsigned char* slm = w8 ? reinterpret_cast<const unsigned char*>(P.S[0] + P.v0) : nullptr;
                        const uint64_t pol_lm = l2_evict_last_policy();
                        const uint32_t a_lane =
                            (uint32_t)((lane & 7) * lmrs + ((lane >> 3) & 1) * part_bytes + (lane >> 4) * 16);
                        int k = 0;
                        for (int r0 = pr.c0; r0 < pr.c1; r0 += pr.rs, ++k) {
                            if (k % nw == warp) {
                                const int nr = min(pr.rs, pr.c1 - r0);
#ifdef GPT2B_PERSIST_TRACE
                                if (lane == 0) { PTRACE_STAGE(1, consumed_n); PTRACE_STAGE(4, consumed_n); }
#endif
                                if (!mbar_wait(&full[cst], cpar)) bad = true;
#ifdef GPT2B_PERSIST_TRACE
                                if (lane == 0) PTRACE_STAGE(2, consumed_n);
#endif
                                const unsigned char* sd = ring + (size_t)cst * lay.stage_bytes;
                                float s0, s1;
                                lm_stage_mma<WK>(smem_addr(sd) + a_lane, w8 ? xh : xs, C, lane, s0, s1);
                                if ((lane & 3) == 0) {
                                    const int g = lane >> 2;
                                    if (2 * g < nr) emit(sd, r0, 2 * g, w8 ? s0 * x_up : s0);
                                    if (2 * g + 1 < nr) emit(sd, r0, 2 * g + 1, w8 ? s1 * x_up : s1);
                                }
                                if (k + NS < nst) {  // refill: stage k + NS into this slot
                                    const int rn = r0 + NS * pr.rs, nrn = min(pr.rs, pr.c1 - rn);
                                    uint32_t sb = 0;
                                    size_t sa = 0;
                                    if (w8) {
                                        sa = ((size_t)rn * 4) & ~(size_t)15;
                                        sb = (uint32_t)((((size_t)(rn + nrn) * 4 + 15) & ~(size_t)15) - sa);
                                    }
                                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // our reads first
                                    __syncwarp();
                                    unsigned char* sdw = ring + (size_t)cst * lay.stage_bytes;
                                    if (lane == 0) mbar_arrive_expect_tx(&full[cst], (uint32_t)(nrn * part_bytes) + sb);
                                    __syncwarp();
                                    if (2 * lane < nrn)
                                        bulk_g2s_hint(sdw + (size_t)lane * lmrs, wlm + (size_t)(rn + 2 * lane) * part_bytes,
                                                      (uint32_t)(min(2, nrn - 2 * lane) * part_bytes), &full[cst], pol_lm);
                                    if (w8 && lane == 0)
                                        bulk_g2s(sdw + kStageUnits * (unit_bytes + 16) + kTailSlot, slm + sa, sb, &full[cst]);
                                }
                                __syncwarp();
                                if (lane == 0) mbar_arrive_cnt(&empty[cst], kCW);
#ifdef GPT2B_PERSIST_TRACE
                                if (lane == 0) PTRACE_STAGE(3, consumed_n);
#endif
                            }
                            if (++cst == NS) { cst = 0; cpar ^= 1u; }
#ifdef GPT2B_PERSIST_TRACE
                            consumed_n++;
#endif
                        }
                    } else if (!MMA && lm) {
                        // the LM head on CUDA cores (FP32 weights), two stages per round: warp w takes
                        // rows w and w + 8 of both (four sums sharing every x load); one K-part per row
                        for (int r0 = pr.c0; r0 < pr.c1; r0 += 2 * pr.rs) {
                            const int na = min(pr.rs, pr.c1 - r0), nb = min(pr.rs, pr.c1 - r0 - pr.rs);
                            const int cb = cst + 1 == NS ? 0 : cst + 1;
                            const uint32_t pb = cst + 1 == NS ? cpar ^ 1u : cpar;
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) { PTRACE_STAGE(1, consumed_n); PTRACE_STAGE(4, consumed_n); }
#endif
                            if (!mbar_wait(&full[cst], cpar)) bad = true;
                            if (nb > 0 && !mbar_wait(&full[cb], pb)) bad = true;
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) PTRACE_STAGE(2, consumed_n);
#endif
                            const unsigned char* sa = ring + (size_t)cst * lay.stage_bytes;
                            const unsigned char* sb = ring + (size_t)cb * lay.stage_bytes;
                            const bool a1v = warp + kCW < na, b0v = warp < nb, b1v = warp + kCW < nb;
                            if (warp < na) {
                                const unsigned char* w0 = sa + (size_t)warp * part_bytes;
                                const unsigned char* w1 = sa + (size_t)(a1v ? warp + kCW : warp) * part_bytes;
                                const unsigned char* w2 = sb + (size_t)(b0v ? warp : 0) * part_bytes;
                                const unsigned char* w3 = sb + (size_t)(b1v ? warp + kCW : 0) * part_bytes;
                                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                                if (nb > 0) {
                                    for (int c = lane; c < pc; c += 32) {
                                        chunk_dot2<WK>(*reinterpret_cast<const uint4*>(w0 + (size_t)c * 16),
                                                       *reinterpret_cast<const uint4*>(w1 + (size_t)c * 16), xs, c, a0, a1);
                                        chunk_dot2<WK>(*reinterpret_cast<const uint4*>(w2 + (size_t)c * 16),
                                                       *reinterpret_cast<const uint4*>(w3 + (size_t)c * 16), xs, c, a2, a3);
                                    }
                                } else {
                                    for (int c = lane; c < pc; c += 32)
                                        chunk_dot2<WK>(*reinterpret_cast<const uint4*>(w0 + (size_t)c * 16),
                                                       *reinterpret_cast<const uint4*>(w1 + (size_t)c * 16), xs, c, a0, a1);
                                }
#pragma unroll
                                for (int o = 16; o > 0; o >>= 1) {
                                    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                                    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
                                    a2 += __shfl_xor_sync(0xffffffffu, a2, o);
                                    a3 += __shfl_xor_sync(0xffffffffu, a3, o);
                                }
                                if (lane == 0) emit(sa, r0, warp, a0);
                                if (lane == 1 && a1v) emit(sa, r0, warp + kCW, a1);
                                if (lane == 2 && b0v) emit(sb, r0 + pr.rs, warp, a2);
                                if (lane == 3 && b1v) emit(sb, r0 + pr.rs, warp + kCW, a3);
                            }
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(&empty[cst]);
                                if (nb > 0) mbar_arrive(&empty[cb]);
                            }
                            if (++cst == NS) { cst = 0; cpar ^= 1u; }
                            if (nb > 0 && ++cst == NS) { cst = 0; cpar ^= 1u; }
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) PTRACE_STAGE(3, consumed_n);
                            consumed_n += nb > 0 ? 2 : 1;
#endif
                        }
                    } else if (!MMA && pr.kparts == 2) {
                        // CUDA cores, rows wider than C: both K-parts of a row block in one round
                        // (warp w: row w, one sum per part, added in part order)
                        for (int r0 = pr.c0; r0 < pr.c1; r0 += pr.rs) {
                            const int nr = min(pr.rs, pr.c1 - r0);
                            const int cb = cst + 1 == NS ? 0 : cst + 1;
                            const uint32_t pb = cst + 1 == NS ? cpar ^ 1u : cpar;
                            if (!mbar_wait(&full[cst], cpar)) bad = true;
                            if (!mbar_wait(&full[cb], pb)) bad = true;
                            const unsigned char* sa = ring + (size_t)cst * lay.stage_bytes;
                            const unsigned char* sb = ring + (size_t)cb * lay.stage_bytes;
                            if (warp < nr) {
                                const unsigned char* wa = sa + (size_t)warp * rstride;
                                const unsigned char* wb2 = sb + (size_t)warp * rstride;
                                float a0 = 0.0f, a1 = 0.0f;
                                for (int c = lane; c < pc; c += 32) {
                                    a0 += chunk_dot<WK>(*reinterpret_cast<const uint4*>(wa + (size_t)c * 16), xs, c);
                                    a1 += chunk_dot<WK>(*reinterpret_cast<const uint4*>(wb2 + (size_t)c * 16), xs, pc + c);
                                }
#pragma unroll
                                for (int o = 16; o > 0; o >>= 1) {
                                    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                                    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
                                }
                                if (lane == 0) emit(sb, r0, warp, (0.0f + a0) + a1);
                            }
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(&empty[cst]);
                                mbar_arrive(&empty[cb]);
                            }
                            for (int k = 0; k < 2; k++)
                                if (++cst == NS) { cst = 0; cpar ^= 1u; }
#ifdef GPT2B_PERSIST_TRACE
                            consumed_n += 2;
#endif
                        }
                    } else
                    for (int r0 = pr.c0; r0 < pr.c1; r0 += pr.rs) {
                        const int nr = min(pr.rs, pr.c1 - r0);
                        float k0 = 0.0f, k1 = 0.0f;  // running row sums over K-parts
                        for (int kq = 0; kq < pr.kparts; kq++) {
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) PTRACE_STAGE(1, consumed_n);
#endif
                            if (!mbar_wait(&full[cst], cpar)) bad = true;
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) PTRACE_STAGE(2, consumed_n);
#endif
                            const unsigned char* sd = ring + (size_t)cst * lay.stage_bytes;
                            const bool last = (kq == pr.kparts - 1);
                            if constexpr (!MMA) {
                                // CUDA cores: warp w takes rows w and w + 8
                                const bool hA = warp < nr, hB = pr.rs == kStageUnits && warp + kCW < nr;
                                if (hA) {
                                    const unsigned char* wa = sd + (size_t)warp * rstride;
                                    const unsigned char* wb2 = sd + (size_t)(warp + kCW) * rstride;
                                    float a0 = 0.0f, a1 = 0.0f;
                                    if (hB) {
                                        for (int c = lane; c < pc; c += 32)
                                            chunk_dot2<WK>(*reinterpret_cast<const uint4*>(wa + (size_t)c * 16),
                                                           *reinterpret_cast<const uint4*>(wb2 + (size_t)c * 16), xs,
                                                           kq * pc + c, a0, a1);
                                    } else {
                                        for (int c = lane; c < pc; c += 32)
                                            a0 += chunk_dot<WK>(*reinterpret_cast<const uint4*>(wa + (size_t)c * 16),
                                                                xs, kq * pc + c);
                                    }
#pragma unroll
                                    for (int o = 16; o > 0; o >>= 1) {
                                        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                                        a1 += __shfl_xor_sync(0xffffffffu, a1, o);
                                    }
                                    k0 += a0;
                                    k1 += a1;
                                    if (last && (lane == 0 || (lane == 1 && hB)))
                                        emit(sd, r0, warp + lane * kCW, lane ? k1 : k0);
                                }
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&empty[cst]);
                            } else {
                                // tensor cores: the 8 warps split K; row sums meet in mred
                                float s0, s1;
                                const unsigned char* xb = w8 ? xh + (size_t)kq * pr.part * 2
                                                             : xs + (size_t)kq * pr.part * 2;
                                const uint32_t a_base =
                                    smem_addr(sd) + (uint32_t)((lane & 15) * rstride + (lane >> 4) * 16);
                                stage_mma<WK>(a_base, xb, pr.part, warp, lane, s0, s1);
                                __syncwarp();
                                // warps 1-7 are done with the stage; warp 0 still reads its tail below
                                if (lane == 0 && warp != 0) mbar_arrive(&empty[cst]);
                                float* mr = mred + (consumed_stages & 1) * (kCW * 16);
                                if ((lane & 3) == 0) {
                                    mr[warp * 16 + (lane >> 2)] = s0;
                                    mr[warp * 16 + (lane >> 2) + 8] = s1;
                                }
                                cta_sync();
                                if (tid < 16) {  // row tid of the stage: the warps' sums in warp order
                                    float v = 0.0f;
#pragma unroll
                                    for (int w = 0; w < kCW; w++) v += mr[w * 16 + tid];
                                    k0 += v;
                                    if (last && tid < nr) emit(sd, r0, tid, w8 ? k0 * x_up : k0);
                                }
                                if (warp == 0) {
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(&empty[cst]);
                                }
                                consumed_stages++;
                            }
#ifdef GPT2B_PERSIST_TRACE
                            if (tid == 0) PTRACE_STAGE(3, consumed_n);
                            consumed_n++;
#endif
                            if (++cst == NS) { cst = 0; cpar ^= 1u; }
                        }
                    }
                }
                if (cta_any(bad)) goto consumer_abort;
                if (lm && tid == 0) {  // every LM stage of this step was consumed and released
                    __threadfence_block();
                    *lm_done = step + 1;
                }
                PTRACE(u * 3 + 1);

                // ---------- after QKV: attention (head ah, split as) ----------
                if (ph == kPhQkv && attn_cta) {
                    const unsigned long long* qkv_w = P.ll_qkv + (size_t)l * P.qkv_rows;
                    const int total = pos + 1;
                    const int chunk = engine_attn_chunk(total, S);
                    const int j0 = as * chunk, j1 = min(j0 + chunk, total);
                    const int n_local = j1 - j0;
                    const int s_eff = min(S, (total + chunk - 1) / chunk);
                    if (tid < 3 * kHSz) {
                        const unsigned long long* src =
                            qkv_w + (size_t)(tid >> 6) * (NH * kHSz) + (size_t)ah * kHSz + (tid & 63);
                        float v = 0.0f;
                        for (uint32_t it = 0;; ++it) {
                            const unsigned long long w = ll_load(src);
                            if ((uint32_t)(w >> 32) == tag) { v = __uint_as_float((uint32_t)w); break; }
                            if (it > plim) { give_up(P.abort_flag, pgp); bad = true; break; }
                            if ((it & 15) == 15 && aborted(P.abort_flag)) { bad = true; break; }
                        }
                        (tid < kHSz ? q_s : (tid < 2 * kHSz ? kcur : vcur))[tid & 63] = v;
                    }
                    if (cta_any(bad)) goto consumer_abort;
                    const bool owns = (pos >= j0 && pos < j1);
                    const size_t lk = (size_t)l * 2 * NHmT;
                    const size_t krow = (size_t)ah * maxT + pos;
                    if (owns) {
                        // append this token's K/V (kv_cache_write_kernel(_w8))
                        if constexpr (k8) {
                            if (tid < 64) {
                                const int which = tid >> 5;
                                const float* src = which ? vcur : kcur;
                                const float v0 = src[lane], v1 = src[lane + 32];
                                const float mx = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
                                const float sc = mx / (KV == KV_FP8 ? 448.0f : 127.0f);
                                const uint8_t c0 = sc > 0.0f ? kv_encode<KV>(v0, sc) : (uint8_t)0;
                                const uint8_t c1 = sc > 0.0f ? kv_encode<KV>(v1, sc) : (uint8_t)0;
                                uint8_t* dst = P.kv + (lk + (which ? NHmT : 0) + krow) * kRowB;
                                dst[lane] = c0;
                                dst[lane + 32] = c1;
                                cur8[which * 64 + lane] = c0;
                                cur8[which * 64 + lane + 32] = c1;
                                if (lane == 0) {
                                    P.kv_scale[lk + (which ? NHmT : 0) + krow] = sc;
                                    cur_sc[which] = sc;
                                }
                            }
                        } else {
                            if (tid < 2 * kHSz) {
                                const int which = tid >> 6, d = tid & 63;
                                KT* dst = reinterpret_cast<KT*>(P.kv + (lk + (which ? NHmT : 0) + krow) * kRowB);
                                dst[d] = from_f<KT>((which ? vcur : kcur)[d]);
                            }
                        }
                        cta_sync();  // cur8 / cur_sc complete; the flag is released after the partials
                    }
                    float m_run = -FLT_MAX, l_run = 0.0f;
                    float acc[kE];
#pragma unroll
                    for (int e = 0; e < kE; e++) acc[e] = 0.0f;
                    const int lp = tid % kLP, rg = tid / kLP;
                    if (n_local > 0) {
                        if (!mbar_wait(kv_bar, (uint32_t)(kv_uses & 1))) bad = true;
                        kv_uses++;
                        const int soff = (int)(((size_t)ah * maxT + j0) & 3);
                        float* ksc = reinterpret_cast<float*>(kvbuf + 2 * kKvRows * kRowB) + soff;
                        float* vsc = ksc + (kKvRows + 8);
                        if (owns) {  // the staged copy holds the stale row of pos: patch it
                            const int r = pos - j0;
                            if constexpr (k8) {
                                if (tid < 128) kvbuf[(tid >> 6) * kKvRows * kRowB + r * kRowB + (tid & 63)] = cur8[tid];
                                if (tid == 0) { ksc[r] = cur_sc[0]; vsc[r] = cur_sc[1]; }
                            } else {
                                if (tid < 2 * kHSz) {
                                    const int which = tid >> 6, d = tid & 63;
                                    reinterpret_cast<KT*>(kvbuf + which * kKvRows * kRowB + r * kRowB)[d] =
                                        from_f<KT>((which ? vcur : kcur)[d]);
                                }
                            }
                        }
                        if (cta_any(bad)) goto consumer_abort;
                        const unsigned char* Kst = kvbuf;
                        const unsigned char* Vst = kvbuf + kKvRows * kRowB;
                        // warp-local softmax: warp w's row groups take rows rbase + rg of every pass;
                        // each warp keeps its own (max, exp-sum, un-normalised out) and the warps'
                        // states merge behind one barrier (the online-softmax combine)
                        float mw = -FLT_MAX;
                        for (int rbase = 0; rbase < n_local; rbase += kRPP) {  // scores
                            const int r = rbase + rg;
                            const bool valid = r < n_local;
                            const uint4 w = valid ? *reinterpret_cast<const uint4*>(Kst + r * kRowB + lp * 16)
                                                  : make_uint4(0u, 0u, 0u, 0u);
                            const float* q = q_s + lp * kE;
                            float d = 0.0f;
                            if constexpr (KV == KV_F32) {
                                d = __uint_as_float(w.x) * q[0] + __uint_as_float(w.y) * q[1] +
                                    __uint_as_float(w.z) * q[2] + __uint_as_float(w.w) * q[3];
                            } else if constexpr (KV == KV_BF16) {
                                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int i = 0; i < 4; i++) d += bf16lo(ww[i]) * q[2 * i] + bf16hi(ww[i]) * q[2 * i + 1];
                            } else {
                                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int i = 0; i < 4; i++)
#pragma unroll
                                    for (int j = 0; j < 4; j++) d += kv_code<KV>(ww[i], j) * q[4 * i + j];
                            }
#pragma unroll
                            for (int o = kLP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                            if (valid) {
                                if constexpr (k8) d *= ksc[r];
                                d *= P.attn_scale;
                                mw = fmaxf(mw, d);
                                if (lp == 0) p_s[r] = d;
                            }
                        }
                        mw = warp_max(mw);
                        __syncwarp();  // this warp's scores in p_s
                        float lw = 0.0f;
                        for (int r = rg; r < n_local; r += kRPP) {  // exp and P.V of the same rows
                            const float p = __expf(p_s[r] - mw);
                            if (lp == 0) lw += p;
                            const uint4 w = *reinterpret_cast<const uint4*>(Vst + r * kRowB + lp * 16);
                            if constexpr (KV == KV_F32) {
                                acc[0] += p * __uint_as_float(w.x); acc[1] += p * __uint_as_float(w.y);
                                acc[2] += p * __uint_as_float(w.z); acc[3] += p * __uint_as_float(w.w);
                            } else if constexpr (KV == KV_BF16) {
                                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int i = 0; i < 4; i++) {
                                    acc[2 * i] += p * bf16lo(ww[i]);
                                    acc[2 * i + 1] += p * bf16hi(ww[i]);
                                }
                            } else {
                                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                                const float pv = p * vsc[r];
#pragma unroll
                                for (int i = 0; i < 4; i++)
#pragma unroll
                                    for (int j = 0; j < 4; j++) acc[4 * i + j] += pv * kv_code<KV>(ww[i], j);
                            }
                        }
                        lw = warp_sum(lw);
#pragma unroll
                        for (int o = kLP; o < 32; o <<= 1)  // the warp's row groups: lanes with equal lp
#pragma unroll
                            for (int e = 0; e < kE; e++) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
                        float* ws = accbuf + warp * (kHSz + 2);
                        if (lane < kLP) {
#pragma unroll
                            for (int e = 0; e < kE; e++) ws[lp * kE + e] = acc[e];
                        }
                        if (lane == 0) { ws[kHSz] = mw; ws[kHSz + 1] = lw; }
                    }
                    cta_sync();  // staged rows consumed; every warp's state in accbuf
                    float o = 0.0f;
                    if (n_local > 0) {
                        float sw[kCW];
#pragma unroll
                        for (int w = 0; w < kCW; w++) m_run = fmaxf(m_run, accbuf[w * (kHSz + 2) + kHSz]);
#pragma unroll
                        for (int w = 0; w < kCW; w++) {
                            sw[w] = __expf(accbuf[w * (kHSz + 2) + kHSz] - m_run);
                            l_run += sw[w] * accbuf[w * (kHSz + 2) + kHSz + 1];
                        }
                        if (tid < kHSz)
#pragma unroll
                            for (int w = 0; w < kCW; w++) o += sw[w] * accbuf[w * (kHSz + 2) + tid];
                    }
                    PTRACE(u * 3 + 2);
                    unsigned long long* part = P.ll_part + ((size_t)l * NH + ah) * S * (kHSz + 2);
                    if (as > 0) {
                        if (n_local > 0) {  // partial (un-normalised out, max, exp-sum) for split 0
                            unsigned long long* dst = part + (size_t)as * (kHSz + 2);
                            if (tid < kHSz) ll_store(dst + tid, o, tag);
                            if (tid == kHSz) ll_store(dst + kHSz, m_run, tag);
                            if (tid == kHSz + 1) ll_store(dst + kHSz + 1, l_run, tag);
                        }
                    } else {
                        // split 0 merges the head's partials and publishes atty
                        const int nw = (s_eff - 1) * (kHSz + 2);  // <= 31 * 66 <= 8 * kCT
                        if (!ll_gather2<WIDE>(P.abort_flag, pgp, plim, part + (kHSz + 2), nw, tag, gv)) bad = true;
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            if (pair_slot(tid, j) < nw) mrg[pair_slot(tid, j)] = gv[j];
                        if (cta_any(bad)) goto consumer_abort;
                        if (tid < kHSz) {
                            // unrolled: the loads and exponentials of several splits in flight together
                            float mg = m_run;
#pragma unroll 4
                            for (int k = 0; k < s_eff - 1; k++) mg = fmaxf(mg, mrg[k * (kHSz + 2) + kHSz]);
                            const float r0 = __expf(m_run - mg);
                            float of = 0.0f + r0 * o, lf = 0.0f + r0 * l_run;
#pragma unroll 4
                            for (int k = 0; k < s_eff - 1; k++) {
                                const float rs = __expf(mrg[k * (kHSz + 2) + kHSz] - mg);
                                of += rs * mrg[k * (kHSz + 2) + tid];
                                lf += rs * mrg[k * (kHSz + 2) + kHSz + 1];
                            }
                            ll_store(P.ll_atty + (size_t)l * P.proj_k + (size_t)ah * kHSz + tid, round_to<XT>(of / lf), tag);
                        }
                    }
                    // off the critical path: the appended K/V row becomes visible before its flag
                    // (release of this step's tag, a max: the flag never goes back), then the next
                    // layer's rows are staged (a failed wait there reaches the next cta_any)
                    if (owns && tid < 2 * kHSz) __threadfence();
                    if (cta_any(bad)) goto consumer_abort;
                    if (tid == 0) {
                        if (owns)
                            asm volatile("red.release.gpu.global.max.u32 [%0], %1;" ::"l"(P.kv_flag + l * NH + ah),
                                         "r"(tag)
                                         : "memory");
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after the patch writes
                        if (l + 1 < L) kv_issue(step, l + 1);
                        else if (step + 1 < P.n_steps) kv_issue(step + 1, 0);
                    }
                }
            }

            // ---------- greedy pick: per-CTA best, all-gather, next token ----------
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {  // lanes 0 and 1 hold candidates
                const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                best_merge(best_v, best_i, ov, oi);
            }
            if (lane == 0) { misc[warp] = best_v; misc_i[16 + warp] = best_i; }
            cta_sync();
            const int NG = (TPG ? P.tp_size : 1) * G;  // (value, index) pairs of every CTA of every rank
            if (tid == 0) {
                float bv = misc[0];
                int bi = misc_i[16];
                for (int w = 1; w < kCW; w++) best_merge(bv, bi, misc[w], misc_i[16 + w]);
                const size_t word = (size_t)kPersistLmStride * ((size_t)P.tp_rank * G + b);
                ll_store_group<TPG>(P.peer_x[0], pgp, P.xoff_lm, word, bv, tag);
                ll_store_group<TPG>(P.peer_x[0], pgp, P.xoff_lm, word + 1, __int_as_float(bi), tag);
            }
            {
                float* gvals = reinterpret_cast<float*>(xs);
                int* gidx = reinterpret_cast<int*>(xs) + NG;
                const bool ok = ll_gather_pairs<TPG>(P.abort_flag, pgp, plim, P.ll_lm, NG, tag, gvals, gidx);
                if (cta_any(!ok)) goto consumer_abort;
                PTRACE(4 * L * 3 + 2);
                float bv = -FLT_MAX;
                int bi = 0x7fffffff;
                for (int k = tid; k < NG; k += kCT) best_merge(bv, bi, gvals[k], gidx[k]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    best_merge(bv, bi, ov, oi);
                }
                if (lane == 0) { misc[32 + warp] = bv; misc_i[48 + warp] = bi; }
                cta_sync();
                bv = misc[32];
                bi = misc_i[48];
                for (int w = 1; w < kCW; w++) best_merge(bv, bi, misc[32 + w], misc_i[48 + w]);
                // teacher-forced prompt positions, as in the LM-head GEMV epilogue
                const int next = (pos + 1 < P.n_prompt) ? P.prompt[pos + 1] : bi;
                if (next < 0 || next >= P.V) {  // no finite logit: every CTA sees the same pick and leaves
                    if (b == 0 && tid == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN);
                    goto consumer_abort;
                }
                if (b == 0 && tid == 0) {
                    P.history[pos + 1] = next;
                    if (step + 1 == P.n_steps) {
                        *P.d_token = next;
                        *P.d_pos = pos + 1;
                        *P.d_epoch = epoch0 + (uint32_t)P.n_steps;
                    }
                }
                tok = next;
                cta_sync();  // misc and xs are reused by the next step
            }
        }
    }
    goto consumer_exit;

consumer_abort:
    if (tid == 0) *stop = 1;  // the producer stops issuing and drains
consumer_exit:
    if (tid == 0 && kv_issued > kv_uses) mbar_wait(kv_bar, (uint32_t)(kv_uses & 1));
    if (tid == 0 && ln_pending) mbar_wait(ln_bar, ln_par);
}

// smem_out != null: report the shared memory of a launch with P.C, P.nsw and
// whether one CTA of it fits on an SM (-1 if not); no launch.
template <int WK, int KV, int MODE>
cudaError_t launch_persist_t(const PersistParams& P, cudaStream_t st, int* smem_out) {
    constexpr bool WIDE = MODE >= 1;
    auto k = decode_persistent_kernel<WK, KV, MODE>;
    static unsigned long long smem_set = 0;
    const PSmem lay = persist_layout<WK, KV>(P.C, P.nsw, WIDE ? P.kv_rows : kNarrowKvRows, P.tp_size);
    cudaError_t e = ensure_smem_limit(k, &smem_set);
    if (e != cudaSuccess) return e;
    if (smem_out) {
        int nb = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, kThreads, lay.total);
        *smem_out = (e == cudaSuccess && nb >= 1) ? lay.total : -1;
        return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P.G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = lay.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: they wait on one another
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, P);
}

cudaError_t persist_dispatch(int wk, int kv, const PersistParams& P, cudaStream_t st, int* smem_out) {
    const int mode = P.tp_size > 1 ? 2 : (persist_narrow(P.C, P.kv_rows, P.tp_size) ? 0 : 1);
#define GPT2B_PK(W_, K_) \
    if (wk == W_ && kv == K_)                                                   \
        return mode == 0 ? launch_persist_t<W_, K_, 0>(P, st, smem_out)       \
                         : (mode == 1 ? launch_persist_t<W_, K_, 1>(P, st, smem_out) : launch_persist_t<W_, K_, 2>(P, st, smem_out));
    GPT2B_PK(WK_F32, KV_F32)
    GPT2B_PK(WK_BF16, KV_BF16)
    GPT2B_PK(WK_I8, KV_BF16)
    GPT2B_PK(WK_I8, KV_I8)
    GPT2B_PK(WK_FP8, KV_BF16)
    GPT2B_PK(WK_FP8, KV_FP8)
#undef GPT2B_PK
    return cudaErrorInvalidValue;
}

}  // namespace

#ifdef GPT2B_PERSIST_TRACE
extern "C" int gpt2b_persist_trace(unsigned long long* host, int* steps, int* ctas, int* events) {
    *steps = kTraceSteps; *ctas = kTraceCtas; *events = kTraceEv;
    return (int)cudaMemcpyFromSymbol(host, g_trace, sizeof(g_trace));
}
extern "C" int gpt2b_persist_trace_stages(unsigned long long* host) {
    return (int)cudaMemcpyFromSymbol(host, g_trace_stage, sizeof(g_trace_stage));
}
#endif

int persist_smem_bytes(int wk, int kv, int C, int nsw, int kv_rows, int tp) {
    PersistParams P;
    P.C = C;
    P.nsw = nsw;
    P.kv_rows = kv_rows;
    P.tp_size = tp;
    int s = -1;
    if (persist_dispatch(wk, kv, P, nullptr, &s) != cudaSuccess) return -1;
    return s;
}

bool persist_supported(int C, int NH, int hs, int maxT, int splits, int nsm, int L) {
    if (L > kMaxLayers) return false;
    if (hs != kHSz || C > kMaxC || C % 64 != 0 || (NH * maxT) % 4 != 0 || nsm > kMaxCtas) return false;
    if (splits < 1 || splits > kMaxSplits || NH * splits > nsm) return false;
    return engine_attn_chunk(maxT, splits) <= kMaxKvRows;
}

// One block per LayerNorm: the exponent e with B = sqrt(C) max|gamma| + max|beta| in
// [2^(13+e), 2^(14+e)).  Since sum_c (r_c - mean)^2 = C var, every LayerNorm output obeys
// |x_c| <= sqrt(C) |gamma_c| + |beta_c| <= B, so x 2^-e stays below 2^14 (a quarter of FP16's
// range, margin for the rounding of the variance).
__global__ void ln_exp_kernel(int* out, const __nv_bfloat16* ln1w, const __nv_bfloat16* ln1b,
                              const __nv_bfloat16* ln2w, const __nv_bfloat16* ln2b, const __nv_bfloat16* lnfw,
                              const __nv_bfloat16* lnfb, int L, int C) {
    __shared__ float scratch[64];
    const int i = blockIdx.x;
    const __nv_bfloat16* w = i == 2 * L ? lnfw : ((i & 1) ? ln2w : ln1w) + (size_t)(i >> 1) * C;
    const __nv_bfloat16* b = i == 2 * L ? lnfb : ((i & 1) ? ln2b : ln1b) + (size_t)(i >> 1) * C;
    float gm = 0.0f, bm = 0.0f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        gm = fmaxf(gm, fabsf(__bfloat162float(w[c])));
        bm = fmaxf(bm, fabsf(__bfloat162float(b[c])));
    }
    gm = warp_max(gm);
    bm = warp_max(bm);
    if ((threadIdx.x & 31) == 0) { scratch[threadIdx.x >> 5] = gm; scratch[32 + (threadIdx.x >> 5)] = bm; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++) { gm = fmaxf(gm, scratch[k]); bm = fmaxf(bm, scratch[32 + k]); }
        gm = fmaxf(gm, scratch[0]);
        bm = fmaxf(bm, scratch[32]);
        const float B = sqrtf((float)C) * gm + bm;
        int e = 0;
        if (B > 0.0f) e = (B <= FLT_MAX) ? ((__float_as_int(B) >> 23) & 0xff) - 127 - 13 : 100;
        out[i] = max(-100, min(100, e));
    }
}

cudaError_t persist_ln_exponents(int* out, const void* ln1w, const void* ln1b, const void* ln2w, const void* ln2b,
                                 const void* lnfw, const void* lnfb, int L, int C, cudaStream_t st) {
    using BF = __nv_bfloat16;
    return launch_k(ln_exp_kernel, dim3(2 * L + 1), dim3(256), 0, st, false, out, (const BF*)ln1w, (const BF*)ln1b,
                    (const BF*)ln2w, (const BF*)ln2b, (const BF*)lnfw, (const BF*)lnfb, L, C);
}

int persist_max_splits() { return kMaxSplits; }
int persist_max_stages() { return kMaxNs; }
bool persist_narrow(int C, int kv_rows, int tp) { return tp <= 1 && C <= kNarrowC && kv_rows <= kNarrowKvRows; }

int persist_stage_bytes(int wk, int C) { return kStageUnits * (C * wkind_bytes(wk) + 16) + kTail; }

cudaError_t launch_persistent(int wk, int kv, const PersistParams& P, cudaStream_t st) {
    return persist_dispatch(wk, kv, P, st, nullptr);
}

}  // namespace gpt2b
