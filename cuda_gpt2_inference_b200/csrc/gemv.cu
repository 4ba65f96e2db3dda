// gemv.cu -- batch-1 decode GEMVs for FP32 / BF16 / INT8 / FP8 weights.
//
// Design (B200, HBM/latency-bound, no tensor cores: one activation vector is
// not a dense contraction):
//   * Warp specialisation: one producer warp streams row tiles of W into a
//     shared-memory ring with cp.async.bulk (rows of a row-major matrix are
//     contiguous, so a tile is one contiguous byte range, plus its 8-bit row
//     scales), completing on per-stage "full" mbarriers; eight consumer warps
//     compute and release stages through "empty" mbarriers.  No block-wide
//     barrier sits in the streaming loop.
//   * Per-layer matrices use one tile per CTA sized to spread the bytes over
//     the SMs, so the whole matrix is in flight at once; the LM head streams
//     ~24 KB tiles through up to 8 stages per SM.
//   * Programmatic dependent launch: the producer never waits on the previous
//     kernel (weights are immutable), and consumers prefetch every parameter
//     they will need (LayerNorm gamma/beta, bias, row scales) before
//     griddepcontrol.wait.  After the wait the activation vector arrives in one
//     round trip (all 16-byte loads in flight, or bulk copies for the
//     attention partials).
//   * Each consumer warp takes a pair of rows (x read once per pair) and, when a
//     tile has fewer than 16 rows, a slice of K.  FP32 accumulation; INT8 and
//     E4M3 codes decode exactly with integer/bit operations (common.cuh).
//   * Streamed 8-bit matrices (the LM head) go through the tensor cores instead:
//     a warp tile is 16 rows copied as 8 row pairs into a padded layout (ldmatrix
//     without bank conflicts), the codes become exact FP16 pairs in registers,
//     x is the B operand's column in FP16 after an exact power-of-two scaling
//     of the CTA's max |x| into [2^14, 2^15), and mma.sync accumulates in FP32.
//     About 25 warp instructions per 512 codes against ~3.5 per code per thread
//     on the CUDA cores, which left the 8-bit stream instruction-bound.
//   * Fused prologues for the engine: residual add + LayerNorm, embedding +
//     LayerNorm, or the LSE merge of the attention split partials -- computed
//     redundantly per CTA from a few KB of L2-resident data instead of separate
//     launches.  Fused LM-head epilogue: logits, per-CTA argmax, last-CTA pick,
//     device-side token/position advance.
#include "common.cuh"
#include "internal.h"

#include <float.h>
#include <stdlib.h>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(gemv_device_error)

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kMaxStages = 8;              // ring depth of kernel A
constexpr int kMaxWarpStages = 4;          // per-warp ring depth of kernel B
constexpr int kRedFloats = 160;            // per-slot partial sums (>= rows per tile + 16)
constexpr int kLnChunks = 2;               // 16-byte LayerNorm chunks per consumer thread (C <= 2048)
constexpr int kBarBytes = 512;             // mbarriers (kernel B: 8 warps x 4 stages + 1)
constexpr int kSmemHeader = kBarBytes + kRedFloats * 4 + 64;

template <int WK> struct WTraits;
template <> struct WTraits<WK_F32> { using XT = float; };
template <> struct WTraits<WK_BF16> { using XT = __nv_bfloat16; };
template <> struct WTraits<WK_I8> { using XT = __nv_bfloat16; };
template <> struct WTraits<WK_FP8> { using XT = __nv_bfloat16; };

// consumer-only barrier (named barrier 1, the 8 consumer warps)
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// all-reduce over the 256 consumer threads through `scratch` (>= 8 floats)
__device__ __forceinline__ float consumer_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) scratch[w] = v;
    consumer_sync();
    float t = (lane < kConsumerWarps) ? scratch[lane] : 0.0f;
    t = warp_sum(t);
    consumer_sync();
    return t;
}

// Dot product of one 16-byte weight chunk of two rows with the matching x.
template <int WK>
__device__ __forceinline__ void chunk_dot2(const uint4& w0, const uint4& w1, const unsigned char* xs, int c,
                                           float& a0, float& a1) {
    if constexpr (WK == WK_F32) {
        const float4 x = *reinterpret_cast<const float4*>(xs + (size_t)c * 16);
        a0 = fmaf(__uint_as_float(w0.x), x.x, a0); a0 = fmaf(__uint_as_float(w0.y), x.y, a0);
        a0 = fmaf(__uint_as_float(w0.z), x.z, a0); a0 = fmaf(__uint_as_float(w0.w), x.w, a0);
        a1 = fmaf(__uint_as_float(w1.x), x.x, a1); a1 = fmaf(__uint_as_float(w1.y), x.y, a1);
        a1 = fmaf(__uint_as_float(w1.z), x.z, a1); a1 = fmaf(__uint_as_float(w1.w), x.w, a1);
    } else if constexpr (WK == WK_BF16) {
        const uint4 x = *reinterpret_cast<const uint4*>(xs + (size_t)c * 16);
        const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
        const uint32_t aw[4] = {w0.x, w0.y, w0.z, w0.w};
        const uint32_t bw[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float xl = bf16lo(xw[i]), xh = bf16hi(xw[i]);
            a0 = fmaf(bf16lo(aw[i]), xl, a0); a0 = fmaf(bf16hi(aw[i]), xh, a0);
            a1 = fmaf(bf16lo(bw[i]), xl, a1); a1 = fmaf(bf16hi(bw[i]), xh, a1);
        }
    } else {
        const uint4 xa = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + (size_t)c * 32 + 16);
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const uint32_t aw[4] = {w0.x, w0.y, w0.z, w0.w};
        const uint32_t bw[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float x0 = bf16lo(xw[2 * i]), x1 = bf16hi(xw[2 * i]);
            const float x2 = bf16lo(xw[2 * i + 1]), x3 = bf16hi(xw[2 * i + 1]);
            if constexpr (WK == WK_I8) {
                const uint32_t p = aw[i] ^ 0x80808080u, q = bw[i] ^ 0x80808080u;
                a0 = fmaf(i8_to_f(p, 0), x0, a0); a0 = fmaf(i8_to_f(p, 1), x1, a0);
                a0 = fmaf(i8_to_f(p, 2), x2, a0); a0 = fmaf(i8_to_f(p, 3), x3, a0);
                a1 = fmaf(i8_to_f(q, 0), x0, a1); a1 = fmaf(i8_to_f(q, 1), x1, a1);
                a1 = fmaf(i8_to_f(q, 2), x2, a1); a1 = fmaf(i8_to_f(q, 3), x3, a1);
            } else {
                a0 = fmaf(e4m3_to_f(aw[i], 0), x0, a0); a0 = fmaf(e4m3_to_f(aw[i], 1), x1, a0);
                a0 = fmaf(e4m3_to_f(aw[i], 2), x2, a0); a0 = fmaf(e4m3_to_f(aw[i], 3), x3, a0);
                a1 = fmaf(e4m3_to_f(bw[i], 0), x0, a1); a1 = fmaf(e4m3_to_f(bw[i], 1), x1, a1);
                a1 = fmaf(e4m3_to_f(bw[i], 2), x2, a1); a1 = fmaf(e4m3_to_f(bw[i], 3), x3, a1);
            }
        }
    }
}

// 16 bytes of activations <-> E floats (E = 4 for float, 8 for bf16)
template <typename XT> struct Vec;
template <> struct Vec<float> {
    static constexpr int E = 4;
    __device__ static void unpack(const uint4& u, float* f) {
        f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
    }
    __device__ static uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
};
template <> struct Vec<__nv_bfloat16> {
    static constexpr int E = 8;
    __device__ static void unpack(const uint4& u, float* f) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) { f[2 * i] = bf16lo(w[i]); f[2 * i + 1] = bf16hi(w[i]); }
    }
    __device__ static uint32_t pack2(float lo, float hi) {
        const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
        const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
        return l | (h << 16);
    }
    __device__ static uint4 pack(const float* f) {
        return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
    }
};

// Embedding chunk (8 or 4 values) of row `tok`, as dequant_wte_kernel stores it
// for 8-bit tables (GEMV_w8.cuh:396): bf16(decode(code) * scale[row]).
template <int WK, typename XT>
__device__ __forceinline__ void emb_chunk(const GemvParams& p, int tok, int c, float* f) {
    constexpr int E = Vec<XT>::E;
    if constexpr (WK == WK_I8 || WK == WK_FP8) {
        const uint2 codes = *reinterpret_cast<const uint2*>(p.wte8 + (size_t)tok * p.K + (size_t)c * E);
        const float s = p.wte_scale[tok];
        const uint32_t cw[2] = {codes.x, codes.y};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t w = cw[i >> 2];
            const float v = (WK == WK_I8) ? (float)(int8_t)((w >> (8 * (i & 3))) & 0xffu) : e4m3_to_f(w, i & 3);
            f[i] = round_to<__nv_bfloat16>(v * s);
        }
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const XT*>(p.wte) + (size_t)tok * p.K +
                                                        (size_t)c * E);
        Vec<XT>::unpack(u, f);
    }
}

// LayerNorm gamma/beta chunks a consumer thread will need (prefetched before
// griddepcontrol.wait: parameters never depend on the previous kernel).
template <int WK, int PRO>
__device__ __forceinline__ void prefetch_ln_params(const GemvParams& p, uint4* lw, uint4* lb) {
    using XT = typename WTraits<WK>::XT;
    if constexpr (PRO == PRO_RES_LN || PRO == PRO_EMB_LN) {
        const int tid = threadIdx.x, nch = p.K / Vec<XT>::E;
#pragma unroll
        for (int j = 0; j < kLnChunks; j++) {
            const int c = tid + j * kConsumers;
            if (c < nch) {
                lw[j] = reinterpret_cast<const uint4*>(p.ln_w)[c];
                lb[j] = reinterpret_cast<const uint4*>(p.ln_b)[c];
            }
        }
    }
}

// The activation vector x (K values) into shared memory, run by the 256
// consumer threads after griddepcontrol.wait: a plain copy with every 16-byte
// load in flight at once, the LSE merge of the attention partials (staged by
// bulk copies), or residual/embedding + LayerNorm.  Ends with a consumer
// barrier.  Returns false if a bounded wait gave up.
template <int WK, int PRO>
__device__ bool build_x(const GemvParams& p, unsigned char* xs, unsigned char* aux, uint64_t* aux_bar, float* misc,
                        const uint4* lw, const uint4* lb) {
    using XT = typename WTraits<WK>::XT;
    constexpr int E = Vec<XT>::E;
    const int tid = threadIdx.x;
    const int x_bytes = ((p.K * (int)sizeof(XT)) + 15) & ~15;
    if constexpr (PRO == PRO_PLAIN) {
        if (p.x_vec) {
            const int nvec = x_bytes / 16;
            const uint4* xv = reinterpret_cast<const uint4*>(p.x);
            uint4* xd = reinterpret_cast<uint4*>(xs);
            for (int base = 0; base < nvec; base += 4 * kConsumers) {
                uint4 r[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int i = base + j * kConsumers + tid;
                    if (i < nvec) r[j] = xv[i];
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int i = base + j * kConsumers + tid;
                    if (i < nvec) xd[i] = r[j];
                }
            }
        } else {
            const XT* x = reinterpret_cast<const XT*>(p.x);
            XT* xd = reinterpret_cast<XT*>(xs);
            for (int k = tid; k < p.K; k += kConsumers) xd[k] = x[k];
        }
    } else if constexpr (PRO == PRO_ATTN_MERGE) {
        // stage all split partials with three bulk copies, then merge
        // (attention_kvcache.cuh:298-318): o = sum e^{m_s-M} o_s / sum e^{m_s-M} l_s
        const int NH = p.attn_heads, S = p.attn_splits;
        const uint32_t ob = (uint32_t)(NH * S * 64 * 4);
        const uint32_t mb = (uint32_t)(((NH * S * 4) + 15) & ~15);
        float* po = reinterpret_cast<float*>(aux);
        float* pm = reinterpret_cast<float*>(aux + ob);
        float* pl = reinterpret_cast<float*>(aux + ob + mb);
        if (tid == 0) {
            mbar_arrive_expect_tx(aux_bar, ob + 2 * mb);
            bulk_g2s(po, p.part_out, ob, aux_bar);
            bulk_g2s(pm, p.part_max, mb, aux_bar);
            bulk_g2s(pl, p.part_lse, mb, aux_bar);
        }
        const int total = *p.d_pos + 1;
        const int chunk = engine_attn_chunk(total, S);
        const int s_eff = min(S, (total + chunk - 1) / chunk);
        if (!mbar_wait(aux_bar, 0)) return false;
        XT* xd = reinterpret_cast<XT*>(xs);
        for (int idx = tid; idx < NH * 64; idx += kConsumers) {
            const int h = idx >> 6, d = idx & 63;
            float m = -FLT_MAX;
            for (int s = 0; s < s_eff; s++) m = fmaxf(m, pm[h * S + s]);
            float o = 0.0f, l = 0.0f;
            for (int s = 0; s < s_eff; s++) {
                const float r = __expf(pm[h * S + s] - m);
                o += r * po[(h * S + s) * 64 + d];
                l += r * pl[h * S + s];
            }
            const XT v = from_f<XT>(o / l);
            xd[idx] = v;
            if (blockIdx.x == 0 && p.atty_out) reinterpret_cast<XT*>(p.atty_out)[idx] = v;
        }
    } else {
        // residual add (or embedding) + LayerNorm, two-pass like the reference
        // (layernorm.cuh:171-241): the sum is rounded to the storage type and
        // the statistics are taken over the rounded values.
        const int C = p.K, nch = C / E;
        float v[kLnChunks][E];
        float sum = 0.0f;
        int tok = 0, pos = 0;
        if constexpr (PRO == PRO_EMB_LN) {
            tok = *p.d_token;
            pos = *p.d_pos;
            if (tok < 0 || tok >= p.vocab) { if (tid == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN); tok = 0; }
            if (pos < 0 || pos >= p.maxT) { if (tid == 0) report_device_error(GPT2B_DEVERR_BAD_POS); pos = 0; }
        }
        uint4 ra[kLnChunks], rb[kLnChunks], rb2[kLnChunks];
        const bool df32 = (PRO == PRO_RES_LN) && p.delta_f32 && E == 8;  // FP32 delta under BF16 activations
#pragma unroll
        for (int j = 0; j < kLnChunks; j++) {  // issue every load before using any
            const int c = tid + j * kConsumers;
            if (c < nch) {
                if constexpr (PRO == PRO_EMB_LN) {
                    rb[j] = reinterpret_cast<const uint4*>(reinterpret_cast<const XT*>(p.wpe) + (size_t)pos * C)[c];
                } else {
                    ra[j] = reinterpret_cast<const uint4*>(p.res_in)[c];
                    if (df32) {
                        rb[j] = reinterpret_cast<const uint4*>(p.delta)[2 * c];
                        rb2[j] = reinterpret_cast<const uint4*>(p.delta)[2 * c + 1];
                    } else {
                        rb[j] = reinterpret_cast<const uint4*>(p.delta)[c];
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kLnChunks; j++) {
            const int c = tid + j * kConsumers;
#pragma unroll
            for (int e = 0; e < E; e++) v[j][e] = 0.0f;
            if (c < nch) {
                float a[E], b[E];
                if constexpr (PRO == PRO_EMB_LN) emb_chunk<WK, XT>(p, tok, c, a);
                else Vec<XT>::unpack(ra[j], a);
                if (df32) {  // the all-reduced FP32 sum, rounded as the single-GPU GEMV stores it
                    Vec<float>::unpack(rb[j], b);
                    Vec<float>::unpack(rb2[j], b + 4);
#pragma unroll
                    for (int e = 0; e < E; e++) b[e] = round_to<XT>(b[e]);
                } else {
                    Vec<XT>::unpack(rb[j], b);
                }
#pragma unroll
                for (int e = 0; e < E; e++) {
                    v[j][e] = round_to<XT>(a[e] + b[e]);
                    sum += v[j][e];
                }
                if (blockIdx.x == 0 && p.res_out) reinterpret_cast<uint4*>(p.res_out)[c] = Vec<XT>::pack(v[j]);
            }
        }
        const float mean = consumer_sum(sum, misc) / (float)C;
        float sq = 0.0f;
#pragma unroll
        for (int j = 0; j < kLnChunks; j++) {
            const int c = tid + j * kConsumers;
            if (c < nch)
#pragma unroll
                for (int e = 0; e < E; e++) { const float d = v[j][e] - mean; sq += d * d; }
        }
        const float rstd = rsqrtf(consumer_sum(sq, misc) / (float)C + 1e-5f);
#pragma unroll
        for (int j = 0; j < kLnChunks; j++) {
            const int c = tid + j * kConsumers;
            if (c < nch) {
                float w[E], b[E], o[E];
                Vec<XT>::unpack(lw[j], w);
                Vec<XT>::unpack(lb[j], b);
#pragma unroll
                for (int e = 0; e < E; e++) o[e] = (rstd * (v[j][e] - mean)) * w[e] + b[e];
                const uint4 packed = Vec<XT>::pack(o);
                reinterpret_cast<uint4*>(xs)[c] = packed;
                if (blockIdx.x == 0 && p.ln_out) reinterpret_cast<uint4*>(p.ln_out)[c] = packed;
            }
        }
    }
    consumer_sync();
    return true;
}

// LM head: reduce the per-thread best (value, index) over the CTA, publish it,
// and let the last CTA to finish pick the token and advance the device state.
__device__ void lmhead_finish(const GemvParams& p, float best_v, int best_i, float* misc) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* sv = misc;
    int* si = reinterpret_cast<int*>(misc + kConsumerWarps);
    __shared__ int s_last;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
    }
    if (lane == 0) { sv[warp] = best_v; si[warp] = best_i; }
    consumer_sync();
    if (tid == 0) {
        float bv = sv[0];
        int bi = si[0];
        for (int w = 1; w < kConsumerWarps; w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        p.part_val[blockIdx.x] = bv;
        p.part_idx[blockIdx.x] = bi;
        __threadfence();
        const unsigned ticket = atomicAdd(p.counter, 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    consumer_sync();
    if (!s_last) return;
    __threadfence();
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int b = tid; b < (int)gridDim.x; b += kConsumers) {
        const float v = __ldcg(&p.part_val[b]);
        const int i = __ldcg(&p.part_idx[b]);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    consumer_sync();
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    consumer_sync();
    if (tid == 0) {
        for (int w = 1; w < kConsumerWarps; w++)
            if (sv[w] > sv[0] || (sv[w] == sv[0] && si[w] < si[0])) { sv[0] = sv[w]; si[0] = si[w]; }
        *p.counter = 0u;
        if (p.pair_out) {  // vocab shard of a tensor-parallel rank: (best, global index) for the all-gather
            p.pair_out[0] = sv[0];
            p.pair_out[1] = __int_as_float(si[0] == 0x7fffffff ? si[0] : si[0] + p.row_offset);
        } else if (p.advance) {
            const int pos = *p.pos_io;
            const int next = (pos + 1 < p.n_prompt) ? p.prompt[pos + 1] : si[0];
            if (p.history) p.history[pos + 1] = next;
            *p.token_io = next;
            *p.pos_io = pos + 1;
        } else if (p.token_io) {
            *p.token_io = si[0];
        }
    }
}

// Shared memory of the FP16 x copy (kernel B, tensor-core form).
__host__ __device__ inline int mma_x_bytes(const GemvParams& p) { return p.mma ? p.K * 2 : 0; }

// Bias / GELU / pre-GELU epilogue of one output row.
template <typename XT, typename OT>
__device__ __forceinline__ void store_row(const GemvParams& p, int row, float acc, float bias) {
    float pre = acc + bias;
    if (p.pre_gelu) reinterpret_cast<OT*>(p.pre_gelu)[row] = from_f<OT>(pre);
    const float o = p.do_gelu ? gelu_tanh(pre) : pre;
    reinterpret_cast<OT*>(p.out)[row] = from_f<OT>(o);
}

// ---------------------------------------------------------------------------
// Kernel A: one row tile per CTA (the per-layer matrices).  A producer warp
// stages the tile (and any further tiles through the ring); the 8 consumer
// warps split the tile's rows into pairs and, for short tiles, split K.
// ---------------------------------------------------------------------------
template <int WK, typename OT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
    using XT = typename WTraits<WK>::XT;
    constexpr int kWB = (WK == WK_F32) ? 4 : (WK == WK_BF16 ? 2 : 1);
    constexpr bool k8 = (WK == WK_I8 || WK == WK_FP8);
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    uint64_t* aux_bar = empty + kMaxStages;
    float* red = reinterpret_cast<float*>(smem + kBarBytes);
    float* misc = red + kRedFloats;  // 16 floats of reduction scratch
    unsigned char* xs = smem + kSmemHeader;
    const int x_bytes = ((p.K * (int)sizeof(XT)) + 15) & ~15;
    unsigned char* aux = xs + x_bytes;
    unsigned char* stages = aux + p.aux_bytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t row_bytes = (size_t)p.K * kWB;
    const int R = p.rows_per_tile, NS = p.nstages, G = gridDim.x;
    const int rows_bytes_tile = (int)(((size_t)R * row_bytes + 15) & ~(size_t)15);

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(aux_bar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {  // producer: weights never depend on other kernels
        if (lane == 0) {
            const unsigned char* Wb = reinterpret_cast<const unsigned char*>(p.W);
            for (int it = 0;; ++it) {
                const int t = blockIdx.x + it * G;
                if (t >= p.ntiles) break;
                const int s = it % NS;
                if (it >= NS && !mbar_wait(&empty[s], (uint32_t)(((it / NS) - 1) & 1))) break;
                const int r0 = t * R, nr = min(R, p.M - r0);
                const uint32_t wbytes = (uint32_t)(nr * row_bytes);
                const uint32_t sbytes = p.scale_in_tile ? (uint32_t)(((nr + 3) & ~3) * 4) : 0u;
                unsigned char* st = stages + (size_t)s * p.tile_bytes;
                mbar_arrive_expect_tx(&full[s], wbytes + sbytes);
                bulk_g2s(st, Wb + (size_t)r0 * row_bytes, wbytes, &full[s]);
                if (sbytes) bulk_g2s(st + rows_bytes_tile, p.scale + r0, sbytes, &full[s]);
            }
        }
        return;
    }

    // consumers: parameters first (bias/scale of a CTA that owns one tile)
    uint4 lw[kLnChunks], lb[kLnChunks];
    prefetch_ln_params<WK, PRO>(p, lw, lb);
    const bool one_tile = (p.ntiles <= G);
    float bias_reg = 0.0f, scale_reg = 1.0f;
    if (one_tile) {
        const int row = blockIdx.x * R + tid;
        if (tid < R && row < p.M) {
            if (p.bias) bias_reg = to_f<XT>(reinterpret_cast<const XT*>(p.bias)[row]);
            if (k8 && !p.scale_in_tile) scale_reg = p.scale[row];
        }
    }
    pdl_wait();
    pdl_trigger();
    if (!build_x<WK, PRO>(p, xs, aux, aux_bar, misc, lw, lb)) return;

    const int nch = (int)(row_bytes / 16);
    float best_v = -FLT_MAX;
    int best_i = 0x7fffffff;
    int it = 0;
    for (int t = blockIdx.x; t < p.ntiles; t += G, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&full[s], (uint32_t)((it / NS) & 1))) return;
        const unsigned char* tile = stages + (size_t)s * p.tile_bytes;
        const int r0 = t * R, nr = min(R, p.M - r0);
        float srow = scale_reg;
        if (k8 && p.scale_in_tile && tid < nr) srow = reinterpret_cast<const float*>(tile + rows_bytes_tile)[tid];
        const int npairs = (nr + 1) >> 1;
        const int splits = npairs >= kConsumerWarps ? 1 : kConsumerWarps / npairs;
        for (int slot = warp; slot < npairs * splits; slot += kConsumerWarps) {
            const int pair = slot / splits, sp = slot % splits;
            const int ra = 2 * pair, rb = min(2 * pair + 1, nr - 1);
            const int cb = (int)((long)sp * nch / splits), ce = (int)((long)(sp + 1) * nch / splits);
            const unsigned char* wa = tile + (size_t)ra * row_bytes;
            const unsigned char* wb = tile + (size_t)rb * row_bytes;
            float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 4
            for (int c = cb + lane; c < ce; c += 32) {
                const uint4 w0 = *reinterpret_cast<const uint4*>(wa + (size_t)c * 16);
                const uint4 w1 = *reinterpret_cast<const uint4*>(wb + (size_t)c * 16);
                chunk_dot2<WK>(w0, w1, xs, c, a0, a1);
            }
            a0 = warp_sum(a0);
            a1 = warp_sum(a1);
            if (lane == 0) {
                red[slot * 2] = a0;
                red[slot * 2 + 1] = a1;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp has finished reading the stage
        consumer_sync();
        for (int r = tid; r < nr; r += kConsumers) {
            const int pair = r >> 1;
            float acc = 0.0f;
            for (int sp = 0; sp < splits; sp++) acc += red[(pair * splits + sp) * 2 + (r & 1)];
            const int row = r0 + r;
            if constexpr (k8) acc *= (one_tile || p.scale_in_tile) ? srow : p.scale[row];
            if constexpr (EPI == EPI_STORE) {
                const float b = p.bias ? (one_tile ? bias_reg : to_f<XT>(reinterpret_cast<const XT*>(p.bias)[row]))
                                       : 0.0f;
                store_row<XT, OT>(p, row, acc, b);
            } else {
                reinterpret_cast<float*>(p.out)[row] = acc;
                if (row < p.vocab && acc > best_v) { best_v = acc; best_i = row; }
            }
        }
        consumer_sync();  // red is reused by the next tile
    }
    if constexpr (EPI == EPI_LMHEAD) lmhead_finish(p, best_v, best_i, misc);
}

// One 16-byte weight chunk of one row against x.
template <int WK>
__device__ __forceinline__ float chunk_dot1(const uint4& w, const unsigned char* xs, int c) {
    float a = 0.0f, b = 0.0f;
    chunk_dot2<WK>(w, w, xs, c, a, b);  // the second row is the same registers; the compiler drops it
    return a;
}

// ---------------------------------------------------------------------------
// Kernel B: streaming (matrices larger than one tile per CTA, e.g. the LM
// head).  Every warp owns a ring of small row tiles: its lane 0 issues the
// bulk copies, the warp waits on its own mbarriers, its lanes are split across
// the tile's rows (32/R lanes per row, short shuffle reductions, two
// accumulators per lane), it writes its rows and re-arms the stage.  No
// block-wide barrier in the streaming loop.  Warp tiles are interleaved over
// all warps of the grid.
// ---------------------------------------------------------------------------
template <int WK, typename OT, int PRO, int EPI>
__global__ void __launch_bounds__(kConsumers) gemv_stream_kernel(const GemvParams p) {
    using XT = typename WTraits<WK>::XT;
    constexpr int kWB = (WK == WK_F32) ? 4 : (WK == WK_BF16 ? 2 : 1);
    constexpr bool k8 = (WK == WK_I8 || WK == WK_FP8);
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [warp][stage]
    uint64_t* aux_bar = full + kConsumerWarps * kMaxWarpStages;
    float* misc = reinterpret_cast<float*>(smem + kBarBytes) + kRedFloats;
    unsigned char* xs = smem + kSmemHeader;
    const int x_bytes = ((p.K * (int)sizeof(XT)) + 15) & ~15;
    unsigned char* aux = xs + x_bytes;
    unsigned char* xh = aux + p.aux_bytes;  // FP16 x of the tensor-core form
    unsigned char* stages = xh + mma_x_bytes(p);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t row_bytes = (size_t)p.K * kWB;
    const bool mma = k8 && p.mma;
    const int R = p.rows_per_tile, NSW = p.nstages;
    // pitch inside a tile: of rows, or in the tensor-core form of row pairs (rows 2p, 2p + 1
    // adjacent, pairs padded to an odd number of 16-byte units)
    const int RS = mma ? p.row_stride : (int)row_bytes;
    const int LPR = 32 / R;  // lanes per row (R is a power of two <= 32)
    const int rows_bytes_tile = mma ? 8 * RS : (int)(((size_t)R * RS + 15) & ~(size_t)15);
    const int gw = blockIdx.x * kConsumerWarps + warp, GW = gridDim.x * kConsumerWarps;
    const int my_tiles = (p.ntiles > gw) ? (p.ntiles - gw + GW - 1) / GW : 0;
    uint64_t* my_full = full + warp * kMaxWarpStages;
    unsigned char* my_stages = stages + (size_t)warp * NSW * p.tile_bytes;
    const unsigned char* Wb = reinterpret_cast<const unsigned char*>(p.W);

    if (tid == 0) {
        for (int i = 0; i < kConsumerWarps * NSW; i++) mbar_init(&full[(i / NSW) * kMaxWarpStages + i % NSW], 1);
        mbar_init(aux_bar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    // Stage warp tile k of this warp: one copy of the contiguous rows (lane 0),
    // or in the tensor-core form one copy per row pair into the padded pitch
    // (lane p copies rows 2p and 2p + 1; lane 0 arms the barrier first).  Called
    // by the whole warp.
    auto issue = [&](int k) {
        const int t = gw + k * GW;
        const int r0 = t * R, nr = min(R, p.M - r0);
        const int s = k % NSW;
        const uint32_t wbytes = (uint32_t)(nr * row_bytes);
        const uint32_t sbytes = p.scale_in_tile ? (uint32_t)(((nr + 3) & ~3) * 4) : 0u;
        unsigned char* st = my_stages + (size_t)s * p.tile_bytes;
        if (lane == 0) mbar_arrive_expect_tx(&my_full[s], wbytes + sbytes);
        if (mma) {
            __syncwarp();
            if (2 * lane < nr)
                bulk_g2s(st + (size_t)lane * RS, Wb + (size_t)(r0 + 2 * lane) * row_bytes,
                         (uint32_t)(min(2, nr - 2 * lane) * row_bytes), &my_full[s]);
        } else if (lane == 0) {
            bulk_g2s(st, Wb + (size_t)r0 * row_bytes, wbytes, &my_full[s]);
        }
        if (lane == 0 && sbytes) bulk_g2s(st + rows_bytes_tile, p.scale + r0, sbytes, &my_full[s]);
    };
    for (int k = 0; k < NSW && k < my_tiles; k++) issue(k);

    uint4 lw[kLnChunks], lb[kLnChunks];
    prefetch_ln_params<WK, PRO>(p, lw, lb);
    pdl_wait();
    pdl_trigger();
    if (!build_x<WK, PRO>(p, xs, aux, aux_bar, misc, lw, lb)) return;

    float x_up = 1.0f;
    if (mma) {
        // x -> FP16 x 2^-e with the CTA's max |x| in [2^14, 2^15): exact for every
        // BF16 value down to 2^-29 of the maximum; row sums are scaled back by 2^e.
        const XT* xv = reinterpret_cast<const XT*>(xs);
        float am = 0.0f;
        for (int k2 = tid; k2 < p.K; k2 += kConsumers) am = fmaxf(am, fabsf(to_f<XT>(xv[k2])));
        am = warp_max(am);
        if (lane == 0) misc[warp] = am;
        consumer_sync();
        am = misc[0];
#pragma unroll
        for (int w = 1; w < kConsumerWarps; w++) am = fmaxf(am, misc[w]);
        int e = 0;
        if (am > 0.0f && am <= FLT_MAX) e = max(-126, min(126, ((__float_as_int(am) >> 23) & 0xff) - 127 - 14));
        const float x_down = __int_as_float((127 - e) << 23);
        x_up = __int_as_float((127 + e) << 23);
        __half2* xh2 = reinterpret_cast<__half2*>(xh);
        for (int k2 = tid; 2 * k2 < p.K; k2 += kConsumers)
            xh2[k2] = __floats2half2_rn(to_f<XT>(xv[2 * k2]) * x_down, to_f<XT>(xv[2 * k2 + 1]) * x_down);
        consumer_sync();
    }

    const int nch = (int)(row_bytes / 16);
    const int rr = lane / LPR, sub = lane % LPR;
    float best_v = -FLT_MAX;
    int best_i = 0x7fffffff;
    // epilogue of one row: 8-bit scale, bias / GELU store or logits + running argmax
    auto finish_row = [&](const unsigned char* tile, int r0, int r, float acc) {
        const int row = r0 + r;
        if constexpr (k8)
            acc *= p.scale_in_tile ? reinterpret_cast<const float*>(tile + rows_bytes_tile)[r] : p.scale[row];
        if constexpr (EPI == EPI_STORE) {
            store_row<XT, OT>(p, row, acc, p.bias ? to_f<XT>(reinterpret_cast<const XT*>(p.bias)[row]) : 0.0f);
        } else {
            reinterpret_cast<float*>(p.out)[row] = acc;
            if (row < p.vocab && acc > best_v) { best_v = acc; best_i = row; }
        }
    };
    // ldmatrix row address of this lane: matrices 0 / 2 (A rows 0-7, bytes 0-15 / 16-31 of a
    // 32-code step) are the even rows 2p, matrices 1 / 3 (A rows 8-15) the odd rows 2p + 1;
    // the pair pitch puts the 8 rows of each matrix in distinct banks
    const uint32_t a_lane = (uint32_t)((lane & 7) * RS + ((lane >> 3) & 1) * row_bytes + (lane >> 4) * 16);
    for (int k = 0; k < my_tiles; k++) {
        const int s = k % NSW;
        if (!mbar_wait(&my_full[s], (uint32_t)((k / NSW) & 1))) return;
        const unsigned char* tile = my_stages + (size_t)s * p.tile_bytes;
        const int t = gw + k * GW;
        const int r0 = t * R, nr = min(R, p.M - r0);
        if constexpr (k8) {
            if (mma) {
                // 16 rows x 32 codes per step: ldmatrix.x4 gives lane (g, q) bytes 4q..4q+3 of tile
                // rows 2g (A row g) and 2g + 1 (A row g + 8) in both 16-byte halves; two MMAs (one
                // per half, separate accumulators) take x values 4q..4q+3 of the half as the B
                // column.  Rows past nr hold stale bytes: their rows of D are discarded (a row of
                // D depends on its row of A only).
                float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t ab = smem_addr(tile) + a_lane;
                const uint2* xw = reinterpret_cast<const uint2*>(xh) + (lane & 3);
                const int nku = p.K >> 5;
#pragma unroll 4
                for (int ku = 0; ku < nku; ku++) {
                    uint32_t q0, q1, q2, q3;
                    ldsm_x4(ab + (uint32_t)ku * 32u, q0, q1, q2, q3);
                    const uint2 x0 = xw[ku * 8], x1 = xw[ku * 8 + 4];
                    mma_f16(d0, code2_to_f16x2<WK == WK_FP8>(q0, false), code2_to_f16x2<WK == WK_FP8>(q1, false),
                            code2_to_f16x2<WK == WK_FP8>(q0, true), code2_to_f16x2<WK == WK_FP8>(q1, true), x0.x,
                            x0.y);
                    mma_f16(d1, code2_to_f16x2<WK == WK_FP8>(q2, false), code2_to_f16x2<WK == WK_FP8>(q3, false),
                            code2_to_f16x2<WK == WK_FP8>(q2, true), code2_to_f16x2<WK == WK_FP8>(q3, true), x1.x,
                            x1.y);
                }
                if ((lane & 3) == 0) {  // column 0 of D: tile rows 2g (d[0]) and 2g + 1 (d[2])
                    const int g = lane >> 2;
                    if (2 * g < nr) finish_row(tile, r0, 2 * g, (d0[0] + d1[0]) * x_up);
                    if (2 * g + 1 < nr) finish_row(tile, r0, 2 * g + 1, (d0[2] + d1[2]) * x_up);
                }
                __syncwarp();
                if (k + NSW < my_tiles) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // our reads before the refill
                    issue(k + NSW);
                }
                continue;
            }
        }
        float acc0 = 0.0f, acc1 = 0.0f;
        if (rr < nr) {
            const unsigned char* wr = tile + (size_t)rr * row_bytes;
            int c = sub;
#pragma unroll 2
            for (; c + LPR < nch; c += 2 * LPR) {
                const uint4 w0 = *reinterpret_cast<const uint4*>(wr + (size_t)c * 16);
                const uint4 w1 = *reinterpret_cast<const uint4*>(wr + (size_t)(c + LPR) * 16);
                acc0 += chunk_dot1<WK>(w0, xs, c);
                acc1 += chunk_dot1<WK>(w1, xs, c + LPR);
            }
            if (c < nch) acc0 += chunk_dot1<WK>(*reinterpret_cast<const uint4*>(wr + (size_t)c * 16), xs, c);
        }
        float acc = acc0 + acc1;
        for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (sub == 0 && rr < nr) finish_row(tile, r0, rr, acc);
        __syncwarp();
        if (k + NSW < my_tiles) {
            if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // our reads before the refill
            issue(k + NSW);
        }
    }
    if constexpr (EPI == EPI_LMHEAD) lmhead_finish(p, best_v, best_i, misc);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t gemv_smem_bytes(const GemvParams& p, int wk) {
    const size_t xb = (size_t)p.K * (wk == WK_F32 ? 4 : 2);
    const size_t rings = (size_t)(p.stream ? kConsumerWarps : 1) * p.nstages * p.tile_bytes;
    return kSmemHeader + ((xb + 15) & ~(size_t)15) + (size_t)p.aux_bytes + mma_x_bytes(p) + rings;
}

// Streaming tuning knobs (read once): GPT2B_GEMV_TILE_KB (warp tile bytes of
// kernel B), GPT2B_GEMV_STAGE_KB (ring bytes per CTA), GPT2B_GEMV_CTAS_PER_SM.
static int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}
// Defaults from a sweep on B200 (tile 6-48 KB, ring 100-200 KB, 1-2 CTAs per SM; the
// 50257 x 768 LM head, BF16 and INT8): 12 KB tiles, 100 KB of ring per CTA and two CTAs
// per SM keep the most bytes in flight with the most independent warps.
static const int g_tile_kb = env_int("GPT2B_GEMV_TILE_KB", 12);
static const int g_stage_kb = env_int("GPT2B_GEMV_STAGE_KB", 100);
static const int g_ctas_per_sm = env_int("GPT2B_GEMV_CTAS_PER_SM", 2);
// GPT2B_GEMV_MMA=0 keeps streamed 8-bit matrices on the CUDA-core form (for A/B timing).
static const int g_gemv_mma = env_int("GPT2B_GEMV_MMA", 1);

bool plan_gemv(GemvParams& p, int wk, int nsm, bool single_wave) {
    const size_t row_bytes = (size_t)p.K * wkind_bytes(wk);
    const size_t kOneTileMax = single_wave ? 96 * 1024 : 32 * 1024;
    if (row_bytes == 0 || row_bytes > 96 * 1024) return false;
    const bool w8 = (wk == WK_I8 || wk == WK_FP8);
    const int r_even = (p.M + nsm - 1) / nsm;
    if ((size_t)r_even * row_bytes <= kOneTileMax && r_even <= kRedFloats - 16) {
        // kernel A: one tile per CTA, the whole matrix in flight at once
        p.stream = 0;
        p.rows_per_tile = r_even;
        p.ntiles = (p.M + r_even - 1) / r_even;
        p.grid = p.ntiles;
        p.nstages = 1;
        p.scale_in_tile = (w8 && r_even % 4 == 0 && p.M % 4 == 0 && aligned16(p.scale)) ? 1 : 0;
        const size_t rows_b = ((size_t)r_even * row_bytes + 15) & ~(size_t)15;
        p.tile_bytes = (int)((rows_b + (p.scale_in_tile ? (size_t)r_even * 4 : 0) + 15) & ~(size_t)15);
    } else {
        // kernel B: per-warp rings of R-row tiles, R a power of two <= 32; 8-bit codes
        // with K a multiple of 32 take the tensor-core form (16-row tiles copied as 8 row
        // pairs, pairs padded to an odd number of 16-byte units so that the 8 rows of every
        // ldmatrix fall in distinct banks)
        p.stream = 1;
        int r = 1;
        while (r < 32 && (size_t)(2 * r) * row_bytes <= (size_t)g_tile_kb * 1024) r *= 2;
        size_t pitch = row_bytes;
        p.mma = 0;
        if (w8 && g_gemv_mma && p.K % 32 == 0) {
            const size_t rs = 2 * row_bytes + 16;  // row-pair pitch: an odd number of 16-byte units
            const size_t tile = 8 * rs + 64;
            if (kSmemHeader + 3 * (size_t)p.K + (size_t)p.aux_bytes + kConsumerWarps * tile + 1024 <=
                (size_t)max_dyn_smem()) {
                p.mma = 1;
                r = 16;
                pitch = rs;
            }
        }
        p.row_stride = (int)pitch;
        p.rows_per_tile = r;
        p.ntiles = (p.M + r - 1) / r;
        p.scale_in_tile = (w8 && r % 4 == 0 && p.M % 4 == 0 && aligned16(p.scale)) ? 1 : 0;
        const size_t rows_b = p.mma ? 8 * pitch : ((size_t)r * pitch + 15) & ~(size_t)15;
        p.tile_bytes = (int)((rows_b + (p.scale_in_tile ? (size_t)r * 4 : 0) + 15) & ~(size_t)15);
        const size_t budget = (size_t)g_stage_kb * 1024;
        p.nstages = (int)std::max<size_t>(1, std::min<size_t>(kMaxWarpStages, budget / ((size_t)kConsumerWarps *
                                                                                          p.tile_bytes)));
        // CTAs per SM: the requested number, or as many as the SM's 228 KB of shared memory holds
        const int fit = (int)(233472 / (gemv_smem_bytes(p, wk) + 1024));
        const int cps = std::max(1, std::min(g_ctas_per_sm, fit));
        const int warps_needed = p.ntiles;
        p.grid = std::max(1, std::min(nsm * cps, (warps_needed + kConsumerWarps - 1) / kConsumerWarps));
    }
    p.x_vec = aligned16(p.x) ? 1 : 0;
    return true;
}

template <int WK, typename OT, int PRO, int EPI>
static cudaError_t launch_one(const GemvParams& p, cudaStream_t s, bool pdl) {
    const size_t smem = gemv_smem_bytes(p, WK);
    if ((int)smem > max_dyn_smem() - 1024) return cudaErrorInvalidValue;
    if (p.stream) {
        auto k = gemv_stream_kernel<WK, OT, PRO, EPI>;
        static unsigned long long smem_set = 0;
        cudaError_t e = ensure_smem_limit(k, &smem_set);
        if (e != cudaSuccess) return e;
        return launch_k(k, dim3(p.grid), dim3(kConsumers), smem, s, pdl, p);
    }
    auto k = gemv_kernel<WK, OT, PRO, EPI>;
    static unsigned long long smem_set = 0;
    cudaError_t e = ensure_smem_limit(k, &smem_set);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(p.grid), dim3(kThreads), smem, s, pdl, p);
}

template <int WK>
static cudaError_t dispatch_wk(const GemvParams& p, bool out_f32, int pro, int epi, cudaStream_t s, bool pdl) {
    using XT = typename WTraits<WK>::XT;
    if (epi == EPI_LMHEAD) {
        if (pro == PRO_RES_LN) return launch_one<WK, float, PRO_RES_LN, EPI_LMHEAD>(p, s, pdl);
        if (pro == PRO_PLAIN) return launch_one<WK, float, PRO_PLAIN, EPI_LMHEAD>(p, s, pdl);
        return cudaErrorInvalidValue;
    }
    if (out_f32) {
        if (pro == PRO_PLAIN) return launch_one<WK, float, PRO_PLAIN, EPI_STORE>(p, s, pdl);
        if (pro == PRO_ATTN_MERGE) return launch_one<WK, float, PRO_ATTN_MERGE, EPI_STORE>(p, s, pdl);
        return cudaErrorInvalidValue;
    }
    switch (pro) {
        case PRO_PLAIN: return launch_one<WK, XT, PRO_PLAIN, EPI_STORE>(p, s, pdl);
        case PRO_RES_LN: return launch_one<WK, XT, PRO_RES_LN, EPI_STORE>(p, s, pdl);
        case PRO_EMB_LN: return launch_one<WK, XT, PRO_EMB_LN, EPI_STORE>(p, s, pdl);
        case PRO_ATTN_MERGE: return launch_one<WK, XT, PRO_ATTN_MERGE, EPI_STORE>(p, s, pdl);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvParams& p, int wk, bool out_f32, int pro, int epi, cudaStream_t s, bool pdl) {
    const int E = (wk == WK_F32) ? 4 : 8;
    if ((pro == PRO_RES_LN || pro == PRO_EMB_LN) && (p.K % E != 0 || p.K / E > kLnChunks * kConsumers))
        return cudaErrorInvalidValue;
    if (pro == PRO_ATTN_MERGE && p.K != p.attn_heads * 64) return cudaErrorInvalidValue;
    switch (wk) {
        case WK_F32: return dispatch_wk<WK_F32>(p, out_f32, pro, epi, s, pdl);
        case WK_BF16: return dispatch_wk<WK_BF16>(p, out_f32, pro, epi, s, pdl);
        case WK_I8: return dispatch_wk<WK_I8>(p, out_f32, pro, epi, s, pdl);
        case WK_FP8: return dispatch_wk<WK_FP8>(p, out_f32, pro, epi, s, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace gpt2b

// ---------------------------------------------------------------------------
// C ABI: the reference operator surface (see include/gpt2_b200.h)
// ---------------------------------------------------------------------------
using namespace gpt2b;

static int gemv_entry(int wk, bool out_f32, void* out, void* pre_gelu, const void* W, const void* x,
                      const float* scale, const void* bias, int M, int K, int do_gelu, cudaStream_t stream) {
    if (M < 0 || K <= 0) return GPT2B_ERR_INVALID_ARG;
    if (M == 0) return GPT2B_OK;
    if (!out || !W || !x) return GPT2B_ERR_INVALID_ARG;
    if ((wk == WK_I8 || wk == WK_FP8) && !scale) return GPT2B_ERR_INVALID_ARG;
    if (((size_t)K * wkind_bytes(wk)) % 16 != 0 || !aligned16(W)) return GPT2B_ERR_ALIGNMENT;
    GemvParams p;
    p.W = W; p.scale = scale; p.bias = bias; p.x = x; p.out = out; p.pre_gelu = pre_gelu;
    p.M = M; p.K = K; p.do_gelu = do_gelu ? 1 : 0;
    if (!plan_gemv(p, wk, sm_count(), false)) return GPT2B_ERR_UNSUPPORTED;
    return status_from(launch_gemv(p, wk, out_f32, PRO_PLAIN, EPI_STORE, stream, false));
}

extern "C" {

int gpt2b_launch_GEMV6_f32(float* out, const float* W, const float* x, int M, int K, gpt2b_stream_t stream) {
    return gemv_entry(WK_F32, true, out, nullptr, W, x, nullptr, nullptr, M, K, 0, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_bf16(float* out, const uint16_t* W, const uint16_t* x, int M, int K, gpt2b_stream_t stream) {
    return gemv_entry(WK_BF16, true, out, nullptr, W, x, nullptr, nullptr, M, K, 0, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_fused_f32(float* out, float* pre_gelu, const float* W, const float* x, const float* bias,
                                 int M, int K, int do_gelu, gpt2b_stream_t stream) {
    return gemv_entry(WK_F32, false, out, pre_gelu, W, x, nullptr, bias, M, K, do_gelu, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_fused_bf16(uint16_t* out, uint16_t* pre_gelu, const uint16_t* W, const uint16_t* x,
                                  const uint16_t* bias, int M, int K, int do_gelu, gpt2b_stream_t stream) {
    return gemv_entry(WK_BF16, false, out, pre_gelu, W, x, nullptr, bias, M, K, do_gelu, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_w8x2_i8(uint16_t* out, uint16_t* pre_gelu, const uint8_t* W, const uint16_t* x,
                               const float* scale, const uint16_t* bias, int M, int K, int do_gelu,
                               gpt2b_stream_t stream) {
    return gemv_entry(WK_I8, false, out, pre_gelu, W, x, scale, bias, M, K, do_gelu, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_w8x2_fp8(uint16_t* out, uint16_t* pre_gelu, const uint8_t* W, const uint16_t* x,
                                const float* scale, const uint16_t* bias, int M, int K, int do_gelu,
                                gpt2b_stream_t stream) {
    return gemv_entry(WK_FP8, false, out, pre_gelu, W, x, scale, bias, M, K, do_gelu, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_w8x2_i8_f32out(float* out, const uint8_t* W, const uint16_t* x, const float* scale, int M,
                                      int K, gpt2b_stream_t stream) {
    return gemv_entry(WK_I8, true, out, nullptr, W, x, scale, nullptr, M, K, 0, (cudaStream_t)stream);
}
int gpt2b_launch_GEMV6_w8x2_fp8_f32out(float* out, const uint8_t* W, const uint16_t* x, const float* scale, int M,
                                       int K, gpt2b_stream_t stream) {
    return gemv_entry(WK_FP8, true, out, nullptr, W, x, scale, nullptr, M, K, 0, (cudaStream_t)stream);
}

}  // extern "C"
