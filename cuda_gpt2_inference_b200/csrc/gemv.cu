// gemv.cu -- batch-1 decode GEMVs for FP32 / BF16 / INT8 / FP8 weights.
//
// Design (B200, HBM-bound, no tensor cores: one activation vector is not a
// dense contraction):
//   * A CTA owns whole row tiles.  Rows of a row-major matrix are contiguous,
//     so a tile is one contiguous byte range that a single elected thread moves
//     into shared memory with one cp.async.bulk, completing on an mbarrier.
//     The whole matrix is in flight at once for the per-layer shapes (one tile
//     per CTA, tiles sized to spread the bytes evenly over the 148 SMs); large
//     matrices (LM head) stream through a 2-3 stage ring.
//   * The weight copies are issued before griddepcontrol.wait, so under
//     programmatic dependent launch a GEMV fetches its weights while the
//     kernel before it is still running; only the activation vector waits.
//   * Each warp takes a pair of rows (x is read once per pair) and, when a
//     tile has fewer than 16 rows, a slice of K so all 8 warps work; FP32
//     accumulation, shuffle reduction, then bias / GELU / pre-GELU epilogue.
//   * Fused prologues for the engine: residual add + LayerNorm (or embedding
//     lookup + LayerNorm) computed redundantly per CTA from ~3 KB of L2-resident
//     data, which removes the separate LN kernels of the reference.
//   * Fused LM-head epilogue: logits, per-CTA argmax, last-CTA reduction and
//     device-side token/position advance (greedy decode without host trips).
#include "common.cuh"
#include "internal.h"

#include <float.h>

namespace gpt2b {

GPT2B_DEFINE_ERROR_READER(gemv_device_error)

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRedFloats = 160;  // per-warp partial sums (>= rows per tile + 16)
constexpr int kMaxLnPer = 8;     // LayerNorm prologue: C <= 8 * 256

template <int WK> struct WTraits;
template <> struct WTraits<WK_F32> { using XT = float; static constexpr int kElemsPerChunk = 4; };
template <> struct WTraits<WK_BF16> { using XT = __nv_bfloat16; static constexpr int kElemsPerChunk = 8; };
template <> struct WTraits<WK_I8> { using XT = __nv_bfloat16; static constexpr int kElemsPerChunk = 16; };
template <> struct WTraits<WK_FP8> { using XT = __nv_bfloat16; static constexpr int kElemsPerChunk = 16; };

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

// Decoded value of element c of embedding row `tok` (PRO_EMB_LN): the
// activation-type table, or the 8-bit code times its row scale rounded to
// bf16 -- exactly what dequant_wte_kernel stores (GEMV_w8.cuh:396).
template <int WK>
__device__ __forceinline__ float emb_value(const GemvParams& p, int tok, int c) {
    using XT = typename WTraits<WK>::XT;
    if constexpr (WK == WK_I8 || WK == WK_FP8) {
        const uint8_t code = p.wte8[(size_t)tok * p.K + c];
        const float v = (WK == WK_I8) ? (float)(int8_t)code : e4m3_to_f((uint32_t)code, 0);
        return round_to<__nv_bfloat16>(v * p.wte_scale[tok]);
    } else {
        return to_f<XT>(reinterpret_cast<const XT*>(p.wte)[(size_t)tok * p.K + c]);
    }
}

template <int WK, typename OT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
    using XT = typename WTraits<WK>::XT;
    constexpr int kWB = (WK == WK_F32) ? 4 : (WK == WK_BF16 ? 2 : 1);
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);            // 4 stages max
    float* red = reinterpret_cast<float*>(smem + 64);               // kRedFloats
    unsigned char* xs = smem + 64 + kRedFloats * 4;                 // K activations
    const int x_bytes = ((p.K * (int)sizeof(XT)) + 15) & ~15;
    unsigned char* stages = xs + x_bytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t row_bytes = (size_t)p.K * kWB;
    const int R = p.rows_per_tile, NS = p.nstages, G = gridDim.x;
    const unsigned char* Wb = reinterpret_cast<const unsigned char*>(p.W);

    // ---- 1. stage the first tiles (weights never depend on other kernels) ----
    if (tid == 0) {
        for (int s = 0; s < NS; s++) mbar_init(&bars[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            const int t = blockIdx.x + s * G;
            if (t >= p.ntiles) break;
            const int r0 = t * R, nr = min(R, p.M - r0);
            const uint32_t bytes = (uint32_t)(nr * row_bytes);
            mbar_arrive_expect_tx(&bars[s], bytes);
            bulk_g2s(stages + (size_t)s * p.tile_bytes, Wb + (size_t)r0 * row_bytes, bytes, &bars[s]);
        }
    }

    // ---- 2. wait for the producer of x, then let the next kernel launch ----
    pdl_wait();
    pdl_trigger();

    // ---- 3. x into shared memory (plain, or residual/embedding + LayerNorm) ----
    XT* xsv = reinterpret_cast<XT*>(xs);
    if constexpr (PRO == PRO_PLAIN) {
        const XT* x = reinterpret_cast<const XT*>(p.x);
        for (int k = tid; k < p.K; k += kThreads) xsv[k] = x[k];
    } else {
        const int C = p.K;
        float v[kMaxLnPer];
        float sum = 0.0f;
        int tok = 0, pos = 0;
        if constexpr (PRO == PRO_EMB_LN) {
            tok = *p.d_token;
            pos = *p.d_pos;
            if (tok < 0 || tok >= p.vocab) { if (tid == 0) report_device_error(GPT2B_DEVERR_BAD_TOKEN); tok = 0; }
            if (pos < 0 || pos >= p.maxT) { if (tid == 0) report_device_error(GPT2B_DEVERR_BAD_POS); pos = 0; }
        }
#pragma unroll
        for (int i = 0; i < kMaxLnPer; i++) {
            const int c = tid + i * kThreads;
            float r = 0.0f;
            if (c < C) {
                if constexpr (PRO == PRO_EMB_LN) {
                    r = emb_value<WK>(p, tok, c) + to_f<XT>(reinterpret_cast<const XT*>(p.wpe)[(size_t)pos * C + c]);
                } else {
                    r = to_f<XT>(reinterpret_cast<const XT*>(p.res_in)[c]) +
                        to_f<XT>(reinterpret_cast<const XT*>(p.delta)[c]);
                }
                r = round_to<XT>(r);  // the residual is stored as floatX and LN reads it back
                if (blockIdx.x == 0 && p.res_out) reinterpret_cast<XT*>(p.res_out)[c] = from_f<XT>(r);
                sum += r;
            }
            v[i] = r;
        }
        const float mean = block_sum(sum, red) / (float)C;
        float sq = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxLnPer; i++) {
            const int c = tid + i * kThreads;
            if (c < C) { const float d = v[i] - mean; sq += d * d; }
        }
        const float var = block_sum(sq, red) / (float)C;
        const float rstd = rsqrtf(var + 1e-5f);
        const XT* lw = reinterpret_cast<const XT*>(p.ln_w);
        const XT* lb = reinterpret_cast<const XT*>(p.ln_b);
#pragma unroll
        for (int i = 0; i < kMaxLnPer; i++) {
            const int c = tid + i * kThreads;
            if (c < C) {
                const float n = rstd * (v[i] - mean);
                const XT o = from_f<XT>(n * to_f<XT>(lw[c]) + to_f<XT>(lb[c]));
                xsv[c] = o;
                if (blockIdx.x == 0 && p.ln_out) reinterpret_cast<XT*>(p.ln_out)[c] = o;
            }
        }
    }
    __syncthreads();

    // ---- 4. tiles ----
    const int nch = (int)(row_bytes / 16);
    float best_v = -FLT_MAX;
    int best_i = 0x7fffffff;
    int it = 0;
    for (int t = blockIdx.x; t < p.ntiles; t += G, ++it) {
        const int s = it % NS;
        const uint32_t parity = (uint32_t)((it / NS) & 1);
        const int r0 = t * R, nr = min(R, p.M - r0);
        const unsigned char* tile = stages + (size_t)s * p.tile_bytes;
        if (!mbar_wait(&bars[s], parity)) return;

        const int npairs = (nr + 1) >> 1;
        const int splits = npairs >= kWarps ? 1 : kWarps / npairs;
        for (int slot = warp; slot < npairs * splits; slot += kWarps) {
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
        __syncthreads();
        // tile fully consumed: refill this stage with tile t + NS*G
        if (tid == 0) {
            const int tn = t + NS * G;
            if (tn < p.ntiles) {
                const int rn = tn * R, nrn = min(R, p.M - rn);
                const uint32_t bytes = (uint32_t)(nrn * row_bytes);
                mbar_arrive_expect_tx(&bars[s], bytes);
                bulk_g2s(stages + (size_t)s * p.tile_bytes, Wb + (size_t)rn * row_bytes, bytes, &bars[s]);
            }
        }
        for (int r = tid; r < nr; r += kThreads) {
            const int pair = r >> 1;
            float acc = 0.0f;
            for (int sp = 0; sp < splits; sp++) acc += red[(pair * splits + sp) * 2 + (r & 1)];
            const int row = r0 + r;
            if constexpr (WK == WK_I8 || WK == WK_FP8) acc *= p.scale[row];
            if constexpr (EPI == EPI_STORE) {
                float pre = acc;
                if (p.bias) pre += to_f<XT>(reinterpret_cast<const XT*>(p.bias)[row]);
                if (p.pre_gelu) reinterpret_cast<OT*>(p.pre_gelu)[row] = from_f<OT>(pre);
                const float o = p.do_gelu ? gelu_tanh(pre) : pre;
                reinterpret_cast<OT*>(p.out)[row] = from_f<OT>(o);
            } else {
                reinterpret_cast<float*>(p.out)[row] = acc;
                if (row < p.vocab && acc > best_v) { best_v = acc; best_i = row; }
            }
        }
        __syncthreads();  // red is reused by the next tile
    }

    if constexpr (EPI == EPI_LMHEAD) {
        // block argmax: largest value, lowest index on ties
        __shared__ float s_v[kWarps];
        __shared__ int s_i[kWarps];
        __shared__ int s_last;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) { s_v[warp] = best_v; s_i[warp] = best_i; }
        __syncthreads();
        if (tid == 0) {
            float bv = s_v[0];
            int bi = s_i[0];
            for (int w = 1; w < kWarps; w++)
                if (s_v[w] > bv || (s_v[w] == bv && s_i[w] < bi)) { bv = s_v[w]; bi = s_i[w]; }
            p.part_val[blockIdx.x] = bv;
            p.part_idx[blockIdx.x] = bi;
            __threadfence();
            const unsigned ticket = atomicAdd(p.counter, 1u);
            s_last = (ticket == gridDim.x - 1);
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            float bv = -FLT_MAX;
            int bi = 0x7fffffff;
            for (int b = tid; b < (int)gridDim.x; b += kThreads) {
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
            if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
            __syncthreads();
            if (tid == 0) {
                for (int w = 1; w < kWarps; w++)
                    if (s_v[w] > s_v[0] || (s_v[w] == s_v[0] && s_i[w] < s_i[0])) { s_v[0] = s_v[w]; s_i[0] = s_i[w]; }
                *p.counter = 0u;
                if (p.advance) {
                    const int pos = *p.pos_io;
                    const int next = (pos + 1 < p.n_prompt) ? p.prompt[pos + 1] : s_i[0];
                    if (p.history) p.history[pos + 1] = next;
                    *p.token_io = next;
                    *p.pos_io = pos + 1;
                } else if (p.token_io) {
                    *p.token_io = s_i[0];
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t gemv_smem_bytes(const GemvParams& p, int wk) {
    const size_t xb = (size_t)p.K * (wk == WK_F32 ? 4 : 2);
    return 64 + kRedFloats * 4 + ((xb + 15) & ~(size_t)15) + (size_t)p.nstages * p.tile_bytes;
}

bool plan_gemv(GemvParams& p, int wk, int nsm, bool single_wave) {
    const size_t row_bytes = (size_t)p.K * wkind_bytes(wk);
    const size_t kTileTarget = 32 * 1024, kTileMax = 96 * 1024;
    if (row_bytes == 0 || row_bytes > kTileMax) return false;
    int r_stream = (int)(kTileTarget / row_bytes);
    if (r_stream < 1) r_stream = 1;
    if (r_stream > kRedFloats - 16) r_stream = kRedFloats - 16;
    const int r_even = (p.M + nsm - 1) / nsm;
    if (r_even <= r_stream || (single_wave && (size_t)r_even * row_bytes <= kTileMax && r_even <= kRedFloats - 16)) {
        p.rows_per_tile = r_even;
        p.ntiles = (p.M + r_even - 1) / r_even;
        p.grid = p.ntiles;
        p.nstages = 1;
    } else {
        p.rows_per_tile = r_stream;
        p.ntiles = (p.M + r_stream - 1) / r_stream;
        p.grid = std::min(p.ntiles, 2 * nsm);
        const int per = (p.ntiles + p.grid - 1) / p.grid;
        p.nstages = std::max(1, std::min(3, per));
    }
    p.tile_bytes = (int)(((size_t)p.rows_per_tile * row_bytes + 15) & ~(size_t)15);
    return true;
}

template <int WK, typename OT, int PRO, int EPI>
static cudaError_t launch_one(const GemvParams& p, cudaStream_t s, bool pdl) {
    auto k = gemv_kernel<WK, OT, PRO, EPI>;
    static unsigned long long smem_set = 0;
    const size_t smem = gemv_smem_bytes(p, WK);
    if ((int)smem > max_dyn_smem()) return cudaErrorInvalidValue;
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
        if (pro != PRO_PLAIN) return cudaErrorInvalidValue;
        return launch_one<WK, float, PRO_PLAIN, EPI_STORE>(p, s, pdl);
    }
    switch (pro) {
        case PRO_PLAIN: return launch_one<WK, XT, PRO_PLAIN, EPI_STORE>(p, s, pdl);
        case PRO_RES_LN: return launch_one<WK, XT, PRO_RES_LN, EPI_STORE>(p, s, pdl);
        case PRO_EMB_LN: return launch_one<WK, XT, PRO_EMB_LN, EPI_STORE>(p, s, pdl);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvParams& p, int wk, bool out_f32, int pro, int epi, cudaStream_t s, bool pdl) {
    if (pro != PRO_PLAIN && p.K > kMaxLnPer * kThreads) return cudaErrorInvalidValue;
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
