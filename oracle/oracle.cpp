/*
 * oracle.cpp -- CPU restatement of the reference GPT-2 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled by oracle/build_oracle.py
 * into oracle/_build/liboracle.so; only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg load it.
 */
#include "oracle.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <math.h>
#include <float.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

/* ------------------------------------------------------------------------ */
/* scalar format helpers                                                     */
/* ------------------------------------------------------------------------ */

/* float -> bf16, round to nearest even: the conversion the reference applies
 * whenever it stores a float into floatX (__float2bfloat16 in cuda_bf16.h). */
extern "C" uint16_t orc_f32_to_bf16_bits(float x) {
    __nv_bfloat16 b = __float2bfloat16(x);
    __nv_bfloat16_raw r = b;
    return r.x;
}
extern "C" float orc_bf16_bits_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
extern "C" float orc_bf16_round(float x) { return orc_bf16_bits_to_f32(orc_f32_to_bf16_bits(x)); }

extern "C" void orc_bf16_to_f32(float* out, const uint16_t* in, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_bf16_bits_to_f32(in[i]);
}
extern "C" void orc_f32_to_bf16(uint16_t* out, const float* in, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_f32_to_bf16_bits(in[i]);
}

/* GEMV_w8.cuh:37-48 -- INT8 codes are two's-complement bytes; FP8 codes are
 * E4M3, which every wider float format represents exactly (the reference goes
 * through bf16; half is used here because its host converter exists). */
static float g_fp8_table[256];
static bool g_fp8_ready = false;
static void fp8_init() {
    if (g_fp8_ready) return;
    for (int i = 0; i < 256; i++) {
        __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)i, __NV_E4M3);
        __half h;
        h = hr;
        g_fp8_table[i] = __half2float(h);
    }
    g_fp8_ready = true;
}
extern "C" float orc_w8_decode(uint8_t code, int fmt) {
    if (fmt == ORC_FMT_FP8) {
        fp8_init();
        return g_fp8_table[code];
    }
    return (float)(int8_t)code;
}

/* Encode one value already divided by its scale.  INT8: round half to even
 * (__float2int_rn) and clamp to [-127,127] (quantize.cu:76-78,
 * attention_kvcache_w8.cuh:61-65).  FP8: saturating E4M3 conversion
 * (quantize.cu:69, attention_kvcache_w8.cuh:56-59). */
static inline uint8_t w8_encode_scaled(float v, int fmt) {
    if (fmt == ORC_FMT_FP8) {
        return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
    }
    int q = (int)nearbyintf(v); /* default FP environment: round to nearest even */
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    return (uint8_t)(int8_t)q;
}

/* ------------------------------------------------------------------------ */
/* per-op loops                                                              */
/* ------------------------------------------------------------------------ */

/* gemv/GEMV.cu:84-93: float accumulation in k order, rows in parallel. */
extern "C" void orc_gemv(float* out, const float* W, const float* x, int M, int K) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float* w = W + (size_t)m * K;
        float sum = 0.0f;
        for (int k = 0; k < K; k++) sum += w[k] * x[k];
        out[m] = sum;
    }
}

/* GPT-2 tanh GELU as written in GEMV.cuh:196-197 and gelu/gelu.cu:31-37. */
static inline float gelu_tanh(float x) {
    float cube = 0.044715f * x * x * x;
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + cube)));
}

extern "C" void orc_gemv_fused(float* out, float* pre_gelu, const float* W, const float* x,
                               const float* bias, int M, int K, int do_gelu) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float* w = W + (size_t)m * K;
        float sum = 0.0f;
        for (int k = 0; k < K; k++) sum += w[k] * x[k];
        float pre = sum;
        if (bias) pre += bias[m];
        if (pre_gelu) pre_gelu[m] = pre;
        out[m] = do_gelu ? gelu_tanh(pre) : pre;
    }
}

extern "C" void orc_gemv_w8(float* out, float* pre_gelu, const uint8_t* W8, int fmt,
                            const float* x, const float* scale, const float* bias,
                            int M, int K, int do_gelu) {
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = orc_w8_decode((uint8_t)i, fmt);
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const uint8_t* w = W8 + (size_t)m * K;
        float sum = 0.0f;
        for (int k = 0; k < K; k++) sum += lut[w[k]] * x[k];
        float pre = sum * scale[m]; /* row scale applied once after the K loop (GEMV_w8.cuh:136) */
        if (bias) pre += bias[m];
        if (pre_gelu) pre_gelu[m] = pre;
        out[m] = do_gelu ? gelu_tanh(pre) : pre;
    }
}

extern "C" void orc_dequant_rows(float* out, const uint8_t* W8, const float* scale, int rows,
                                 int cols, int fmt) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        for (int c = 0; c < cols; c++) {
            size_t i = (size_t)r * cols + c;
            out[i] = orc_bf16_round(orc_w8_decode(W8[i], fmt) * scale[r]);
        }
    }
}

/* quantize.cu:41-81: amax over the row, s = amax / 127 (INT8) or / 448 (FP8),
 * s = 1 for an all-zero row, codes = encode(w / s). */
extern "C" void orc_quant_rows(const float* W, uint8_t* W8, float* scale, int M, int K, int fmt) {
    const float full = (fmt == ORC_FMT_FP8) ? 448.0f : 127.0f;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float* w = W + (size_t)m * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = fmaxf(amax, fabsf(w[k]));
        float s = (amax == 0.0f) ? 1.0f : (amax / full);
        scale[m] = s;
        for (int k = 0; k < K; k++) W8[(size_t)m * K + k] = w8_encode_scaled(w[k] / s, fmt);
    }
}

/* attention_kvcache_w8.cuh:115-155: amax starts at 0, scale = amax / LIMIT
 * (no zero guard), codes are 0 when scale is not positive. */
extern "C" void orc_kv_encode_row(const float* x, int hs, int fmt, uint8_t* codes, float* scale) {
    const float limit = (fmt == ORC_FMT_FP8) ? 448.0f : 127.0f;
    float mx = 0.0f;
    for (int d = 0; d < hs; d++) mx = fmaxf(mx, fabsf(x[d]));
    float s = mx / limit;
    *scale = s;
    for (int d = 0; d < hs; d++) codes[d] = (s > 0.0f) ? w8_encode_scaled(x[d] / s, fmt) : (uint8_t)0;
}

/* attention_kvcache/attention_kvcache.cu:74-103.  The reference re-evaluates
 * expf(score - max) once per output channel; the value is the same each time,
 * so it is computed once here and the accumulation order is unchanged. */
extern "C" void orc_attention_kv(float* out, const float* qkv, const float* kv_cache,
                                 int B, int seq_len, int NH, int hs, int maxT, float scale) {
    std::vector<float> scores(seq_len > 0 ? seq_len : 1), ex(seq_len > 0 ? seq_len : 1);
    for (int b = 0; b < B; b++) {
        for (int h = 0; h < NH; h++) {
            const float* q = qkv + (size_t)b * 3 * NH * hs + (size_t)h * hs;
            const float* kc = kv_cache + ((size_t)b * NH + h) * maxT * hs;
            const float* vc = kv_cache + (size_t)B * NH * maxT * hs + ((size_t)b * NH + h) * maxT * hs;
            float maxval = -FLT_MAX;
            for (int j = 0; j < seq_len; j++) {
                float sum = 0.0f;
                for (int d = 0; d < hs; d++) sum += q[d] * kc[(size_t)j * hs + d];
                scores[j] = sum * scale;
                maxval = fmaxf(maxval, scores[j]);
            }
            for (int j = 0; j < seq_len; j++) ex[j] = expf(scores[j] - maxval);
            for (int d = 0; d < hs; d++) {
                float acc = 0.0f, expsum = 0.0f;
                for (int j = 0; j < seq_len; j++) {
                    acc += ex[j] * vc[(size_t)j * hs + d];
                    expsum += ex[j];
                }
                out[((size_t)b * NH + h) * hs + d] = acc / expsum;
            }
        }
    }
}

extern "C" void orc_attention_kv_w8(float* out, const float* qkv, const uint8_t* kv_cache,
                                    const float* kv_scale, int fmt, int B, int seq_len, int NH,
                                    int hs, int maxT, float scale) {
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = orc_w8_decode((uint8_t)i, fmt);
    std::vector<float> scores(seq_len > 0 ? seq_len : 1), ex(seq_len > 0 ? seq_len : 1);
    const size_t vofs = (size_t)B * NH * maxT * hs, vsofs = (size_t)B * NH * maxT;
    for (int b = 0; b < B; b++) {
        for (int h = 0; h < NH; h++) {
            const float* q = qkv + (size_t)b * 3 * NH * hs + (size_t)h * hs;
            const size_t row0 = ((size_t)b * NH + h) * maxT;
            float maxval = -FLT_MAX;
            for (int j = 0; j < seq_len; j++) {
                const uint8_t* kr = kv_cache + (row0 + j) * hs;
                float sum = 0.0f;
                for (int d = 0; d < hs; d++) sum += q[d] * lut[kr[d]];
                scores[j] = sum * kv_scale[row0 + j] * scale;
                maxval = fmaxf(maxval, scores[j]);
            }
            for (int j = 0; j < seq_len; j++) ex[j] = expf(scores[j] - maxval);
            for (int d = 0; d < hs; d++) {
                float acc = 0.0f, expsum = 0.0f;
                for (int j = 0; j < seq_len; j++) {
                    float v = lut[kv_cache[vofs + (row0 + j) * hs + d]] * kv_scale[vsofs + row0 + j];
                    acc += ex[j] * v;
                    expsum += ex[j];
                }
                out[((size_t)b * NH + h) * hs + d] = acc / expsum;
            }
        }
    }
}

/* fused/fused.cu:50-80 */
extern "C" void orc_layernorm(float* out, float* mean, float* rstd, const float* inp,
                              const float* weight, const float* bias, int N, int C) {
    const float eps = 1e-5f;
    for (int n = 0; n < N; n++) {
        const float* x = inp + (size_t)n * C;
        float m = 0.0f;
        for (int i = 0; i < C; i++) m += x[i];
        m = m / C;
        float v = 0.0f;
        for (int i = 0; i < C; i++) {
            float xs = x[i] - m;
            v += xs * xs;
        }
        v = v / C;
        float s = 1.0f / sqrtf(v + eps);
        float* o = out + (size_t)n * C;
        for (int i = 0; i < C; i++) o[i] = (s * (x[i] - m)) * weight[i] + bias[i];
        if (mean) mean[n] = m;
        if (rstd) rstd[n] = s;
    }
}

extern "C" void orc_residual(float* out, const float* a, const float* b, int N) {
    for (int i = 0; i < N; i++) out[i] = a[i] + b[i];
}

extern "C" void orc_gelu(float* out, const float* inp, int N) {
    for (int i = 0; i < N; i++) out[i] = gelu_tanh(inp[i]);
}

extern "C" void orc_encoder_kv(float* out, const int* tokens, const float* wte, const float* wpe,
                               int pos, int B, int C) {
    for (int b = 0; b < B; b++)
        for (int c = 0; c < C; c++)
            out[(size_t)b * C + c] = wte[(size_t)tokens[b] * C + c] + wpe[(size_t)pos * C + c];
}

extern "C" int orc_argmax(const float* logits, int V) {
    int best = 0;
    for (int i = 1; i < V; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* ------------------------------------------------------------------------ */
/* whole model                                                               */
/* ------------------------------------------------------------------------ */

struct orc_model {
    int maxT, V, L, NH, C, Vp, hs;
    int wmode, kvmode, fmt;
    /* non-linear parameters, decoded to float (gpt2_model.h:41-58 order) */
    std::vector<float> wpe, ln1w, ln1b, qkvb, attprojb, ln2w, ln2b, fcb, fcprojb, lnfw, lnfb;
    std::vector<float> wte_emb; /* embedding table as the encoder sees it */
    /* linear weights: float (F32/BF16 modes) or codes + scales (8-bit modes) */
    std::vector<float> wte_f, qkvw_f, attprojw_f, fcw_f, fcprojw_f;
    std::vector<uint8_t> wte_8, qkvw_8, attprojw_8, fcw_8, fcprojw_8;
    std::vector<float> wte_s, qkvw_s, attprojw_s, fcw_s, fcprojw_s;
    /* KV cache, reference layout per layer [K: NH*maxT*hs][V: same] (B = 1) */
    std::vector<float> kv_f;
    std::vector<uint8_t> kv_8;
    std::vector<float> kv_s;
    /* activations of the last step, for probes */
    std::vector<float> encoded, ln1, qkv, atty, residual2, ln2, fch, fch_gelu, residual3, lnf;
    std::vector<float> tmp;
};

static inline float rx(const orc_model* m, float v) {
    return m->wmode == ORC_W_F32 ? v : orc_bf16_round(v);
}
static void rx_vec(const orc_model* m, float* v, size_t n) {
    if (m->wmode == ORC_W_F32) return;
    for (size_t i = 0; i < n; i++) v[i] = orc_bf16_round(v[i]);
}

namespace {
struct Reader {
    const uint8_t* p;
    size_t left;
    bool ok = true;
    const uint8_t* take(size_t n) {
        if (n > left) { ok = false; return nullptr; }
        const uint8_t* r = p;
        p += n;
        left -= n;
        return r;
    }
};
}  // namespace

static bool read_float_tensor(Reader& r, std::vector<float>& dst, size_t n, bool bf16) {
    dst.resize(n);
    if (bf16) {
        const uint8_t* src = r.take(n * 2);
        if (!src) return false;
        std::vector<uint16_t> tmp(n);
        memcpy(tmp.data(), src, n * 2);
        orc_bf16_to_f32(dst.data(), tmp.data(), n);
    } else {
        const uint8_t* src = r.take(n * 4);
        if (!src) return false;
        memcpy(dst.data(), src, n * 4);
    }
    return true;
}

static bool read_code_tensor(Reader& r, std::vector<uint8_t>& dst, size_t n) {
    const uint8_t* src = r.take(n);
    if (!src) return false;
    dst.assign(src, src + n);
    return true;
}

extern "C" orc_model* orc_model_from_buffer(const void* image, size_t nbytes, int wmode,
                                            const float* scales, size_t nscales, int kvmode,
                                            const char** err) {
    const char* dummy;
    if (!err) err = &dummy;
    *err = nullptr;
    if (nbytes < 1024) { *err = "image shorter than the 256-int header"; return nullptr; }
    int hdr[256];
    memcpy(hdr, image, 1024);
    /* gpt2_model.h:276-296 */
    if (hdr[0] != 20251103) { *err = "bad magic"; return nullptr; }
    const int want_version = (wmode == ORC_W_F32) ? 3 : 5;
    if (hdr[1] != want_version) { *err = "version does not match the weight mode"; return nullptr; }
    orc_model* m = new orc_model();
    m->maxT = hdr[2]; m->V = hdr[3]; m->L = hdr[4]; m->NH = hdr[5]; m->C = hdr[6]; m->Vp = hdr[7];
    if (m->maxT <= 0 || m->V <= 0 || m->L <= 0 || m->NH <= 0 || m->C <= 0 || m->Vp < m->V ||
        m->C % m->NH != 0) {
        *err = "bad dimensions in header";
        delete m;
        return nullptr;
    }
    m->hs = m->C / m->NH;
    m->wmode = wmode;
    m->kvmode = kvmode;
    m->fmt = (wmode == ORC_W_FP8) ? ORC_FMT_FP8 : ORC_FMT_INT8;
    const size_t C = m->C, L = m->L, Vp = m->Vp, maxT = m->maxT;
    const bool w8 = (wmode == ORC_W_INT8 || wmode == ORC_W_FP8);
    const bool bf16 = (wmode != ORC_W_F32);
    if (kvmode == ORC_KV_8BIT && !w8) { *err = "8-bit KV needs an 8-bit weight mode"; delete m; return nullptr; }

    Reader r{(const uint8_t*)image + 1024, nbytes - 1024};
    bool ok = true;
    auto lin = [&](std::vector<float>& f, std::vector<uint8_t>& q, size_t n) {
        if (w8) ok = ok && read_code_tensor(r, q, n);
        else ok = ok && read_float_tensor(r, f, n, bf16);
    };
    /* fill_in_parameter_sizes order (gpt2_model.h:63-87) */
    lin(m->wte_f, m->wte_8, Vp * C);
    ok = ok && read_float_tensor(r, m->wpe, maxT * C, bf16);
    ok = ok && read_float_tensor(r, m->ln1w, L * C, bf16);
    ok = ok && read_float_tensor(r, m->ln1b, L * C, bf16);
    lin(m->qkvw_f, m->qkvw_8, L * 3 * C * C);
    ok = ok && read_float_tensor(r, m->qkvb, L * 3 * C, bf16);
    lin(m->attprojw_f, m->attprojw_8, L * C * C);
    ok = ok && read_float_tensor(r, m->attprojb, L * C, bf16);
    ok = ok && read_float_tensor(r, m->ln2w, L * C, bf16);
    ok = ok && read_float_tensor(r, m->ln2b, L * C, bf16);
    lin(m->fcw_f, m->fcw_8, L * 4 * C * C);
    ok = ok && read_float_tensor(r, m->fcb, L * 4 * C, bf16);
    lin(m->fcprojw_f, m->fcprojw_8, L * C * 4 * C);
    ok = ok && read_float_tensor(r, m->fcprojb, L * C, bf16);
    ok = ok && read_float_tensor(r, m->lnfw, C, bf16);
    ok = ok && read_float_tensor(r, m->lnfb, C, bf16);
    if (!ok) { *err = "image truncated"; delete m; return nullptr; }

    if (w8) {
        /* scale file: float per row in group order (quantize.cu:226-229) */
        const size_t need = Vp + L * 3 * C + L * C + L * 4 * C + L * C;
        if (!scales || nscales != need) { *err = "scale count does not match the model"; delete m; return nullptr; }
        const float* s = scales;
        m->wte_s.assign(s, s + Vp); s += Vp;
        m->qkvw_s.assign(s, s + L * 3 * C); s += L * 3 * C;
        m->attprojw_s.assign(s, s + L * C); s += L * C;
        m->fcw_s.assign(s, s + L * 4 * C); s += L * 4 * C;
        m->fcprojw_s.assign(s, s + L * C);
        /* dequant_wte_kernel fills the embedding slot (inference_gpt2_opt.cu:214) */
        m->wte_emb.resize(Vp * C);
        orc_dequant_rows(m->wte_emb.data(), m->wte_8.data(), m->wte_s.data(), (int)Vp, (int)C, m->fmt);
    } else {
        m->wte_emb = m->wte_f;
    }
    const size_t kv_elems = L * 2 * (size_t)m->NH * maxT * m->hs;
    if (kvmode == ORC_KV_8BIT) {
        m->kv_8.assign(kv_elems, 0);
        m->kv_s.assign(L * 2 * (size_t)m->NH * maxT, 0.0f);
    } else {
        m->kv_f.assign(kv_elems, 0.0f);
    }
    m->encoded.resize(C);
    m->ln1.resize(L * C);
    m->qkv.resize(L * 3 * C);
    m->atty.resize(L * C);
    m->residual2.resize(L * C);
    m->ln2.resize(L * C);
    m->fch.resize(L * 4 * C);
    m->fch_gelu.resize(L * 4 * C);
    m->residual3.resize(L * C);
    m->lnf.resize(C);
    m->tmp.resize(4 * C > Vp ? 4 * C : Vp);
    return m;
}

extern "C" void orc_model_free(orc_model* m) { delete m; }

extern "C" void orc_model_config(const orc_model* m, int cfg[6]) {
    cfg[0] = m->maxT; cfg[1] = m->V; cfg[2] = m->L; cfg[3] = m->NH; cfg[4] = m->C; cfg[5] = m->Vp;
}

extern "C" void orc_model_reset(orc_model* m) {
    std::fill(m->kv_f.begin(), m->kv_f.end(), 0.0f);
    std::fill(m->kv_8.begin(), m->kv_8.end(), (uint8_t)0);
    std::fill(m->kv_s.begin(), m->kv_s.end(), 0.0f);
}

/* One Linear: GEMV6_fused (F32/BF16) or GEMV6_w8x2 (8-bit) semantics. */
static void linear(const orc_model* m, float* out, float* pre_gelu, const std::vector<float>& Wf,
                   const std::vector<uint8_t>& W8, const std::vector<float>& S, size_t w_off,
                   size_t s_off, const float* x, const float* bias, int M, int K, int do_gelu) {
    if (m->wmode == ORC_W_INT8 || m->wmode == ORC_W_FP8)
        orc_gemv_w8(out, pre_gelu, W8.data() + w_off, m->fmt, x, S.data() + s_off, bias, M, K, do_gelu);
    else
        orc_gemv_fused(out, pre_gelu, Wf.data() + w_off, x, bias, M, K, do_gelu);
}

extern "C" int orc_model_step(orc_model* m, int token, int pos, float* logits) {
    if (token < 0 || token >= m->V || pos < 0 || pos >= m->maxT) return 1;
    const int C = m->C, L = m->L, NH = m->NH, hs = m->hs, maxT = m->maxT;
    const float attn_scale = 1.0f / sqrtf((float)hs);
    /* encoder_forward_kv (encoder.cuh:67-85) */
    for (int c = 0; c < C; c++)
        m->encoded[c] = rx(m, m->wte_emb[(size_t)token * C + c] + m->wpe[(size_t)pos * C + c]);
    /* layer-0 LN1 (inference_gpt2_opt.cu:259) */
    orc_layernorm(m->ln1.data(), nullptr, nullptr, m->encoded.data(), m->ln1w.data(), m->ln1b.data(), 1, C);
    rx_vec(m, m->ln1.data(), C);
    std::vector<float> proj(C), fcproj(C), pre(4 * C), att(C);
    for (int l = 0; l < L; l++) {
        float* ln1 = m->ln1.data() + (size_t)l * C;
        float* qkv = m->qkv.data() + (size_t)l * 3 * C;
        float* atty = m->atty.data() + (size_t)l * C;
        float* res2 = m->residual2.data() + (size_t)l * C;
        float* ln2 = m->ln2.data() + (size_t)l * C;
        float* fch = m->fch.data() + (size_t)l * 4 * C;
        float* fchg = m->fch_gelu.data() + (size_t)l * 4 * C;
        float* res3 = m->residual3.data() + (size_t)l * C;
        const float* residual = (l == 0) ? m->encoded.data() : m->residual3.data() + (size_t)(l - 1) * C;

        /* QKV (inference_gpt2_opt.cu:290-296) */
        linear(m, qkv, nullptr, m->qkvw_f, m->qkvw_8, m->qkvw_s, (size_t)l * 3 * C * C, (size_t)l * 3 * C,
               ln1, m->qkvb.data() + (size_t)l * 3 * C, 3 * C, C, 0);
        rx_vec(m, qkv, 3 * C);

        /* KV append at pos (attention_kvcache.cuh:46-64 / _w8.cuh:115-155) and
         * attention over [0, pos] (fused_single / split+merge give the same math). */
        const size_t layer_kv = (size_t)l * 2 * NH * maxT * hs;
        const size_t layer_sc = (size_t)l * 2 * NH * maxT;
        if (m->kvmode == ORC_KV_8BIT) {
            for (int h = 0; h < NH; h++) {
                const size_t row = (size_t)h * maxT + pos;
                orc_kv_encode_row(qkv + C + h * hs, hs, m->fmt, m->kv_8.data() + layer_kv + row * hs,
                                  m->kv_s.data() + layer_sc + row);
                orc_kv_encode_row(qkv + 2 * C + h * hs, hs, m->fmt,
                                  m->kv_8.data() + layer_kv + (size_t)NH * maxT * hs + row * hs,
                                  m->kv_s.data() + layer_sc + (size_t)NH * maxT + row);
            }
            orc_attention_kv_w8(att.data(), qkv, m->kv_8.data() + layer_kv, m->kv_s.data() + layer_sc, m->fmt,
                                1, pos + 1, NH, hs, maxT, attn_scale);
        } else {
            for (int h = 0; h < NH; h++) {
                const size_t row = (size_t)h * maxT + pos;
                memcpy(m->kv_f.data() + layer_kv + row * hs, qkv + C + h * hs, hs * sizeof(float));
                memcpy(m->kv_f.data() + layer_kv + (size_t)NH * maxT * hs + row * hs, qkv + 2 * C + h * hs,
                       hs * sizeof(float));
            }
            orc_attention_kv(att.data(), qkv, m->kv_f.data() + layer_kv, 1, pos + 1, NH, hs, maxT, attn_scale);
        }
        for (int c = 0; c < C; c++) atty[c] = rx(m, att[c]);

        /* attention projection + residual + LN2 (inference_gpt2_opt.cu:349-358) */
        linear(m, proj.data(), nullptr, m->attprojw_f, m->attprojw_8, m->attprojw_s, (size_t)l * C * C,
               (size_t)l * C, atty, m->attprojb.data() + (size_t)l * C, C, C, 0);
        rx_vec(m, proj.data(), C);
        for (int c = 0; c < C; c++) res2[c] = rx(m, residual[c] + proj[c]);
        orc_layernorm(ln2, nullptr, nullptr, res2, m->ln2w.data() + (size_t)l * C, m->ln2b.data() + (size_t)l * C,
                      1, C);
        rx_vec(m, ln2, C);

        /* MLP (inference_gpt2_opt.cu:360-374): pre-GELU and GELU are both taken
         * from the float pre-activation, then stored as floatX. */
        linear(m, fchg, pre.data(), m->fcw_f, m->fcw_8, m->fcw_s, (size_t)l * 4 * C * C, (size_t)l * 4 * C, ln2,
               m->fcb.data() + (size_t)l * 4 * C, 4 * C, C, 1);
        for (int i = 0; i < 4 * C; i++) { fch[i] = rx(m, pre[i]); fchg[i] = rx(m, fchg[i]); }
        linear(m, fcproj.data(), nullptr, m->fcprojw_f, m->fcprojw_8, m->fcprojw_s, (size_t)l * C * 4 * C,
               (size_t)l * C, fchg, m->fcprojb.data() + (size_t)l * C, C, 4 * C, 0);
        rx_vec(m, fcproj.data(), C);
        for (int c = 0; c < C; c++) res3[c] = rx(m, res2[c] + fcproj[c]);
        /* next LN1, or the final LN (inference_gpt2_opt.cu:376-388) */
        if (l + 1 < L) {
            orc_layernorm(m->ln1.data() + (size_t)(l + 1) * C, nullptr, nullptr, res3,
                          m->ln1w.data() + (size_t)(l + 1) * C, m->ln1b.data() + (size_t)(l + 1) * C, 1, C);
            rx_vec(m, m->ln1.data() + (size_t)(l + 1) * C, C);
        } else {
            orc_layernorm(m->lnf.data(), nullptr, nullptr, res3, m->lnfw.data(), m->lnfb.data(), 1, C);
            rx_vec(m, m->lnf.data(), C);
        }
    }
    /* LM head over the tied embedding, float logits (inference_gpt2_opt.cu:391-399) */
    float* out = logits ? logits : m->tmp.data();
    if (m->wmode == ORC_W_INT8 || m->wmode == ORC_W_FP8)
        orc_gemv_w8(out, nullptr, m->wte_8.data(), m->fmt, m->lnf.data(), m->wte_s.data(), nullptr, m->Vp, C, 0);
    else
        orc_gemv(out, m->wte_f.data(), m->lnf.data(), m->Vp, C);
    return 0;
}

extern "C" int orc_model_generate(orc_model* m, const int* prompt, int n_prompt, int n_gen,
                                  int* out_tokens, float* logits_out) {
    if (n_prompt < 1 || n_gen < 0 || n_prompt + n_gen > m->maxT) return 1;
    std::vector<float> logits(m->Vp);
    int tok = prompt[0];
    int produced = 0;
    for (int pos = 0; pos < n_prompt + n_gen; pos++) {
        float* lg = logits_out ? logits_out + (size_t)pos * m->Vp : logits.data();
        int rc = orc_model_step(m, tok, pos, lg);
        if (rc) return rc;
        if (pos + 1 < n_prompt) {
            tok = prompt[pos + 1];
        } else {
            tok = orc_argmax(lg, m->V); /* the pick reads only the real vocabulary */
            out_tokens[produced++] = tok;
        }
    }
    return 0;
}

extern "C" int orc_model_probe(const orc_model* m, const char* name, int layer, float* out) {
    const int C = m->C;
    struct { const char* n; const std::vector<float>* v; int w; bool per_layer; } tab[] = {
        {"encoded", &m->encoded, C, false},     {"ln1", &m->ln1, C, true},
        {"qkv", &m->qkv, 3 * C, true},          {"atty", &m->atty, C, true},
        {"residual2", &m->residual2, C, true},  {"ln2", &m->ln2, C, true},
        {"fch", &m->fch, 4 * C, true},          {"fch_gelu", &m->fch_gelu, 4 * C, true},
        {"residual3", &m->residual3, C, true},  {"lnf", &m->lnf, C, false},
    };
    for (auto& t : tab) {
        if (strcmp(t.n, name) != 0) continue;
        size_t off = t.per_layer ? (size_t)layer * t.w : 0;
        if (t.per_layer && (layer < 0 || layer >= m->L)) return -1;
        memcpy(out, t.v->data() + off, t.w * sizeof(float));
        return t.w;
    }
    return -1;
}
