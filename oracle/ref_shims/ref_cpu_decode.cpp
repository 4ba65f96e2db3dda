/* The reference's CPU decode path: the reference ships no whole-model CPU
 * decoder, so this file composes the reference's own CPU loops (compiled from
 * source into the sibling shim libraries) in the kernel order of
 * forward_kv_graph_ready (inference_gpt2_opt.cu:235-400), FP32 throughout.
 * Linear layers use GEMV_cpu (gemv/GEMV.cu:84-93, OpenMP over rows) plus the
 * bias add of GEMV.cuh:192; matmul_forward_cpu parallelises only over B*T and
 * would run on one thread at batch 1.
 * TEST INFRASTRUCTURE: bench.py's reference arm and cpu_baseline leg time it. */
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

extern "C" {
void ref_gemv_cpu_f32(float* out, const float* W, const float* x, int M, int K);
void ref_attention_kv_cpu(float* out, const float* qkv, const float* kv_cache, int B, int seq_len, int NH,
                          int hs, int maxT, float scale);
void ref_residual_cpu(float* out, const float* a, const float* b, int N);
void ref_layernorm_cpu(float* out, float* mean, float* rstd, const float* inp, const float* weight,
                       const float* bias, int B, int T, int C);
void ref_gelu_cpu(float* out, const float* inp, int N);
void ref_encoder_cpu(float* out, const int* inp, const float* wte, const float* wpe, int B, int T, int C);
}

#define REFAPI extern "C" __attribute__((visibility("default")))

struct RefDecoder {
    int maxT, V, L, NH, C, Vp, hs;
    const float* p[16]; /* gpt2_model.h:41-58 order */
    std::vector<float> kv, enc, ln, qkv, atty, proj, res2, res3, fch, fchg, fcproj, logits, mean, rstd;
};

/* params: the 16 FP32 tensors back to back, as after a v3 header. */
REFAPI void* ref_decoder_create(const int* cfg6, const float* params) {
    RefDecoder* d = new RefDecoder();
    d->maxT = cfg6[0]; d->V = cfg6[1]; d->L = cfg6[2]; d->NH = cfg6[3]; d->C = cfg6[4]; d->Vp = cfg6[5];
    d->hs = d->C / d->NH;
    const size_t C = d->C, L = d->L, Vp = d->Vp, maxT = d->maxT;
    const size_t sz[16] = {Vp * C, maxT * C, L * C, L * C, L * 3 * C * C, L * 3 * C, L * C * C, L * C,
                           L * C, L * C, L * 4 * C * C, L * 4 * C, L * C * 4 * C, L * C, C, C};
    const float* it = params;
    for (int i = 0; i < 16; i++) { d->p[i] = it; it += sz[i]; }
    d->kv.assign(L * 2 * (size_t)d->NH * maxT * d->hs, 0.0f);
    d->enc.resize(C); d->ln.resize(C); d->qkv.resize(3 * C); d->atty.resize(C); d->proj.resize(C);
    d->res2.resize(C); d->res3.resize(C); d->fch.resize(4 * C); d->fchg.resize(4 * C); d->fcproj.resize(C);
    d->logits.resize(Vp); d->mean.resize(1); d->rstd.resize(1);
    return d;
}

REFAPI void ref_decoder_free(void* h) { delete (RefDecoder*)h; }

/* OpenMP threads of the GEMV loops (a launcher may have set OMP_NUM_THREADS=1
 * for its ranks); returns the count now in effect. */
REFAPI int ref_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}

static void linear(RefDecoder* d, float* out, const float* W, const float* b, const float* x, int M, int K) {
    ref_gemv_cpu_f32(out, W, x, M, K);
    for (int m = 0; m < M; m++) out[m] += b[m];
}

/* One forward; returns the greedy pick over the real vocabulary. */
REFAPI int ref_decoder_step(void* h, int token, int pos, float* logits_out) {
    RefDecoder* d = (RefDecoder*)h;
    const int C = d->C, NH = d->NH, hs = d->hs, maxT = d->maxT;
    const float *wte = d->p[0], *wpe = d->p[1], *ln1w = d->p[2], *ln1b = d->p[3], *qkvw = d->p[4],
                *qkvb = d->p[5], *apw = d->p[6], *apb = d->p[7], *ln2w = d->p[8], *ln2b = d->p[9],
                *fcw = d->p[10], *fcb = d->p[11], *fpw = d->p[12], *fpb = d->p[13], *lnfw = d->p[14],
                *lnfb = d->p[15];
    ref_encoder_cpu(d->enc.data(), &token, wte, wpe + (size_t)pos * C, 1, 1, C);
    ref_layernorm_cpu(d->ln.data(), d->mean.data(), d->rstd.data(), d->enc.data(), ln1w, ln1b, 1, 1, C);
    const float* residual = d->enc.data();
    for (int l = 0; l < d->L; l++) {
        linear(d, d->qkv.data(), qkvw + (size_t)l * 3 * C * C, qkvb + (size_t)l * 3 * C, d->ln.data(), 3 * C, C);
        float* kvl = d->kv.data() + (size_t)l * 2 * NH * maxT * hs;
        for (int h = 0; h < NH; h++) {
            memcpy(kvl + ((size_t)h * maxT + pos) * hs, d->qkv.data() + C + h * hs, hs * sizeof(float));
            memcpy(kvl + (size_t)NH * maxT * hs + ((size_t)h * maxT + pos) * hs, d->qkv.data() + 2 * C + h * hs,
                   hs * sizeof(float));
        }
        ref_attention_kv_cpu(d->atty.data(), d->qkv.data(), kvl, 1, pos + 1, NH, hs, maxT, 1.f / sqrtf((float)hs));
        linear(d, d->proj.data(), apw + (size_t)l * C * C, apb + (size_t)l * C, d->atty.data(), C, C);
        ref_residual_cpu(d->res2.data(), residual, d->proj.data(), C);
        ref_layernorm_cpu(d->ln.data(), d->mean.data(), d->rstd.data(), d->res2.data(), ln2w + (size_t)l * C,
                          ln2b + (size_t)l * C, 1, 1, C);
        linear(d, d->fch.data(), fcw + (size_t)l * 4 * C * C, fcb + (size_t)l * 4 * C, d->ln.data(), 4 * C, C);
        ref_gelu_cpu(d->fchg.data(), d->fch.data(), 4 * C);
        linear(d, d->fcproj.data(), fpw + (size_t)l * C * 4 * C, fpb + (size_t)l * C, d->fchg.data(), C, 4 * C);
        ref_residual_cpu(d->res3.data(), d->res2.data(), d->fcproj.data(), C);
        if (l + 1 < d->L)
            ref_layernorm_cpu(d->ln.data(), d->mean.data(), d->rstd.data(), d->res3.data(),
                              ln1w + (size_t)(l + 1) * C, ln1b + (size_t)(l + 1) * C, 1, 1, C);
        else
            ref_layernorm_cpu(d->ln.data(), d->mean.data(), d->rstd.data(), d->res3.data(), lnfw, lnfb, 1, 1, C);
        std::swap(d->enc, d->res3); /* the next layer's residual input */
        residual = d->enc.data();
    }
    ref_gemv_cpu_f32(d->logits.data(), wte, d->ln.data(), d->Vp, C);
    if (logits_out) memcpy(logits_out, d->logits.data(), (size_t)d->Vp * sizeof(float));
    int best = 0;
    for (int i = 1; i < d->V; i++)
        if (d->logits[i] > d->logits[best]) best = i;
    return best;
}
