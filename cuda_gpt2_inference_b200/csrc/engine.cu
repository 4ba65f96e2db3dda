// engine.cu -- whole-model batch-1 decode engine (host C++).
//
// Replaces the reference's forward_kv_graph_ready / graph_capture_all /
// run_generation_once_graph (inference_gpt2_opt.cu:235-596) and its loaders
// (gpt2_build_from_checkpoint, gpt2_model.h:268-303; gpt2_build_w8,
// inference_gpt2_opt.cu:143-219).
//
// One decode step is 5 kernels per layer + 1 (the reference launches 8-9 per
// layer + 3):
//   QKV GEMV   prologue: residual add + LN1 (layer 0: embedding + LN1)
//   attention  KV append + flash-decoding + merge, one launch
//   proj GEMV  + bias
//   FC GEMV    prologue: residual add + LN2; epilogue: bias, GELU, pre-GELU
//   FCproj     + bias
//   LM head    prologue: residual add + final LN; epilogue: logits, greedy
//              pick, next token / position written on the device
// Kernels are chained with programmatic dependent launch (each stages its
// weights before waiting on the previous kernel) and several steps are
// captured into one CUDA graph; because token and position live in device
// memory and are advanced by the LM head, a graph replays any number of
// steps with no host round trip.
//
// Memory layout in HBM: one parameter arena with the 16 tensors of
// gpt2_model.h:41-58 in file order (8-bit modes keep the 5 Linear groups as
// 1-byte codes in their slots, followed by the 5 per-row scale arrays); one
// activation arena; one KV arena [layer][K|V][head][maxT][hs] (+ scales).
#include "common.cuh"
#include "internal.h"

#if GPT2B_HAVE_NCCL
#include <nccl.h>
#endif

#include <math.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>

#include <algorithm>
#include <string>
#include <vector>

using namespace gpt2b;

struct gpt2b_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    gpt2b_config cfg{};
    int wmode = 0, kvmode = 0, wk = 0, kvk = 0;
    bool w8 = false;
    size_t xbytes = 2;  // activation element size
    // arenas
    unsigned char* params = nullptr;
    unsigned char* acts = nullptr;
    unsigned char* kv = nullptr;
    size_t params_bytes = 0, acts_bytes = 0, kv_bytes = 0;
    // parameter pointers (file order)
    unsigned char* p[16] = {};
    float* sc[5] = {};  // wte, qkvw, attprojw, fcw, fcprojw row scales
    // activations
    unsigned char *encoded, *ln1, *qkv, *atty, *res2, *ln2, *fch, *fch_gelu, *res3, *lnf, *proj_out, *fcproj_out;
    float* logits;
    float *part_out, *part_max, *part_lse;
    float* lm_val;
    int* lm_idx;
    unsigned* lm_counter;
    int *d_token, *d_pos, *d_history, *d_prompt, *d_nprompt;
    // kv cache
    unsigned char* kv_cache = nullptr;
    float* kv_scale = nullptr;
    size_t kv_layer_elems = 0, kv_layer_scales = 0;
    // plans
    std::vector<GemvParams> qkv_p, proj_p, fc_p, fcproj_p;
    GemvParams lm_p;
    int splits = 1;
    bool use_graph = true, use_pdl = true;
    int steps_per_graph = 8;
    cudaGraphExec_t graph_multi = nullptr, graph_one = nullptr;
    bool graphs_valid = false;
    // persistent decode kernel (persistent.cu): its exchange arena and params
    bool persist_ok = false, use_persistent = false;
    unsigned char* xchg = nullptr;
    size_t xchg_bytes = 0;
    PersistParams pp;
    // tensor parallelism (tp_size 1: single GPU): this rank's heads, FC rows and vocab rows
    int tp_rank = 0, tp_size = 1;
    int h0 = 0, nh_l = 0, f0 = 0, f_l = 0, v0 = 0, v_rows = 0;
    float* proj_f32 = nullptr;     // row-parallel partial sums (C floats), all-reduced in place
    float* fcproj_f32 = nullptr;
    float* lm_pair = nullptr;      // (best logit, global index) of this rank's vocab rows
    float* lm_pairs = nullptr;     // every rank's pair
    float* logits_full = nullptr;  // all-gathered logits (Vp) for host copies and sampling
    bool tp_connected = false;     // peers' exchange arenas mapped (persistent kernel usable)
    // prompt prefill on the tensor cores (prefill.cu): set up at the first prompt
    bool prefill_ok = false, use_prefill = false, prefill_ready = false;
    unsigned char* pf_mem = nullptr;  // activation rows [maxT] x (C | C | 3C | C | C | 4C), then maxT x Vp logits
    PrefillPlan pf;
    unsigned char* peer_map[8] = {};  // IPC mappings of the other ranks' arenas
#if GPT2B_HAVE_NCCL
    ncclComm_t comm = nullptr;
#endif
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Element counts of the 16 parameter tensors (gpt2_model.h:63-87).
void param_sizes(const gpt2b_config& c, size_t n[16]) {
    const size_t C = c.channels, L = c.num_layers, Vp = c.padded_vocab_size, maxT = c.max_seq_len;
    const size_t v[16] = {Vp * C, maxT * C, L * C, L * C, L * 3 * C * C, L * 3 * C, L * C * C, L * C,
                          L * C, L * C, L * 4 * C * C, L * 4 * C, L * C * 4 * C, L * C, C, C};
    for (int i = 0; i < 16; i++) n[i] = v[i];
}
// tensors stored as 8-bit codes in the mixed file (quantize.cu:190-196)
const int kLinearSlot[16] = {0, -1, -1, -1, 1, -1, 2, -1, -1, -1, 3, -1, 4, -1, -1, -1};

// Tensor-parallel shard of one rank (the Megatron column/row split, for decode):
// QKV and FC column-parallel (heads, FC rows), attention projection and FC
// projection row-parallel (their K slices), LM head vocab-parallel.  25 heads
// split unevenly (13/12, 7/6/6/6, 4/3x7); FC rows and vocab rows evenly.
struct TpPlan {
    int h0, nh_l, f0, f_l, v0, v_rows;
};
bool tp_plan(const gpt2b_config& c, int rank, int size, TpPlan* pl) {
    const int NH = c.num_heads, F = 4 * c.channels, Vp = c.padded_vocab_size;
    if (size < 1 || rank < 0 || rank >= size || size > NH) return false;
    if (size > 1 && (F % (16 * size) != 0 || Vp % size != 0)) return false;
    const int q = NH / size, r = NH % size;
    pl->nh_l = q + (rank < r ? 1 : 0);
    pl->h0 = rank * q + (rank < r ? rank : r);
    pl->f_l = F / size;
    pl->f0 = rank * pl->f_l;
    pl->v_rows = Vp / size;
    pl->v0 = rank * pl->v_rows;
    return true;
}

// Element counts of this rank's 16 parameter tensors and 5 scale arrays.
void local_sizes(const gpt2b_config& c, const TpPlan& pl, size_t n[16], size_t ns[5]) {
    const size_t C = c.channels, L = c.num_layers, Vp = c.padded_vocab_size, maxT = c.max_seq_len;
    const size_t Q = 3 * (size_t)pl.nh_l * 64, A = (size_t)pl.nh_l * 64, F = pl.f_l;
    const size_t v[16] = {Vp * C, maxT * C, L * C, L * C, L * Q * C, L * Q, L * C * A, L * C,
                          L * C, L * C, L * F * C, L * F, L * C * F, L * C, C, C};
    for (int i = 0; i < 16; i++) n[i] = v[i];
    const size_t w[5] = {Vp, L * Q, L * C, L * F, L * C};
    for (int g = 0; g < 5; g++) ns[g] = w[g];
}

// Copies this rank's slices of the full (file-order) tensors into `out`
// (local tensors in file order, element sizes as stored) and of the scale
// groups into `out_sc`.  Row-parallel biases are kept by rank 0 only (the
// other ranks hold zeros) so the all-reduced sum carries them once.
void tp_shard(const unsigned char* image, const float* scales, const gpt2b_config& c, bool w8, size_t xb,
              const TpPlan& pl, int rank, std::vector<unsigned char>& out, std::vector<float>& out_sc) {
    const size_t C = c.channels, L = c.num_layers, NH64 = (size_t)c.num_heads * 64, F4 = 4 * C;
    size_t nf[16], nl[16], nsl[5];
    param_sizes(c, nf);
    local_sizes(c, pl, nl, nsl);
    size_t total = 0;
    for (int i = 0; i < 16; i++) total += nl[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb);
    out.assign(total, 0);
    const unsigned char* src = image + 1024;
    unsigned char* dst = out.data();
    const size_t h0 = (size_t)pl.h0 * 64, hl = (size_t)pl.nh_l * 64, f0 = pl.f0, fl = pl.f_l;
    for (int i = 0; i < 16; i++) {
        const size_t eb = (w8 && kLinearSlot[i] >= 0) ? 1 : xb;
        auto rows = [&](size_t nrow_full, size_t r0, size_t nr, size_t row_elems) {  // [L][nrow_full][row]
            for (size_t l = 0; l < L; l++) {
                memcpy(dst, src + (l * nrow_full + r0) * row_elems * eb, nr * row_elems * eb);
                dst += nr * row_elems * eb;
            }
        };
        auto cols = [&](size_t nrow, size_t ncol_full, size_t k0, size_t nk) {  // [L][nrow][ncol_full]
            for (size_t l = 0; l < L; l++)
                for (size_t r = 0; r < nrow; r++) {
                    memcpy(dst, src + ((l * nrow + r) * ncol_full + k0) * eb, nk * eb);
                    dst += nk * eb;
                }
        };
        switch (i) {
            case 4:  // qkvw [L][3C][C]: q, k, v rows of this rank's heads
            case 5:  // qkvb [L][3C]
                for (size_t l = 0; l < L; l++)
                    for (size_t part = 0; part < 3; part++) {
                        const size_t re = (i == 4) ? C : 1;
                        memcpy(dst, src + ((l * 3 + part) * NH64 + h0) * re * eb, hl * re * eb);
                        dst += hl * re * eb;
                    }
                break;
            case 6: cols(C, C, h0, hl); break;               // attprojw [L][C][C]: K slice of the heads
            case 10: rows(F4, f0, fl, C); break;             // fcw [L][4C][C]: FC rows
            case 11: rows(F4, f0, fl, 1); break;             // fcb [L][4C]
            case 12: cols(C, F4, f0, fl); break;             // fcprojw [L][C][4C]: K slice
            case 7:                                          // attprojb, fcprojb: rank 0 only
            case 13:
                if (rank == 0) memcpy(dst, src, nf[i] * eb);
                dst += nf[i] * eb;
                break;
            default: memcpy(dst, src, nf[i] * eb); dst += nf[i] * eb; break;
        }
        src += nf[i] * eb;
    }
    out_sc.clear();
    if (!w8) return;
    size_t nsf[5] = {(size_t)c.padded_vocab_size, L * 3 * C, L * C, L * F4, L * C};
    const float* s = scales;
    for (int g = 0; g < 5; g++) {
        if (g == 1) {
            for (size_t l = 0; l < L; l++)
                for (size_t part = 0; part < 3; part++)
                    out_sc.insert(out_sc.end(), s + (l * 3 + part) * NH64 + h0, s + (l * 3 + part) * NH64 + h0 + hl);
        } else if (g == 3) {
            for (size_t l = 0; l < L; l++) out_sc.insert(out_sc.end(), s + l * F4 + f0, s + l * F4 + f0 + fl);
        } else {
            out_sc.insert(out_sc.end(), s, s + nsf[g]);
        }
        s += nsf[g];
    }
}

int check_header(const int* hdr, int wmode, gpt2b_config* cfg) {
    if (hdr[0] != 20251103) return GPT2B_ERR_FORMAT;
    const int want = (wmode == GPT2B_W_F32) ? 3 : 5;
    if (hdr[1] != want) return GPT2B_ERR_FORMAT;
    cfg->max_seq_len = hdr[2];
    cfg->vocab_size = hdr[3];
    cfg->num_layers = hdr[4];
    cfg->num_heads = hdr[5];
    cfg->channels = hdr[6];
    cfg->padded_vocab_size = hdr[7];
    if (cfg->max_seq_len <= 0 || cfg->vocab_size <= 0 || cfg->num_layers <= 0 || cfg->num_heads <= 0 ||
        cfg->channels <= 0 || cfg->padded_vocab_size < cfg->vocab_size || cfg->channels % cfg->num_heads != 0)
        return GPT2B_ERR_FORMAT;
    return GPT2B_OK;
}

void free_engine(gpt2b_engine* e) {
    if (!e) return;
    DeviceGuard g(e->device);
    if (e->graph_multi) cudaGraphExecDestroy(e->graph_multi);  // graphs holding collectives go first
    if (e->graph_one) cudaGraphExecDestroy(e->graph_one);
#if GPT2B_HAVE_NCCL
    if (e->comm) ncclCommDestroy(e->comm);
#endif
    for (int r = 0; r < 8; r++)
        if (e->peer_map[r]) cudaIpcCloseMemHandle(e->peer_map[r]);
    if (e->params) cudaFree(e->params);
    if (e->acts) cudaFree(e->acts);
    if (e->kv) cudaFree(e->kv);
    if (e->xchg) cudaFree(e->xchg);
    if (e->pf_mem) cudaFree(e->pf_mem);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

// Picks the next token from every tensor-parallel rank's (best logit, global
// index) pair -- first maximum, lowest index on ties, the order the
// single-GPU LM head uses -- and advances token, position and history.
__global__ void tp_pick_kernel(const float* pairs, int n, const int* prompt, int n_prompt, int* token, int* pos,
                               int* history) {
    float bv = pairs[0];
    int bi = __float_as_int(pairs[1]);
    for (int r = 1; r < n; r++) {
        const float v = pairs[2 * r];
        const int i = __float_as_int(pairs[2 * r + 1]);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    const int p = *pos;
    const int next = (p + 1 < n_prompt) ? prompt[p + 1] : bi;
    history[p + 1] = next;
    *token = next;
    *pos = p + 1;
}

// Sum of this rank's FP32 partials over the tensor-parallel group, in place.
cudaError_t tp_allreduce(gpt2b_engine* e, float* buf, size_t n) {
#if GPT2B_HAVE_NCCL
    return ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, e->comm, e->stream) == ncclSuccess ? cudaSuccess
                                                                                           : cudaErrorUnknown;
#else
    (void)e; (void)buf; (void)n;
    return cudaErrorNotSupported;
#endif
}
cudaError_t tp_allgather(gpt2b_engine* e, const float* send, float* recv, size_t n) {
#if GPT2B_HAVE_NCCL
    return ncclAllGather(send, recv, n, ncclFloat, e->comm, e->stream) == ncclSuccess ? cudaSuccess
                                                                                    : cudaErrorUnknown;
#else
    (void)e; (void)send; (void)recv; (void)n;
    return cudaErrorNotSupported;
#endif
}

// Launches one decode step (5L + 1 kernels; with tensor parallelism also 2L
// all-reduces, the pair all-gather and the pick) on e->stream.
cudaError_t launch_step(gpt2b_engine* e) {
    const int L = e->cfg.num_layers, C = e->cfg.channels;
    const bool tp = e->tp_size > 1;
    const bool pdl = e->use_pdl;
    cudaError_t err;
    for (int l = 0; l < L; l++) {
        err = launch_gemv(e->qkv_p[l], e->wk, false, l == 0 ? PRO_EMB_LN : PRO_RES_LN, EPI_STORE, e->stream,
                          pdl && !(tp && l > 0));
        if (err != cudaSuccess) return err;
        unsigned char* kv_l = e->kv_cache + (size_t)l * e->kv_layer_elems * (e->kvk >= KV_I8 ? 1 : e->xbytes);
        float* ks_l = e->kv_scale ? e->kv_scale + (size_t)l * e->kv_layer_scales : nullptr;
        err = launch_attention_engine(e->kvk, e->qkv, kv_l, ks_l, e->d_pos, e->nh_l, e->cfg.max_seq_len,
                                      e->splits, e->part_out, e->part_max, e->part_lse, e->stream, pdl);
        if (err != cudaSuccess) return err;
        err = launch_gemv(e->proj_p[l], e->wk, tp, PRO_ATTN_MERGE, EPI_STORE, e->stream, pdl);
        if (err != cudaSuccess) return err;
        if (tp && (err = tp_allreduce(e, e->proj_f32, C)) != cudaSuccess) return err;
        err = launch_gemv(e->fc_p[l], e->wk, false, PRO_RES_LN, EPI_STORE, e->stream, pdl && !tp);
        if (err != cudaSuccess) return err;
        err = launch_gemv(e->fcproj_p[l], e->wk, tp, PRO_PLAIN, EPI_STORE, e->stream, pdl);
        if (err != cudaSuccess) return err;
        if (tp && (err = tp_allreduce(e, e->fcproj_f32, C)) != cudaSuccess) return err;
    }
    err = launch_gemv(e->lm_p, e->wk, true, PRO_RES_LN, EPI_LMHEAD, e->stream, pdl && !tp);
    if (err != cudaSuccess || !tp) return err;
    if ((err = tp_allgather(e, e->lm_pair, e->lm_pairs, 2)) != cudaSuccess) return err;
    return launch_k(tp_pick_kernel, dim3(1), dim3(1), 0, e->stream, false, (const float*)e->lm_pairs, e->tp_size,
                    (const int*)e->d_prompt, e->lm_p.n_prompt, e->d_token, e->d_pos, e->d_history);
}

cudaError_t capture(gpt2b_engine* e, int steps, cudaGraphExec_t* out) {
    cudaGraph_t g;
    cudaError_t err = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return err;
    for (int s = 0; s < steps && err == cudaSuccess; s++) err = launch_step(e);
    cudaError_t end = cudaStreamEndCapture(e->stream, &g);
    if (err != cudaSuccess) { if (end == cudaSuccess) cudaGraphDestroy(g); return err; }
    if (end != cudaSuccess) return end;
    err = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return err;
}

cudaError_t ensure_graphs(gpt2b_engine* e) {
    if (e->graphs_valid) return cudaSuccess;
    if (e->graph_multi) { cudaGraphExecDestroy(e->graph_multi); e->graph_multi = nullptr; }
    if (e->graph_one) { cudaGraphExecDestroy(e->graph_one); e->graph_one = nullptr; }
    cudaError_t err = capture(e, 1, &e->graph_one);
    if (err == cudaSuccess && e->steps_per_graph > 1) err = capture(e, e->steps_per_graph, &e->graph_multi);
    if (err == cudaSuccess) e->graphs_valid = true;
    return err;
}

// The prefill plan: activation rows for maxT prompt tokens, the logits of
// every prompt row, and the tensor maps of every GEMM operand (weights of
// every layer, activations over maxT rows), built once at the first prompt.
cudaError_t ensure_prefill(gpt2b_engine* e) {
    if (e->prefill_ready) return cudaSuccess;
    const gpt2b_config& c = e->cfg;
    const size_t C = c.channels, L = c.num_layers, maxT = c.max_seq_len, Vp = c.padded_vocab_size;
    const size_t wb = (size_t)wkind_bytes(e->wk), xb = e->xbytes;
    const size_t widths[6] = {C, C, 3 * C, C, C, 4 * C};  // res, x, qkv, atty, proj, f
    size_t off[7], total = 0;
    for (int i = 0; i < 6; i++) { off[i] = total; total += align256(maxT * widths[i] * 2); }
    off[6] = total;
    total += align256(maxT * Vp * 4);
    cudaError_t err = cudaMalloc(&e->pf_mem, total);
    if (err != cudaSuccess) return err;
    if ((err = cudaMemset(e->pf_mem, 0, total)) != cudaSuccess) return err;
    PrefillPlan& P = e->pf;
    P.wk = e->wk; P.kvk = e->kvk; P.C = (int)C; P.NH = c.num_heads; P.L = (int)L; P.V = c.vocab_size;
    P.Vp = (int)Vp; P.maxT = (int)maxT;
    P.attn_scale = 1.0f / sqrtf((float)(C / c.num_heads));
    P.res = e->pf_mem + off[0]; P.x = e->pf_mem + off[1]; P.qkv = e->pf_mem + off[2];
    P.atty = e->pf_mem + off[3]; P.proj = e->pf_mem + off[4]; P.f = e->pf_mem + off[5];
    P.logits_rows = reinterpret_cast<float*>(e->pf_mem + off[6]);
    P.tokens = e->d_prompt;
    P.wte = e->p[0]; P.wte_scale = e->w8 ? e->sc[0] : nullptr; P.wpe = e->p[1];
    P.lnfw = e->p[14]; P.lnfb = e->p[15];
    P.logits_last = e->logits; P.d_token = e->d_token; P.d_pos = e->d_pos; P.history = e->d_history;
    const int iC = (int)C, iM = (int)maxT;
    bool ok = tc_maps(&P.a_x, nullptr, e->wk, P.x, iM, nullptr, 0, iC, false) &&
              tc_maps(&P.a_atty, nullptr, e->wk, P.atty, iM, nullptr, 0, iC, false) &&
              tc_maps(&P.a_f, nullptr, e->wk, P.f, iM, nullptr, 0, 4 * iC, false) &&
              tc_maps(nullptr, &P.w_lm, e->wk, nullptr, 0, e->p[0], (int)Vp, iC, true);
    P.s_lm = e->w8 ? e->sc[0] : nullptr;
    P.layers.assign(L, PrefillLayer());
    const size_t kvb = (e->kvk >= KV_I8) ? 1 : xb;
    for (size_t l = 0; l < L && ok; l++) {
        PrefillLayer& Y = P.layers[l];
        ok = tc_maps(nullptr, &Y.w_qkv, e->wk, nullptr, 0, e->p[4] + l * 3 * C * C * wb, 3 * iC, iC, false) &&
             tc_maps(nullptr, &Y.w_proj, e->wk, nullptr, 0, e->p[6] + l * C * C * wb, iC, iC, false) &&
             tc_maps(nullptr, &Y.w_fc, e->wk, nullptr, 0, e->p[10] + l * 4 * C * C * wb, 4 * iC, iC, false) &&
             tc_maps(nullptr, &Y.w_fcproj, e->wk, nullptr, 0, e->p[12] + l * 4 * C * C * wb, iC, 4 * iC, false);
        Y.qkvb = e->p[5] + l * 3 * C * xb; Y.projb = e->p[7] + l * C * xb;
        Y.fcb = e->p[11] + l * 4 * C * xb; Y.fcprojb = e->p[13] + l * C * xb;
        if (e->w8) {
            Y.s_qkv = e->sc[1] + l * 3 * C; Y.s_proj = e->sc[2] + l * C;
            Y.s_fc = e->sc[3] + l * 4 * C; Y.s_fcproj = e->sc[4] + l * C;
        }
        Y.ln1w = e->p[2] + l * C * xb; Y.ln1b = e->p[3] + l * C * xb;
        Y.ln2w = e->p[8] + l * C * xb; Y.ln2b = e->p[9] + l * C * xb;
        Y.kv = e->kv_cache + l * e->kv_layer_elems * kvb;
        Y.kv_scale = e->kv_scale ? e->kv_scale + l * e->kv_layer_scales : nullptr;
    }
    if (!ok) return cudaErrorNotSupported;
    e->prefill_ready = true;
    return cudaSuccess;
}

// n forwards from the device-resident token/position.
cudaError_t run_steps(gpt2b_engine* e, int n) {
    if (e->use_persistent) {
        if (n <= 0) return cudaSuccess;
        cudaError_t err = cudaMemsetAsync(e->pp.abort_flag, 0, sizeof(int), e->stream);
        if (err != cudaSuccess) return err;
        PersistParams p = e->pp;
        p.n_steps = n;
        p.n_prompt = e->lm_p.n_prompt;
        return launch_persistent(e->wk, e->kvk, p, e->stream);
    }
    if (!e->use_graph) {
        for (int i = 0; i < n; i++) {
            cudaError_t err = launch_step(e);
            if (err != cudaSuccess) return err;
        }
        return cudaSuccess;
    }
    cudaError_t err = ensure_graphs(e);
    if (err != cudaSuccess) return err;
    int left = n;
    if (e->graph_multi)
        for (; left >= e->steps_per_graph; left -= e->steps_per_graph) {
            err = cudaGraphLaunch(e->graph_multi, e->stream);
            if (err != cudaSuccess) return err;
        }
    for (; left > 0; left--) {
        err = cudaGraphLaunch(e->graph_one, e->stream);
        if (err != cudaSuccess) return err;
    }
    return cudaSuccess;
}

__global__ void set_history_kernel(int* history, const int* d_token, const int* d_pos) {
    history[*d_pos] = *d_token;
}

// Plans the persistent decode kernel when the shape allows it: splits per
// head (as many as fill the SMs, at most 96 positions each), ring stages (as
// many as fit in shared memory, at most kPersistRingBytes of weights), and the zero-initialised exchange
// arena: tagged words per layer and phase, per-(layer, head) KV flags, the
// epoch counter and the abort flag.
cudaError_t setup_persistent(gpt2b_engine* e, int nsm) {
    const gpt2b_config& c = e->cfg;
    const int C = c.channels, L = c.num_layers, maxT = c.max_seq_len, TP = e->tp_size;
    const int NHl = e->nh_l;  // this rank's heads
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, e->device);
    const int S = std::min(nsm / NHl, persist_max_splits());
    if (!coop || TP > 8 || !persist_supported(C, NHl, 64, maxT, S, nsm, L)) return cudaSuccess;
    const int kv_rows = engine_attn_chunk(maxT, S);
    // ring: as many stages as fit in shared memory (the LM head streams through all of
    // them); the layer phases run at most kPersistRingBytes of weights ahead (a deeper
    // look-ahead there only adds traffic while the CTAs wait on exchange words).  The
    // narrow kernels with 8-bit weights keep the ring at that depth: their LM head
    // measured 9-12 % slower per token with 14 stages than with 8 (BF16 narrow, 4 -> 7
    // stages: -0.7 %; GPT-2-XL wide: -2 %)
    int nsw = 0;
    for (int k = persist_max_stages(); k >= 2 && !nsw; k--) {
        const int b = persist_smem_bytes(e->wk, e->kvk, C, k, kv_rows, TP);
        if (b > 0 && b <= max_dyn_smem()) nsw = k;
    }
    if (!nsw) return cudaSuccess;
    const int lookahead = std::max(2, std::min(nsw, kPersistRingBytes / persist_stage_bytes(e->wk, C)));
    if (e->w8 && persist_narrow(C, kv_rows, TP)) nsw = lookahead;
    const int G = nsm;
    const int Q = 3 * NHl * 64, A = NHl * 64, F = e->f_l;
    // exchange arena: the cross-GPU parts first, at offsets every rank shares
    // (abort flag, projection and FC-projection partials [L][TP][C], LM pairs
    // [TP][G] one per kPersistLmStride words), then this rank's own words and flags
    const size_t n_grp = (size_t)L * TP * C, n_lm = (size_t)kPersistLmStride * TP * G;
    const size_t n_qkv = (size_t)L * Q, n_att = (size_t)L * A, n_fc = (size_t)L * F;
    const size_t n_part = (size_t)L * NHl * S * (64 + 2);
    const size_t off_proj = 256, off_fcproj = off_proj + n_grp * 8, off_lm = off_fcproj + n_grp * 8;
    const size_t off_own = align256(off_lm + n_lm * 8);
    const size_t own_words = n_qkv + n_att + n_part + n_fc;
    const size_t off_flags = align256(off_own + own_words * 8);
    const size_t flags = (size_t)L * NHl;
    const size_t off_epoch = align256(off_flags + flags * 4);  // the epoch counter (256 bytes)
    const size_t off_lnexp = off_epoch + 256;                   // LayerNorm exponents (8-bit weights)
    const size_t bytes = align256(off_lnexp + (2 * (size_t)L + 1) * 4);
    cudaError_t err = cudaMalloc(&e->xchg, bytes);
    if (err != cudaSuccess) return err;
    if ((err = cudaMemset(e->xchg, 0, bytes)) != cudaSuccess) return err;
    e->xchg_bytes = bytes;
    PersistParams& p = e->pp;
    p.ln_exp = reinterpret_cast<const int*>(e->xchg + off_lnexp);
    if (e->w8) {  // the tensor-core stages of 8-bit weights scale x by 2^-e before FP16
        err = persist_ln_exponents(reinterpret_cast<int*>(e->xchg + off_lnexp), e->p[2], e->p[3], e->p[8], e->p[9],
                                   e->p[14], e->p[15], L, C, nullptr);
        if (err == cudaSuccess) err = cudaDeviceSynchronize();
        if (err != cudaSuccess) return err;
    }
    p.abort_flag = reinterpret_cast<int*>(e->xchg);
    p.ll_proj = reinterpret_cast<unsigned long long*>(e->xchg + off_proj);
    p.ll_fcproj = reinterpret_cast<unsigned long long*>(e->xchg + off_fcproj);
    p.ll_lm = reinterpret_cast<unsigned long long*>(e->xchg + off_lm);
    p.xoff_abort = 0; p.xoff_proj = off_proj; p.xoff_fcproj = off_fcproj; p.xoff_lm = off_lm;
    unsigned long long* w = reinterpret_cast<unsigned long long*>(e->xchg + off_own);
    p.ll_qkv = w; w += n_qkv;
    p.ll_atty = w; w += n_att;
    p.ll_part = w; w += n_part;
    p.ll_fc = w;
    p.kv_flag = reinterpret_cast<unsigned*>(e->xchg + off_flags);
    p.d_epoch = reinterpret_cast<unsigned*>(e->xchg + off_epoch);
    for (int r = 0; r < 8; r++) p.peer_x[r] = nullptr;
    p.peer_x[TP > 1 ? e->tp_rank : 0] = e->xchg;
    p.tp_rank = TP > 1 ? e->tp_rank : 0;
    p.tp_size = TP;
    p.C = C; p.L = L; p.NH = NHl; p.V = c.vocab_size; p.Vp = c.padded_vocab_size; p.maxT = maxT;
    p.splits = S; p.nsw = nsw; p.G = G; p.kv_rows = kv_rows; p.lookahead = lookahead;
    p.qkv_rows = Q; p.proj_k = A; p.fc_rows = F; p.fcproj_k = F; p.v_rows = e->v_rows; p.v0 = e->v0;
    p.attn_scale = 1.0f / sqrtf(64.0f);
    p.W[0] = e->p[0]; p.W[1] = e->p[4]; p.W[2] = e->p[6]; p.W[3] = e->p[10]; p.W[4] = e->p[12];
    for (int g = 0; g < 5; g++) p.S[g] = e->sc[g];
    p.wpe = e->p[1];
    p.ln1w = e->p[2]; p.ln1b = e->p[3]; p.qkvb = e->p[5]; p.attprojb = e->p[7];
    p.ln2w = e->p[8]; p.ln2b = e->p[9]; p.fcb = e->p[11]; p.fcprojb = e->p[13];
    p.lnfw = e->p[14]; p.lnfb = e->p[15];
    p.kv = e->kv_cache;
    p.kv_scale = e->kv_scale;
    p.d_token = e->d_token; p.d_pos = e->d_pos; p.history = e->d_history; p.prompt = e->d_prompt;
    p.logits = e->logits;
    // single GPU: ready; tensor parallel: after gpt2b_engine_tp_connect maps the peers' arenas
    e->persist_ok = (TP == 1);
    e->use_persistent = (TP == 1);
    return cudaSuccess;
}

int build_engine(const unsigned char* image, size_t nbytes, const float* scales, size_t nscales, int wmode,
                 int kvmode, int tp_rank, int tp_size, const void* nccl_id, gpt2b_engine** out) {
    if (!out) return GPT2B_ERR_INVALID_ARG;
    *out = nullptr;
    if (wmode < GPT2B_W_F32 || wmode > GPT2B_W_FP8 || (kvmode != GPT2B_KV_FLOATX && kvmode != GPT2B_KV_8BIT))
        return GPT2B_ERR_INVALID_ARG;
    const bool w8 = (wmode == GPT2B_W_INT8 || wmode == GPT2B_W_FP8);
    if (kvmode == GPT2B_KV_8BIT && !w8) return GPT2B_ERR_UNSUPPORTED;  // Makefile:102-103
    if (!image || nbytes < 1024) return GPT2B_ERR_FORMAT;
    int hdr[256];
    memcpy(hdr, image, sizeof(hdr));
    gpt2b_config cfg;
    int rc = check_header(hdr, wmode, &cfg);
    if (rc) return rc;
    const int C = cfg.channels, L = cfg.num_layers, NH = cfg.num_heads, maxT = cfg.max_seq_len;
    const int Vp = cfg.padded_vocab_size, hs = C / NH;
    if (hs != 64 || C > 2048 || maxT % 16 != 0) return GPT2B_ERR_UNSUPPORTED;

    size_t n[16];
    param_sizes(cfg, n);
    const size_t xb = (wmode == GPT2B_W_F32) ? 4 : 2;
    size_t file_bytes = 1024;
    for (int i = 0; i < 16; i++) file_bytes += n[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb);
    if (nbytes != file_bytes) return GPT2B_ERR_FORMAT;
    const size_t n_scales = (size_t)Vp + (size_t)L * 3 * C + (size_t)L * C + (size_t)L * 4 * C + (size_t)L * C;
    if (w8 && (!scales || nscales != n_scales)) return GPT2B_ERR_FORMAT;
    TpPlan pl;
    if (!tp_plan(cfg, tp_rank, tp_size, &pl)) return GPT2B_ERR_UNSUPPORTED;
#if !GPT2B_HAVE_NCCL
    if (tp_size > 1) return GPT2B_ERR_UNSUPPORTED;
#endif
    if (tp_size > 1 && !nccl_id) return GPT2B_ERR_INVALID_ARG;
    size_t nl[16], nsl[5];
    local_sizes(cfg, pl, nl, nsl);
    // this rank's tensors (the image itself on a single GPU)
    std::vector<unsigned char> shard;
    std::vector<float> shard_sc;
    const unsigned char* src_params = image + 1024;
    const float* src_scales = scales;
    if (tp_size > 1) {
        tp_shard(image, scales, cfg, w8, xb, pl, tp_rank, shard, shard_sc);
        src_params = shard.data();
        src_scales = shard_sc.data();
    }
    const int NHl = pl.nh_l, Fl = pl.f_l;

    gpt2b_engine* e = new gpt2b_engine();
    cudaGetDevice(&e->device);
    e->cfg = cfg;
    e->wmode = wmode;
    e->kvmode = kvmode;
    e->w8 = w8;
    e->xbytes = xb;
    e->wk = (wmode == GPT2B_W_F32) ? WK_F32 : (wmode == GPT2B_W_BF16 ? WK_BF16 : (wmode == GPT2B_W_INT8 ? WK_I8 : WK_FP8));
    e->tp_rank = tp_rank;
    e->tp_size = tp_size;
    e->h0 = pl.h0; e->nh_l = pl.nh_l; e->f0 = pl.f0; e->f_l = pl.f_l; e->v0 = pl.v0; e->v_rows = pl.v_rows;
    if (kvmode == GPT2B_KV_8BIT) e->kvk = (wmode == GPT2B_W_FP8) ? KV_FP8 : KV_I8;
    else e->kvk = (wmode == GPT2B_W_F32) ? KV_F32 : KV_BF16;

    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    auto fail = [&](cudaError_t x) { free_engine(e); return status_from(x); };
    if (err != cudaSuccess) return fail(err);

#if GPT2B_HAVE_NCCL
    if (tp_size > 1) {  // collective: every rank of the group calls this together
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        if (ncclCommInitRank(&e->comm, tp_size, id, tp_rank) != ncclSuccess) {
            e->comm = nullptr;
            free_engine(e);
            return GPT2B_ERR_NCCL;
        }
    }
#endif

    // ---- parameter arena (this rank's shard) ----
    size_t off[16], total = 0;
    for (int i = 0; i < 16; i++) {
        off[i] = total;
        total = align256(total + nl[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb));
    }
    size_t sc_off[5];
    if (w8)
        for (int g = 0; g < 5; g++) { sc_off[g] = total; total = align256(total + nsl[g] * 4); }
    e->params_bytes = total;
    if ((err = cudaMalloc(&e->params, total)) != cudaSuccess) return fail(err);
    const unsigned char* src = src_params;
    for (int i = 0; i < 16; i++) {
        const size_t b = nl[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb);
        e->p[i] = e->params + off[i];
        if ((err = cudaMemcpy(e->p[i], src, b, cudaMemcpyHostToDevice)) != cudaSuccess) return fail(err);
        src += b;
    }
    if (w8) {
        const float* s = src_scales;
        for (int g = 0; g < 5; g++) {
            e->sc[g] = reinterpret_cast<float*>(e->params + sc_off[g]);
            if ((err = cudaMemcpy(e->sc[g], s, nsl[g] * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return fail(err);
            s += nsl[g];
        }
    }

    // ---- activation arena ----
    const int nsm = sm_count();
    const int max_chunk = attn_engine_max_chunk(e->kvk);
    int splits = std::max((maxT + max_chunk - 1) / max_chunk, nsm / NHl);
    if (splits < 1) splits = 1;
    // engine chunks are multiples of 16 positions and at most max_chunk
    while (splits > 1 && ((((maxT + splits - 1) / splits) + 15) & ~15) > max_chunk) splits++;
    e->splits = splits;
    const int lm_grid_max = 2 * nsm;
    struct Slot { unsigned char** ptr; size_t bytes; };
    unsigned char *logits_b, *po_b, *pm_b, *pl_b, *lmv_b, *lmi_b, *lmc_b, *tok_b, *pos_b, *hist_b, *pr_b, *np_b;
    unsigned char *pf_b, *fpf_b, *pair_b, *pairs_b, *lfull_b;
    const bool tp = tp_size > 1;
    std::vector<Slot> slots = {
        {&e->encoded, C * xb},        {&e->ln1, (size_t)L * C * xb},   {&e->qkv, 3 * (size_t)NHl * hs * xb},
        {&e->atty, (size_t)L * NHl * hs * xb}, {&e->res2, (size_t)L * C * xb}, {&e->ln2, (size_t)L * C * xb},
        {&e->fch, (size_t)L * Fl * xb}, {&e->fch_gelu, (size_t)Fl * xb}, {&e->res3, (size_t)L * C * xb},
        {&e->lnf, C * xb},            {&e->proj_out, C * xb},          {&e->fcproj_out, C * xb},
        {&logits_b, (size_t)pl.v_rows * 4},  {&po_b, (size_t)NHl * splits * hs * 4}, {&pm_b, (size_t)NHl * splits * 4},
        {&pl_b, (size_t)NHl * splits * 4}, {&lmv_b, (size_t)lm_grid_max * 4},
        {&lmi_b, (size_t)lm_grid_max * 4}, {&lmc_b, 16},               {&tok_b, 16},
        {&pos_b, 16},                 {&hist_b, (size_t)(maxT + 1) * 4}, {&pr_b, (size_t)maxT * 4},
        {&np_b, 16},
        {&pf_b, tp ? (size_t)C * 4 : 16}, {&fpf_b, tp ? (size_t)C * 4 : 16}, {&pair_b, 16},
        {&pairs_b, (size_t)tp_size * 8}, {&lfull_b, tp ? (size_t)Vp * 4 : 16}};
    size_t at = 0;
    for (auto& s : slots) at = align256(at + s.bytes);
    e->acts_bytes = at;
    if ((err = cudaMalloc(&e->acts, at)) != cudaSuccess) return fail(err);
    if ((err = cudaMemset(e->acts, 0, at)) != cudaSuccess) return fail(err);
    at = 0;
    for (auto& s : slots) { *s.ptr = e->acts + at; at = align256(at + s.bytes); }
    e->logits = reinterpret_cast<float*>(logits_b);
    e->part_out = reinterpret_cast<float*>(po_b);
    e->part_max = reinterpret_cast<float*>(pm_b);
    e->part_lse = reinterpret_cast<float*>(pl_b);
    e->lm_val = reinterpret_cast<float*>(lmv_b);
    e->lm_idx = reinterpret_cast<int*>(lmi_b);
    e->lm_counter = reinterpret_cast<unsigned*>(lmc_b);
    e->d_token = reinterpret_cast<int*>(tok_b);
    e->d_pos = reinterpret_cast<int*>(pos_b);
    e->d_history = reinterpret_cast<int*>(hist_b);
    e->d_prompt = reinterpret_cast<int*>(pr_b);
    e->d_nprompt = reinterpret_cast<int*>(np_b);
    if (tp) {
        e->proj_f32 = reinterpret_cast<float*>(pf_b);
        e->fcproj_f32 = reinterpret_cast<float*>(fpf_b);
        e->lm_pair = reinterpret_cast<float*>(pair_b);
        e->lm_pairs = reinterpret_cast<float*>(pairs_b);
        e->logits_full = reinterpret_cast<float*>(lfull_b);
    }

    // ---- KV arena ----
    e->kv_layer_elems = 2 * (size_t)NHl * maxT * hs;
    e->kv_layer_scales = (e->kvk >= KV_I8) ? 2 * (size_t)NHl * maxT : 0;
    const size_t kv_elem_b = (e->kvk >= KV_I8) ? 1 : xb;
    size_t kvb = align256((size_t)L * e->kv_layer_elems * kv_elem_b);
    const size_t sc_at = kvb;
    kvb += align256((size_t)L * e->kv_layer_scales * 4);
    e->kv_bytes = kvb;
    if ((err = cudaMalloc(&e->kv, kvb)) != cudaSuccess) return fail(err);
    if ((err = cudaMemset(e->kv, 0, kvb)) != cudaSuccess) return fail(err);
    e->kv_cache = e->kv;
    e->kv_scale = e->kv_layer_scales ? reinterpret_cast<float*>(e->kv + sc_at) : nullptr;

    // ---- GEMV plans ----
    const int wk = e->wk;
    const size_t wb = (size_t)wkind_bytes(wk);
    e->qkv_p.resize(L);
    e->proj_p.resize(L);
    e->fc_p.resize(L);
    e->fcproj_p.resize(L);
    const size_t Q = 3 * (size_t)NHl * hs, A = (size_t)NHl * hs;  // local QKV rows, projection K
    for (int l = 0; l < L; l++) {
        GemvParams q;
        q.W = e->p[4] + (size_t)l * Q * C * wb;
        q.scale = w8 ? e->sc[1] + (size_t)l * Q : nullptr;
        q.bias = e->p[5] + (size_t)l * Q * xb;
        q.out = e->qkv;
        q.M = (int)Q; q.K = C;
        q.ln_w = e->p[2] + (size_t)l * C * xb;
        q.ln_b = e->p[3] + (size_t)l * C * xb;
        q.ln_out = e->ln1 + (size_t)l * C * xb;
        if (l == 0) {
            q.d_token = e->d_token; q.d_pos = e->d_pos;
            q.wte = w8 ? nullptr : e->p[0];
            q.wte8 = w8 ? e->p[0] : nullptr;
            q.wte_scale = w8 ? e->sc[0] : nullptr;
            q.wpe = e->p[1];
            q.vocab = cfg.vocab_size; q.maxT = maxT;
            q.res_out = e->encoded;
        } else {
            q.res_in = e->res2 + (size_t)(l - 1) * C * xb;
            q.delta = tp ? (const void*)e->fcproj_f32 : (const void*)e->fcproj_out;
            q.delta_f32 = tp ? 1 : 0;
            q.res_out = e->res3 + (size_t)(l - 1) * C * xb;
        }
        plan_gemv(q, wk, nsm, true);
        e->qkv_p[l] = q;

        GemvParams pr;
        pr.W = e->p[6] + (size_t)l * C * A * wb;
        pr.scale = w8 ? e->sc[2] + (size_t)l * C : nullptr;
        pr.bias = e->p[7] + (size_t)l * C * xb;
        pr.part_out = e->part_out;  // x = merge of the attention partials (PRO_ATTN_MERGE)
        pr.part_max = e->part_max;
        pr.part_lse = e->part_lse;
        pr.attn_heads = NHl;
        pr.attn_splits = splits;
        pr.d_pos = e->d_pos;
        pr.atty_out = e->atty + (size_t)l * A * xb;
        pr.aux_bytes = NHl * splits * 64 * 4 + 2 * (((NHl * splits * 4) + 15) & ~15);
        pr.out = tp ? (void*)e->proj_f32 : (void*)e->proj_out;  // row-parallel: FP32 partial sums
        pr.M = C; pr.K = (int)A;
        plan_gemv(pr, wk, nsm, true);
        e->proj_p[l] = pr;

        GemvParams f;
        f.W = e->p[10] + (size_t)l * Fl * C * wb;
        f.scale = w8 ? e->sc[3] + (size_t)l * Fl : nullptr;
        f.bias = e->p[11] + (size_t)l * Fl * xb;
        f.out = e->fch_gelu;
        f.pre_gelu = e->fch + (size_t)l * Fl * xb;
        f.do_gelu = 1;
        f.M = Fl; f.K = C;
        f.res_in = (l == 0) ? e->encoded : e->res3 + (size_t)(l - 1) * C * xb;
        f.delta = tp ? (const void*)e->proj_f32 : (const void*)e->proj_out;
        f.delta_f32 = tp ? 1 : 0;
        f.res_out = e->res2 + (size_t)l * C * xb;
        f.ln_out = e->ln2 + (size_t)l * C * xb;
        f.ln_w = e->p[8] + (size_t)l * C * xb;
        f.ln_b = e->p[9] + (size_t)l * C * xb;
        plan_gemv(f, wk, nsm, true);
        e->fc_p[l] = f;

        GemvParams fp;
        fp.W = e->p[12] + (size_t)l * C * Fl * wb;
        fp.scale = w8 ? e->sc[4] + (size_t)l * C : nullptr;
        fp.bias = e->p[13] + (size_t)l * C * xb;
        fp.x = e->fch_gelu;
        fp.out = tp ? (void*)e->fcproj_f32 : (void*)e->fcproj_out;
        fp.M = C; fp.K = Fl;
        plan_gemv(fp, wk, nsm, true);
        e->fcproj_p[l] = fp;
    }
    GemvParams lm;  // this rank's vocab rows [v0, v0 + v_rows) of the tied wte
    lm.W = e->p[0] + (size_t)pl.v0 * C * wb;
    lm.scale = w8 ? e->sc[0] + pl.v0 : nullptr;
    lm.out = e->logits;
    lm.M = pl.v_rows; lm.K = C;
    lm.res_in = e->res2 + (size_t)(L - 1) * C * xb;
    lm.delta = tp ? (const void*)e->fcproj_f32 : (const void*)e->fcproj_out;
    lm.delta_f32 = tp ? 1 : 0;
    lm.res_out = e->res3 + (size_t)(L - 1) * C * xb;
    lm.ln_out = e->lnf;
    lm.ln_w = e->p[14];
    lm.ln_b = e->p[15];
    lm.vocab = std::max(0, std::min(cfg.vocab_size - pl.v0, pl.v_rows));  // valid rows of the shard
    lm.part_val = e->lm_val; lm.part_idx = e->lm_idx; lm.counter = e->lm_counter;
    if (tp) { lm.pair_out = e->lm_pair; lm.row_offset = pl.v0; }
    lm.token_io = e->d_token; lm.pos_io = e->d_pos; lm.history = e->d_history;
    lm.prompt = e->d_prompt;
    lm.n_prompt = 0;
    plan_gemv(lm, wk, nsm, false);
    if (lm.grid > lm_grid_max) return fail(cudaErrorInvalidConfiguration);
    e->lm_p = lm;
    if ((err = setup_persistent(e, nsm)) != cudaSuccess) return fail(err);
    e->prefill_ok = e->use_prefill =
        !tp && prefill_supported(e->wk, e->kvk, C, cfg.num_heads, cfg.max_seq_len);
    *out = e;
    return GPT2B_OK;
}

bool read_file(const char* path, std::vector<unsigned char>& buf) {
    FILE* f = fopen(path, "rb");
    if (!f) return false;
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz < 0) { fclose(f); return false; }
    buf.resize((size_t)sz);
    size_t got = sz ? fread(buf.data(), 1, (size_t)sz, f) : 0;
    fclose(f);
    return got == (size_t)sz;
}

}  // namespace

// The LM head's prompt length is a kernel parameter captured into the graphs;
// changing it invalidates them.
static void set_prompt_len(gpt2b_engine* e, int n_prompt) {
    if (e->lm_p.n_prompt != n_prompt) {
        e->lm_p.n_prompt = n_prompt;
        e->graphs_valid = false;
    }
}

extern "C" {

int gpt2b_read_header(const char* path, int* version, gpt2b_config* cfg) {
    if (!path || !cfg) return GPT2B_ERR_INVALID_ARG;
    FILE* f = fopen(path, "rb");
    if (!f) return GPT2B_ERR_FILE;
    int hdr[256];
    size_t got = fread(hdr, sizeof(int), 256, f);
    fclose(f);
    if (got != 256) return GPT2B_ERR_FORMAT;
    if (hdr[0] != 20251103 || (hdr[1] != 3 && hdr[1] != 5)) return GPT2B_ERR_FORMAT;
    if (version) *version = hdr[1];
    return check_header(hdr, hdr[1] == 3 ? GPT2B_W_F32 : GPT2B_W_BF16, cfg);
}

int gpt2b_engine_create_from_buffer(const void* image, size_t nbytes, const float* scales, size_t nscales, int wmode,
                                    int kvmode, gpt2b_engine** out) {
    return build_engine(static_cast<const unsigned char*>(image), nbytes, scales, nscales, wmode, kvmode, 0, 1, nullptr,
                        out);
}

int gpt2b_engine_create_tp_from_buffer(const void* image, size_t nbytes, const float* scales, size_t nscales,
                                       int wmode, int kvmode, int tp_rank, int tp_size, const void* nccl_id,
                                       gpt2b_engine** out) {
    return build_engine(static_cast<const unsigned char*>(image), nbytes, scales, nscales, wmode, kvmode, tp_rank,
                        tp_size, nccl_id, out);
}

int gpt2b_engine_tp_ipc_handle(gpt2b_engine* e, void* handle_out) {
    if (!e || !handle_out) return GPT2B_ERR_INVALID_ARG;
    if (e->tp_size < 2 || !e->xchg) return GPT2B_ERR_UNSUPPORTED;
    DeviceGuard g(e->device);
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, e->xchg);
    if (err != cudaSuccess) return status_from(err);
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return GPT2B_OK;
}

int gpt2b_engine_tp_connect(gpt2b_engine* e, const void* handles, int n) {
    if (!e || !handles) return GPT2B_ERR_INVALID_ARG;
    if (e->tp_size < 2 || !e->xchg) return GPT2B_ERR_UNSUPPORTED;
    if (n != e->tp_size) return GPT2B_ERR_INVALID_ARG;
    if (e->tp_connected) return GPT2B_OK;
    DeviceGuard g(e->device);
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < n; r++) {
        if (r == e->tp_rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)r * 64, 64);
        void* ptr = nullptr;
        cudaError_t err = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) return status_from(err);
        e->peer_map[r] = static_cast<unsigned char*>(ptr);
        e->pp.peer_x[r] = e->peer_map[r];
    }
    e->tp_connected = true;
    e->persist_ok = true;
    e->use_persistent = true;
    return GPT2B_OK;
}

int gpt2b_nccl_unique_id(void* id_out) {
    if (!id_out) return GPT2B_ERR_INVALID_ARG;
#if GPT2B_HAVE_NCCL
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return GPT2B_ERR_NCCL;
    memcpy(id_out, &id, sizeof(id));
    return GPT2B_OK;
#else
    return GPT2B_ERR_UNSUPPORTED;
#endif
}

int gpt2b_tp_plan(const gpt2b_config* cfg, int tp_rank, int tp_size, int* out6) {
    if (!cfg || !out6) return GPT2B_ERR_INVALID_ARG;
    TpPlan pl;
    if (!tp_plan(*cfg, tp_rank, tp_size, &pl)) return GPT2B_ERR_UNSUPPORTED;
    const int v[6] = {pl.h0, pl.nh_l, pl.f0, pl.f_l, pl.v0, pl.v_rows};
    memcpy(out6, v, sizeof(v));
    return GPT2B_OK;
}

int gpt2b_tp_shard_image(const void* image, size_t nbytes, const float* scales, size_t nscales, int wmode,
                         int tp_rank, int tp_size, void* out_params, size_t* out_bytes, float* out_scales,
                         size_t* out_nscales) {
    if (!image || !out_bytes || !out_nscales || nbytes < 1024) return GPT2B_ERR_INVALID_ARG;
    if (wmode < GPT2B_W_F32 || wmode > GPT2B_W_FP8) return GPT2B_ERR_INVALID_ARG;
    const bool w8 = (wmode == GPT2B_W_INT8 || wmode == GPT2B_W_FP8);
    int hdr[256];
    memcpy(hdr, image, sizeof(hdr));
    gpt2b_config cfg;
    int rc = check_header(hdr, wmode, &cfg);
    if (rc) return rc;
    size_t n[16];
    param_sizes(cfg, n);
    const size_t xb = (wmode == GPT2B_W_F32) ? 4 : 2;
    size_t file_bytes = 1024;
    for (int i = 0; i < 16; i++) file_bytes += n[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb);
    if (nbytes != file_bytes) return GPT2B_ERR_FORMAT;
    const size_t C = cfg.channels, L = cfg.num_layers;
    const size_t n_scales = (size_t)cfg.padded_vocab_size + L * 3 * C + L * C + L * 4 * C + L * C;
    if (w8 && (!scales || nscales != n_scales)) return GPT2B_ERR_FORMAT;
    TpPlan pl;
    if (!tp_plan(cfg, tp_rank, tp_size, &pl)) return GPT2B_ERR_UNSUPPORTED;
    size_t nl[16], nsl[5], total = 0, total_sc = 0;
    local_sizes(cfg, pl, nl, nsl);
    for (int i = 0; i < 16; i++) total += nl[i] * ((w8 && kLinearSlot[i] >= 0) ? 1 : xb);
    if (w8)
        for (int g = 0; g < 5; g++) total_sc += nsl[g];
    if (!out_params) {  // size query
        *out_bytes = total;
        *out_nscales = total_sc;
        return GPT2B_OK;
    }
    if (*out_bytes < total || (w8 && (!out_scales || *out_nscales < total_sc))) return GPT2B_ERR_INVALID_ARG;
    std::vector<unsigned char> sh;
    std::vector<float> ssc;
    tp_shard(static_cast<const unsigned char*>(image), scales, cfg, w8, xb, pl, tp_rank, sh, ssc);
    memcpy(out_params, sh.data(), sh.size());
    if (w8) memcpy(out_scales, ssc.data(), ssc.size() * sizeof(float));
    *out_bytes = total;
    *out_nscales = total_sc;
    return GPT2B_OK;
}

int gpt2b_engine_create_from_file(const char* model_path, const char* scale_path, int wmode, int kvmode,
                                  gpt2b_engine** out) {
    if (!model_path || !out) return GPT2B_ERR_INVALID_ARG;
    std::vector<unsigned char> img;
    if (!read_file(model_path, img)) return GPT2B_ERR_FILE;
    std::vector<unsigned char> sc;
    const bool w8 = (wmode == GPT2B_W_INT8 || wmode == GPT2B_W_FP8);
    if (w8) {
        std::string sp;
        if (scale_path) sp = scale_path;
        else {  // inference_gpt2_opt.cu:666-668
            std::string m = model_path;
            if (m.size() < 4) return GPT2B_ERR_FILE;
            sp = m.substr(0, m.size() - 4) + "_scales.bin";
        }
        if (!read_file(sp.c_str(), sc)) return GPT2B_ERR_FILE;
        if (sc.size() % 4) return GPT2B_ERR_FORMAT;
    }
    return build_engine(img.data(), img.size(), w8 ? reinterpret_cast<const float*>(sc.data()) : nullptr,
                        sc.size() / 4, wmode, kvmode, 0, 1, nullptr, out);
}

int gpt2b_engine_destroy(gpt2b_engine* e) {
    if (!e) return GPT2B_ERR_INVALID_ARG;
    {
        DeviceGuard g(e->device);
        cudaStreamSynchronize(e->stream);
    }
    free_engine(e);
    return GPT2B_OK;
}

int gpt2b_engine_config(const gpt2b_engine* e, gpt2b_config* cfg) {
    if (!e || !cfg) return GPT2B_ERR_INVALID_ARG;
    *cfg = e->cfg;
    return GPT2B_OK;
}

int gpt2b_engine_set_option(gpt2b_engine* e, int option, int value) {
    if (!e) return GPT2B_ERR_INVALID_ARG;
    switch (option) {
        case GPT2B_OPT_USE_GRAPH: e->use_graph = value != 0; break;
        case GPT2B_OPT_USE_PDL: e->use_pdl = value != 0; e->graphs_valid = false; break;
        case GPT2B_OPT_SPLITS: {
            const int maxT = e->cfg.max_seq_len, mc = attn_engine_max_chunk(e->kvk);
            if (value < 1 || ((((maxT + value - 1) / value) + 15) & ~15) > mc) return GPT2B_ERR_INVALID_ARG;
            if (value > e->splits) return GPT2B_ERR_INVALID_ARG;  // partial buffers are sized at creation
            e->splits = value;
            e->graphs_valid = false;
            break;
        }
        case GPT2B_OPT_STEPS_PER_GRAPH:
            if (value < 1 || value > 64) return GPT2B_ERR_INVALID_ARG;
            e->steps_per_graph = value;
            e->graphs_valid = false;
            break;
        case GPT2B_OPT_PERSISTENT:
            if (value && !e->persist_ok) return GPT2B_ERR_UNSUPPORTED;  // (tensor parallel: connect first)
            e->use_persistent = value != 0;
            break;
        case GPT2B_OPT_PREFILL:
            if (value && !e->prefill_ok) return GPT2B_ERR_UNSUPPORTED;
            e->use_prefill = value != 0;
            break;
        case GPT2B_OPT_POLL_LIMIT:
            if (value < 1024) return GPT2B_ERR_INVALID_ARG;
            e->pp.poll_limit = (uint32_t)value;
            break;
        default: return GPT2B_ERR_INVALID_ARG;
    }
    return GPT2B_OK;
}

int gpt2b_engine_stream(const gpt2b_engine* e, gpt2b_stream_t* stream) {
    if (!e || !stream) return GPT2B_ERR_INVALID_ARG;
    *stream = (gpt2b_stream_t)e->stream;
    return GPT2B_OK;
}

int gpt2b_engine_device_buffers(const gpt2b_engine* e, float** logits, int** token, int** pos, int** history) {
    if (!e) return GPT2B_ERR_INVALID_ARG;
    if (logits) *logits = e->tp_size > 1 ? e->logits_full : e->logits;
    if (token) *token = e->d_token;
    if (pos) *pos = e->d_pos;
    if (history) *history = e->d_history;
    return GPT2B_OK;
}

int gpt2b_engine_kernels_per_step(const gpt2b_engine* e, int* n) {
    if (!e || !n) return GPT2B_ERR_INVALID_ARG;
    *n = e->use_persistent ? 0 : 5 * e->cfg.num_layers + 1 + (e->tp_size > 1 ? 1 : 0);
    return GPT2B_OK;
}

int gpt2b_engine_forward(gpt2b_engine* e, int token, int pos) {
    if (!e) return GPT2B_ERR_INVALID_ARG;
    if (token < 0 || token >= e->cfg.vocab_size || pos < 0 || pos >= e->cfg.max_seq_len) return GPT2B_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    set_prompt_len(e, 0);
    const int tp[2] = {token, pos};
    cudaError_t err = cudaMemcpyAsync(e->d_token, &tp[0], sizeof(int), cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_pos, &tp[1], sizeof(int), cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = run_steps(e, 1);
    if (err == cudaSuccess && e->tp_size > 1) err = tp_allgather(e, e->logits, e->logits_full, (size_t)e->v_rows);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    return status_from(err);
}

int gpt2b_engine_decode(gpt2b_engine* e, int n_steps) {
    if (!e || n_steps < 0) return GPT2B_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    return status_from(run_steps(e, n_steps));
}

int gpt2b_engine_history(gpt2b_engine* e, int* out_host, int first, int count) {
    if (!e || !out_host || first < 0 || count < 0 || first + count > e->cfg.max_seq_len + 1)
        return GPT2B_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    cudaError_t err = cudaStreamSynchronize(e->stream);
    if (err == cudaSuccess)
        err = cudaMemcpy(out_host, e->d_history + first, (size_t)count * sizeof(int), cudaMemcpyDeviceToHost);
    return status_from(err);
}

int gpt2b_engine_set_position(gpt2b_engine* e, int token, int pos) {
    if (!e) return GPT2B_ERR_INVALID_ARG;
    if (token < 0 || token >= e->cfg.vocab_size || pos < 0 || pos >= e->cfg.max_seq_len) return GPT2B_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    const int tp[2] = {token, pos};  // pageable source: the stream is synchronised before returning
    cudaError_t err = cudaMemcpyAsync(e->d_token, &tp[0], sizeof(int), cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_pos, &tp[1], sizeof(int), cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    return status_from(err);
}

int gpt2b_engine_generate(gpt2b_engine* e, const int* prompt, int n_prompt, int n_gen, int* out_tokens,
                          float* logits_host, int sample, unsigned long long seed) {
    if (!e || !prompt || !out_tokens || n_prompt < 1 || n_gen < 0) return GPT2B_ERR_INVALID_ARG;
    const int maxT = e->cfg.max_seq_len, V = e->cfg.vocab_size, Vp = e->cfg.padded_vocab_size;
    if (n_prompt + n_gen > maxT) return GPT2B_ERR_INVALID_ARG;
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= V) return GPT2B_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    set_prompt_len(e, n_prompt);
    cudaStream_t st = e->stream;
    const int zero = 0;
    cudaError_t err = cudaMemcpyAsync(e->d_prompt, prompt, (size_t)n_prompt * sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_token, prompt, sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_pos, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_history, prompt, sizeof(int), cudaMemcpyHostToDevice, st);
    const int total = n_prompt + n_gen;
    int first = 0;  // forwards already done
    if (err == cudaSuccess && e->use_prefill && n_prompt >= 2) {
        // the whole prompt as tensor-core GEMMs: positions 0..n_prompt-1 in one pass
        err = ensure_prefill(e);
        if (err == cudaSuccess) err = run_prefill(e->pf, n_prompt, st);
        if (err == cudaSuccess && logits_host)
            err = cudaMemcpyAsync(logits_host, e->pf.logits_rows, (size_t)n_prompt * Vp * 4, cudaMemcpyDeviceToHost, st);
        if (err == cudaSuccess && sample) {  // the token after the prompt is drawn, not picked
            int rc = gpt2b_gpu_sample_softmax(e->d_token, e->logits, 1, V, seed, n_prompt, (gpt2b_stream_t)st);
            if (rc) return rc;
            err = launch_k(set_history_kernel, dim3(1), dim3(1), 0, st, false, e->d_history, e->d_token, e->d_pos);
        }
        first = n_prompt;
    }
    if (err == cudaSuccess) {
        if (!logits_host && !sample) {
            err = run_steps(e, total - first);  // device-resident: no host round trip per token
        } else {
            for (int s = first; s < total && err == cudaSuccess; s++) {
                err = run_steps(e, 1);
                float* lg = e->logits;  // all Vp logits (tensor parallel: gathered from the vocab shards)
                if (err == cudaSuccess && e->tp_size > 1) {
                    err = tp_allgather(e, e->logits, e->logits_full, (size_t)e->v_rows);
                    lg = e->logits_full;
                }
                if (err == cudaSuccess && sample && s + 1 >= n_prompt) {
                    // replace the greedy pick by a softmax sample (step = position of the new token);
                    // every rank draws the same (seed, step) sample from the same logits
                    int rc = gpt2b_gpu_sample_softmax(e->d_token, lg, 1, V, seed, s + 1, (gpt2b_stream_t)st);
                    if (rc) return rc;
                    err = launch_k(set_history_kernel, dim3(1), dim3(1), 0, st, false, e->d_history, e->d_token, e->d_pos);
                }
                if (err == cudaSuccess && logits_host)
                    err = cudaMemcpyAsync(logits_host + (size_t)s * Vp, lg, (size_t)Vp * 4, cudaMemcpyDeviceToHost, st);
            }
        }
    }
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(out_tokens, e->d_history + n_prompt, (size_t)(n_gen + 1) * sizeof(int),
                              cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) return status_from(err);
    int dev = 0;
    gpt2b_device_error(&dev);
    return dev ? GPT2B_ERR_DEVICE : GPT2B_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// verification dumps (Inference_gpt2/dump_utils.h)
// ---------------------------------------------------------------------------
namespace {

bool mkdir_p(const std::string& dir) {
    std::string cur;
    for (size_t i = 0; i < dir.size(); i++) {
        cur += dir[i];
        if ((dir[i] == '/' && i > 0) || i + 1 == dir.size()) {
            if (mkdir(cur.c_str(), 0755) != 0) {
                struct stat st;
                if (stat(cur.c_str(), &st) != 0 || !S_ISDIR(st.st_mode)) return false;
            }
        }
    }
    return true;
}

bool write_file(const std::string& path, const void* data, size_t bytes) {
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = fwrite(data, 1, bytes, f) == bytes;
    return fclose(f) == 0 && ok;
}

}  // namespace

extern "C" int gpt2b_engine_generate_dump(gpt2b_engine* e, const int* prompt, int n_prompt, int n_gen,
                                          int* out_tokens, int sample, unsigned long long seed,
                                          const gpt2b_dump_config* dump, float* nll_out) {
    if (!e || !prompt || !out_tokens || !dump || n_prompt < 1 || n_gen < 0) return GPT2B_ERR_INVALID_ARG;
    const int maxT = e->cfg.max_seq_len, V = e->cfg.vocab_size;
    const int total = n_prompt + n_gen;
    if (total > maxT || dump->ppl_len < 0 || dump->ppl_len > total || dump->n_steps < 0 ||
        (dump->n_steps && !dump->steps))
        return GPT2B_ERR_INVALID_ARG;
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= V) return GPT2B_ERR_INVALID_ARG;
    std::string dir, prefix = dump->prefix ? dump->prefix : "gpt2b";
    if (dump->dir) {
        dir = dump->dir;
        if (!mkdir_p(dir)) return GPT2B_ERR_FILE;
        if (dir.back() != '/') dir += '/';
    }
    DeviceGuard g(e->device);
    cudaStream_t st = e->stream;
    float* d_nll = nullptr;
    cudaError_t err = cudaSuccess;
    if (dump->ppl_len > 0) err = cudaMalloc(&d_nll, (size_t)dump->ppl_len * sizeof(float));
    set_prompt_len(e, n_prompt);
    const int zero = 0;
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(e->d_prompt, prompt, (size_t)n_prompt * sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_token, prompt, sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_pos, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->d_history, prompt, sizeof(int), cudaMemcpyHostToDevice, st);
    std::vector<float> lg(V);
    std::vector<int> hist;
    int rc = GPT2B_OK;
    // the prompt as in gpt2b_engine_generate: one tensor-core pass when prefill is on, and
    // step t <= n_prompt then reads row t - 1 of the prompt logits
    const bool pf = e->use_prefill && n_prompt >= 2;
    if (pf && err == cudaSuccess) {
        err = ensure_prefill(e);
        if (err == cudaSuccess) err = run_prefill(e->pf, n_prompt, st);
    }
    for (int t = 1; t <= total && err == cudaSuccess && rc == GPT2B_OK; t++) {
        const bool in_prompt = pf && t <= n_prompt;
        const float* logits = in_prompt ? e->pf.logits_rows + (size_t)(t - 1) * e->cfg.padded_vocab_size : e->logits;
        if (!in_prompt) err = run_steps(e, 1);  // the forward at position t - 1
        if (err == cudaSuccess && !in_prompt && e->tp_size > 1) {
            err = tp_allgather(e, e->logits, e->logits_full, (size_t)e->v_rows);
            logits = e->logits_full;
        }
        if (err == cudaSuccess && sample && t >= n_prompt) {
            rc = gpt2b_gpu_sample_softmax(e->d_token, logits, 1, V, seed, t, (gpt2b_stream_t)st);
            if (rc == GPT2B_OK)
                err = launch_k(set_history_kernel, dim3(1), dim3(1), 0, st, false, e->d_history, e->d_token, e->d_pos);
        }
        if (err == cudaSuccess && rc == GPT2B_OK && t <= dump->ppl_len)
            err = in_prompt ? launch_nll(d_nll, logits, V, nullptr, e->d_history, nullptr, t, st)
                            : launch_nll(d_nll, logits, V, nullptr, e->d_history, e->d_pos, 0, st);
        const bool want_step = std::find(dump->steps, dump->steps + dump->n_steps, t) != dump->steps + dump->n_steps;
        if (err == cudaSuccess && rc == GPT2B_OK && !dir.empty() && ((dump->logits_t1 && t == 1) || want_step)) {
            err = cudaMemcpyAsync(lg.data(), logits, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost, st);
            hist.resize(t);
            if (err == cudaSuccess)
                err = cudaMemcpyAsync(hist.data(), e->d_history, (size_t)t * sizeof(int), cudaMemcpyDeviceToHost, st);
            if (err == cudaSuccess) err = cudaStreamSynchronize(st);
            if (err == cudaSuccess && dump->logits_t1 && t == 1 &&
                !write_file(dir + prefix + "_logits_t1.bin", lg.data(), lg.size() * sizeof(float)))
                rc = GPT2B_ERR_FILE;
            if (err == cudaSuccess && want_step) {
                const std::string ts = std::to_string(t);
                if (!write_file(dir + prefix + "_logits_step" + ts + ".bin", lg.data(), lg.size() * sizeof(float)) ||
                    !write_file(dir + prefix + "_inputs_step" + ts + ".bin", hist.data(), hist.size() * sizeof(int)))
                    rc = GPT2B_ERR_FILE;
            }
        }
    }
    std::vector<float> nll(dump->ppl_len);
    std::vector<int> ptoks(dump->ppl_len);
    if (err == cudaSuccess && rc == GPT2B_OK) {
        err = cudaMemcpyAsync(out_tokens, e->d_history + n_prompt, (size_t)(n_gen + 1) * sizeof(int),
                              cudaMemcpyDeviceToHost, st);
        if (err == cudaSuccess && dump->ppl_len > 0) {
            err = cudaMemcpyAsync(nll.data(), d_nll, nll.size() * sizeof(float), cudaMemcpyDeviceToHost, st);
            if (err == cudaSuccess)
                err = cudaMemcpyAsync(ptoks.data(), e->d_history + 1, ptoks.size() * sizeof(int),
                                      cudaMemcpyDeviceToHost, st);
        }
        if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    }
    if (d_nll) cudaFree(d_nll);
    if (err != cudaSuccess) return status_from(err);
    if (rc != GPT2B_OK) return rc;
    int dev = 0;
    gpt2b_device_error(&dev);
    if (dev) return GPT2B_ERR_DEVICE;
    if (dump->ppl_len > 0) {
        if (nll_out) memcpy(nll_out, nll.data(), nll.size() * sizeof(float));
        if (!dir.empty() &&
            (!write_file(dir + "ppl_" + prefix + "_nll.bin", nll.data(), nll.size() * sizeof(float)) ||
             !write_file(dir + "ppl_" + prefix + "_tokens.bin", ptoks.data(), ptoks.size() * sizeof(int))))
            return GPT2B_ERR_FILE;
    }
    return GPT2B_OK;
}
