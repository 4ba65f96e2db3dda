// internal.h -- interfaces between the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace gpt2b {

enum WKind { WK_F32 = 0, WK_BF16 = 1, WK_I8 = 2, WK_FP8 = 3 };
// x-vector source of a GEMV launch
enum Prologue {
    PRO_PLAIN = 0,      // x read from memory
    PRO_RES_LN = 1,     // r = res_in + delta (stored), x = LayerNorm(r)
    PRO_EMB_LN = 2,     // e = wte[token] + wpe[pos] (stored), x = LayerNorm(e)
    PRO_ATTN_MERGE = 3  // x = LSE merge of the attention split partials (stored as atty)
};
// output of a GEMV launch
enum Epilogue {
    EPI_STORE = 0,   // out = gelu?(W.x*scale + b), optional pre_gelu
    EPI_LMHEAD = 1   // float logits + greedy pick + device-side token/position advance
};

inline int wkind_bytes(int wk) { return wk == WK_F32 ? 4 : (wk == WK_BF16 ? 2 : 1); }

// Position chunking of the engine's flash-decoding attention: `splits` CTAs
// per head, chunks a multiple of 16 positions.  Shared by the attention kernel
// (which writes the partials) and the GEMV prologue that merges them.
__host__ __device__ inline int engine_attn_chunk(int total, int splits) {
    int chunk = (total + splits - 1) / splits;
    chunk = (chunk + 15) & ~15;
    return chunk < 16 ? 16 : chunk;
}

struct GemvParams {
    // the matrix-vector product
    const void* W = nullptr;      // M x K row-major, storage per WKind
    const float* scale = nullptr; // per-row scale (8-bit kinds)
    const void* bias = nullptr;   // M, activation type; may be null
    const void* x = nullptr;      // K, activation type (PRO_PLAIN)
    void* out = nullptr;          // M, output type
    void* pre_gelu = nullptr;     // M, output type; may be null
    int M = 0, K = 0, do_gelu = 0;
    // tiling (filled by plan_gemv)
    int rows_per_tile = 0, ntiles = 0, nstages = 1, tile_bytes = 0, grid = 0;
    int stream = 0;               // 0: one tile per CTA (kernel A); 1: per-warp streaming rings (kernel B)
    int scale_in_tile = 0;        // 8-bit row scales travel with the weight tile
    int mma = 0;                  // kernel B, 8-bit codes: 16-row tiles through mma.sync (x as scaled FP16)
    int row_stride = 0;           // bytes between rows of a tile in shared memory (mma: padded)
    int x_vec = 0;                // x is 16-byte aligned (vector loads)
    int aux_bytes = 0;            // shared memory for PRO_ATTN_MERGE partials
    // PRO_RES_LN / PRO_EMB_LN
    const void* res_in = nullptr;  // C, activation type
    const void* delta = nullptr;   // C, activation type (FP32 when delta_f32)
    int delta_f32 = 0;             // delta is an FP32 all-reduced sum, rounded to the activation type on use
    void* res_out = nullptr;       // C, written by block 0
    void* ln_out = nullptr;        // C, written by block 0 (may be null)
    const void* ln_w = nullptr;
    const void* ln_b = nullptr;
    const int* d_token = nullptr;
    const int* d_pos = nullptr;
    const void* wte = nullptr;          // Vp x C activation type (F32/BF16 kinds)
    const uint8_t* wte8 = nullptr;      // Vp x C codes (8-bit kinds)
    const float* wte_scale = nullptr;   // Vp
    const void* wpe = nullptr;          // maxT x C
    int vocab = 0, maxT = 0;
    // PRO_ATTN_MERGE: partials [head][split] (+ [head][split][64] for out)
    const float* part_out = nullptr;
    const float* part_max = nullptr;
    const float* part_lse = nullptr;
    void* atty_out = nullptr;     // merged attention output (block 0), activation type
    int attn_heads = 0, attn_splits = 0;
    // EPI_LMHEAD
    float* part_val = nullptr;    // >= grid
    int* part_idx = nullptr;      // >= grid
    unsigned* counter = nullptr;  // zero between launches (the last block resets it)
    int* token_io = nullptr;
    int* pos_io = nullptr;
    int* history = nullptr;       // maxT + 1 ints
    const int* prompt = nullptr;  // device prompt, n_prompt ints
    int n_prompt = 0;
    int advance = 1;              // 1: write next token and pos+1; 0: only the logits
    float* pair_out = nullptr;    // tensor parallel: (best value, global index bits) instead of advancing
    int row_offset = 0;           // global index of local row 0 (vocab shard)
};

// KV-cache storage kinds
enum KvKind { KV_F32 = 0, KV_BF16 = 1, KV_I8 = 2, KV_FP8 = 3 };

// Decode attention for the engine: fused KV append + flash-decoding over
// `splits` CTAs per head; writes the per-split partials (un-normalised out,
// max, exp-sum) that the following projection GEMV merges (PRO_ATTN_MERGE).
// kv_layer / kv_scale_layer point at one layer's [K|V] cache and scales.
cudaError_t launch_attention_engine(int kv, const void* qkv, void* kv_layer, float* kv_scale_layer, const int* d_pos,
                                    int NH, int maxT, int splits, float* part_out, float* part_max, float* part_lse,
                                    cudaStream_t st, bool pdl);
int attn_engine_max_chunk(int kv);  // positions one engine CTA stages at once

// Negative log-likelihood of a token under softmax(logits[0..V)) (sampler.cu):
// token *tok -> out[0], or hist[p] -> out[p - 1] with p = *pos (pos non-null) or fixed_pos.
cudaError_t launch_nll(float* out, const float* logits, int V, const int* tok, const int* hist, const int* pos,
                       int fixed_pos, cudaStream_t st);

// Persistent decode kernel (persistent.cu): every step of a decode call in
// one cooperative launch of G CTAs (one per SM).
struct PersistParams {
    int C = 0, L = 0, NH = 0, V = 0, Vp = 0, maxT = 0, splits = 0, nsw = 0, G = 0;
    int kv_rows = 0;  // positions one attention CTA stages (the largest chunk at maxT)
    int lookahead = 0;  // stages the producer runs ahead in the layer phases (the LM head uses all nsw)
    // this rank's matrix shapes (single GPU: 3C, C, 4C, 4C, Vp, 0) and tensor-parallel group;
    // NH above is this rank's head count
    int qkv_rows = 0, proj_k = 0, fc_rows = 0, fcproj_k = 0, v_rows = 0, v0 = 0;
    int tp_rank = 0, tp_size = 1;
    // exchange arena of every rank (own included; peers through IPC mappings) and the
    // offsets of the cross-GPU parts: abort flag, projection / FC-projection partials
    // [L][tp][C], LM pairs [tp][G][2]
    unsigned char* peer_x[8] = {};
    size_t xoff_abort = 0, xoff_proj = 0, xoff_fcproj = 0, xoff_lm = 0;
    float attn_scale = 0.125f;
    // parameters: layer-0 bases of the stacked tensors, storage per weight kind
    const unsigned char* W[5] = {};  // wte, qkvw, attprojw, fcw, fcprojw
    const float* S[5] = {};          // their per-row scales (8-bit kinds)
    const void* wpe = nullptr;
    const void *ln1w = nullptr, *ln1b = nullptr, *qkvb = nullptr, *attprojb = nullptr, *ln2w = nullptr,
               *ln2b = nullptr, *fcb = nullptr, *fcprojb = nullptr, *lnfw = nullptr, *lnfb = nullptr;
    // KV cache [layer][K|V][head][maxT][hs] and 8-bit scales [layer][K|V][head][maxT]
    unsigned char* kv = nullptr;
    float* kv_scale = nullptr;
    // exchange words (step tag << 32 | float bits), zero-initialised; ll_proj, ll_fcproj and
    // ll_lm are this rank's copies of the cross-GPU parts
    unsigned long long *ll_qkv = nullptr, *ll_atty = nullptr, *ll_part = nullptr, *ll_proj = nullptr,
                       *ll_fc = nullptr, *ll_fcproj = nullptr, *ll_lm = nullptr;
    unsigned* kv_flag = nullptr;  // [layer][head]: last epoch whose KV append is complete
    // step state (device)
    int* d_token = nullptr;
    int* d_pos = nullptr;
    int* history = nullptr;
    const int* prompt = nullptr;
    int n_prompt = 0;
    unsigned* d_epoch = nullptr;  // advanced by n_steps per call
    int* abort_flag = nullptr;    // zero at launch
    uint32_t poll_limit = 1u << 22;  // polls of one exchange wait before it gives up (GPT2B_OPT_POLL_LIMIT)
    // 8-bit weights on tensor-core stages: per LayerNorm (LN1 and LN2 of layer l at 2l and 2l+1,
    // the final LN at 2L) the exponent e with sqrt(C) max|gamma| + max|beta| < 2^(14+e), a bound
    // of |x| (persist_ln_exponents)
    const int* ln_exp = nullptr;
    float* logits = nullptr;      // Vp floats of the last step
    int n_steps = 0;
};
// exchange words between the (value, index) pairs of the LM-head pick: one CTA's
// pair per 128-byte line (a line shared by several writers is slow to poll)
constexpr int kPersistLmStride = 16;
bool persist_supported(int C, int NH, int hs, int maxT, int splits, int nsm, int L);
// Fills out[2L+1] with the LayerNorm exponents of PersistParams::ln_exp from BF16 LayerNorm
// parameters (ln1w/ln1b/ln2w/ln2b: L x C, lnfw/lnfb: C).
cudaError_t persist_ln_exponents(int* out, const void* ln1w, const void* ln1b, const void* ln2w, const void* ln2b,
                                 const void* lnfw, const void* lnfb, int L, int C, cudaStream_t st);
int persist_max_splits();
int persist_max_stages();
bool persist_narrow(int C, int kv_rows, int tp);  // the launch takes the narrow (CUDA-core) kernel
int persist_stage_bytes(int wk, int C);  // one ring stage: 16 row-units of C weights + bias/scale tail
// Weight bytes the ring holds at most: deeper look-ahead measured slower on B200 (GPT-2 124M:
// 4 BF16 / 8 INT8 stages beat the 7 / 14 that fit; the extra copies only add HBM traffic
// while the CTAs wait on exchange words).
constexpr int kPersistRingBytes = 104 * 1024;
int persist_smem_bytes(int wk, int kv, int C, int nsw, int kv_rows, int tp);  // -1: unsupported, or no fit
cudaError_t launch_persistent(int wk, int kv, const PersistParams& P, cudaStream_t st);

// per-translation-unit device error readers
int gemv_device_error();
int attention_device_error();
int norm_device_error();
int sampler_device_error();
int persistent_device_error();

// Chooses rows per tile / stages / grid for an M x K matrix of kind wk.
// Returns false when the shape cannot be tiled (row larger than a tile).
bool plan_gemv(GemvParams& p, int wk, int nsm, bool single_wave);
size_t gemv_smem_bytes(const GemvParams& p, int wk);
// Dispatches to the kernel instance for (wk, output float?, prologue, epilogue).
cudaError_t launch_gemv(const GemvParams& p, int wk, bool out_f32, int pro, int epi, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------------------
// Prompt prefill on the tensor cores (prefill.cu)
// ---------------------------------------------------------------------------
// One tcgen05 GEMM launch: out[T x N] = epilogue(A[T x K] . W[N x K]^T).
struct TcGemmArgs {
    int T = 0, N = 0, K = 0;      // token rows, output columns, reduction
    const void* bias = nullptr;   // N, BF16 (may be null)
    const float* scale = nullptr; // N per-row scales of 8-bit weights
    void* out = nullptr;          // T x ldo: BF16, or FP32 for the LM-head form
    void* pre_gelu = nullptr;     // T x ldo BF16 pre-activation (may be null)
    int ldo = 0;
    int do_gelu = 0;
};
// Tensor maps of one GEMM (A: BF16 activations [act_rows x K], B: weights
// [N x K] BF16 or 8-bit codes); either pointer may be null to skip its map.
bool tc_maps(CUtensorMap* a, CUtensorMap* b, int wk, const void* act, int act_rows, const void* W, int N, int K,
             bool out_f32);
cudaError_t launch_tc_gemm(int wk, const CUtensorMap& a, const CUtensorMap& b, const TcGemmArgs& g, bool out_f32,
                           cudaStream_t st);

struct PrefillLayer {
    CUtensorMap w_qkv, w_proj, w_fc, w_fcproj;  // weight maps of this layer
    const void *qkvb = nullptr, *projb = nullptr, *fcb = nullptr, *fcprojb = nullptr;
    const float *s_qkv = nullptr, *s_proj = nullptr, *s_fc = nullptr, *s_fcproj = nullptr;  // 8-bit row scales
    const void *ln1w = nullptr, *ln1b = nullptr, *ln2w = nullptr, *ln2b = nullptr;
    unsigned char* kv = nullptr;  // this layer's [K|V][head][maxT][64] cache
    float* kv_scale = nullptr;    // and its 8-bit row scales [K|V][head][maxT]
};
struct PrefillPlan {
    int wk = 0, kvk = 0, C = 0, NH = 0, L = 0, V = 0, Vp = 0, maxT = 0;
    float attn_scale = 0.125f;
    // activation maps over maxT rows: x (LayerNorm outputs), atty, f (GELU outputs)
    CUtensorMap a_x, a_atty, a_f, w_lm;
    const float* s_lm = nullptr;
    void *res = nullptr, *x = nullptr, *qkv = nullptr, *atty = nullptr, *proj = nullptr, *f = nullptr;  // BF16 rows
    float* logits_rows = nullptr;  // maxT x Vp
    const int* tokens = nullptr;   // device prompt
    const void* wte = nullptr;     // BF16 rows or 8-bit codes
    const float* wte_scale = nullptr;
    const void* wpe = nullptr;
    const void *lnfw = nullptr, *lnfb = nullptr;
    float* logits_last = nullptr;  // the engine's logits (Vp) receive row T-1
    int *d_token = nullptr, *d_pos = nullptr, *history = nullptr;
    std::vector<PrefillLayer> layers;
};
bool prefill_supported(int wk, int kvk, int C, int NH, int maxT);
// The whole prompt (positions 0..T-1) in one pass: KV cache filled, logits of
// every prompt row in logits_rows, the engine's token/position/history
// advanced to position T with the greedy pick of row T-1.
cudaError_t run_prefill(const PrefillPlan& P, int T, cudaStream_t st);
int prefill_device_error();

}  // namespace gpt2b
