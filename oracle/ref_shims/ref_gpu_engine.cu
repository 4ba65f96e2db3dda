/* The reference decode engine (inference_gpt2_opt.cu) compiled in place for
 * sm_100a with one of the reference's precision flag sets (Makefile:78-105).
 * Its main() is renamed; the entry points below drive the reference's own
 * loader (gpt2_build_from_checkpoint / gpt2_build_w8), its one-step forward
 * forward_kv_graph_ready (with is_capturing=true, i.e. the split+merge path the
 * CUDA graphs use, :336-341) and its stock graph generation loop
 * run_generation_once_graph (:525-596).
 * TEST INFRASTRUCTURE: a second oracle and the timing bar on the GPU box. */
#include "ref_api.h"
#include "fp8_compat.h"
#include <unistd.h>
#define main ref_opt_main
#include "inference_gpt2_opt.cu"
#undef main

static GPT2 g_ref_model;
static floatX* g_ref_kv = nullptr;
static float* g_ref_po = nullptr;
static float* g_ref_pl = nullptr;
static float* g_ref_pm = nullptr;
static const int g_ref_S = 8; /* inference_gpt2_opt.cu:711 */

REFAPI int ref_engine_init(const char* model_path, int use_w8) {
    common_start(false);
    gpt2_init_common(&g_ref_model);
#ifdef USE_W8
    if (use_w8) {
        g_use_w8 = true;
        std::string w8_path = model_path;
        std::string scale_path = w8_path.substr(0, w8_path.size() - 4) + "_scales.bin";
        gpt2_build_w8(&g_ref_model, w8_path.c_str(), scale_path.c_str());
    } else
#endif
    {
        (void)use_w8;
        gpt2_build_from_checkpoint(&g_ref_model, model_path);
    }
    gpt2_allocate_state(&g_ref_model, 1, 1);
    const GPT2Config& c = g_ref_model.config;
    size_t kv_bytes = 2 * (size_t)c.num_layers * c.num_heads * c.max_seq_len * (c.channels / c.num_heads) *
                      sizeof(floatX);
#if defined(USE_KV_W8)
    if (g_use_w8) kv_bytes /= 2;
    if (g_use_w8)
        cudaCheck(cudaMalloc((void**)&g_kv_scale, 2 * (size_t)c.num_layers * c.num_heads * c.max_seq_len *
                                                      sizeof(float)));
#endif
    cudaCheck(cudaMalloc((void**)&g_ref_kv, kv_bytes));
    cudaCheck(cudaMalloc((void**)&g_ref_po, c.num_heads * g_ref_S * (c.channels / c.num_heads) * sizeof(float)));
    cudaCheck(cudaMalloc((void**)&g_ref_pl, c.num_heads * g_ref_S * sizeof(float)));
    cudaCheck(cudaMalloc((void**)&g_ref_pm, c.num_heads * g_ref_S * sizeof(float)));
    return 0;
}

REFAPI void ref_engine_config(int* cfg) {
    const GPT2Config& c = g_ref_model.config;
    cfg[0] = c.max_seq_len; cfg[1] = c.vocab_size; cfg[2] = c.num_layers;
    cfg[3] = c.num_heads; cfg[4] = c.channels; cfg[5] = c.padded_vocab_size;
}

/* One forward of `token` at position `pos`; copies Vp float logits to host. */
REFAPI int ref_engine_step(int token, int pos, float* logits_host) {
    cudaCheck(cudaMemcpy(g_ref_model.inputs, &token, sizeof(int), cudaMemcpyHostToDevice));
    cudaCheck(cudaMemcpyToSymbol(g_cur_len, &pos, sizeof(int)));
    forward_kv_graph_ready(&g_ref_model, pos, g_ref_kv, g_ref_po, g_ref_pl, g_ref_pm, g_ref_S, main_stream, true);
    cudaCheck(cudaStreamSynchronize(main_stream));
    if (logits_host)
        cudaCheck(cudaMemcpy(logits_host, g_ref_model.acts.logits,
                             (size_t)g_ref_model.config.padded_vocab_size * sizeof(float), cudaMemcpyDeviceToHost));
    return 0;
}

/* The reference's own --graph --bench loop: capture both graphs, then `runs`
 * timed generations of genT-1 tokens each (run_generation_once_graph).  Writes
 * the wall ms of every run.  The loop writes its t=1 logits dump under the
 * current directory, so it runs from `workdir`. */
REFAPI int ref_engine_bench_graph(int genT, int runs, double* wall_ms, const char* workdir) {
    char old[4096];
    if (!getcwd(old, sizeof(old))) return 1;
    if (workdir && chdir(workdir) != 0) return 2;
    graph_capture_all(&g_ref_model, g_ref_kv, g_ref_po, g_ref_pl, g_ref_pm, g_ref_S, main_stream);
    const int maxT = g_ref_model.config.max_seq_len;
    int* gen_tokens = (int*)malloc((size_t)(maxT + 1) * sizeof(int));
    int* d_token;
    cudaCheck(cudaMalloc((void**)&d_token, sizeof(int)));
    Tokenizer tok;
    memset(&tok, 0, sizeof(tok));
    for (int r = 0; r < runs; r++)
        wall_ms[r] = run_generation_once_graph(&g_ref_model, &tok, gen_tokens, d_token, genT, 50256, true,
                                               g_ref_kv, g_ref_po, g_ref_pl, g_ref_pm, g_ref_S);
    cudaCheck(cudaFree(d_token));
    free(gen_tokens);
    if (chdir(old) != 0) return 3;
    return 0;
}
