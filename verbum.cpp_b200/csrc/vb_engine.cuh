// vb_engine.cuh -- device-resident state of one decode engine (one GPU).
#pragma once

#include <vector>

#include "vb_kernels.cuh"

// HBM layout (all row-major, HF [out, in] orientation):
//   wqkv  [L][(H+2KVH)*D, hidden]   q | k | v rows of each layer stacked
//   wo    [L][hidden, H*D]
//   wgu   [L][2*ffn, hidden]        gate row j at 2j, up row j at 2j+1
//   wd    [L][hidden, ffn]
// (INT8 mode: the same shapes as int8 plus one f32 scale per row.)
//   embed [vocab, hidden] f32 (tied lm_head)
//   kc/vc [L][B][KVH][max_seq][D] f32 -- one contiguous stream per (layer,
//          sequence, kv head), so a split of the attention reads one span.
struct vb_layer_dev {
    float* in_norm;
    float* post_norm;
    float* q_norm;
    float* k_norm;
    float* wqkv;
    float* wo;
    float* wgu;
    float* wd;
    int8_t* qqkv;
    int8_t* qo;
    int8_t* qgu;
    int8_t* qd;
    float* sqkv;
    float* so;
    float* sgu;
    float* sd;
};

struct vb_engine {
    vb_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    bool quantized = false;
    int path = 1;          // effective step path (1, 2)
    bool path_auto = true; // pick the path per weight format at graph build

    // sizes
    int qkv_rows = 0;    // (H + 2 KVH) * D
    int q_width = 0;     // H * D
    int kv_width = 0;    // KVH * D
    size_t per_layer_f32 = 0;  // floats of projections per layer
    size_t per_layer_i8 = 0;   // bytes of int8 projections per layer
    size_t per_layer_rows = 0; // scale entries per layer

    // weights
    float* embed = nullptr;
    float* final_norm = nullptr;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    float* norms = nullptr;    // all per-layer norm vectors
    float* wf32 = nullptr;     // all f32 projections
    int8_t* wi8 = nullptr;     // all int8 projections
    float* wscale = nullptr;   // all scales
    // opt-in INT8 copy of the tied lm_head (the embedding lookup stays f32)
    void* stage = nullptr;     // bf16 upload staging
    size_t stage_bytes = 0;
    int8_t* lm_q8 = nullptr;
    float* lm_sc = nullptr;
    bool lm_int8 = false;
    std::vector<vb_layer_dev> L;
    std::vector<int> layer_set;
    bool globals_set = false;

    // cache (batch 1)
    int max_seq = 0;
    int len = 0;
    float* kc = nullptr;
    float* vc = nullptr;

    // scratch
    float* x = nullptr;
    float* qkv = nullptr;
    float* q = nullptr;
    float* ctx = nullptr;
    float* h = nullptr;
    float* logits = nullptr;
    float* attn_ws = nullptr;
    int attn_splits = 1;
    float* part_val = nullptr;
    int* part_idx = nullptr;
    int* d_tok = nullptr;
    int* d_pos = nullptr;
    int* d_next = nullptr;
    int* d_err = nullptr;
    int* d_hist = nullptr;     // decode history [max_seq]
    int* d_step = nullptr;     // decode history write index
    int* h_pinned_i = nullptr; // pinned host staging
    float* h_logits = nullptr;

    cudaGraphExec_t graph = nullptr;
    int graph_nodes = 0;
    int* d_prompt = nullptr;   // prefill tokens [max_seq]

    // clustered persistent step (vb_mega2.cu)
    void* mega2 = nullptr;
    bool trace_on = false;
};

namespace vb {
// Enqueue one full decode step (token in d_tok, position in d_pos) using the
// per-op kernels.  Leaves logits in e->logits and the greedy pick in d_next,
// then advances d_pos / d_tok and appends the pick to the history.
vb_status enqueue_step_ops(vb_engine* e, cudaStream_t s);
// Clustered persistent step (vb_mega2.cu). Returns VB_ERR_UNSUPPORTED when
// the shapes are outside what it handles.
vb_status mega2_prepare(vb_engine* e);
vb_status mega2_enqueue_step(vb_engine* e, cudaStream_t s);
void mega2_release(vb_engine* e);
void mega2_reset_counters(vb_engine* e);
// Sets the clustered step's failure-test hook word (ordered on s).
vb_status mega2_set_fault(int v, cudaStream_t s);
int mega2_read_trace(vb_engine* e, unsigned long long* host, int cap);
std::string mega2_debug(vb_engine* e);
vb_status engine_check_err(vb_engine* e);
void build_rope_table_host(int head_dim, int max_pos, float theta, float* c, float* s);
// Device sampling (vb_sample.cu).
bool sampler_greedy(const vb_sampler* sp);
// n draws of the sampler's generator, uploaded for the next n samples.
vb_status sampler_draws(vb_sampler* sp, int n, cudaStream_t s);
// Sample logits [vocab] with draw `draw`; the pick goes to *out and, when tok
// is set, into tok / next and hist[*step - 1].
vb_status launch_sample(vb_sampler* sp, const float* logits, int64_t vocab, int draw, int* out, int* tok, int* next,
                        int* hist, const int* step, int hist_cap, cudaStream_t s);
}  // namespace vb
