// vb_engine.cu -- batch-1 decode engine: weights, KV cache and scratch in
// HBM; one step = embedding -> L x (fused-norm QKV GEMV, q/k norm + RoPE + KV
// append, split-K attention, o_proj + residual, fused-norm gate/up + SwiGLU,
// down + residual) -> fused-norm lm_head with argmax partials -> argmax.
// The step reads its token and position from device memory, so the whole
// step is captured once in a CUDA graph and replayed; greedy decode feeds
// each argmax back on the device with no host round trip.
//
// Mirrors verbum::Model (core/include/verbum/model.h:47-116): to_cuda
// (model.cpp:367-443), reset_cache (277-282), step / step_cuda (284-311,
// 446-497), quantize (313-338), weight_bytes (340-365).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <string>

#include <stdlib.h>

#include "vb_engine.cuh"

namespace vb {

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

template <class T>
vb_status dalloc(T** p, size_t count, const char* what) {
    *p = nullptr;
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, what);
    return VB_OK;
}

template <class T>
void dfree(T*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

// pos += 1, token = pick, history[step++] = pick  (single thread).
__global__ void engine_advance_kernel(int* pos, int* tok, const int* next, int* hist,
                                      int* step, int hist_cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const int t = *next;
        *pos += 1;
        *tok = t;
        const int s = *step;
        if (s >= 0 && s < hist_cap) hist[s] = t;
        *step = s + 1;
    }
}

void free_cache(vb_engine* e) {
    dfree(e->kc);
    dfree(e->vc);
    dfree(e->attn_ws);
    dfree(e->d_hist);
    dfree(e->d_prompt);
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
}

}  // namespace

void build_rope_table_host(int head_dim, int max_pos, float theta, float* c, float* s) {
    // nn.cpp:44-74: inv_freq = 1 / theta^(2i/D) in double, angle in double,
    // cos/sin rounded to float, the same value stored for i and i + D/2.
    const int half = head_dim / 2;
    for (int pos = 0; pos < max_pos; pos++) {
        for (int i = 0; i < half; i++) {
            const double inv_freq =
                1.0 / std::pow((double)theta, (double)(2 * i) / (double)head_dim);
            const double angle = (double)pos * inv_freq;
            const float cv = (float)std::cos(angle);
            const float sv = (float)std::sin(angle);
            const size_t b = (size_t)pos * head_dim;
            c[b + i] = cv;
            c[b + i + half] = cv;
            s[b + i] = sv;
            s[b + i + half] = sv;
        }
    }
}

vb_status engine_check_err(vb_engine* e) {
    int err = 0;
    VB_CUDA_TRY(cudaMemcpy(&err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err == kErrNone) return VB_OK;
    const std::string where = mega2_debug(e);
    cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream);
    cudaStreamSynchronize(e->stream);
    mega2_reset_counters(e);  // a step that stopped early leaves its tickets set
    switch (err) {
        case kErrBadToken:
            return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
        case kErrCacheFull: return fail(VB_ERR_CACHE_FULL, "kv cache is full");
        case kErrBarrierTimeout:
            return fail(VB_ERR_TIMEOUT, "fused step: grid barrier wait timed out" + where);
        case kErrPipeTimeout:
            return fail(VB_ERR_TIMEOUT, "fused step: stage pipeline wait timed out" + where);
        default: return fail(VB_ERR_CUDA, "device error word set: " + std::to_string(err));
    }
}

// A layer projection of the per-op step: the prefetching GEMV (weights in
// shared memory before it waits for the previous kernel) when its slices fit,
// the streaming GEMV otherwise.
// Weights of GEMV number j of the step (4 per layer: q|k|v, o, gate|up,
// down; then the lm_head): base pointer and bytes, for the L2 look-ahead.
static void step_weights(const vb_engine* e, int j, const void** w, size_t* bytes) {
    const vb_config& c = e->cfg;
    const bool q8 = e->quantized;
    const size_t es = q8 ? 1 : 4, hd = c.hidden;
    *w = nullptr;
    *bytes = 0;
    const int l = j / 4, k = j % 4;
    if (l >= c.layers) {  // the lm_head: its first part (it streams the rest at full rate)
        const size_t lm = (size_t)c.vocab * hd * (e->lm_int8 ? 1 : 4);
        const size_t part = (size_t)48 << 20;
        const size_t off = (size_t)(j - 4 * c.layers) * part;
        if (off < lm) {
            *w = static_cast<const char*>(e->lm_int8 ? (const void*)e->lm_q8 : (const void*)e->embed) + off;
            *bytes = lm - off < part ? lm - off : part;
        }
        return;
    }
    const vb_layer_dev& L = e->L[l];
    switch (k) {
        case 0: *w = q8 ? (const void*)L.qqkv : (const void*)L.wqkv; *bytes = (size_t)e->qkv_rows * hd * es; break;
        case 1: *w = q8 ? (const void*)L.qo : (const void*)L.wo; *bytes = hd * e->q_width * es; break;
        case 2: *w = q8 ? (const void*)L.qgu : (const void*)L.wgu; *bytes = 2 * (size_t)c.ffn * hd * es; break;
        default: *w = q8 ? (const void*)L.qd : (const void*)L.wd; *bytes = hd * (size_t)c.ffn * es; break;
    }
}

// step_gemv takes the prefetching GEMV for this shape
static bool step_gemv_pf_fits(const vb_engine*, int N, int K, bool q8, int epi) {
    return K <= 4096 && gemv_pf_parts(N, K, q8, epi) > 0;
}

static vb_status step_gemv(vb_engine* e, int j, GemvArgs g, bool q8, int pro, int epi, cudaStream_t s) {
    g.err = e->d_err;
    // two GEMVs ahead (measured: without it INT8 per-op 1005 against 1033 tok/s)
    // (one or three ahead measured the same within 2 %)
    step_weights(e, j + 2, &g.l2_ahead, &g.l2_ahead_bytes);
    if (step_gemv_pf_fits(e, g.N, g.K, q8, epi)) return launch_gemv_pf(g, q8, pro, epi, s);
    return launch_gemv(g, q8, pro, epi, s);
}

// The projection k of layer l (0 q|k|v with the input RMSNorm, 1 o with the
// residual, 2 gate/up with the post-attention RMSNorm and SwiGLU, 3 down with
// the residual) as a batch-1 GEMV.
static GemvArgs layer_gemv(const vb_engine* e, int l, int k, int* pro, int* epi) {
    const vb_config& c = e->cfg;
    const bool q8 = e->quantized;
    const vb_layer_dev& L = e->L[l];
    GemvArgs g{};
    g.eps = c.eps;
    g.err = e->d_err;
    switch (k) {
        case 0: {
            const size_t layer_kv = (size_t)c.kv_heads * e->max_seq * c.head_dim;
            g.x = e->x;
            g.norm_w = L.in_norm;
            g.W = q8 ? (const void*)L.qqkv : (const void*)L.wqkv;
            g.scales = L.sqkv;
            g.y = e->qkv;
            g.N = e->qkv_rows;
            g.K = c.hidden;
            // this layer's cached K / V rows into L2 for the attention after it
            g.kv_k = e->kc + l * layer_kv;
            g.kv_v = e->vc + l * layer_kv;
            g.kv_pos = e->d_pos;
            g.kv_heads = c.kv_heads;
            g.kv_stride_h = (int64_t)e->max_seq * c.head_dim;
            *pro = kProRms;
            *epi = kEpiStore;
            break;
        }
        case 1:
            g.x = e->ctx;
            g.attn_parts = e->attn_ws;
            g.attn_splits = e->attn_splits;
            g.W = q8 ? (const void*)L.qo : (const void*)L.wo;
            g.scales = L.so;
            g.y = e->x;
            g.N = c.hidden;
            g.K = e->q_width;
            *pro = kProNone;
            *epi = kEpiResidual;
            break;
        case 2:
            g.x = e->x;
            g.norm_w = L.post_norm;
            g.W = q8 ? (const void*)L.qgu : (const void*)L.wgu;
            g.scales = L.sgu;
            g.y = e->h;
            g.N = 2 * c.ffn;
            g.K = c.hidden;
            *pro = kProRms;
            *epi = kEpiSwiGLU;
            break;
        default:
            g.x = e->h;
            g.W = q8 ? (const void*)L.qd : (const void*)L.wd;
            g.scales = L.sd;
            g.y = e->x;
            g.N = c.hidden;
            g.K = c.ffn;
            *pro = kProNone;
            *epi = kEpiResidual;
            break;
    }
    return g;
}

// One decode step of the per-op path.  Per layer: q|k|v GEMV -> split
// attention (q/k norm, RoPE and cache append inside) [-> split merge] -> o ->
// gate/up -> down.  (o, gate/up, down and the next layer's q|k|v as one launch
// with grid barriers between them, every INT8 slice in shared memory from
// the start, measured slower: INT8 per-op 1181 -> 885 tok/s.)
vb_status enqueue_step_ops(vb_engine* e, cudaStream_t s) {
    const vb_config& c = e->cfg;
    const bool q8 = e->quantized;
    vb_status st;
    if ((st = launch_embed(e->embed, e->d_tok, 1, c.hidden, c.vocab, e->x, e->d_err, s))) return st;
    const size_t layer_kv = (size_t)c.kv_heads * e->max_seq * c.head_dim;
    // With few splits the o projection merges the split partials in its
    // prologue: one launch fewer on the step's dependency chain (f32 at
    // 3 splits, context <= 168: 1136 -> 1162 tok/s).  Every CTA merges all
    // heads, a serial pass over the splits: at 13 splits (INT8, context
    // ~770) that measured slower than the merge launch (1185 -> 1052).
    const bool merge_in_o = e->attn_splits <= 4 && step_gemv_pf_fits(e, c.hidden, e->q_width, q8, kEpiResidual);
    for (int l = 0; l < c.layers; l++) {
        const vb_layer_dev& L = e->L[l];
        int pro = 0, epi = 0;
        {
            const GemvArgs g = layer_gemv(e, l, 0, &pro, &epi);
            if ((st = step_gemv(e, 4 * l + 0, g, q8, pro, epi, s))) return st;
        }

        QkNormArgs qa{};
        qa.qkv = e->qkv;
        qa.q_norm = L.q_norm;
        qa.k_norm = L.k_norm;
        qa.cos_tab = e->rope_cos;
        qa.sin_tab = e->rope_sin;
        qa.pos = e->d_pos;
        qa.q_out = e->q;
        qa.kc = e->kc + l * layer_kv;
        qa.vc = e->vc + l * layer_kv;
        qa.stride_b = (int64_t)layer_kv;
        qa.stride_pos = c.head_dim;
        qa.stride_h = (int64_t)e->max_seq * c.head_dim;
        qa.B = 1;
        qa.H = c.heads;
        qa.KVH = c.kv_heads;
        qa.D = c.head_dim;
        qa.rope_positions = std::min(c.rope_positions, e->max_seq);
        qa.eps = c.eps;
        qa.err = e->d_err;

        // the q/k norm, RoPE and cache append run inside the attention kernel
        AttnArgs aa{};
        aa.fuse_qk = 1;
        aa.qk = qa;
        aa.q = e->q;
        aa.k = qa.kc;
        aa.v = qa.vc;
        aa.out = e->ctx;
        aa.lens = nullptr;
        aa.pos = e->d_pos;
        aa.B = 1;
        aa.H = c.heads;
        aa.KVH = c.kv_heads;
        aa.D = c.head_dim;
        aa.n_max = e->max_seq;
        aa.stride_b = qa.stride_b;
        aa.stride_pos = qa.stride_pos;
        aa.stride_h = qa.stride_h;
        aa.splits = e->attn_splits;
        aa.ws = e->attn_ws;
        // the positions come from the previous step: the first cached rows and
        // the rope row are requested before the kernel waits for q|k|v
        // (INT8 per-op step 1059 -> 1085 tok/s).  Merging the splits in the
        // last split CTA instead of the merge kernel measured slower (1031):
        // its fence and ticket round trip cost more than the launch.
        aa.pos_stable = 1;
        aa.no_merge = merge_in_o ? 1 : 0;
        if ((st = launch_attention(aa, s))) return st;

        for (int k = 1; k <= 3; k++) {
            GemvArgs g = layer_gemv(e, l, k, &pro, &epi);
            if (k == 1 && merge_in_o) pro = kProMerge;
            if ((st = step_gemv(e, 4 * l + k, g, q8, pro, epi, s))) return st;
        }
    }
    GemvArgs lm{};
    lm.x = e->x;
    lm.norm_w = e->final_norm;
    lm.eps = c.eps;
    lm.W = e->lm_int8 ? static_cast<const void*>(e->lm_q8) : static_cast<const void*>(e->embed);
    lm.scales = e->lm_int8 ? e->lm_sc : nullptr;
    lm.y = e->logits;
    lm.N = c.vocab;
    lm.K = c.hidden;
    lm.part_val = e->part_val;
    lm.part_idx = e->part_idx;
    int parts = 0;
    if ((st = launch_gemv(lm, e->lm_int8, kProRms, kEpiArgmax, s, &parts))) return st;
    if ((st = launch_argmax_parts(e->part_val, e->part_idx, parts, e->d_next, s))) return st;
    engine_advance_kernel<<<1, 32, 0, s>>>(e->d_pos, e->d_tok, e->d_next, e->d_hist, e->d_step,
                                           e->max_seq);
    VB_LAUNCH_CHECK("engine_advance_kernel");
    return VB_OK;
}

// One decode step on e->stream: the captured graph, or (VB_STEP_DIRECT=1 in
// the environment, for profilers that cannot follow a cooperative launch
// inside a graph) the same launches issued directly.
static vb_status launch_step(vb_engine* e) {
    static const bool direct = [] {
        const char* v = getenv("VB_STEP_DIRECT");
        return v && v[0] == '1';
    }();
    // failure-path test: the armed step's CTA 0 waits for an exchange word
    // nothing writes (the hook word is written and complete before the launch)
    const bool inject = e->path == 2 && e->mega2 && fault_take(kFaultStepExchange);
    if (inject) {
        vb_status st = mega2_set_fault(1, e->stream);
        if (st) return st;
        VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    }
    vb_status st = VB_OK;
    if (!direct) {
        const cudaError_t ce = cudaGraphLaunch(e->graph, e->stream);
        if (ce != cudaSuccess) st = cuda_fail(ce, "cudaGraphLaunch");
    } else {
        st = (e->path == 2 && e->mega2) ? mega2_enqueue_step(e, e->stream) : enqueue_step_ops(e, e->stream);
    }
    if (inject) {
        const vb_status s2 = mega2_set_fault(0, e->stream);
        if (!st) st = s2;
    }
    return st;
}

static vb_status ensure_graph(vb_engine* e) {
    if (e->graph) return VB_OK;
    cudaGraph_t g = nullptr;
    VB_CUDA_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    vb_status st = (e->path == 2 && e->mega2) ? mega2_enqueue_step(e, e->stream)
                                              : enqueue_step_ops(e, e->stream);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    e->graph_nodes = (int)nn;
    ce = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) {
        e->graph = nullptr;
        return cuda_fail(ce, "cudaGraphInstantiate");
    }
    return VB_OK;
}

static vb_status check_ready(vb_engine* e) {
    if (!e->globals_set) return fail(VB_ERR_STATE, "engine weights not uploaded (set_globals)");
    for (int l = 0; l < e->cfg.layers; l++)
        if (!e->layer_set[l]) return fail(VB_ERR_STATE, "layer " + std::to_string(l) + " not uploaded");
    if (!e->kc) return fail(VB_ERR_NO_CACHE, "call reset_cache() first");
    return VB_OK;
}

}  // namespace vb

using namespace vb;

extern "C" {

vb_status vb_engine_create(const vb_config* cfg, int device, vb_engine** out) {
    if (!cfg || !out) return fail(VB_ERR_ARG, "null argument");
    *out = nullptr;
    const vb_config& c = *cfg;
    if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.ffn <= 0 ||
        c.vocab <= 0 || c.rope_positions <= 0)
        return fail(VB_ERR_ARG, "config has a non-positive dimension");
    if (c.head_dim != 128) return fail(VB_ERR_UNSUPPORTED, "head_dim must be 128");
    if (c.heads % c.kv_heads) return fail(VB_ERR_ARG, "attention heads must be a multiple of kv heads");
    const int G = c.heads / c.kv_heads;
    if (G != 1 && G != 2 && G != 4) return fail(VB_ERR_UNSUPPORTED, "GQA group must be 1, 2 or 4");
    if (c.hidden % 32 || c.ffn % 32) return fail(VB_ERR_UNSUPPORTED, "hidden and ffn must be multiples of 32");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(VB_ERR_CUDA, "no CUDA device found");
    if (device < 0 || device >= ndev) return fail(VB_ERR_ARG, "device index out of range");
    DeviceGuard dg(device);

    vb_engine* e = new vb_engine();
    e->cfg = c;
    e->device = device;
    e->qkv_rows = (c.heads + 2 * c.kv_heads) * c.head_dim;
    e->q_width = c.heads * c.head_dim;
    e->kv_width = c.kv_heads * c.head_dim;
    const size_t hd = c.hidden;
    e->per_layer_f32 = (size_t)e->qkv_rows * hd + hd * e->q_width + 2 * (size_t)c.ffn * hd +
                       hd * (size_t)c.ffn;
    e->per_layer_i8 = e->per_layer_f32;
    e->per_layer_rows = (size_t)e->qkv_rows + hd + 2 * (size_t)c.ffn + hd;
    e->L.resize(c.layers);
    e->layer_set.assign(c.layers, 0);

    vb_status st = VB_OK;
    auto bail = [&](vb_status s) {
        vb_engine_destroy(e);
        return s;
    };
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(VB_ERR_CUDA, "cudaStreamCreate failed"));
    if ((st = dalloc(&e->embed, (size_t)c.vocab * hd, "embed"))) return bail(st);
    if ((st = dalloc(&e->final_norm, hd, "final_norm"))) return bail(st);
    const size_t rope_n = (size_t)c.rope_positions * c.head_dim;
    if ((st = dalloc(&e->rope_cos, rope_n, "rope"))) return bail(st);
    if ((st = dalloc(&e->rope_sin, rope_n, "rope"))) return bail(st);
    {
        std::vector<float> hc(rope_n), hs(rope_n);
        build_rope_table_host(c.head_dim, c.rope_positions, c.theta, hc.data(), hs.data());
        if (cudaMemcpy(e->rope_cos, hc.data(), rope_n * 4, cudaMemcpyHostToDevice) ||
            cudaMemcpy(e->rope_sin, hs.data(), rope_n * 4, cudaMemcpyHostToDevice))
            return bail(fail(VB_ERR_CUDA, "rope table upload failed"));
    }
    const size_t norms_per_layer = 2 * hd + 2 * (size_t)c.head_dim;
    if ((st = dalloc(&e->norms, norms_per_layer * c.layers, "norms"))) return bail(st);
    if ((st = dalloc(&e->wf32, e->per_layer_f32 * c.layers, "f32 projections"))) return bail(st);
    for (int l = 0; l < c.layers; l++) {
        vb_layer_dev& L = e->L[l];
        float* nb = e->norms + norms_per_layer * l;
        L.in_norm = nb;
        L.post_norm = nb + hd;
        L.q_norm = nb + 2 * hd;
        L.k_norm = nb + 2 * hd + c.head_dim;
        float* wb = e->wf32 + e->per_layer_f32 * l;
        L.wqkv = wb;
        L.wo = L.wqkv + (size_t)e->qkv_rows * hd;
        L.wgu = L.wo + hd * e->q_width;
        L.wd = L.wgu + 2 * (size_t)c.ffn * hd;
    }
    if ((st = dalloc(&e->x, hd, "x"))) return bail(st);
    if ((st = dalloc(&e->qkv, e->qkv_rows, "qkv"))) return bail(st);
    if ((st = dalloc(&e->q, e->q_width, "q"))) return bail(st);
    if ((st = dalloc(&e->ctx, e->q_width, "ctx"))) return bail(st);
    if ((st = dalloc(&e->h, c.ffn, "h"))) return bail(st);
    if ((st = dalloc(&e->logits, c.vocab, "logits"))) return bail(st);
    const int parts = std::max(gemv_grid(c.vocab, false, kEpiArgmax), gemv_grid(c.vocab, true, kEpiArgmax));
    if ((st = dalloc(&e->part_val, parts, "argmax parts"))) return bail(st);
    if ((st = dalloc(&e->part_idx, parts, "argmax parts"))) return bail(st);
    if ((st = dalloc(&e->d_tok, 1, "tok"))) return bail(st);
    if ((st = dalloc(&e->d_pos, 1, "pos"))) return bail(st);
    if ((st = dalloc(&e->d_next, 1, "next"))) return bail(st);
    if ((st = dalloc(&e->d_err, 1, "err"))) return bail(st);
    if ((st = dalloc(&e->d_step, 1, "step"))) return bail(st);
    // every memset goes on the engine's own stream (non-blocking: it does not
    // order with the legacy default stream) and is waited for here
    if (cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream) ||
        cudaMemsetAsync(e->d_pos, 0, sizeof(int), e->stream) ||
        cudaStreamSynchronize(e->stream))
        return bail(fail(VB_ERR_CUDA, "engine state init failed"));
    if (cudaMallocHost(&e->h_pinned_i, 64 * sizeof(int)) != cudaSuccess)
        return bail(fail(VB_ERR_CUDA, "cudaMallocHost failed"));
    *out = e;
    return VB_OK;
}

vb_status vb_engine_destroy(vb_engine* e) {
    if (!e) return VB_OK;
    DeviceGuard dg(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    mega2_release(e);
    free_cache(e);
    dfree(e->embed); dfree(e->final_norm); dfree(e->rope_cos); dfree(e->rope_sin);
    dfree(e->norms); dfree(e->wf32); dfree(e->wi8); dfree(e->wscale); dfree(e->lm_q8); dfree(e->lm_sc);
    if (e->stage) cudaFree(e->stage);
    dfree(e->x); dfree(e->qkv); dfree(e->q); dfree(e->ctx); dfree(e->h); dfree(e->logits);
    dfree(e->part_val); dfree(e->part_idx); dfree(e->d_tok); dfree(e->d_pos); dfree(e->d_next);
    dfree(e->d_err); dfree(e->d_step);
    if (e->h_pinned_i) cudaFreeHost(e->h_pinned_i);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return VB_OK;
}

vb_status vb_engine_set_globals(vb_engine* e, const float* embed, const float* final_norm) {
    if (!e || !embed || !final_norm) return fail(VB_ERR_ARG, "null argument");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    VB_CUDA_TRY(cudaMemcpy(e->embed, embed, (size_t)c.vocab * c.hidden * 4, cudaMemcpyHostToDevice));
    VB_CUDA_TRY(cudaMemcpy(e->final_norm, final_norm, (size_t)c.hidden * 4, cudaMemcpyHostToDevice));
    e->globals_set = true;
    return VB_OK;
}

namespace vb {
namespace {
// dst[r * ld + k] = widen(src[r * cols + k]) for r < rows, k < cols.
__global__ void widen_bf16_kernel(const uint16_t* src, int64_t rows, int64_t cols, float* dst, int64_t ld) {
    const int64_t n = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, k = i - r * cols;
        dst[r * ld + k] = __uint_as_float((unsigned)src[i] << 16);
    }
}
}  // namespace

// Uploads a bf16 [rows][cols] host tensor through a device staging buffer and
// widens it into dst (row stride ld floats).
vb_status upload_bf16(vb_engine* e, const uint16_t* host, int64_t rows, int64_t cols, float* dst, int64_t ld) {
    const size_t bytes = (size_t)rows * cols * 2;
    if (e->stage_bytes < bytes) {
        if (e->stage) cudaFree(e->stage);
        e->stage = nullptr;
        e->stage_bytes = 0;
        VB_CUDA_TRY(cudaMalloc(&e->stage, bytes));
        e->stage_bytes = bytes;
    }
    VB_CUDA_TRY(cudaMemcpyAsync(e->stage, host, bytes, cudaMemcpyHostToDevice, e->stream));
    widen_bf16_kernel<<<1184, 256, 0, e->stream>>>(static_cast<const uint16_t*>(e->stage), rows, cols, dst, ld);
    VB_LAUNCH_CHECK("widen_bf16_kernel");
    // the staging buffer is reused by the next call: keep the copies ordered
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    return VB_OK;
}
}  // namespace vb

vb_status vb_engine_set_globals_bf16(vb_engine* e, const uint16_t* embed, const uint16_t* final_norm) {
    if (!e || !embed || !final_norm) return fail(VB_ERR_ARG, "null argument");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    vb_status st;
    if ((st = upload_bf16(e, embed, c.vocab, c.hidden, e->embed, c.hidden))) return st;
    if ((st = upload_bf16(e, final_norm, 1, c.hidden, e->final_norm, c.hidden))) return st;
    e->globals_set = true;
    return VB_OK;
}

vb_status vb_engine_set_layer_bf16(vb_engine* e, int layer, const vb_layer_host_bf16* w) {
    if (!e || !w) return fail(VB_ERR_ARG, "null argument");
    if (layer < 0 || layer >= e->cfg.layers) return fail(VB_ERR_ARG, "layer index out of range");
    if (e->quantized) return fail(VB_ERR_STATE, "engine already quantized; upload f32 layers first");
    if (!w->input_norm || !w->post_norm || !w->wq || !w->wk || !w->wv || !w->wo || !w->q_norm ||
        !w->k_norm || !w->wg || !w->wu || !w->wd)
        return fail(VB_ERR_ARG, "null weight pointer");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    const int64_t hd = c.hidden, D = c.head_dim;
    vb_layer_dev& L = e->L[layer];
    vb_status st;
    if ((st = upload_bf16(e, w->input_norm, 1, hd, L.in_norm, hd)) ||
        (st = upload_bf16(e, w->post_norm, 1, hd, L.post_norm, hd)) ||
        (st = upload_bf16(e, w->q_norm, 1, D, L.q_norm, D)) || (st = upload_bf16(e, w->k_norm, 1, D, L.k_norm, D)) ||
        (st = upload_bf16(e, w->wq, e->q_width, hd, L.wqkv, hd)) ||
        (st = upload_bf16(e, w->wk, e->kv_width, hd, L.wqkv + (size_t)e->q_width * hd, hd)) ||
        (st = upload_bf16(e, w->wv, e->kv_width, hd, L.wqkv + (size_t)(e->q_width + e->kv_width) * hd, hd)) ||
        (st = upload_bf16(e, w->wo, hd, e->q_width, L.wo, e->q_width)) ||
        // gate row j -> row 2j, up row j -> row 2j+1
        (st = upload_bf16(e, w->wg, c.ffn, hd, L.wgu, 2 * hd)) ||
        (st = upload_bf16(e, w->wu, c.ffn, hd, L.wgu + hd, 2 * hd)) ||
        (st = upload_bf16(e, w->wd, hd, c.ffn, L.wd, c.ffn)))
        return st;
    e->layer_set[layer] = 1;
    return VB_OK;
}

vb_status vb_engine_set_layer(vb_engine* e, int layer, const vb_layer_host* w) {
    if (!e || !w) return fail(VB_ERR_ARG, "null argument");
    if (layer < 0 || layer >= e->cfg.layers) return fail(VB_ERR_ARG, "layer index out of range");
    if (e->quantized) return fail(VB_ERR_STATE, "engine already quantized; upload f32 layers first");
    if (!w->input_norm || !w->post_norm || !w->wq || !w->wk || !w->wv || !w->wo || !w->q_norm ||
        !w->k_norm || !w->wg || !w->wu || !w->wd)
        return fail(VB_ERR_ARG, "null weight pointer");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    const size_t hd = c.hidden, D = c.head_dim;
    vb_layer_dev& L = e->L[layer];
    auto up = [](void* d, const void* h, size_t bytes) {
        return cudaMemcpy(d, h, bytes, cudaMemcpyHostToDevice);
    };
    VB_CUDA_TRY(up(L.in_norm, w->input_norm, hd * 4));
    VB_CUDA_TRY(up(L.post_norm, w->post_norm, hd * 4));
    VB_CUDA_TRY(up(L.q_norm, w->q_norm, D * 4));
    VB_CUDA_TRY(up(L.k_norm, w->k_norm, D * 4));
    VB_CUDA_TRY(up(L.wqkv, w->wq, (size_t)e->q_width * hd * 4));
    VB_CUDA_TRY(up(L.wqkv + (size_t)e->q_width * hd, w->wk, (size_t)e->kv_width * hd * 4));
    VB_CUDA_TRY(up(L.wqkv + (size_t)(e->q_width + e->kv_width) * hd, w->wv,
                   (size_t)e->kv_width * hd * 4));
    VB_CUDA_TRY(up(L.wo, w->wo, hd * e->q_width * 4));
    // gate row j -> row 2j, up row j -> row 2j+1
    VB_CUDA_TRY(cudaMemcpy2D(L.wgu, 2 * hd * 4, w->wg, hd * 4, hd * 4, c.ffn,
                             cudaMemcpyHostToDevice));
    VB_CUDA_TRY(cudaMemcpy2D(L.wgu + hd, 2 * hd * 4, w->wu, hd * 4, hd * 4, c.ffn,
                             cudaMemcpyHostToDevice));
    VB_CUDA_TRY(up(L.wd, w->wd, hd * (size_t)c.ffn * 4));
    e->layer_set[layer] = 1;
    return VB_OK;
}

namespace vb {
namespace {
// INT8 storage of every layer (same layout the device quantizer writes) with
// the per-layer pointers set; releases the f32 projections.
vb_status alloc_int8_layers(vb_engine* e) {
    const vb_config& c = e->cfg;
    const size_t hd = c.hidden;
    vb_status st;
    if ((st = dalloc(&e->wi8, e->per_layer_i8 * c.layers, "int8 projections"))) return st;
    if ((st = dalloc(&e->wscale, e->per_layer_rows * c.layers, "scales"))) return st;
    for (int l = 0; l < c.layers; l++) {
        vb_layer_dev& L = e->L[l];
        int8_t* qb = e->wi8 + e->per_layer_i8 * l;
        float* sb = e->wscale + e->per_layer_rows * l;
        L.qqkv = qb;
        L.qo = L.qqkv + (size_t)e->qkv_rows * hd;
        L.qgu = L.qo + hd * e->q_width;
        L.qd = L.qgu + 2 * (size_t)c.ffn * hd;
        L.sqkv = sb;
        L.so = L.sqkv + e->qkv_rows;
        L.sgu = L.so + hd;
        L.sd = L.sgu + 2 * c.ffn;
    }
    return VB_OK;
}

void drop_step_state(vb_engine* e) {
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    mega2_release(e);
}
}  // namespace
}  // namespace vb

vb_status vb_engine_set_layer_q8(vb_engine* e, int layer, const vb_layer_host_q8* w) {
    if (!e || !w) return fail(VB_ERR_ARG, "null argument");
    if (layer < 0 || layer >= e->cfg.layers) return fail(VB_ERR_ARG, "layer index out of range");
    if (!w->input_norm || !w->post_norm || !w->q_norm || !w->k_norm || !w->wq || !w->wk || !w->wv || !w->wo ||
        !w->wg || !w->wu || !w->wd || !w->sq || !w->sk || !w->sv || !w->so || !w->sg || !w->su || !w->sd)
        return fail(VB_ERR_ARG, "null weight pointer");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    const size_t hd = c.hidden, D = c.head_dim, qw = e->q_width, kw = e->kv_width, F = c.ffn;
    vb_status st;
    if (!e->quantized) {
        // switching to INT8 uploads: every layer comes through this call now
        for (int l = 0; l < c.layers; l++) e->layer_set[l] = 0;
        if ((st = alloc_int8_layers(e))) return st;
        dfree(e->wf32);
        for (auto& L : e->L) L.wqkv = L.wo = L.wgu = L.wd = nullptr;
        e->quantized = true;
        drop_step_state(e);
    }
    vb_layer_dev& L = e->L[layer];
    auto up = [](void* d, const void* h, size_t bytes) { return cudaMemcpy(d, h, bytes, cudaMemcpyHostToDevice); };
    VB_CUDA_TRY(up(L.in_norm, w->input_norm, hd * 4));
    VB_CUDA_TRY(up(L.post_norm, w->post_norm, hd * 4));
    VB_CUDA_TRY(up(L.q_norm, w->q_norm, D * 4));
    VB_CUDA_TRY(up(L.k_norm, w->k_norm, D * 4));
    // q | k | v rows stacked, with their scales
    VB_CUDA_TRY(up(L.qqkv, w->wq, qw * hd));
    VB_CUDA_TRY(up(L.qqkv + qw * hd, w->wk, kw * hd));
    VB_CUDA_TRY(up(L.qqkv + (qw + kw) * hd, w->wv, kw * hd));
    VB_CUDA_TRY(up(L.sqkv, w->sq, qw * 4));
    VB_CUDA_TRY(up(L.sqkv + qw, w->sk, kw * 4));
    VB_CUDA_TRY(up(L.sqkv + qw + kw, w->sv, kw * 4));
    VB_CUDA_TRY(up(L.qo, w->wo, hd * qw));
    VB_CUDA_TRY(up(L.so, w->so, hd * 4));
    // gate row j -> row 2j, up row j -> row 2j+1 (scales alike)
    VB_CUDA_TRY(cudaMemcpy2D(L.qgu, 2 * hd, w->wg, hd, hd, F, cudaMemcpyHostToDevice));
    VB_CUDA_TRY(cudaMemcpy2D(L.qgu + hd, 2 * hd, w->wu, hd, hd, F, cudaMemcpyHostToDevice));
    VB_CUDA_TRY(cudaMemcpy2D(L.sgu, 8, w->sg, 4, 4, F, cudaMemcpyHostToDevice));
    VB_CUDA_TRY(cudaMemcpy2D(L.sgu + 1, 8, w->su, 4, 4, F, cudaMemcpyHostToDevice));
    VB_CUDA_TRY(up(L.qd, w->wd, hd * F));
    VB_CUDA_TRY(up(L.sd, w->sd, hd * 4));
    e->layer_set[layer] = 1;
    return VB_OK;
}

vb_status vb_engine_quantize(vb_engine* e) {
    if (!e) return fail(VB_ERR_ARG, "null engine");
    if (e->quantized) return VB_OK;  // model.cpp:314
    for (int l = 0; l < e->cfg.layers; l++)
        if (!e->layer_set[l]) return fail(VB_ERR_STATE, "quantize before all layers are uploaded");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    const size_t hd = c.hidden;
    vb_status st;
    if ((st = alloc_int8_layers(e))) return st;
    for (int l = 0; l < c.layers; l++) {
        vb_layer_dev& L = e->L[l];
        if ((st = launch_quantize_rows(L.wqkv, e->qkv_rows, hd, L.qqkv, L.sqkv, e->stream))) return st;
        if ((st = launch_quantize_rows(L.wo, hd, e->q_width, L.qo, L.so, e->stream))) return st;
        if ((st = launch_quantize_rows(L.wgu, 2 * c.ffn, hd, L.qgu, L.sgu, e->stream))) return st;
        if ((st = launch_quantize_rows(L.wd, hd, c.ffn, L.qd, L.sd, e->stream))) return st;
    }
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    // model.cpp:329-335: the f32 originals are released.
    dfree(e->wf32);
    for (auto& L : e->L) L.wqkv = L.wo = L.wgu = L.wd = nullptr;
    e->quantized = true;
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    mega2_release(e);
    return VB_OK;
}

int vb_engine_is_quantized(const vb_engine* e) { return e && e->quantized ? 1 : 0; }

vb_status vb_engine_quantize_lm_head(vb_engine* e) {
    if (!e) return fail(VB_ERR_ARG, "null engine");
    if (e->lm_int8) return VB_OK;
    if (!e->globals_set) return fail(VB_ERR_STATE, "engine weights not uploaded");
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    vb_status st;
    if ((st = dalloc(&e->lm_q8, (size_t)c.vocab * c.hidden, "int8 lm_head"))) return st;
    if ((st = dalloc(&e->lm_sc, (size_t)c.vocab, "lm_head scales"))) return st;
    if ((st = launch_quantize_rows(e->embed, c.vocab, c.hidden, e->lm_q8, e->lm_sc, e->stream))) return st;
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->lm_int8 = true;
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    mega2_release(e);
    return VB_OK;
}

int vb_engine_lm_head_int8(const vb_engine* e) { return e && e->lm_int8 ? 1 : 0; }

size_t vb_engine_weight_bytes(const vb_engine* e) {
    if (!e) return 0;
    const vb_config& c = e->cfg;
    size_t total = ((size_t)c.vocab * c.hidden + c.hidden) * 4;
    total += (size_t)c.layers * (2 * (size_t)c.hidden + 2 * (size_t)c.head_dim) * 4;
    if (e->quantized)
        total += (size_t)c.layers * (e->per_layer_i8 + e->per_layer_rows * 4);
    else
        total += (size_t)c.layers * e->per_layer_f32 * 4;
    return total;
}

vb_status vb_engine_reset_cache(vb_engine* e, int max_seq) {
    if (!e) return fail(VB_ERR_ARG, "null engine");
    if (max_seq <= 0) return fail(VB_ERR_ARG, "max_seq must be positive");
    DeviceGuard dg(e->device);
    cudaStreamSynchronize(e->stream);
    const vb_config& c = e->cfg;
    if (e->kc && e->max_seq == max_seq) {
        // same geometry: keep the buffers, zero them (generate.cpp:19-21)
        const size_t n = (size_t)c.layers * c.kv_heads * max_seq * c.head_dim;
        VB_CUDA_TRY(cudaMemsetAsync(e->kc, 0, n * 4, e->stream));
        VB_CUDA_TRY(cudaMemsetAsync(e->vc, 0, n * 4, e->stream));
    } else {
        free_cache(e);
        mega2_release(e);
        const size_t n = (size_t)c.layers * c.kv_heads * max_seq * c.head_dim;
        vb_status st;
        if ((st = dalloc(&e->kc, n, "kv cache"))) return st;
        if ((st = dalloc(&e->vc, n, "kv cache"))) return st;
        VB_CUDA_TRY(cudaMemsetAsync(e->kc, 0, n * 4, e->stream));
        VB_CUDA_TRY(cudaMemsetAsync(e->vc, 0, n * 4, e->stream));
        e->max_seq = max_seq;
        e->attn_splits = attn_splits_for(1, c.kv_heads, max_seq);
        if ((st = dalloc(&e->attn_ws, attn_ws_bytes(1, c.heads, e->attn_splits) / 4 + 1, "attn ws")))
            return st;
        if ((st = dalloc(&e->d_hist, max_seq, "history"))) return st;
        if ((st = dalloc(&e->d_prompt, max_seq, "prompt"))) return st;
    }
    VB_CUDA_TRY(cudaMemsetAsync(e->d_pos, 0, sizeof(int), e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->len = 0;
    return VB_OK;
}

int vb_engine_cache_len(const vb_engine* e) { return e ? e->len : 0; }

// The automatic step path: the one measured fastest on B200 for the weight
// format (f32: the per-op graph, 985 against 867 tok/s for the clustered
// step; INT8: the clustered step, 1175 against 943).  A clustered step whose
// shape requirements are not met falls back to the per-op graph.
static int auto_path(const vb_engine* e) { return e->quantized ? 2 : 1; }

static vb_status pre_step(vb_engine* e, int n_tokens) {
    vb_status st = check_ready(e);
    if (st) return st;
    if (e->len + n_tokens > e->max_seq) return fail(VB_ERR_CACHE_FULL, "kv cache is full");
    if (e->len + n_tokens > e->cfg.rope_positions)
        return fail(VB_ERR_ROPE, "position is outside the rope table");
    if (e->path_auto && !e->graph) e->path = auto_path(e);
    if (e->path == 2 && !e->mega2) {
        st = mega2_prepare(e);
        if (st == VB_ERR_UNSUPPORTED) e->path = 1;
        else if (st) return st;
    }
    return ensure_graph(e);
}

vb_status vb_engine_step(vb_engine* e, int token, float* logits_host) {
    if (!e || !logits_host) return fail(VB_ERR_ARG, "null argument");
    DeviceGuard dg(e->device);
    vb_status st = pre_step(e, 1);
    if (st) return st;
    if (token < 0 || token >= e->cfg.vocab)
        return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    e->h_pinned_i[0] = token;
    e->h_pinned_i[1] = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_tok, e->h_pinned_i, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_step, e->h_pinned_i + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    if ((st = launch_step(e))) return st;
    VB_CUDA_TRY(cudaMemcpyAsync(logits_host, e->logits, (size_t)e->cfg.vocab * 4,
                                cudaMemcpyDeviceToHost, e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if ((st = engine_check_err(e))) return st;
    e->len += 1;
    return VB_OK;
}

vb_status vb_engine_decode(vb_engine* e, int first_token, int n, int* tokens_host,
                           float* logits_host) {
    if (!e) return fail(VB_ERR_ARG, "null engine");
    if (n <= 0) return VB_OK;
    DeviceGuard dg(e->device);
    vb_status st = pre_step(e, n);
    if (st) return st;
    if (first_token < 0 || first_token >= e->cfg.vocab)
        return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    e->h_pinned_i[0] = first_token;
    e->h_pinned_i[1] = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_tok, e->h_pinned_i, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_step, e->h_pinned_i + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < n; i++)
        if ((st = launch_step(e))) return st;
    if (tokens_host)
        VB_CUDA_TRY(cudaMemcpyAsync(tokens_host, e->d_hist, (size_t)n * sizeof(int),
                                    cudaMemcpyDeviceToHost, e->stream));
    if (logits_host)
        VB_CUDA_TRY(cudaMemcpyAsync(logits_host, e->logits, (size_t)e->cfg.vocab * 4,
                                    cudaMemcpyDeviceToHost, e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if ((st = engine_check_err(e))) return st;
    e->len += n;
    return VB_OK;
}

vb_status vb_engine_decode_sampled(vb_engine* e, vb_sampler* sp, int first_token, int n, int* tokens_host) {
    if (!e || !sp) return fail(VB_ERR_ARG, "null argument");
    if (sampler_greedy(sp)) return vb_engine_decode(e, first_token, n, tokens_host, nullptr);
    if (n <= 0) return VB_OK;
    DeviceGuard dg(e->device);
    vb_status st = pre_step(e, n);
    if (st) return st;
    if (first_token < 0 || first_token >= e->cfg.vocab)
        return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    if ((st = sampler_draws(sp, n, e->stream))) return st;
    e->h_pinned_i[0] = first_token;
    e->h_pinned_i[1] = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_tok, e->h_pinned_i, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_step, e->h_pinned_i + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < n; i++) {
        // the step leaves the logits and its greedy pick; the sample replaces the pick
        if ((st = launch_step(e))) return st;
        if ((st = launch_sample(sp, e->logits, e->cfg.vocab, i, e->d_next, e->d_tok, e->d_next, e->d_hist, e->d_step,
                                e->max_seq, e->stream)))
            return st;
    }
    if (tokens_host)
        VB_CUDA_TRY(cudaMemcpyAsync(tokens_host, e->d_hist, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost,
                                    e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if ((st = engine_check_err(e))) return st;
    e->len += n;
    return VB_OK;
}

vb_status vb_engine_prefill(vb_engine* e, const int* tokens_host, int n, float* logits_host) {
    if (!e || !tokens_host) return fail(VB_ERR_ARG, "null argument");
    if (n <= 0) return VB_OK;
    DeviceGuard dg(e->device);
    vb_status st = pre_step(e, n);
    if (st) return st;
    for (int i = 0; i < n; i++)
        if (tokens_host[i] < 0 || tokens_host[i] >= e->cfg.vocab)
            return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_prompt, tokens_host, sizeof(int) * n, cudaMemcpyHostToDevice,
                                e->stream));
    e->h_pinned_i[1] = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(e->d_step, e->h_pinned_i + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < n; i++) {
        VB_CUDA_TRY(cudaMemcpyAsync(e->d_tok, e->d_prompt + i, sizeof(int),
                                    cudaMemcpyDeviceToDevice, e->stream));
        if ((st = launch_step(e))) return st;
    }
    if (logits_host)
        VB_CUDA_TRY(cudaMemcpyAsync(logits_host, e->logits, (size_t)e->cfg.vocab * 4,
                                    cudaMemcpyDeviceToHost, e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if ((st = engine_check_err(e))) return st;
    e->len += n;
    return VB_OK;
}

int vb_engine_graph_nodes(const vb_engine* e) { return e ? e->graph_nodes : 0; }

int vb_engine_path(const vb_engine* e) { return !e ? 0 : (e->path_auto && !e->graph) ? auto_path(e) : e->path; }

vb_status vb_engine_read_kv(const vb_engine* e, int layer, int which, float* host) {
    if (!e || !host) return fail(VB_ERR_ARG, "null argument");
    if (!e->kc) return fail(VB_ERR_NO_CACHE, "call reset_cache() first");
    if (layer < 0 || layer >= e->cfg.layers) return fail(VB_ERR_ARG, "layer index out of range");
    if (e->len == 0) return VB_OK;
    DeviceGuard dg(e->device);
    const vb_config& c = e->cfg;
    const size_t layer_kv = (size_t)c.kv_heads * e->max_seq * c.head_dim;
    const float* base = (which == 0 ? e->kc : e->vc) + layer * layer_kv;
    VB_CUDA_TRY(cudaStreamSynchronize(e->stream));
    for (int h = 0; h < c.kv_heads; h++) {
        VB_CUDA_TRY(cudaMemcpy2D(host + (size_t)h * c.head_dim, (size_t)e->kv_width * 4,
                                 base + (size_t)h * e->max_seq * c.head_dim,
                                 (size_t)c.head_dim * 4, (size_t)c.head_dim * 4, e->len,
                                 cudaMemcpyDeviceToHost));
    }
    return VB_OK;
}

vb_status vb_engine_set_path(vb_engine* e, int path) {
    if (!e || path < -1 || path == 0 || path > 2) return fail(VB_ERR_ARG, "path must be -1 (automatic), 1 or 2");
    DeviceGuard dg(e->device);
    cudaStreamSynchronize(e->stream);
    e->path_auto = path < 0;
    if (e->path_auto || e->path != path) {
        if (!e->path_auto) e->path = path;
        if (e->graph) cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    return VB_OK;
}

void* vb_engine_stream(vb_engine* e) { return e ? (void*)e->stream : nullptr; }

vb_status vb_engine_set_trace(vb_engine* e, int on) {
    if (!e) return fail(VB_ERR_ARG, "null engine");
    DeviceGuard dg(e->device);
    if (e->trace_on != (on != 0)) {
        cudaStreamSynchronize(e->stream);
        e->trace_on = on != 0;
        mega2_release(e);
        if (e->graph) cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    return VB_OK;
}

int vb_engine_read_trace(vb_engine* e, uint64_t* out, int cap) {
    if (!e || !out || cap <= 0) return 0;
    DeviceGuard dg(e->device);
    return mega2_read_trace(e, reinterpret_cast<unsigned long long*>(out), cap);
}

}  // extern "C"
