// vb_batch.cu -- batched independent-sequence decode: B sequences share one
// engine's weights (read once per step for all B rows) and each owns a KV
// cache.  Per layer: rmsnorm rows -> QKV GEMM -> q/k norm + RoPE + append ->
// split-K attention over B caches -> o GEMM + residual -> rmsnorm -> gate/up
// GEMM + SwiGLU -> down GEMM + residual; then final norm -> lm_head GEMM ->
// per-row argmax.  The step is graph-captured and replayed.
//
// The GEMMs run on the tensor cores (vb_tcgemm.cu): the batch keeps bf16
// copies of the projections (exact for INT8 values; a hi+lo pair for f32
// weights and the tied lm_head), each GEMM's activations are split into bf16
// hi+lo, and the split-K partials are summed with the INT8 scales and the
// epilogue (store, residual add, SwiGLU) by the reduce kernel.
#include <algorithm>
#include <string>
#include <vector>

#include "vb_engine.cuh"

struct vb_batch {
    vb_engine* e = nullptr;
    int B = 0;
    int max_seq = 0;
    int len = 0;
    float* kc = nullptr;
    float* vc = nullptr;
    float* x = nullptr;
    float* xn = nullptr;
    float* q = nullptr;
    float* ctx = nullptr;
    float* h = nullptr;
    float* logits = nullptr;
    float* attn_ws = nullptr;
    int attn_splits = 1;
    float* gemm_ws = nullptr;
    size_t gemm_ws_floats = 0;
    int* d_tok = nullptr;
    int* d_pos = nullptr;
    int* d_next = nullptr;
    unsigned long long* d_keys = nullptr;  // [B] argmax keys of the decode step (zero between steps)
    int* d_err = nullptr;
    int* h_io = nullptr;  // pinned [2*B + 1]: tokens in, next tokens out, error word
    cudaGraphExec_t graph = nullptr;
    bool graph_q8 = false;
    bool graph_lm8 = false;
    int graph_nodes = 0;
    void* arena = nullptr;    // prefill buffers, kept for the next prefill
    size_t arena_bytes = 0;
    // tensor-core operands
    std::vector<void*> tcw;   // per layer: qkv, o, gu, d -> {hi, lo}
    void* lm_hi = nullptr;
    void* lm_lo = nullptr;
    bool tc_q8 = false;       // which weights tcw holds
    bool tc_lm8 = false;      // lm_hi holds the INT8 lm_head (exact in bf16), lm_lo unused
    bool tc_ready = false;
    void* a_hi = nullptr;     // [64][hidden] bf16 split of the normed input (QKV, gate/up, lm_head)
    void* a_lo = nullptr;
    void* y_hi = nullptr;     // [64][max(H*D, ffn)] bf16 split of ctx (o_proj) or h (down)
    void* y_lo = nullptr;
};

namespace vb {
namespace {

template <class T>
vb_status balloc(T** p, size_t count, const char* what) {
    *p = nullptr;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), (count ? count : 1) * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, what);
    return VB_OK;
}
template <class T>
void bfree(T*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

void free_tc_weights(vb_batch* b) {
    for (void*& p : b->tcw)
        if (p) cudaFree(p), p = nullptr;
    b->tcw.clear();
    b->tc_ready = false;
}

// bf16 tensor-core copies of the current weights (rebuilt when the engine is
// quantised after the batch was made); the lm_head pair is built once.
vb_status batch_tc_weights(vb_batch* b) {
    vb_engine* e = b->e;
    if (b->tc_ready && b->tc_q8 == e->quantized && b->tc_lm8 == e->lm_int8) return VB_OK;
    const vb_config& c = e->cfg;
    cudaStream_t s = e->stream;
    const bool q8 = e->quantized;
    free_tc_weights(b);
    b->tcw.assign((size_t)c.layers * 8, nullptr);
    const int Ns[4] = {e->qkv_rows, c.hidden, 2 * c.ffn, c.hidden};
    const int Ks[4] = {c.hidden, e->q_width, c.hidden, c.ffn};
    vb_status st;
    for (int l = 0; l < c.layers; l++) {
        const vb_layer_dev& L = e->L[l];
        const void* src[4] = {q8 ? (const void*)L.qqkv : (const void*)L.wqkv, q8 ? (const void*)L.qo : (const void*)L.wo,
                              q8 ? (const void*)L.qgu : (const void*)L.wgu, q8 ? (const void*)L.qd : (const void*)L.wd};
        for (int j = 0; j < 4; j++) {
            const size_t n = (size_t)Ns[j] * Ks[j];
            void** hl = &b->tcw[(size_t)l * 8 + 2 * j];
            VB_CUDA_TRY(cudaMalloc(&hl[0], n * 2));
            if (!q8) VB_CUDA_TRY(cudaMalloc(&hl[1], n * 2));
            if ((st = launch_weights_bf16(src[j], q8, n, hl[0], hl[1], s))) return st;
        }
    }
    if (!b->lm_hi || b->tc_lm8 != e->lm_int8) {
        const size_t n = (size_t)c.vocab * c.hidden;
        if (!b->lm_hi) VB_CUDA_TRY(cudaMalloc(&b->lm_hi, n * 2));
        if (!b->lm_lo) VB_CUDA_TRY(cudaMalloc(&b->lm_lo, n * 2));
        if (e->lm_int8) {
            if ((st = launch_weights_bf16(e->lm_q8, true, n, b->lm_hi, nullptr, s))) return st;
        } else if ((st = launch_weights_bf16(e->embed, false, n, b->lm_hi, b->lm_lo, s))) {
            return st;
        }
        b->tc_lm8 = e->lm_int8;
    }
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    b->tc_q8 = q8;
    b->tc_ready = true;
    return VB_OK;
}

vb_status enqueue_batch_step(vb_batch* b, cudaStream_t s) {
    vb_engine* e = b->e;
    const vb_config& c = e->cfg;
    const bool q8 = e->quantized;
    const int B = b->B;
    vb_status st;
    if ((st = launch_embed(e->embed, b->d_tok, B, c.hidden, c.vocab, b->x, b->d_err, s))) return st;
    const size_t per_seq = (size_t)c.kv_heads * b->max_seq * c.head_dim;
    const size_t layer_kv = per_seq * B;
    // C (epilogue) A . W^T on the tensor cores from A's bf16 split (ahi, alo)
    auto gemm = [&](const void* ahi, const void* alo, void* const* w, const float* sc, float* C, int N, int K,
                    int ldc, int epi, bool wq8, void* ohi, void* olo, bool partials = false,
                    const QkNormArgs* qk = nullptr) {
        TcGemmArgs t{};
        t.w_hi = w[0];
        t.w_lo = wq8 ? nullptr : w[1];
        t.a_hi = ahi;
        t.a_lo = alo;
        t.M = B;
        t.N = N;
        t.K = K;
        t.ws = b->gemm_ws;
        t.ws_floats = b->gemm_ws_floats;
        t.scales = wq8 ? sc : nullptr;
        t.C = C;
        t.ldc = ldc;
        t.epi = epi;
        t.out_hi = ohi;
        t.out_lo = olo;
        t.partials_only = partials;
        t.err = b->d_err;
        t.qk = qk;
        return launch_tc_gemm(t, s);
    };
    // The q|k|v GEMM sums its splits inside thread-block clusters and applies
    // the q/k norm + RoPE + append itself (or, past 8 splits, leaves them to the
    // q/k-norm kernel); the o and down partials are left in the GEMM workspace
    // and summed by the residual add + the next RMSNorm (nn.cpp:8-42) + bf16 split.
    const bool qk_fused = tc_gemm_cluster_reduce(B, e->qkv_rows, c.hidden, !q8);
    const float* parts = b->gemm_ws;
    if ((st = launch_rmsnorm_rows(b->x, e->L[0].in_norm, b->xn, B, c.hidden, c.eps, s, b->a_hi, b->a_lo)))
        return st;
    for (int l = 0; l < c.layers; l++) {
        const vb_layer_dev& L = e->L[l];
        void* const* tw = &b->tcw[(size_t)l * 8];
        QkNormArgs qa{};
        qa.parts = parts;
        qa.splits = tc_gemm_splits(e->qkv_rows, c.hidden, !q8);
        qa.scales = q8 ? L.sqkv : nullptr;
        qa.q_norm = L.q_norm;
        qa.k_norm = L.k_norm;
        qa.cos_tab = e->rope_cos;
        qa.sin_tab = e->rope_sin;
        qa.pos = b->d_pos;
        qa.q_out = b->q;
        qa.kc = b->kc + l * layer_kv;
        qa.vc = b->vc + l * layer_kv;
        qa.stride_b = (int64_t)per_seq;
        qa.stride_pos = c.head_dim;
        qa.stride_h = (int64_t)b->max_seq * c.head_dim;
        qa.B = B;
        qa.H = c.heads;
        qa.KVH = c.kv_heads;
        qa.D = c.head_dim;
        qa.rope_positions = c.rope_positions < b->max_seq ? c.rope_positions : b->max_seq;
        qa.eps = c.eps;
        qa.err = b->d_err;
        // (Inside the attention (fuse_qk) each of the 2560 CTAs would redo the
        // q norm from the partials before streaming its cache slice: measured
        // 1% slower at 64 sequences than a separate kernel.)
        if (qk_fused) {
            if ((st = gemm(b->a_hi, b->a_lo, tw + 0, L.sqkv, nullptr, e->qkv_rows, c.hidden, e->qkv_rows, kEpiQkNorm,
                           q8, nullptr, nullptr, false, &qa)))
                return st;
        } else {
            if ((st = gemm(b->a_hi, b->a_lo, tw + 0, L.sqkv, nullptr, e->qkv_rows, c.hidden, e->qkv_rows, kEpiStore,
                           q8, nullptr, nullptr, true)))
                return st;
            if ((st = launch_qk_norm_rope_append(qa, s))) return st;
        }
        AttnArgs aa{};
        aa.q = b->q;
        aa.k = qa.kc;
        aa.v = qa.vc;
        aa.out = b->ctx;
        aa.pos = b->d_pos;
        aa.B = B;
        aa.H = c.heads;
        aa.KVH = c.kv_heads;
        aa.D = c.head_dim;
        aa.n_max = b->max_seq;
        aa.stride_b = qa.stride_b;
        aa.stride_pos = qa.stride_pos;
        aa.stride_h = qa.stride_h;
        aa.splits = b->attn_splits;
        aa.ws = b->attn_ws;
        aa.out_hi = b->y_hi;
        aa.out_lo = b->y_lo;
        if ((st = launch_attention(aa, s))) return st;
        if ((st = gemm(b->y_hi, b->y_lo, tw + 2, L.so, nullptr, c.hidden, e->q_width, c.hidden, kEpiResidual, q8,
                       nullptr, nullptr, true)))
            return st;
        if ((st = launch_reduce_residual_norm(b->x, parts, tc_gemm_splits(c.hidden, e->q_width, !q8), q8 ? L.so : nullptr,
                                              L.post_norm, b->xn, b->a_hi, b->a_lo, B, c.hidden, c.eps, s)))
            return st;
        if ((st = gemm(b->a_hi, b->a_lo, tw + 4, L.sgu, b->h, 2 * c.ffn, c.hidden, c.ffn, kEpiSwiGLU, q8, b->y_hi,
                       b->y_lo)))
            return st;
        if ((st = gemm(b->y_hi, b->y_lo, tw + 6, L.sd, nullptr, c.hidden, c.ffn, c.hidden, kEpiResidual, q8, nullptr,
                       nullptr, true)))
            return st;
        const float* next_norm = l + 1 < c.layers ? e->L[l + 1].in_norm : e->final_norm;
        if ((st = launch_reduce_residual_norm(b->x, parts, tc_gemm_splits(c.hidden, c.ffn, !q8), q8 ? L.sd : nullptr,
                                              next_norm, b->xn, b->a_hi, b->a_lo, B, c.hidden, c.eps, s)))
            return st;
    }
    {
        void* const lm[2] = {b->lm_hi, b->lm_lo};
        if ((st = gemm(b->a_hi, b->a_lo, lm, e->lm_sc, b->logits, c.vocab, c.hidden, c.vocab, kEpiStore,
                       e->lm_int8, nullptr, nullptr)))
            return st;
    }
    // (one CTA per row measured ~33 us a step; 16 CTAs per row fold into keys)
    if ((st = launch_argmax_rows_keys(b->logits, B, c.vocab, b->d_keys, s))) return st;
    return launch_advance_keys(b->d_pos, b->d_tok, b->d_next, b->d_keys, B, s);
}

// Device buffers of one prompt chunk of R = B * C rows (row b*C + c is
// position p0 + c of sequence b).
struct PrefillBufs {
    float *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *ctx = nullptr, *h = nullptr, *ws = nullptr;
    size_t ws_floats = 0;
    void* att = nullptr;  // bf16 copies for the tensor-core prompt attention
    void *a_hi = nullptr, *a_lo = nullptr, *y_hi = nullptr, *y_lo = nullptr;
    int *tok = nullptr, *pos = nullptr;
};

// embed_text's pooling (model.cpp:191-233): pool[b][d] += sum over the chunk's
// positions of xn[b*C + c][d], in position order, one thread per (b, d).
__global__ void pool_rows_kernel(const float* xn, int B, int C, int dim, float* pool) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * dim) return;
    const int b = i / dim, d = i - b * dim;
    float acc = pool[i];
    for (int c = 0; c < C; c++) acc += xn[((size_t)b * C + c) * dim + d];
    pool[i] = acc;
}

// Mean (x 1/n in float) and L2 normalisation (double norm, float 1/norm) of
// each pooled row.  One block of 1024 threads per row.
__global__ void __launch_bounds__(1024) pool_finish_kernel(float* pool, int dim, int n) {
    __shared__ double red[32];
    float* v = pool + (size_t)blockIdx.x * dim;
    const float inv = 1.0f / (float)n;
    double ss = 0.0;
    for (int d = threadIdx.x; d < dim; d += 1024) {
        const float x = v[d] * inv;
        v[d] = x;
        ss += (double)x * (double)x;
    }
    ss = block_sum_d<1024>(ss, red);
    const double norm = sqrt(ss);
    if (norm > 0) {
        const float nf = (float)(1.0 / norm);
        for (int d = threadIdx.x; d < dim; d += 1024) v[d] *= nf;
    }
}

// Prefill of P positions for all B sequences (tokens_host [P][B]) as whole
// chunks: the projections of all chunk rows run as tensor-core GEMMs (weights
// read once per chunk instead of once per position), the q/k norm + RoPE +
// append over all rows, then causal flash attention over the cache.  The same
// layer arithmetic as the decode step (model.cpp:240-254, generate.cpp:42-107)
// in a different summation order.  Afterwards the decode state is what P
// decode steps leave: logits and greedy picks of the last position, tokens =
// picks, positions advanced by P.
vb_status batch_prefill_chunks(vb_batch* b, const int* tokens_host, int P, float* pool = nullptr) {
    vb_engine* e = b->e;
    const vb_config& c = e->cfg;
    const bool q8 = e->quantized;
    const int B = b->B, H = c.hidden;
    // positions per chunk: up to 128k rows, so a 64 x 2048 prompt is one chunk
    // (VB_PREFILL_ROWS overrides the row budget)
    int rows = 131072;
    if (const char* v = getenv("VB_PREFILL_ROWS"))
        if (atoi(v) > 0) rows = atoi(v);
    const int C = std::min(P, std::max(1, rows / B));
    const int R = B * C, R64 = std::max(R, 64);
    const int ky = std::max(e->q_width, c.ffn);
    cudaStream_t s = e->stream;
    // the whole prompt from position 0 in one chunk: attention on the tensor cores
    const bool tc_att = b->len == 0 && C == P && c.heads == 2 * c.kv_heads && c.head_dim == 128;
    // one arena for every buffer (kept in the batch and reused by the next prefill)
    PrefillBufs pb;
    {
        const int nk[4][2] = {{e->qkv_rows, H}, {H, e->q_width}, {2 * c.ffn, H}, {H, c.ffn}};
        for (const auto& g : nk)  // split-K partials: GEMMs of at most 64 rows use split-K
            pb.ws_floats = std::max(pb.ws_floats, tc_gemm_ws_floats(std::min(R, 64), g[0], g[1]));
    }
    const size_t sz[] = {
        (size_t)R * H * 4,              // x
        pool ? (size_t)R * H * 4 : 0,   // xn (f32 final norm rows for embed_text)
        (size_t)R * e->qkv_rows * 4,    // qkv
        tc_att ? 0 : (size_t)R * e->q_width * 4,  // q (f32, CUDA-core attention only)
        tc_att ? 0 : (size_t)R * e->q_width * 4,  // ctx (f32 attention output, CUDA-core form only)
        (size_t)R * c.ffn * 4,          // h
        pb.ws_floats * 4,               // ws
        tc_att ? prompt_attention_tc_bytes(B, P, c.heads, c.kv_heads) : 0,  // att
        (size_t)R64 * H * 2,            // a_hi
        (size_t)R64 * H * 2,            // a_lo
        (size_t)R64 * ky * 2,           // y_hi
        (size_t)R64 * ky * 2,           // y_lo
        (size_t)R * 4,                  // tok
        (size_t)R * 4,                  // pos
    };
    constexpr int kN = sizeof(sz) / sizeof(sz[0]);
    size_t total = 0;
    for (size_t z : sz) total += (z + 255) / 256 * 256;
    if (b->arena_bytes < total) {
        if (b->arena) cudaFree(b->arena);
        b->arena = nullptr;
        b->arena_bytes = 0;
        const cudaError_t ce = cudaMalloc(&b->arena, total);
        if (ce != cudaSuccess) return cuda_fail(ce, "prefill buffers");
        b->arena_bytes = total;
    }
    {
        void* ptr[kN];
        char* cur = static_cast<char*>(b->arena);
        for (int i = 0; i < kN; i++) {
            ptr[i] = sz[i] ? cur : nullptr;
            cur += (sz[i] + 255) / 256 * 256;
        }
        pb.x = static_cast<float*>(ptr[0]);
        pb.xn = static_cast<float*>(ptr[1]);
        pb.qkv = static_cast<float*>(ptr[2]);
        pb.q = static_cast<float*>(ptr[3]);
        pb.ctx = static_cast<float*>(ptr[4]);
        pb.h = static_cast<float*>(ptr[5]);
        pb.ws = static_cast<float*>(ptr[6]);
        pb.att = ptr[7];
        pb.a_hi = ptr[8];
        pb.a_lo = ptr[9];
        pb.y_hi = ptr[10];
        pb.y_lo = ptr[11];
        pb.tok = static_cast<int*>(ptr[12]);
        pb.pos = static_cast<int*>(ptr[13]);
    }
    vb_status st;
    if (R < 64) {
        // rows past R of a single 64-row tile are read by the MMA: keep them finite
        for (void* p : {pb.a_hi, pb.a_lo}) VB_CUDA_TRY(cudaMemsetAsync(p, 0, (size_t)R64 * H * 2, s));
        for (void* p : {pb.y_hi, pb.y_lo}) VB_CUDA_TRY(cudaMemsetAsync(p, 0, (size_t)R64 * ky * 2, s));
    }
    auto gemm = [&](int M, const void* ahi, const void* alo, void* const* w, const float* sc, float* Cm, int N, int K,
                    int ldc, int epi, bool wq8, void* ohi, void* olo) {
        TcGemmArgs t{};
        t.w_hi = w[0];
        t.w_lo = wq8 ? nullptr : w[1];
        t.a_hi = ahi;
        t.a_lo = alo;
        t.M = M;
        t.N = N;
        t.K = K;
        t.ws = pb.ws;
        t.ws_floats = pb.ws_floats;
        t.scales = wq8 ? sc : nullptr;
        t.C = Cm;
        t.ldc = ldc;
        t.epi = epi;
        t.out_hi = ohi;
        t.out_lo = olo;
        t.err = b->d_err;
        return launch_tc_gemm(t, s);
    };
    const size_t per_seq = (size_t)c.kv_heads * b->max_seq * c.head_dim;
    const size_t layer_kv = per_seq * B;
    std::vector<int> htok(R), hpos(R);
    int Cn = 0;
    for (int p0 = 0; p0 < P; p0 += C) {
        Cn = std::min(C, P - p0);
        const int Rn = B * Cn, start = b->len + p0;
        for (int sq = 0; sq < B; sq++)
            for (int i = 0; i < Cn; i++) {
                htok[(size_t)sq * Cn + i] = tokens_host[(size_t)(p0 + i) * B + sq];
                hpos[(size_t)sq * Cn + i] = start + i;
            }
        VB_CUDA_TRY(cudaMemcpyAsync(pb.tok, htok.data(), sizeof(int) * Rn, cudaMemcpyHostToDevice, s));
        VB_CUDA_TRY(cudaMemcpyAsync(pb.pos, hpos.data(), sizeof(int) * Rn, cudaMemcpyHostToDevice, s));
        // the host arrays are rewritten for the next chunk: wait for the copies
        VB_CUDA_TRY(cudaStreamSynchronize(s));
        if ((st = launch_embed(e->embed, pb.tok, Rn, H, c.vocab, pb.x, b->d_err, s))) return st;
        for (int l = 0; l < c.layers; l++) {
            const vb_layer_dev& L = e->L[l];
            void* const* tw = &b->tcw[(size_t)l * 8];
            // (the GEMMs read the bf16 split only)
            if ((st = launch_rmsnorm_rows(pb.x, L.in_norm, nullptr, Rn, H, c.eps, s, pb.a_hi, pb.a_lo))) return st;
            if ((st = gemm(Rn, pb.a_hi, pb.a_lo, tw + 0, L.sqkv, pb.qkv, e->qkv_rows, H, e->qkv_rows, kEpiStore, q8,
                           nullptr, nullptr)))
                return st;
            QkNormArgs qa{};
            qa.qkv = pb.qkv;
            qa.rows_per_seq = Cn;
            qa.q_norm = L.q_norm;
            qa.k_norm = L.k_norm;
            qa.cos_tab = e->rope_cos;
            qa.sin_tab = e->rope_sin;
            qa.pos = pb.pos;
            qa.q_out = pb.q;
            qa.kc = b->kc + l * layer_kv;
            qa.vc = b->vc + l * layer_kv;
            qa.stride_b = (int64_t)per_seq;
            qa.stride_pos = c.head_dim;
            qa.stride_h = (int64_t)b->max_seq * c.head_dim;
            qa.B = Rn;
            qa.H = c.heads;
            qa.KVH = c.kv_heads;
            qa.D = c.head_dim;
            qa.rope_positions = c.rope_positions < b->max_seq ? c.rope_positions : b->max_seq;
            qa.eps = c.eps;
            qa.err = b->d_err;
            if (tc_att) {
                const PromptCopies cp = prompt_attention_copies(pb.att, B, P, c.heads, c.kv_heads);
                qa.q_hi = cp.q_hi;
                qa.q_lo = cp.q_lo;
                qa.k_hi = cp.k_hi;
                qa.k_lo = cp.k_lo;
                qa.kbf_rows = P;
            }
            if ((st = launch_qk_norm_rope_append(qa, s))) return st;
            PrefillAttnArgs pa{};
            pa.q = pb.q;
            pa.k = qa.kc;
            pa.v = qa.vc;
            pa.stride_b = qa.stride_b;
            pa.stride_h = qa.stride_h;
            pa.B = B;
            pa.C = Cn;
            pa.p0 = start;
            pa.H = c.heads;
            pa.KVH = c.kv_heads;
            pa.D = c.head_dim;
            pa.out = pb.ctx;
            pa.out_hi = pb.y_hi;
            pa.out_lo = pb.y_lo;
            pa.err = b->d_err;
            if (tc_att) {
                pa.out = nullptr;  // the o_proj reads the split only
                if ((st = launch_prompt_attention_tc(pa, pb.q, pb.att, s, true))) return st;
            } else if ((st = launch_prefill_attention(pa, s))) {
                return st;
            }
            if ((st = gemm(Rn, pb.y_hi, pb.y_lo, tw + 2, L.so, pb.x, H, e->q_width, H, kEpiResidual, q8, nullptr,
                           nullptr)))
                return st;
            if ((st = launch_rmsnorm_rows(pb.x, L.post_norm, nullptr, Rn, H, c.eps, s, pb.a_hi, pb.a_lo))) return st;
            // the down projection reads the bf16 split of h: its f32 copy only where the
            // small-M (split-K) form needs an output
            float* hf = (Rn >= 128 && 2 * c.ffn >= 256) ? nullptr : pb.h;
            if ((st = gemm(Rn, pb.a_hi, pb.a_lo, tw + 4, L.sgu, hf, 2 * c.ffn, H, c.ffn, kEpiSwiGLU, q8, pb.y_hi,
                           pb.y_lo)))
                return st;
            if ((st = gemm(Rn, pb.y_hi, pb.y_lo, tw + 6, L.sd, pb.x, H, c.ffn, H, kEpiResidual, q8, nullptr,
                           nullptr)))
                return st;
        }
        if (pool) {  // embed_text: final norm of every row, summed per sequence
            if ((st = launch_rmsnorm_rows(pb.x, e->final_norm, pb.xn, Rn, H, c.eps, s))) return st;
            pool_rows_kernel<<<(B * H + 255) / 256, 256, 0, s>>>(pb.xn, B, Cn, H, pool);
            VB_LAUNCH_CHECK("pool_rows_kernel");
        }
    }
    if (pool) {
        pool_finish_kernel<<<B, 1024, 0, s>>>(pool, H, P);
        VB_LAUNCH_CHECK("pool_finish_kernel");
        VB_CUDA_TRY(cudaStreamSynchronize(s));
        return VB_OK;
    }
    // the last position of every sequence: final norm, lm_head, greedy pick
    VB_CUDA_TRY(cudaMemcpy2DAsync(b->x, sizeof(float) * H, pb.x + (size_t)(Cn - 1) * H, sizeof(float) * H * Cn,
                                  sizeof(float) * H, B, cudaMemcpyDeviceToDevice, s));
    if ((st = launch_rmsnorm_rows(b->x, e->final_norm, b->xn, B, H, c.eps, s, b->a_hi, b->a_lo))) return st;
    void* const lm[2] = {b->lm_hi, b->lm_lo};
    if ((st = gemm(B, b->a_hi, b->a_lo, lm, e->lm_sc, b->logits, c.vocab, H, c.vocab, kEpiStore, e->lm_int8,
                   nullptr, nullptr)))
        return st;
    if ((st = launch_argmax_rows(b->logits, B, c.vocab, b->d_next, s))) return st;
    // decode state after P steps: tokens = picks, positions += P
    for (int sq = 0; sq < B; sq++) htok[sq] = b->len + P;
    VB_CUDA_TRY(cudaMemcpyAsync(b->d_pos, htok.data(), sizeof(int) * B, cudaMemcpyHostToDevice, s));
    VB_CUDA_TRY(cudaMemcpyAsync(b->d_tok, b->d_next, sizeof(int) * B, cudaMemcpyDeviceToDevice, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    return VB_OK;
}

vb_status batch_graph(vb_batch* b) {
    if (b->graph && b->graph_q8 == b->e->quantized && b->graph_lm8 == b->e->lm_int8) return VB_OK;
    if (vb_status ws = batch_tc_weights(b)) return ws;
    if (b->graph) cudaGraphExecDestroy(b->graph);
    b->graph = nullptr;
    cudaStream_t s = b->e->stream;
    cudaGraph_t g = nullptr;
    VB_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    vb_status st = enqueue_batch_step(b, s);
    cudaError_t ce = cudaStreamEndCapture(s, &g);
    if (st) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    b->graph_nodes = (int)nn;
    ce = cudaGraphInstantiate(&b->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) {
        b->graph = nullptr;
        return cuda_fail(ce, "cudaGraphInstantiate");
    }
    b->graph_q8 = b->e->quantized;
    b->graph_lm8 = b->e->lm_int8;
    // upload now so the first launch does not pay for it
    ce = cudaGraphUpload(b->graph, s);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphUpload");
    return VB_OK;
}

// Maps the device error word (read by the caller after its stream sync) to a status.
vb_status batch_err_status(vb_batch* b, int err) {
    if (!err) return VB_OK;
    cudaMemsetAsync(b->d_err, 0, sizeof(int), b->e->stream);
    cudaStreamSynchronize(b->e->stream);
    if (err == kErrBadToken) return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    if (err == kErrCacheFull) return fail(VB_ERR_CACHE_FULL, "kv cache is full");
    return fail(VB_ERR_CUDA, "device error word set: " + std::to_string(err));
}

struct Dev {
    int prev = -1;
    explicit Dev(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~Dev() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" {

vb_status vb_batch_create(vb_engine* e, int batch, int max_seq, vb_batch** out) {
    if (!e || !out) return fail(VB_ERR_ARG, "null argument");
    *out = nullptr;
    if (batch <= 0 || batch > 64) return fail(VB_ERR_UNSUPPORTED, "batch must be 1..64");
    if (max_seq <= 0) return fail(VB_ERR_ARG, "max_seq must be positive");
    Dev dg(e->device);
    const vb_config& c = e->cfg;
    vb_batch* b = new vb_batch();
    b->e = e;
    b->B = batch;
    b->max_seq = max_seq;
    auto bail = [&](vb_status s) {
        vb_batch_destroy(b);
        return s;
    };
    const size_t kvn = (size_t)c.layers * batch * c.kv_heads * max_seq * c.head_dim;
    vb_status st;
    if ((st = balloc(&b->kc, kvn, "batch kv cache"))) return bail(st);
    if ((st = balloc(&b->vc, kvn, "batch kv cache"))) return bail(st);
    cudaStream_t es = e->stream;  // non-blocking: memsets must be ordered on it
    if (cudaMemsetAsync(b->kc, 0, kvn * 4, es) || cudaMemsetAsync(b->vc, 0, kvn * 4, es))
        return bail(fail(VB_ERR_CUDA, "kv cache memset failed"));
    if ((st = balloc(&b->x, (size_t)batch * c.hidden, "x"))) return bail(st);
    if ((st = balloc(&b->xn, (size_t)batch * c.hidden, "xn"))) return bail(st);
    if ((st = balloc(&b->q, (size_t)batch * e->q_width, "q"))) return bail(st);
    if ((st = balloc(&b->ctx, (size_t)batch * e->q_width, "ctx"))) return bail(st);
    if ((st = balloc(&b->h, (size_t)batch * c.ffn, "h"))) return bail(st);
    if ((st = balloc(&b->logits, (size_t)batch * c.vocab, "logits"))) return bail(st);
    b->attn_splits = attn_splits_for(batch, c.kv_heads, max_seq);
    if ((st = balloc(&b->attn_ws, attn_ws_bytes(batch, c.heads, b->attn_splits) / 4 + 1, "attn ws")))
        return bail(st);
    if (c.hidden % 64 || e->q_width % 64 || c.ffn % 64)
        return bail(fail(VB_ERR_UNSUPPORTED, "batch: tensor-core GEMMs need hidden, heads*head_dim, ffn % 64 == 0"));
    size_t ws = 0;
    auto upd = [&](int N, int K) {
        const size_t w = tc_gemm_ws_floats(batch, N, K);
        if (w > ws) ws = w;
    };
    upd(e->qkv_rows, c.hidden);
    upd(c.hidden, e->q_width);
    upd(2 * c.ffn, c.hidden);
    upd(c.hidden, c.ffn);
    upd(c.vocab, c.hidden);
    b->gemm_ws_floats = ws;
    if ((st = balloc(&b->gemm_ws, ws, "gemm ws"))) return bail(st);
    {
        const int ky = std::max(e->q_width, c.ffn);
        unsigned short *ah = nullptr, *al = nullptr, *yh = nullptr, *yl = nullptr;
        if ((st = balloc(&ah, (size_t)64 * c.hidden, "activation split"))) return bail(st);
        b->a_hi = ah;
        if ((st = balloc(&al, (size_t)64 * c.hidden, "activation split"))) return bail(st);
        b->a_lo = al;
        if ((st = balloc(&yh, (size_t)64 * ky, "activation split"))) return bail(st);
        b->y_hi = yh;
        if ((st = balloc(&yl, (size_t)64 * ky, "activation split"))) return bail(st);
        b->y_lo = yl;
        // rows >= batch are read by the MMA (their outputs are dropped): keep them finite
        if (cudaMemsetAsync(ah, 0, (size_t)128 * c.hidden, es) || cudaMemsetAsync(al, 0, (size_t)128 * c.hidden, es) ||
            cudaMemsetAsync(yh, 0, (size_t)128 * ky, es) || cudaMemsetAsync(yl, 0, (size_t)128 * ky, es))
            return bail(fail(VB_ERR_CUDA, "activation split memset failed"));

    }
    if ((st = balloc(&b->d_tok, batch, "tok"))) return bail(st);
    if ((st = balloc(&b->d_pos, batch, "pos"))) return bail(st);
    if ((st = balloc(&b->d_next, batch, "next"))) return bail(st);
    if ((st = balloc(&b->d_keys, batch, "argmax keys"))) return bail(st);
    if (cudaMemsetAsync(b->d_keys, 0, sizeof(unsigned long long) * batch, es))
        return bail(fail(VB_ERR_CUDA, "argmax keys memset failed"));
    if ((st = balloc(&b->d_err, 1, "err"))) return bail(st);
    if (cudaMemsetAsync(b->d_pos, 0, sizeof(int) * batch, es) ||
        cudaMemsetAsync(b->d_tok, 0, sizeof(int) * batch, es) ||
        cudaMemsetAsync(b->d_err, 0, sizeof(int), es) || cudaStreamSynchronize(es))
        return bail(fail(VB_ERR_CUDA, "batch state init failed"));
    if (cudaMallocHost(&b->h_io, sizeof(int) * (2 * batch + 1)) != cudaSuccess)
        return bail(fail(VB_ERR_CUDA, "cudaMallocHost failed"));
    *out = b;
    return VB_OK;
}

vb_status vb_batch_destroy(vb_batch* b) {
    if (!b) return VB_OK;
    Dev dg(b->e->device);
    cudaStreamSynchronize(b->e->stream);
    if (b->graph) cudaGraphExecDestroy(b->graph);
    bfree(b->kc); bfree(b->vc); bfree(b->x); bfree(b->xn); bfree(b->q);
    bfree(b->ctx); bfree(b->h); bfree(b->logits); bfree(b->attn_ws); bfree(b->gemm_ws);
    bfree(b->d_tok); bfree(b->d_pos); bfree(b->d_next); bfree(b->d_keys); bfree(b->d_err);
    if (b->arena) cudaFree(b->arena);
    free_tc_weights(b);
    bfree(b->lm_hi); bfree(b->lm_lo); bfree(b->a_hi); bfree(b->a_lo); bfree(b->y_hi); bfree(b->y_lo);
    if (b->h_io) cudaFreeHost(b->h_io);
    delete b;
    return VB_OK;
}

static vb_status batch_pre(vb_batch* b, int n) {
    vb_engine* e = b->e;
    if (!e->globals_set) return fail(VB_ERR_STATE, "engine weights not uploaded");
    for (int l = 0; l < e->cfg.layers; l++)
        if (!e->layer_set[l]) return fail(VB_ERR_STATE, "layer not uploaded");
    if (b->len + n > b->max_seq) return fail(VB_ERR_CACHE_FULL, "kv cache is full");
    if (b->len + n > e->cfg.rope_positions)
        return fail(VB_ERR_ROPE, "position is outside the rope table");
    return batch_graph(b);
}

vb_status vb_batch_step(vb_batch* b, const int* tokens_host, float* logits_host, int* next_host) {
    if (!b || !tokens_host) return fail(VB_ERR_ARG, "null argument");
    Dev dg(b->e->device);
    vb_status st = batch_pre(b, 1);
    if (st) return st;
    for (int i = 0; i < b->B; i++) {
        if (tokens_host[i] < 0 || tokens_host[i] >= b->e->cfg.vocab)
            return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
        b->h_io[i] = tokens_host[i];
    }
    cudaStream_t s = b->e->stream;
    VB_CUDA_TRY(cudaMemcpyAsync(b->d_tok, b->h_io, sizeof(int) * b->B, cudaMemcpyHostToDevice, s));
    VB_CUDA_TRY(cudaGraphLaunch(b->graph, s));
    if (logits_host)
        VB_CUDA_TRY(cudaMemcpyAsync(logits_host, b->logits, sizeof(float) * b->B * b->e->cfg.vocab,
                                    cudaMemcpyDeviceToHost, s));
    if (next_host)
        VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + b->B, b->d_next, sizeof(int) * b->B,
                                    cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + 2 * b->B, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    if ((st = batch_err_status(b, b->h_io[2 * b->B]))) return st;
    if (next_host)
        for (int i = 0; i < b->B; i++) next_host[i] = b->h_io[b->B + i];
    b->len += 1;
    return VB_OK;
}

vb_status vb_batch_decode(vb_batch* b, const int* tokens_host, int n, int* next_host) {
    if (!b) return fail(VB_ERR_ARG, "null batch");
    if (n <= 0) return VB_OK;
    Dev dg(b->e->device);
    vb_status st = batch_pre(b, n);
    if (st) return st;
    cudaStream_t s = b->e->stream;
    if (tokens_host) {
        for (int i = 0; i < b->B; i++) {
            if (tokens_host[i] < 0 || tokens_host[i] >= b->e->cfg.vocab)
                return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
            b->h_io[i] = tokens_host[i];
        }
        VB_CUDA_TRY(cudaMemcpyAsync(b->d_tok, b->h_io, sizeof(int) * b->B, cudaMemcpyHostToDevice, s));
    }
    for (int i = 0; i < n; i++) VB_CUDA_TRY(cudaGraphLaunch(b->graph, s));
    if (next_host)
        VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + b->B, b->d_next, sizeof(int) * b->B,
                                    cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + 2 * b->B, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    if ((st = batch_err_status(b, b->h_io[2 * b->B]))) return st;
    if (next_host)
        for (int i = 0; i < b->B; i++) next_host[i] = b->h_io[b->B + i];
    b->len += n;
    return VB_OK;
}

vb_status vb_batch_prefill(vb_batch* b, const int* tokens_host, int P, int* next_host) {
    if (!b || !tokens_host) return fail(VB_ERR_ARG, "null argument");
    if (P <= 0) return VB_OK;
    Dev dg(b->e->device);
    vb_status st = batch_pre(b, P);
    if (st) return st;
    const size_t n = (size_t)P * b->B;
    for (size_t i = 0; i < n; i++)
        if (tokens_host[i] < 0 || tokens_host[i] >= b->e->cfg.vocab)
            return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    if ((st = batch_prefill_chunks(b, tokens_host, P))) return st;
    cudaStream_t s = b->e->stream;
    if (next_host)
        VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + b->B, b->d_next, sizeof(int) * b->B,
                                    cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaMemcpyAsync(b->h_io + 2 * b->B, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    if ((st = batch_err_status(b, b->h_io[2 * b->B]))) return st;
    if (next_host)
        for (int i = 0; i < b->B; i++) next_host[i] = b->h_io[b->B + i];
    b->len += P;
    return VB_OK;
}

int vb_batch_graph_nodes(const vb_batch* b) { return b ? b->graph_nodes : 0; }

int vb_batch_cache_len(const vb_batch* b) { return b ? b->len : 0; }

vb_status vb_batch_reset(vb_batch* b) {
    if (!b) return fail(VB_ERR_ARG, "null batch");
    Dev dg(b->e->device);
    cudaStreamSynchronize(b->e->stream);
    const vb_config& c = b->e->cfg;
    const size_t kvn = (size_t)c.layers * b->B * c.kv_heads * b->max_seq * c.head_dim;
    VB_CUDA_TRY(cudaMemsetAsync(b->kc, 0, kvn * 4, b->e->stream));
    VB_CUDA_TRY(cudaMemsetAsync(b->vc, 0, kvn * 4, b->e->stream));
    VB_CUDA_TRY(cudaMemsetAsync(b->d_pos, 0, sizeof(int) * b->B, b->e->stream));
    VB_CUDA_TRY(cudaStreamSynchronize(b->e->stream));
    b->len = 0;
    return VB_OK;
}

// Model::embed_text (model.cpp:191-233) on the device: the whole prompt's
// layers through the prefill path (a temporary one-sequence batch whose cache
// holds the n positions), the final norm of every position, mean pooling and
// L2 normalisation.  Like the reference, f32 projections only.
vb_status vb_engine_embed_text(vb_engine* e, const int* ids, int n, float* out_host) {
    if (!e || !out_host) return fail(VB_ERR_ARG, "null argument");
    if (e->quantized) return fail(VB_ERR_STATE, "embed_text needs the f32 path");
    if (!ids || n <= 0) return fail(VB_ERR_ARG, "embed_text got no tokens");
    if (!e->globals_set) return fail(VB_ERR_STATE, "engine weights not uploaded");
    for (int l = 0; l < e->cfg.layers; l++)
        if (!e->layer_set[l]) return fail(VB_ERR_STATE, "layer not uploaded");
    if (n > e->cfg.rope_positions) return fail(VB_ERR_ROPE, "position is outside the rope table");
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= e->cfg.vocab)
            return fail(VB_ERR_TOKEN, "token id out of range for the embedding table");
    Dev dg(e->device);
    vb_batch* b = nullptr;
    vb_status st = vb_batch_create(e, 1, n, &b);
    if (st) return st;
    float* pool = nullptr;
    const size_t dim = e->cfg.hidden;
    if ((st = balloc(&pool, dim, "embed_text pool")) == VB_OK &&
        (st = cudaMemsetAsync(pool, 0, dim * 4, e->stream) ? fail(VB_ERR_CUDA, "memset") : VB_OK) == VB_OK &&
        (st = batch_tc_weights(b)) == VB_OK && (st = batch_prefill_chunks(b, ids, n, pool)) == VB_OK) {
        const cudaError_t ce = cudaMemcpy(out_host, pool, dim * 4, cudaMemcpyDeviceToHost);
        if (ce != cudaSuccess) st = cuda_fail(ce, "embed_text copy");
        int err = 0;
        if (!st && cudaMemcpy(&err, b->d_err, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && err)
            st = batch_err_status(b, err);
    }
    bfree(pool);
    vb_batch_destroy(b);
    return st;
}

vb_status vb_batch_truncate(vb_batch* b, int len) {
    if (!b) return fail(VB_ERR_ARG, "null batch");
    if (len < 0 || len > b->len) return fail(VB_ERR_ARG, "truncate: length outside [0, cache length]");
    Dev dg(b->e->device);
    cudaStream_t s = b->e->stream;
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    // positions >= len are overwritten before attention reads them again
    for (int i = 0; i < b->B; i++) b->h_io[i] = len;
    VB_CUDA_TRY(cudaMemcpyAsync(b->d_pos, b->h_io, sizeof(int) * b->B, cudaMemcpyHostToDevice, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    b->len = len;
    return VB_OK;
}

}  // extern "C"
