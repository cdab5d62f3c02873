// ref_shim.cpp -- extern "C" access to the UNMODIFIED reference engine.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own sources (core/src/*.cpp, read in place, never copied)
// into oracle/_ref/libverbum_ref.so.  Tests use it to pin the C oracle bit for
// bit; bench.py's reference arm times Model::step through it.
//
// Every entry point calls straight into the reference's public API:
//   verbum::Model (core/include/verbum/model.h:47-116), quantize_rows /
//   matmul_nt_q8 (quant.h:42-50), matmul_nt (ops.h:19), rmsnorm /
//   build_rope_table / apply_rope (nn.h:17-40), Sampler (generate.h:56-67).
// The single exception is ref_model_set_cache_len: to time a decode step at a
// long context without a token-by-token CPU prefill of thousands of tokens,
// it sets each layer's KVCache::len (Model::caches_ is private, so this
// translation unit opens the class's access).  The cache contents stay what
// reset_cache() left (zeros); the arithmetic cost of Model::step at that
// length is unchanged, which is all the timing needs.

// Standard headers first so that their own classes keep their access rules.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <ctime>
#include <unordered_map>
#include <utility>
#include <vector>

#define private public
#include "verbum/model.h"
#undef private
#include "verbum/generate.h"
#include "verbum/nn.h"
#include "verbum/ops.h"
#include "verbum/quant.h"

namespace {
thread_local std::string g_err;
template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

void* ref_model_open(const char* dir) {
    verbum::Model* m = nullptr;
    if (guarded([&] { m = new verbum::Model(dir); })) return nullptr;
    return m;
}

void ref_model_free(void* h) { delete static_cast<verbum::Model*>(h); }

int ref_model_quantize(void* h) {
    return guarded([&] { static_cast<verbum::Model*>(h)->quantize(); });
}

int ref_model_reset_cache(void* h, int max_seq) {
    return guarded([&] { static_cast<verbum::Model*>(h)->reset_cache(max_seq); });
}

int ref_model_step(void* h, int token, float* logits) {
    auto* m = static_cast<verbum::Model*>(h);
    return guarded([&] {
        verbum::Tensor out({1, (int64_t)m->config().vocab_size});
        m->step(token, out);
        std::memcpy(logits, out.data(), sizeof(float) * (size_t)out.numel());
    });
}

// Greedy decode loop shaped like tools/bench.cpp:50-69: one logits Tensor
// reused every step, Sampler with temperature 0, each step() timed alone.
int ref_model_greedy_steps(void* h, int first_token, int n_steps, int* tokens_out,
                           double* step_seconds) {
    auto* m = static_cast<verbum::Model*>(h);
    return guarded([&] {
        const int64_t vocab = m->config().vocab_size;
        verbum::Tensor logits({1, vocab});
        verbum::SamplerConfig sc;
        sc.temperature = 0.0f;
        verbum::Sampler sampler(sc);
        int tok = first_token;
        for (int i = 0; i < n_steps; i++) {
            timespec t0{}, t1{};
            clock_gettime(CLOCK_MONOTONIC, &t0);
            m->step(tok, logits);
            clock_gettime(CLOCK_MONOTONIC, &t1);
            if (step_seconds)
                step_seconds[i] = (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
            tok = sampler.sample(logits.data(), vocab);
            if (tokens_out) tokens_out[i] = tok;
        }
    });
}

int ref_model_embed_text(void* h, const int* ids, int n, float* out) {
    return guarded([&] {
        auto v = static_cast<verbum::Model*>(h)->embed_text(std::vector<int>(ids, ids + n));
        std::memcpy(out, v.data(), sizeof(float) * v.size());
    });
}

int ref_model_set_cache_len(void* h, int len) {
    auto* m = static_cast<verbum::Model*>(h);
    return guarded([&] {
        if (m->caches_.empty()) throw std::runtime_error("call reset_cache() first");
        for (auto& c : m->caches_) {
            if (len < 0 || len > c.max_seq) throw std::runtime_error("len out of range");
            c.len = len;
        }
    });
}

int ref_model_cache_len(void* h) {
    auto* m = static_cast<verbum::Model*>(h);
    return m->caches_.empty() ? 0 : m->caches_[0].len;
}

unsigned long long ref_model_weight_bytes(void* h) {
    return static_cast<verbum::Model*>(h)->weight_bytes();
}

int ref_model_is_quantized(void* h) {
    return static_cast<verbum::Model*>(h)->is_quantized() ? 1 : 0;
}

// Copies layer `layer`'s quantized projection `which` (0 q,1 k,2 v,3 o,4 gate,
// 5 up,6 down) as stored by Model::quantize().
int ref_model_quant_tensor(void* h, int layer, int which, int8_t* q, float* scales) {
    auto* m = static_cast<verbum::Model*>(h);
    return guarded([&] {
        if (!m->quantized_) throw std::runtime_error("not quantized");
        const verbum::QuantLayer& Q = m->qlayers_.at((size_t)layer);
        const verbum::QuantTensor* t[7] = {&Q.q_proj, &Q.k_proj, &Q.v_proj, &Q.o_proj,
                                           &Q.gate_proj, &Q.up_proj, &Q.down_proj};
        if (which < 0 || which > 6) throw std::runtime_error("bad tensor index");
        std::memcpy(q, t[which]->data.data(), t[which]->data.size());
        std::memcpy(scales, t[which]->scales.data(), t[which]->scales.size() * sizeof(float));
    });
}

// Copies layer `layer`'s K (which==0) or V cache, [max_seq, KVH*D].
int ref_model_kv(void* h, int layer, int which, float* out) {
    auto* m = static_cast<verbum::Model*>(h);
    return guarded([&] {
        const verbum::KVCache& c = m->caches_.at((size_t)layer);
        const auto& src = which == 0 ? c.k : c.v;
        std::memcpy(out, src.data(), src.size() * sizeof(float));
    });
}

int ref_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q,
                      float* scales) {
    return guarded([&] {
        verbum::Tensor w({rows, cols}, std::vector<float>(W, W + rows * cols));
        verbum::QuantTensor t = verbum::quantize_rows(w);
        std::memcpy(q, t.data.data(), t.data.size());
        std::memcpy(scales, t.scales.data(), t.scales.size() * sizeof(float));
    });
}

int ref_matmul_nt(const float* A, const float* B, float* C, int64_t M, int64_t N,
                  int64_t K) {
    return guarded([&] {
        verbum::Tensor a({M, K}, std::vector<float>(A, A + M * K));
        verbum::Tensor b({N, K}, std::vector<float>(B, B + N * K));
        verbum::Tensor c({M, N});
        verbum::matmul_nt(a, b, c);
        std::memcpy(C, c.data(), sizeof(float) * (size_t)(M * N));
    });
}

int ref_matmul_nt_q8(const float* A, const int8_t* Bq, const float* S, float* C,
                     int64_t M, int64_t N, int64_t K) {
    return guarded([&] {
        verbum::Tensor a({M, K}, std::vector<float>(A, A + M * K));
        verbum::QuantTensor b;
        b.rows = N;
        b.cols = K;
        b.data.assign(Bq, Bq + N * K);
        b.scales.assign(S, S + N);
        verbum::Tensor c({M, N});
        verbum::matmul_nt_q8(a, b, c);
        std::memcpy(C, c.data(), sizeof(float) * (size_t)(M * N));
    });
}

int ref_rmsnorm(const float* x, const float* w, float eps, float* out, int64_t rows,
                int64_t dim) {
    return guarded([&] {
        verbum::Tensor xt({rows, dim}, std::vector<float>(x, x + rows * dim));
        verbum::Tensor o({rows, dim});
        verbum::rmsnorm(xt, std::vector<float>(w, w + dim), eps, o);
        std::memcpy(out, o.data(), sizeof(float) * (size_t)(rows * dim));
    });
}

int ref_rope_table(int head_dim, int max_pos, float theta, float* cos_tab,
                   float* sin_tab) {
    return guarded([&] {
        verbum::RopeTable t = verbum::build_rope_table(head_dim, max_pos, theta);
        std::memcpy(cos_tab, t.cos.data(), t.cos.size() * sizeof(float));
        std::memcpy(sin_tab, t.sin.data(), t.sin.size() * sizeof(float));
    });
}

int ref_apply_rope(float* x, int64_t heads, int head_dim, int pos, int max_pos,
                   float theta) {
    return guarded([&] {
        verbum::RopeTable t = verbum::build_rope_table(head_dim, max_pos, theta);
        verbum::Tensor xt({heads, (int64_t)head_dim},
                          std::vector<float>(x, x + heads * head_dim));
        verbum::apply_rope(xt, pos, t);
        std::memcpy(x, xt.data(), sizeof(float) * (size_t)(heads * head_dim));
    });
}

int ref_greedy(const float* logits, int64_t vocab) {
    verbum::SamplerConfig sc;
    sc.temperature = 0.0f;
    verbum::Sampler s(sc);
    return s.sample(logits, vocab);
}

// One Sampler, n calls: row i of logits [n][vocab] -> out[i].
int ref_sample_seq(float temperature, int top_k, float top_p, uint64_t seed, const float* logits, int64_t vocab,
                   int n, int* out) {
    return guarded([&] {
        verbum::SamplerConfig sc;
        sc.temperature = temperature;
        sc.top_k = top_k;
        sc.top_p = top_p;
        sc.seed = seed;
        verbum::Sampler s(sc);
        for (int i = 0; i < n; i++) out[i] = s.sample(logits + (size_t)i * vocab, vocab);
    });
}

}  // extern "C"
