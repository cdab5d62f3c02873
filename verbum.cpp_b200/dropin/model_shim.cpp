// model_shim.cpp -- extern "C" face of verbum::Model and verbum::Sampler
// (core/include/verbum/model.h:47-116, generate.h:49-67) for tests that
// drive the drop-in builds through ctypes.  Compiled against whichever
// model.h the build uses (the reference's own, or the engine-backed patch);
// every C++ exception becomes a non-zero return and its message.
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>

#include "verbum/generate.h"
#include "verbum/model.h"
#include "verbum/tensor.h"

namespace {
thread_local std::string g_err;

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
    } catch (...) {
        g_err = "unknown exception";
    }
    return -1;
}
}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* vbm_last_error() { return g_err.c_str(); }

__attribute__((visibility("default"))) void* vbm_create(const char* dir) {
    verbum::Model* m = nullptr;
    if (guard([&] { m = new verbum::Model(dir); })) return nullptr;
    return m;
}

__attribute__((visibility("default"))) void vbm_free(void* h) { delete static_cast<verbum::Model*>(h); }

__attribute__((visibility("default"))) int vbm_quantize(void* h) {
    return guard([&] { static_cast<verbum::Model*>(h)->quantize(); });
}

__attribute__((visibility("default"))) int vbm_reset_cache(void* h, int max_seq) {
    return guard([&] { static_cast<verbum::Model*>(h)->reset_cache(max_seq); });
}

__attribute__((visibility("default"))) int vbm_to_cuda(void* h) {
    return guard([&] { static_cast<verbum::Model*>(h)->to_cuda(); });
}

__attribute__((visibility("default"))) int vbm_is_cuda(void* h) {
    return static_cast<verbum::Model*>(h)->is_cuda() ? 1 : 0;
}

__attribute__((visibility("default"))) int vbm_is_quantized(void* h) {
    return static_cast<verbum::Model*>(h)->is_quantized() ? 1 : 0;
}

__attribute__((visibility("default"))) size_t vbm_weight_bytes(void* h) {
    return static_cast<verbum::Model*>(h)->weight_bytes();
}

__attribute__((visibility("default"))) int vbm_vocab(void* h) {
    return static_cast<verbum::Model*>(h)->config().vocab_size;
}

// Model::step: one token, logits [vocab] copied to out.
__attribute__((visibility("default"))) int vbm_step(void* h, int token, float* out) {
    return guard([&] {
        auto* m = static_cast<verbum::Model*>(h);
        const int64_t V = m->config().vocab_size;
        verbum::Tensor logits({1, V});
        m->step(token, logits);
        std::memcpy(out, logits.data(), sizeof(float) * (size_t)V);
    });
}

__attribute__((visibility("default"))) void* vbm_sampler_create(float temperature, int top_k, float top_p,
                                                                uint64_t seed) {
    verbum::SamplerConfig c;
    c.temperature = temperature;
    c.top_k = top_k;
    c.top_p = top_p;
    c.seed = seed;
    return new verbum::Sampler(c);
}

__attribute__((visibility("default"))) int vbm_sampler_sample(void* s, const float* logits, int64_t vocab) {
    return static_cast<verbum::Sampler*>(s)->sample(logits, vocab);
}

__attribute__((visibility("default"))) void vbm_sampler_free(void* s) { delete static_cast<verbum::Sampler*>(s); }

}  // extern "C"
