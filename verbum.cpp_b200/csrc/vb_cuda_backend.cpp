// vb_cuda_backend.cpp -- the reference's launcher API (cuda_backend.h:7-43)
// on this library's C ABI, so the reference's own Model::to_cuda /
// step_cuda (core/src/model.cpp:367-497) run on the sm_100a kernels when
// model.cpp is compiled with VERBUM_CUDA and linked against this library.
#include <stdexcept>
#include <string>

#include "verbum_b200_backend.hpp"

namespace verbum {
namespace {

void check(vb_status s, const char* what) {
    if (s != VB_OK) throw std::runtime_error(std::string(what) + ": " + vb_last_error());
}

}  // namespace

bool cuda_available() { return vb_device_count() > 0; }

const char* cuda_device_name() {
    static thread_local char name[256];
    name[0] = 0;
    if (vb_device_count() > 0) vb_device_name(0, name, sizeof name);
    return name;
}

size_t cuda_free_memory() {
    size_t b = 0;
    if (vb_device_count() > 0) check(vb_free_memory(0, &b), "cuda_free_memory");
    return b;
}

CudaBuffer cuda_alloc(size_t bytes) {
    CudaBuffer b;
    check(vb_alloc(&b.ptr, bytes), "cuda_alloc");
    b.bytes = bytes;
    return b;
}

void cuda_free(CudaBuffer& b) {
    if (b.ptr) check(vb_free(b.ptr), "cuda_free");
    b.ptr = nullptr;
    b.bytes = 0;
}

void cuda_upload(CudaBuffer& dst, const void* host, size_t bytes) {
    check(vb_upload(dst.ptr, host, bytes, nullptr), "cuda_upload");
}

void cuda_download(void* host, const CudaBuffer& src, size_t bytes) {
    check(vb_download(host, src.ptr, bytes, nullptr), "cuda_download");
}

void cuda_zero(CudaBuffer& b) { check(vb_zero(b.ptr, b.bytes, nullptr), "cuda_zero"); }

void cuda_sync() { check(vb_sync(nullptr), "cuda_sync"); }

void cuda_matmul_nt(const CudaBuffer& a, const CudaBuffer& b, CudaBuffer& c, int M, int N, int K) {
    check(vb_matmul_nt_f32(static_cast<const float*>(a.ptr), static_cast<const float*>(b.ptr),
                           static_cast<float*>(c.ptr), M, N, K, nullptr),
          "cuda_matmul_nt");
}

void cuda_rmsnorm(const CudaBuffer& x, const CudaBuffer& w, CudaBuffer& out, int rows, int dim, float eps) {
    check(vb_rmsnorm(static_cast<const float*>(x.ptr), static_cast<const float*>(w.ptr),
                     static_cast<float*>(out.ptr), rows, dim, eps, nullptr),
          "cuda_rmsnorm");
}

void cuda_rope(CudaBuffer& x, const CudaBuffer& cos_tab, const CudaBuffer& sin_tab, int pos, int heads, int D) {
    check(vb_rope(static_cast<float*>(x.ptr), static_cast<const float*>(cos_tab.ptr),
                  static_cast<const float*>(sin_tab.ptr), pos, heads, D, nullptr),
          "cuda_rope");
}

void cuda_silu_mul(CudaBuffer& gate, const CudaBuffer& up, int n) {
    check(vb_silu_mul(static_cast<float*>(gate.ptr), static_cast<const float*>(up.ptr), n, nullptr),
          "cuda_silu_mul");
}

void cuda_add(CudaBuffer& a, const CudaBuffer& b, int n) {
    check(vb_add(static_cast<float*>(a.ptr), static_cast<const float*>(b.ptr), n, nullptr), "cuda_add");
}

void cuda_attn_decode(const CudaBuffer& q, const CudaBuffer& kcache, const CudaBuffer& vcache, CudaBuffer& out,
                      int H, int KVH, int D, int n) {
    check(vb_attn_decode(static_cast<const float*>(q.ptr), static_cast<const float*>(kcache.ptr),
                         static_cast<const float*>(vcache.ptr), static_cast<float*>(out.ptr), H, KVH, D, n,
                         nullptr),
          "cuda_attn_decode");
}

void cuda_cache_append(CudaBuffer& kcache, CudaBuffer& vcache, const CudaBuffer& knew, const CudaBuffer& vnew,
                       int pos, int width) {
    check(vb_cache_append(static_cast<float*>(kcache.ptr), static_cast<float*>(vcache.ptr),
                          static_cast<const float*>(knew.ptr), static_cast<const float*>(vnew.ptr), pos, width,
                          nullptr),
          "cuda_cache_append");
}

}  // namespace verbum
