/*
 * verbum_b200_backend.hpp -- the reference's CUDA launcher API, implemented
 * by this library (C++ only).
 *
 * verbum.cpp's CUDA path is Model::to_cuda / Model::step_cuda
 * (core/src/model.cpp:367-497) calling the launchers declared in
 * core/include/verbum/cuda_backend.h:7-43.  libverbum_b200.so defines those
 * same functions, with the same names, namespace and signatures (a C++ ABI:
 * these have to match the reference's declarations symbol for symbol), on top
 * of the C ABI in verbum_b200.h.  So the reference's unmodified model.cpp,
 * compiled with VERBUM_CUDA and linked against this library instead of its
 * kernels/cuda_ops.cu, runs its own step loop on the B200 kernels.
 *
 * Differences from the reference's implementation, each deliberate:
 * failures throw std::runtime_error (the reference's CUDA_CHECK aborts the
 * process, kernels/cuda_ops.cu:9-16); cuda_attn_decode has no context-length
 * limit (split-K); every call runs on the legacy default stream and the
 * copies are synchronous, as the reference's cudaMemcpy calls are.
 */
#pragma once

#include <cstddef>

#include "verbum_b200.h"

namespace verbum {

struct CudaBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
};

VB_API bool cuda_available();
VB_API const char* cuda_device_name();
VB_API size_t cuda_free_memory();

VB_API CudaBuffer cuda_alloc(size_t bytes);
VB_API void cuda_free(CudaBuffer& b);
VB_API void cuda_upload(CudaBuffer& dst, const void* host, size_t bytes);
VB_API void cuda_download(void* host, const CudaBuffer& src, size_t bytes);
VB_API void cuda_zero(CudaBuffer& b);
VB_API void cuda_sync();

VB_API void cuda_matmul_nt(const CudaBuffer& a, const CudaBuffer& b, CudaBuffer& c, int M, int N, int K);
VB_API void cuda_rmsnorm(const CudaBuffer& x, const CudaBuffer& w, CudaBuffer& out, int rows, int dim, float eps);
VB_API void cuda_rope(CudaBuffer& x, const CudaBuffer& cos_tab, const CudaBuffer& sin_tab, int pos, int heads, int D);
VB_API void cuda_silu_mul(CudaBuffer& gate, const CudaBuffer& up, int n);
VB_API void cuda_add(CudaBuffer& a, const CudaBuffer& b, int n);
VB_API void cuda_attn_decode(const CudaBuffer& q, const CudaBuffer& kcache, const CudaBuffer& vcache, CudaBuffer& out,
                             int H, int KVH, int D, int n);
VB_API void cuda_cache_append(CudaBuffer& kcache, CudaBuffer& vcache, const CudaBuffer& knew, const CudaBuffer& vnew,
                              int pos, int width);

}  // namespace verbum
