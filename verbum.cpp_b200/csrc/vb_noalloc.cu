// vb_noalloc.cu -- single-sequence decode attention that never allocates
// device memory.
//
// vb_attn_decode keeps its split-K partials in a buffer the library
// cudaMalloc's on first use.  Some callers cannot let a library do that: a
// host framework that owns every byte of device memory through its own pool
// and budgets it up front, a plugin whose enqueue call is forbidden to
// allocate, or a latency-critical loop that must not hit cudaMalloc's implicit
// device synchronisation or its failure modes in the middle of serving.  For
// them, vb_attn_decode_noalloc runs the same kernels with the partials in a
// fixed array compiled into this library.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "vb_kernels.cuh"

namespace vb {
namespace {

// 1 MiB: the split partials (H * splits * 132 floats) plus one length word.
// Every GPU that loads the library holds this array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};
CUcontext g_ctx[kMaxDevices] = {};

// In host code the array's name is only a host-side stand-in; the device
// address has to be looked up with the device current.  The lookup is done on
// the first call on a device and again whenever the device's current context
// is not the one the address was taken in (after a cudaDeviceReset the module
// is loaded anew into a new context).
// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link the driver library directly).
PFN_cuCtxGetCurrent_v4000 ctx_get_fn() {
    static PFN_cuCtxGetCurrent_v4000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    }();
    return fn;
}

vb_status scratch_address(void** out) {
    int dev = 0;
    VB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(VB_ERR_UNSUPPORTED, "device index above 63");
    const PFN_cuCtxGetCurrent_v4000 get_ctx = ctx_get_fn();
    if (!get_ctx) return fail(VB_ERR_CUDA, "cuCtxGetCurrent unavailable");
    CUcontext ctx = nullptr;
    if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(VB_ERR_CUDA, "cuCtxGetCurrent failed");
    if (!ctx) {
        // no context on this thread yet: cudaSetDevice makes the device's
        // primary context current (CUDA 12 and later initialise it there)
        VB_CUDA_TRY(cudaSetDevice(dev));
        if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
            return fail(VB_ERR_CUDA, "no current CUDA context for the noalloc scratch lookup");
    }
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[dev] || g_ctx[dev] != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_addr[dev] = p;
        g_ctx[dev] = ctx;
    }
    *out = g_addr[dev];
    return VB_OK;
}

__global__ void noalloc_set_len_kernel(int* dst, int n) { *dst = n; }

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" vb_status vb_attn_decode_noalloc(const float* q, const float* kcache,
                                            const float* vcache, float* out, int H, int KVH,
                                            int D, int n, void* stream) {
    if (!q || !kcache || !vcache || !out) return fail(VB_ERR_ARG, "null pointer");
    if (n <= 0 || H <= 0 || KVH <= 0) return fail(VB_ERR_ARG, "attention: non-positive shape");
    if (D != 128) return fail(VB_ERR_UNSUPPORTED, "attention: head_dim must be 128");
    // The split count the allocating entry point would use, capped at what the
    // static array holds: the split kernel takes any count (each split covers
    // ceil(n / splits) positions), so long contexts run with longer splits
    // instead of being refused.  Only a head count too large for even one
    // split is refused.
    const size_t per_split = attn_ws_bytes(1, H, 1);
    const size_t fit = (kNoAllocScratchBytes - 512) / per_split;
    if (fit < 1)
        return fail(VB_ERR_UNSUPPORTED,
                    "attention with " + std::to_string(H) + " heads needs " +
                        std::to_string(per_split + 512) +
                        " bytes of scratch for one split, more than the 1 MiB static buffer of "
                        "vb_attn_decode_noalloc (use vb_attn_decode)");
    int splits = attn_splits_for(1, KVH, n);
    if ((size_t)splits > fit) splits = (int)fit;
    const size_t part_bytes = attn_ws_bytes(1, H, splits);
    const size_t len_off = (part_bytes + 255) / 256 * 256;  // <= 1 MiB - 256
    void* base = nullptr;
    vb_status st = scratch_address(&base);
    if (st) return st;
    int* lens = reinterpret_cast<int*>(static_cast<char*>(base) + len_off);
    cudaStream_t s = as_stream(stream);
    // The partials need no clearing: every split writes its whole slot before
    // the merge reads it.  Only the length word is per call, written here.
    noalloc_set_len_kernel<<<1, 1, 0, s>>>(lens, n);
    VB_LAUNCH_CHECK("noalloc_set_len_kernel");
    AttnArgs a{};
    a.q = q; a.k = kcache; a.v = vcache; a.out = out; a.lens = lens;
    a.B = 1; a.H = H; a.KVH = KVH; a.D = D; a.n_max = n;
    a.stride_b = 0; a.stride_pos = (int64_t)KVH * D; a.stride_h = D;
    a.splits = splits;
    a.ws = static_cast<float*>(base);
    return launch_attention(a, s);
}
