// vb_capi.cu -- extern "C" kernel entry points, memory helpers and error
// state of the C ABI declared in include/verbum_b200.h.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "vb_kernels.cuh"

namespace vb {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

vb_status fail(vb_status code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

vb_status cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return VB_ERR_CUDA;
}

namespace {

// Per-device scratch for vb_attn_decode's split partials: allocated on first
// use, grown on demand, kept for the life of the process.
struct AttnScratch {
    std::mutex mu;
    std::vector<void*> ptr;
    std::vector<size_t> bytes;
};
AttnScratch& attn_scratch() {
    static AttnScratch s;
    return s;
}

vb_status scratch_for(size_t need, void** out) {
    int dev = 0;
    VB_CUDA_TRY(cudaGetDevice(&dev));
    AttnScratch& s = attn_scratch();
    std::lock_guard<std::mutex> lk(s.mu);
    if ((int)s.ptr.size() <= dev) {
        s.ptr.resize(dev + 1, nullptr);
        s.bytes.resize(dev + 1, 0);
    }
    if (s.bytes[dev] < need) {
        if (s.ptr[dev]) {
            cudaDeviceSynchronize();
            cudaFree(s.ptr[dev]);
        }
        s.ptr[dev] = nullptr;
        s.bytes[dev] = 0;
        VB_CUDA_TRY(cudaMalloc(&s.ptr[dev], need));
        s.bytes[dev] = need;
    }
    *out = s.ptr[dev];
    return VB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::atomic<int> g_fault_site{kFaultNone};

}  // namespace

bool fault_take(int site) {
    int want = site;
    return site != kFaultNone && g_fault_site.compare_exchange_strong(want, kFaultNone);
}
}  // namespace vb

using namespace vb;

extern "C" {

const char* vb_last_error(void) { return g_last_error.c_str(); }

const char* vb_version(void) { return "verbum-b200 0.1 (sm_100a)"; }

vb_status vb_debug_arm_fault(int site) {
    if (site < kFaultNone || site > kFaultGemmStage) return fail(VB_ERR_ARG, "fault site must be 0, 1 or 2");
    g_fault_site.store(site);
    return VB_OK;
}

int vb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

vb_status vb_device_name(int dev, char* buf, size_t len) {
    if (!buf || len == 0) return fail(VB_ERR_ARG, "null buffer");
    cudaDeviceProp p;
    VB_CUDA_TRY(cudaGetDeviceProperties(&p, dev));
    snprintf(buf, len, "%s", p.name);
    return VB_OK;
}

vb_status vb_free_memory(int dev, size_t* free_bytes) {
    if (!free_bytes) return fail(VB_ERR_ARG, "null argument");
    int prev = 0;
    VB_CUDA_TRY(cudaGetDevice(&prev));
    VB_CUDA_TRY(cudaSetDevice(dev));
    size_t f = 0, t = 0;
    cudaError_t e = cudaMemGetInfo(&f, &t);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemGetInfo");
    *free_bytes = f;
    return VB_OK;
}

vb_status vb_alloc(void** ptr, size_t bytes) {
    if (!ptr) return fail(VB_ERR_ARG, "null argument");
    VB_CUDA_TRY(cudaMalloc(ptr, bytes ? bytes : 1));
    return VB_OK;
}

vb_status vb_free(void* ptr) {
    if (ptr) VB_CUDA_TRY(cudaFree(ptr));
    return VB_OK;
}

vb_status vb_upload(void* dst, const void* host, size_t bytes, void* stream) {
    VB_CUDA_TRY(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    VB_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    return VB_OK;
}

vb_status vb_download(void* host, const void* src, size_t bytes, void* stream) {
    VB_CUDA_TRY(cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    VB_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    return VB_OK;
}

vb_status vb_zero(void* dst, size_t bytes, void* stream) {
    VB_CUDA_TRY(cudaMemsetAsync(dst, 0, bytes, as_stream(stream)));
    return VB_OK;
}

vb_status vb_sync(void* stream) {
    VB_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    return VB_OK;
}

vb_status vb_matmul_nt_f32(const float* A, const float* W, float* C, int M, int N, int K,
                           void* stream) {
    if (!A || !W || !C) return fail(VB_ERR_ARG, "null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return fail(VB_ERR_ARG, "matmul_nt: non-positive shape");
    if (!aligned16(A) || !aligned16(W) || K % 4) return fail(VB_ERR_UNSUPPORTED, "matmul_nt: needs 16-byte alignment and K % 4 == 0");
    cudaStream_t s = as_stream(stream);
    if (M == 1) {
        GemvArgs g{};
        g.x = A;
        g.W = W;
        g.y = C;
        g.N = N;
        g.K = K;
        // weights that fit one prefetched slice per SM: the prefetching GEMV
        // (its weights stream in while the previous kernel on the stream runs)
        if (K <= 4096 && gemv_pf_parts(N, K, false, kEpiStore) == 1) return launch_gemv_pf(g, false, kProNone, kEpiStore, s);
        return launch_gemv(g, false, kProNone, kEpiStore, s);
    }
    if (M <= 64 && K % 32 == 0) {
        void* ws = nullptr;
        const size_t wf = gemm_ws_floats(M, N, K, false);
        vb_status st = scratch_for(wf * 4, &ws);
        if (st) return st;
        GemmArgs g{};
        g.A = A; g.W = W; g.C = C; g.M = M; g.N = N; g.K = K; g.ldc = N;
        g.ws = static_cast<float*>(ws);
        g.ws_floats = wf;
        return launch_gemm(g, false, kEpiStore, s);
    }
    for (int m = 0; m < M; m++) {
        GemvArgs g{};
        g.x = A + (size_t)m * K;
        g.W = W;
        g.y = C + (size_t)m * N;
        g.N = N;
        g.K = K;
        vb_status st = launch_gemv(g, false, kProNone, kEpiStore, s);
        if (st) return st;
    }
    return VB_OK;
}

vb_status vb_matmul_nt_q8(const float* A, const int8_t* Wq, const float* scales, float* C,
                          int M, int N, int K, void* stream) {
    if (!A || !Wq || !scales || !C) return fail(VB_ERR_ARG, "null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return fail(VB_ERR_ARG, "matmul_nt_q8: non-positive shape");
    if (!aligned16(A) || !aligned16(Wq) || K % 16) return fail(VB_ERR_UNSUPPORTED, "matmul_nt_q8: needs 16-byte alignment and K % 16 == 0");
    cudaStream_t s = as_stream(stream);
    if (M == 1) {
        GemvArgs g{};
        g.x = A;
        g.W = Wq;
        g.scales = scales;
        g.y = C;
        g.N = N;
        g.K = K;
        if (K <= 4096 && gemv_pf_parts(N, K, true, kEpiStore) == 1) return launch_gemv_pf(g, true, kProNone, kEpiStore, s);
        return launch_gemv(g, true, kProNone, kEpiStore, s);
    }
    if (M <= 64 && K % 32 == 0) {
        void* ws = nullptr;
        const size_t wf = gemm_ws_floats(M, N, K, true);
        vb_status st = scratch_for(wf * 4, &ws);
        if (st) return st;
        GemmArgs g{};
        g.A = A; g.W = Wq; g.scales = scales; g.C = C; g.M = M; g.N = N; g.K = K; g.ldc = N;
        g.ws = static_cast<float*>(ws);
        g.ws_floats = wf;
        return launch_gemm(g, true, kEpiStore, s);
    }
    for (int m = 0; m < M; m++) {
        GemvArgs g{};
        g.x = A + (size_t)m * K;
        g.W = Wq;
        g.scales = scales;
        g.y = C + (size_t)m * N;
        g.N = N;
        g.K = K;
        vb_status st = launch_gemv(g, true, kProNone, kEpiStore, s);
        if (st) return st;
    }
    return VB_OK;
}

vb_status vb_matmul_nt_tc(const float* A, const void* W, const float* scales, float* C, int M, int N, int K,
                          int w_int8, void* stream) {
    if (!A || !W || !C || (w_int8 && !scales)) return fail(VB_ERR_ARG, "null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || K % 64)
        return fail(VB_ERR_UNSUPPORTED, "matmul_nt_tc: needs M >= 1 and K % 64 == 0");
    cudaStream_t s = as_stream(stream);
    const size_t wf = M <= 64 ? tc_gemm_ws_floats(M, N, K) : 0;
    const size_t a_bytes = (size_t)std::max(M, 64) * K * 2, w_bytes = (size_t)N * K * 2;
    const size_t off_ahi = 256;
    const size_t off_alo = off_ahi + a_bytes, off_whi = off_alo + a_bytes;
    const size_t off_wlo = off_whi + w_bytes, off_ws = off_wlo + (w_int8 ? 0 : w_bytes);
    void* base = nullptr;
    vb_status st = scratch_for(off_ws + wf * 4, &base);
    if (st) return st;
    char* b = static_cast<char*>(base);
    int* err = reinterpret_cast<int*>(b);
    VB_CUDA_TRY(cudaMemsetAsync(b, 0, sizeof(int), s));  // error word
    if ((st = launch_split_bf16(A, M, K, K, b + off_ahi, b + off_alo, s))) return st;
    if ((st = launch_weights_bf16(W, w_int8 != 0, (size_t)N * K, b + off_whi, w_int8 ? nullptr : b + off_wlo, s)))
        return st;
    TcGemmArgs t{};
    t.w_hi = b + off_whi;
    t.w_lo = w_int8 ? nullptr : b + off_wlo;
    t.a_hi = b + off_ahi;
    t.a_lo = b + off_alo;
    t.M = M;
    t.N = N;
    t.K = K;
    t.ws = reinterpret_cast<float*>(b + off_ws);
    t.ws_floats = wf;
    t.scales = w_int8 ? scales : nullptr;
    t.C = C;
    t.ldc = N;
    t.epi = kEpiStore;
    t.err = err;
    if ((st = launch_tc_gemm(t, s))) return st;
    int h_err = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    if (h_err) return fail(VB_ERR_TIMEOUT, "matmul_nt_tc: a bounded wait in the kernel gave up");
    return VB_OK;
}

vb_status vb_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q, float* scales,
                           void* stream) {
    if (!W || !q || !scales) return fail(VB_ERR_ARG, "null pointer");
    return launch_quantize_rows(W, rows, cols, q, scales, as_stream(stream));
}

vb_status vb_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps,
                     void* stream) {
    if (!x || !w || !out) return fail(VB_ERR_ARG, "null pointer");
    return launch_rmsnorm_rows(x, w, out, rows, dim, eps, as_stream(stream));
}

vb_status vb_rope(float* x, const float* cos_tab, const float* sin_tab, int pos, int heads, int D,
                  void* stream) {
    if (!x || !cos_tab || !sin_tab) return fail(VB_ERR_ARG, "null pointer");
    if (pos < 0) return fail(VB_ERR_ROPE, "position is outside the rope table");
    return launch_rope(x, cos_tab, sin_tab, pos, heads, D, as_stream(stream));
}

vb_status vb_silu_mul(float* gate, const float* up, int n, void* stream) {
    if (!gate || !up) return fail(VB_ERR_ARG, "null pointer");
    return launch_silu_mul(gate, up, n, as_stream(stream));
}

vb_status vb_add(float* a, const float* b, int n, void* stream) {
    if (!a || !b) return fail(VB_ERR_ARG, "null pointer");
    return launch_add(a, b, n, as_stream(stream));
}

vb_status vb_cache_append(float* kcache, float* vcache, const float* knew, const float* vnew,
                          int pos, int width, void* stream) {
    if (!kcache || !vcache || !knew || !vnew) return fail(VB_ERR_ARG, "null pointer");
    return launch_cache_append(kcache, vcache, knew, vnew, pos, width, as_stream(stream));
}

size_t vb_attn_workspace_bytes(int B, int H, int n_max) {
    if (B <= 0 || H <= 0 || n_max <= 0) return 0;
    // splits depend on KVH only through the grid target; size for KVH = 1
    // (the most splits), which bounds every KVH.
    return attn_ws_bytes(B, H, attn_splits_for(B, 1, n_max));
}

vb_status vb_attn_decode_batched(const float* q, const float* k, const float* v, float* out,
                                 const int* lens, int B, int H, int KVH, int D, int n_max,
                                 int64_t stride_b, int64_t stride_pos, int64_t stride_h,
                                 void* workspace, void* stream) {
    if (!q || !k || !v || !out || !lens || !workspace) return fail(VB_ERR_ARG, "null pointer");
    if (B <= 0 || H <= 0 || KVH <= 0 || n_max <= 0) return fail(VB_ERR_ARG, "attention: non-positive shape");
    if (D != 128) return fail(VB_ERR_UNSUPPORTED, "attention: head_dim must be 128");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(workspace) ||
        (stride_b | stride_pos | stride_h) & 3)
        return fail(VB_ERR_UNSUPPORTED, "attention: 16-byte alignment required");
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = out; a.lens = lens;
    a.B = B; a.H = H; a.KVH = KVH; a.D = D; a.n_max = n_max;
    a.stride_b = stride_b; a.stride_pos = stride_pos; a.stride_h = stride_h;
    a.splits = attn_splits_for(B, KVH, n_max);
    a.ws = static_cast<float*>(workspace);
    return launch_attention(a, as_stream(stream));
}

vb_status vb_attn_prefill(const float* q, const float* k, const float* v, float* out, int B, int C, int p0,
                          int H, int KVH, int D, int64_t stride_b, int64_t stride_h, void* stream) {
    if (!q || !k || !v || !out) return fail(VB_ERR_ARG, "null pointer");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (stride_b | stride_h) & 3)
        return fail(VB_ERR_UNSUPPORTED, "attention: 16-byte alignment required");
    PrefillAttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = out;
    a.stride_b = stride_b; a.stride_h = stride_h;
    a.B = B; a.C = C; a.p0 = p0; a.H = H; a.KVH = KVH; a.D = D;
    if (p0 != 0 || H != 2 * KVH || D != 128 || B <= 0 || C <= 0) return launch_prefill_attention(a, as_stream(stream));
    // a prompt from position 0: the tensor-core form (bf16 hi/lo copies in the scratch buffer)
    cudaStream_t s = as_stream(stream);
    const size_t split = (size_t)B * C * H * D * 2;
    const size_t need = 256 + 2 * split + prompt_attention_tc_bytes(B, C, H, KVH);
    void* base = nullptr;
    vb_status st = scratch_for(need, &base);
    if (st) return st;
    char* sc = static_cast<char*>(base);
    int* err = reinterpret_cast<int*>(sc);
    VB_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), s));
    a.err = err;
    a.out_hi = sc + 256;
    a.out_lo = sc + 256 + split;
    if ((st = launch_prompt_attention_tc(a, q, sc + 256 + 2 * split, s))) return st;
    int h_err = 0;
    VB_CUDA_TRY(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    if (h_err) return fail(VB_ERR_TIMEOUT, "attn_prefill: a bounded wait in the kernel gave up");
    return VB_OK;
}

vb_status vb_attn_decode(const float* q, const float* kcache, const float* vcache, float* out,
                         int H, int KVH, int D, int n, void* stream) {
    if (!q || !kcache || !vcache || !out) return fail(VB_ERR_ARG, "null pointer");
    if (n <= 0 || H <= 0 || KVH <= 0) return fail(VB_ERR_ARG, "attention: non-positive shape");
    if (D != 128) return fail(VB_ERR_UNSUPPORTED, "attention: head_dim must be 128");
    const int splits = attn_splits_for(1, KVH, n);
    const size_t need = attn_ws_bytes(1, H, splits) + 256;
    void* ws = nullptr;
    vb_status st = scratch_for(need, &ws);
    if (st) return st;
    // the length lives in the scratch tail so the kernel reads it from device
    int* lens = reinterpret_cast<int*>(static_cast<char*>(ws) + need - 256);
    cudaStream_t s = as_stream(stream);
    VB_CUDA_TRY(cudaMemcpyAsync(lens, &n, sizeof(int), cudaMemcpyHostToDevice, s));
    AttnArgs a{};
    a.q = q; a.k = kcache; a.v = vcache; a.out = out; a.lens = lens;
    a.B = 1; a.H = H; a.KVH = KVH; a.D = D; a.n_max = n;
    a.stride_b = 0; a.stride_pos = (int64_t)KVH * D; a.stride_h = D;
    a.splits = splits;
    a.ws = static_cast<float*>(ws);
    return launch_attention(a, s);
}

vb_status vb_argmax_rows(const float* logits, int rows, int64_t n, int* out_idx, void* stream) {
    if (!logits || !out_idx) return fail(VB_ERR_ARG, "null pointer");
    return launch_argmax_rows(logits, rows, n, out_idx, as_stream(stream));
}

}  // extern "C"
