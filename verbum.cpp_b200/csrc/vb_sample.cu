// vb_sample.cu -- Sampler::sample (generate.cpp:197-252) on the device, with
// the random draw taken on the host from the same generator the reference
// uses, so a seeded sampler picks the reference's tokens.
//
// The reference: temperature <= 0 or top_k == 1 -> greedy argmax (no draw);
// otherwise (logit, index) pairs partially sorted by logit, descending, the
// first keep = top_k (or all) kept; e_i = exp((v_i - v_0) / T) in float, their
// sum in double, p_i = float(e_i / sum); top_p < 1 keeps the shortest prefix
// whose double cumulative sum reaches top_p and renormalises it; then one
// uniform double r from std::mt19937_64 picks the first i with r <= the
// cumulative sum (else the last kept).
//
// Device form: a radix sort of all (logit, index) pairs (CUB, descending,
// ties keep index order) and one finishing block.  For keep <= 1024 one thread
// runs the reference's loops in the reference's order (the only difference is
// CUDA's expf against the host libm's, at most an ulp or two); for larger keep
// the block computes the same sums as parallel reductions and scans (the double
// sums differ from the sequential ones in their last bits).  The host draws r
// with std::mt19937_64 and std::uniform_real_distribution<double>, one draw per
// non-greedy sample, exactly as the reference does.
#include <cub/cub.cuh>

#include <random>

#include "vb_engine.cuh"

struct vb_sampler {
    float temperature = 0.8f;
    int top_k = 40;
    float top_p = 0.95f;
    std::mt19937_64 rng;
    int device = -1;
    int64_t cap = 0;  // vocabulary the buffers are sized for
    void* temp = nullptr;
    size_t temp_bytes = 0;
    float* keys = nullptr;    // sorted logits
    int* vals_in = nullptr;   // 0 .. vocab - 1
    int* vals_out = nullptr;  // sorted indices
    float* prob = nullptr;    // probabilities (large keep)
    double* d_r = nullptr;    // draws of the current call
    int r_cap = 0;
    int* d_tok = nullptr;
    int* h_tok = nullptr;  // pinned
};

namespace vb {
namespace {

constexpr int kSeqKeep = 1024;  // keep <= this: the reference's loops on one thread

__global__ void iota_kernel(int* v, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int)i;
}

// Block-wide inclusive scan of one double per thread (1024 threads); returns
// the thread's inclusive prefix, *total gets the block sum.
__device__ double block_scan_d(double x, double* sh, double* total) {
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        double s = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh[lane] = s;
    }
    __syncthreads();
    const double r = x + (w > 0 ? sh[w - 1] : 0.0);
    *total = sh[31];
    __syncthreads();
    return r;
}

// One block of 1024 threads over the sorted pairs.  Writes the pick to *out
// and, when tok is set, feeds it back as the engine's next token (tok, next)
// and records it at hist[*step - 1] (the step already advanced by the decode
// graph).
__global__ void __launch_bounds__(1024)
    sample_finish_kernel(const float* keys, const int* vals, int64_t vocab, float T, int top_k, float top_p,
                         const double* r_ptr, float* prob, int* out, int* tok, int* next, int* hist, const int* step,
                         int hist_cap) {
    __shared__ float p[kSeqKeep];
    __shared__ double sh[32];
    __shared__ int found;
    const int t = threadIdx.x;
    int64_t keep = vocab;
    if (top_k > 0 && top_k < keep) keep = top_k;
    const float m = keys[0];
    const double r = *r_ptr;
    int pick = vals[keep - 1];
    if (keep <= kSeqKeep) {
        if (t == 0) {
            double sum = 0.0;
            for (int i = 0; i < keep; i++) {
                p[i] = expf(__fdiv_rn(__fsub_rn(keys[i], m), T));
                sum += (double)p[i];
            }
            for (int i = 0; i < keep; i++) p[i] = (float)((double)p[i] / sum);
            int kept = (int)keep;
            if (top_p < 1.0f) {
                double cum = 0.0;
                for (int i = 0; i < keep; i++) {
                    cum += (double)p[i];
                    if (cum >= (double)top_p) {
                        kept = i + 1;
                        break;
                    }
                }
                double renorm = 0.0;
                for (int i = 0; i < kept; i++) renorm += (double)p[i];
                for (int i = 0; i < kept; i++) p[i] = (float)((double)p[i] / renorm);
            }
            double cum = 0.0;
            pick = vals[kept - 1];
            for (int i = 0; i < kept; i++) {
                cum += (double)p[i];
                if (r <= cum) {
                    pick = vals[i];
                    break;
                }
            }
            found = pick;
        }
        __syncthreads();
        pick = found;
    } else {
        // e_i and their sum
        double part = 0.0;
        for (int64_t i = t; i < keep; i += 1024) {
            const float e = expf(__fdiv_rn(__fsub_rn(keys[i], m), T));
            prob[i] = e;
            part += (double)e;
        }
        double sum;
        block_scan_d(part, sh, &sum);
        for (int64_t i = t; i < keep; i += 1024) prob[i] = (float)((double)prob[i] / sum);
        __syncthreads();
        int64_t kept = keep;
        if (top_p < 1.0f) {
            // first i whose cumulative sum reaches top_p, chunk by chunk
            if (t == 0) found = -1;
            __syncthreads();
            double carry = 0.0;
            for (int64_t c0 = 0; c0 < keep; c0 += 1024) {
                const int64_t i = c0 + t;
                const double x = i < keep ? (double)prob[i] : 0.0;
                double tot;
                const double inc = carry + block_scan_d(x, sh, &tot);
                if (i < keep && inc >= (double)top_p) atomicMin(reinterpret_cast<unsigned*>(&found), (unsigned)t);
                __syncthreads();
                if (found >= 0) {
                    kept = c0 + found + 1;
                    break;
                }
                carry += tot;
            }
            double rp = 0.0;
            for (int64_t i = t; i < kept; i += 1024) rp += (double)prob[i];
            double renorm;
            block_scan_d(rp, sh, &renorm);
            for (int64_t i = t; i < kept; i += 1024) prob[i] = (float)((double)prob[i] / renorm);
            __syncthreads();
        }
        if (t == 0) found = -1;
        __syncthreads();
        double carry = 0.0;
        pick = vals[kept - 1];
        for (int64_t c0 = 0; c0 < kept; c0 += 1024) {
            const int64_t i = c0 + t;
            const double x = i < kept ? (double)prob[i] : 0.0;
            double tot;
            const double inc = carry + block_scan_d(x, sh, &tot);
            if (i < kept && r <= inc) atomicMin(reinterpret_cast<unsigned*>(&found), (unsigned)t);
            __syncthreads();
            if (found >= 0) {
                pick = vals[c0 + found];
                break;
            }
            carry += tot;
        }
    }
    if (t == 0) {
        *out = pick;
        if (tok) {
            *tok = pick;
            *next = pick;
            const int s = *step - 1;
            if (s >= 0 && s < hist_cap) hist[s] = pick;
        }
    }
}

vb_status sampler_buffers(vb_sampler* sp, int64_t vocab, cudaStream_t s) {
    int dev = 0;
    VB_CUDA_TRY(cudaGetDevice(&dev));
    if (sp->cap >= vocab && sp->device == dev) return VB_OK;
    if (sp->device >= 0 && sp->device != dev) return fail(VB_ERR_ARG, "sampler: used on another device");
    for (void* p : {(void*)sp->keys, (void*)sp->vals_in, (void*)sp->vals_out, (void*)sp->prob, sp->temp})
        if (p) cudaFree(p);
    sp->keys = nullptr;
    sp->vals_in = sp->vals_out = nullptr;
    sp->prob = nullptr;
    sp->temp = nullptr;
    size_t tb = 0;
    VB_CUDA_TRY(cub::DeviceRadixSort::SortPairsDescending(nullptr, tb, (const float*)nullptr, (float*)nullptr,
                                                          (const int*)nullptr, (int*)nullptr, (int)vocab));
    VB_CUDA_TRY(cudaMalloc(&sp->temp, tb));
    VB_CUDA_TRY(cudaMalloc(&sp->keys, sizeof(float) * vocab));
    VB_CUDA_TRY(cudaMalloc(&sp->vals_in, sizeof(int) * vocab));
    VB_CUDA_TRY(cudaMalloc(&sp->vals_out, sizeof(int) * vocab));
    VB_CUDA_TRY(cudaMalloc(&sp->prob, sizeof(float) * vocab));
    if (!sp->d_tok) VB_CUDA_TRY(cudaMalloc(&sp->d_tok, sizeof(int)));
    if (!sp->h_tok) VB_CUDA_TRY(cudaMallocHost(&sp->h_tok, sizeof(int)));
    sp->temp_bytes = tb;
    iota_kernel<<<64, 256, 0, s>>>(sp->vals_in, vocab);
    VB_LAUNCH_CHECK("iota_kernel");
    sp->cap = vocab;
    sp->device = dev;
    return VB_OK;
}

}  // namespace

bool sampler_greedy(const vb_sampler* sp) { return sp->temperature <= 0.0f || sp->top_k == 1; }

vb_status sampler_draws(vb_sampler* sp, int n, cudaStream_t s) {
    if (sp->r_cap < n) {
        if (sp->d_r) cudaFree(sp->d_r);
        sp->d_r = nullptr;
        sp->r_cap = 0;
        VB_CUDA_TRY(cudaMalloc(&sp->d_r, sizeof(double) * n));
        sp->r_cap = n;
    }
    std::vector<double> r(n);
    for (int i = 0; i < n; i++) {
        std::uniform_real_distribution<double> dist(0.0, 1.0);
        r[i] = dist(sp->rng);
    }
    VB_CUDA_TRY(cudaMemcpyAsync(sp->d_r, r.data(), sizeof(double) * n, cudaMemcpyHostToDevice, s));
    // the host vector dies here: wait for the copy
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    return VB_OK;
}

// Sort + finish for draw `draw` (of the last sampler_draws); see the kernel for
// the engine feedback arguments.
vb_status launch_sample(vb_sampler* sp, const float* logits, int64_t vocab, int draw, int* out, int* tok, int* next,
                        int* hist, const int* step, int hist_cap, cudaStream_t s) {
    vb_status st;
    if ((st = sampler_buffers(sp, vocab, s))) return st;
    size_t tb = sp->temp_bytes;
    VB_CUDA_TRY(cub::DeviceRadixSort::SortPairsDescending(sp->temp, tb, logits, sp->keys, sp->vals_in, sp->vals_out,
                                                          (int)vocab, 0, 32, s));
    sample_finish_kernel<<<1, 1024, 0, s>>>(sp->keys, sp->vals_out, vocab, sp->temperature, sp->top_k, sp->top_p,
                                            sp->d_r + draw, sp->prob, out, tok, next, hist, step, hist_cap);
    VB_LAUNCH_CHECK("sample_finish_kernel");
    return VB_OK;
}

}  // namespace vb

using namespace vb;

extern "C" {

vb_status vb_sampler_create(float temperature, int top_k, float top_p, uint64_t seed, vb_sampler** out) {
    if (!out) return fail(VB_ERR_ARG, "null argument");
    *out = nullptr;
    if (top_k < 0) return fail(VB_ERR_ARG, "sampler: top_k < 0");
    vb_sampler* sp = new vb_sampler();
    sp->temperature = temperature;
    sp->top_k = top_k;
    sp->top_p = top_p;
    sp->rng.seed(seed);
    *out = sp;
    return VB_OK;
}

vb_status vb_sampler_destroy(vb_sampler* sp) {
    if (!sp) return VB_OK;
    for (void* p : {(void*)sp->keys, (void*)sp->vals_in, (void*)sp->vals_out, (void*)sp->prob, sp->temp,
                    (void*)sp->d_r, (void*)sp->d_tok})
        if (p) cudaFree(p);
    if (sp->h_tok) cudaFreeHost(sp->h_tok);
    delete sp;
    return VB_OK;
}

vb_status vb_sampler_sample(vb_sampler* sp, const float* logits, int64_t vocab, void* stream, int* token) {
    if (!sp || !logits || !token) return fail(VB_ERR_ARG, "null argument");
    if (vocab <= 0 || vocab > INT32_MAX) return fail(VB_ERR_ARG, "sampler: vocab out of range");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    vb_status st;
    if ((st = sampler_buffers(sp, vocab, s))) return st;
    if (sampler_greedy(sp)) {
        if ((st = launch_argmax_rows(logits, 1, vocab, sp->d_tok, s))) return st;
    } else {
        if ((st = sampler_draws(sp, 1, s))) return st;
        if ((st = launch_sample(sp, logits, vocab, 0, sp->d_tok, nullptr, nullptr, nullptr, nullptr, 0, s)))
            return st;
    }
    VB_CUDA_TRY(cudaMemcpyAsync(sp->h_tok, sp->d_tok, sizeof(int), cudaMemcpyDeviceToHost, s));
    VB_CUDA_TRY(cudaStreamSynchronize(s));
    *token = *sp->h_tok;
    return VB_OK;
}

}  // extern "C"
