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
// Device form: for top_k <= 1024 a radix select (two 4096-bin histograms of
// the logits' order-preserving keys, 12 bits each, find the 24-bit bin
// holding the k-th largest; the keys at or above it are compacted and sorted
// in one block); otherwise a
// radix sort of all (logit, index) pairs (CUB, descending, ties keep index
// order).  Then one finishing block.  For keep <= 1024 one thread
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
    unsigned* hist = nullptr; // two 4096-bin key histograms, candidate count, threshold
    unsigned long long* cand = nullptr;  // [kCand] packed candidates
    unsigned* sel = nullptr;  // bitmap of picked indices (selection fallback)
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

// ---- top-k by radix select (top_k <= 1024) ----------------------------------
constexpr int kBins = 4096;
constexpr int kCand = 4096;  // candidates sorted in shared memory

// Order-preserving key: larger float -> larger unsigned.
__device__ __forceinline__ unsigned fkey(float x) {
    const unsigned u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float funkey(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
// Candidate: (key descending, index ascending) as one ascending 64-bit value.
__device__ __forceinline__ unsigned long long pack_cand(unsigned key, int idx) {
    return ((unsigned long long)(~key) << 32) | (unsigned)idx;
}

// Histogram of 12 key bits.  Level 0: bits [20, 32) of every key; level 1:
// bits [8, 20) of the keys whose top 12 bits equal the level-0 bin in
// thr[0] >> 20.  Same-bin updates of a warp are combined before the
// shared-memory atomic (logits crowd into few bins).
__global__ void __launch_bounds__(256) topk_hist_kernel(const float* x, int64_t n, unsigned* hist, int level,
                                                        const unsigned* thr) {
    __shared__ unsigned h[kBins];
    for (int i = threadIdx.x; i < kBins; i += 256) h[i] = 0;
    __syncthreads();
    const unsigned top = level ? (*thr >> 20) : 0u;
    const int64_t n_pad = (n + 255) / 256 * 256;
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n_pad; i += (int64_t)gridDim.x * 256) {
        int bin = -1;
        if (i < n) {
            const unsigned key = fkey(x[i]);
            if (level == 0) bin = (int)(key >> 20);
            else if ((key >> 20) == top) bin = (int)((key >> 8) & 0xFFFu);
        }
        const unsigned same = __match_any_sync(0xffffffffu, bin);
        if (bin >= 0 && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&h[bin], (unsigned)__popc(same));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kBins; i += 256)
        if (h[i]) atomicAdd(&hist[i], h[i]);
}

// Bin b* holding the k-th largest key: sum of the bins above it < k <= that
// sum plus its own count.  One block of 1024 threads, 4 bins per thread from
// the top.
__device__ unsigned topk_threshold(const unsigned* hist, int k, unsigned* sh) {
    const int t = threadIdx.x;
    unsigned c[4], s = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        c[j] = hist[kBins - 1 - (4 * t + j)];
        s += c[j];
    }
    // inclusive scan of s over the block (threads in descending-bin order)
    const int lane = t & 31, w = t >> 5;
    unsigned x = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        unsigned v = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        sh[lane] = v;
    }
    __syncthreads();
    const unsigned before = x - s + (w > 0 ? sh[w - 1] : 0u);
    __syncthreads();
    if (t == 0) sh[32] = 0;
    __syncthreads();
    unsigned run = before;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (run < (unsigned)k && run + c[j] >= (unsigned)k) {
            sh[32] = (unsigned)(kBins - 1 - (4 * t + j));
            sh[33] = run;  // keys in the bins above
        }
        run += c[j];
    }
    __syncthreads();
    return sh[32] << 20;
}

// Level 0: thr[0] = the bin of the k-th largest key (<< 20) and thr[1] = the
// number of keys in bins above it.  Level 1: thr[0] |= the level-1 bin (<< 8)
// holding the (k - thr[1])-th largest of the level-0 bin's keys.
__global__ void __launch_bounds__(1024) topk_thr_kernel(const unsigned* hist, int k, int level, unsigned* thr) {
    __shared__ unsigned sh[34];
    const int kk = level ? k - (int)thr[1] : k;
    const unsigned b = topk_threshold(hist, kk, sh);  // bin << 20
    if (threadIdx.x == 0) {
        if (level == 0) {
            thr[0] = b;
            thr[1] = sh[33];
        } else {
            thr[0] |= (b >> 20) << 8;
        }
    }
}

__global__ void __launch_bounds__(256) topk_compact_kernel(const float* x, int64_t n, const unsigned* thr_ptr,
                                                           unsigned* count, unsigned long long* cand) {
    const unsigned T = *thr_ptr;  // keys >= T: the k largest and the rest of their level-1 bin
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        const unsigned key = fkey(x[i]);
        if (key >= T) {
            const unsigned pos = atomicAdd(count, 1u);
            if (pos < (unsigned)kCand) cand[pos] = pack_cand(key, (int)i);
        }
    }
}

// Sequential finish (keep <= 1024) over sorted keys/vals in any memory: the
// reference's loops in its order.  Returns the pick.
__device__ int finish_seq(const float* keys, const int* vals, int keep, float T, float top_p, double r, float* p) {
    const float m = keys[0];
    double sum = 0.0;
    for (int i = 0; i < keep; i++) {
        p[i] = expf(__fdiv_rn(__fsub_rn(keys[i], m), T));
        sum += (double)p[i];
    }
    for (int i = 0; i < keep; i++) p[i] = (float)((double)p[i] / sum);
    int kept = keep;
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
    for (int i = 0; i < kept; i++) {
        cum += (double)p[i];
        if (r <= cum) return vals[i];
    }
    return vals[kept - 1];
}

// Top-k path: sort the candidates (<= kCand) in shared memory, or, when more
// keys than kCand tie at the threshold bin, select the k largest by k rounds of
// a block argmax (lowest index first on ties); then the sequential finish.
__global__ void __launch_bounds__(1024)
    topk_finish_kernel(const float* x, int64_t n, const unsigned* count, const unsigned long long* cand, int k,
                       float T, float top_p, const double* r_ptr, unsigned* sel, int* out, int* tok, int* next,
                       int* hist, const int* step, int hist_cap) {
    __shared__ unsigned long long c[kCand];
    __shared__ float kv[1024];
    __shared__ int ki[1024];
    __shared__ float p[1024];
    __shared__ unsigned long long best[32];
    const int t = threadIdx.x;
    const unsigned cnt = *count;
    if (cnt <= (unsigned)kCand) {
        // bitonic sort (ascending) of the candidates padded to a power of two
        int n2 = 2;
        while (n2 < (int)cnt) n2 <<= 1;
        for (int i = t; i < n2; i += 1024) c[i] = i < (int)cnt ? cand[i] : ~0ull;
        __syncthreads();
        for (int size = 2; size <= n2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = t; i < n2 / 2; i += 1024) {
                    const int lo = 2 * i - (i & (stride - 1));
                    const int hi = lo + stride;
                    const bool up = (lo & size) == 0;
                    const unsigned long long a = c[lo], b = c[hi];
                    if ((a > b) == up) {
                        c[lo] = b;
                        c[hi] = a;
                    }
                }
                __syncthreads();
            }
        for (int i = t; i < k; i += 1024) {
            kv[i] = funkey(~(unsigned)(c[i] >> 32));
            ki[i] = (int)(unsigned)(c[i] & 0xFFFFFFFFull);
        }
    } else {
        for (int64_t i = t; i < (n + 31) / 32; i += 1024) sel[i] = 0u;
        __syncthreads();
        for (int j = 0; j < k; j++) {
            unsigned long long b = ~0ull;
            for (int64_t i = t; i < n; i += 1024)
                if (!(sel[i >> 5] & (1u << (i & 31)))) {
                    const unsigned long long pc = pack_cand(fkey(x[i]), (int)i);
                    b = pc < b ? pc : b;
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long y = __shfl_xor_sync(0xffffffffu, b, o);
                b = y < b ? y : b;
            }
            if ((t & 31) == 0) best[t >> 5] = b;
            __syncthreads();
            if (t < 32) {
                b = best[t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long y = __shfl_xor_sync(0xffffffffu, b, o);
                    b = y < b ? y : b;
                }
                if (t == 0) {
                    const int idx = (int)(unsigned)(b & 0xFFFFFFFFull);
                    kv[j] = funkey(~(unsigned)(b >> 32));
                    ki[j] = idx;
                    sel[idx >> 5] |= 1u << (idx & 31);
                }
            }
            __syncthreads();
        }
    }
    __syncthreads();
    if (t == 0) {
        const int pick = finish_seq(kv, ki, k, T, top_p, *r_ptr, p);
        *out = pick;
        if (tok) {
            *tok = pick;
            *next = pick;
            const int st = *step - 1;
            if (st >= 0 && st < hist_cap) hist[st] = pick;
        }
    }
}

vb_status sampler_buffers(vb_sampler* sp, int64_t vocab, cudaStream_t s) {
    int dev = 0;
    VB_CUDA_TRY(cudaGetDevice(&dev));
    if (sp->cap >= vocab && sp->device == dev) return VB_OK;
    if (sp->device >= 0 && sp->device != dev) return fail(VB_ERR_ARG, "sampler: used on another device");
    for (void* p : {(void*)sp->keys, (void*)sp->vals_in, (void*)sp->vals_out, (void*)sp->prob, sp->temp,
                    (void*)sp->hist, (void*)sp->cand, (void*)sp->sel})
        if (p) cudaFree(p);
    sp->hist = nullptr;
    sp->cand = nullptr;
    sp->sel = nullptr;
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
    VB_CUDA_TRY(cudaMalloc(&sp->hist, sizeof(unsigned) * (2 * kBins + 4)));
    VB_CUDA_TRY(cudaMalloc(&sp->cand, sizeof(unsigned long long) * kCand));
    VB_CUDA_TRY(cudaMalloc(&sp->sel, sizeof(unsigned) * ((vocab + 31) / 32)));
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
    if (sp->top_k > 0 && sp->top_k <= 1024 && sp->top_k < vocab) {
        // hist: [0, 4096) level 0, [4096, 8192) level 1, [8192] count, [8193, 8195) threshold
        unsigned* h0 = sp->hist;
        unsigned* h1 = sp->hist + kBins;
        unsigned* cnt = sp->hist + 2 * kBins;
        unsigned* thr = cnt + 1;
        VB_CUDA_TRY(cudaMemsetAsync(sp->hist, 0, sizeof(unsigned) * (2 * kBins + 4), s));
        topk_hist_kernel<<<148, 256, 0, s>>>(logits, vocab, h0, 0, thr);
        VB_LAUNCH_CHECK("topk_hist_kernel");
        topk_thr_kernel<<<1, 1024, 0, s>>>(h0, sp->top_k, 0, thr);
        VB_LAUNCH_CHECK("topk_thr_kernel");
        topk_hist_kernel<<<148, 256, 0, s>>>(logits, vocab, h1, 1, thr);
        VB_LAUNCH_CHECK("topk_hist_kernel");
        topk_thr_kernel<<<1, 1024, 0, s>>>(h1, sp->top_k, 1, thr);
        VB_LAUNCH_CHECK("topk_thr_kernel");
        topk_compact_kernel<<<148, 256, 0, s>>>(logits, vocab, thr, cnt, sp->cand);
        VB_LAUNCH_CHECK("topk_compact_kernel");
        topk_finish_kernel<<<1, 1024, 0, s>>>(logits, vocab, cnt, sp->cand, sp->top_k, sp->temperature,
                                              sp->top_p, sp->d_r + draw, sp->sel, out, tok, next, hist, step,
                                              hist_cap);
        VB_LAUNCH_CHECK("topk_finish_kernel");
        return VB_OK;
    }
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
                    (void*)sp->d_r, (void*)sp->d_tok, (void*)sp->hist, (void*)sp->cand, (void*)sp->sel})
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
