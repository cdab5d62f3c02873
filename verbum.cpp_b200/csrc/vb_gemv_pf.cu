// vb_gemv_pf.cu -- batch-1 GEMV whose weights are in shared memory before it
// waits for the kernel in front of it.
//
// y = W . x for one activation row (ops.cpp:42-70 matmul_nt, quant.cpp:43-70
// matmul_nt_q8), the projections of one decode step.  One CTA per SM owns a
// contiguous slice of W's rows (at most kPfSliceBytes).  Its first act is to
// request the whole slice with bulk copies; only then does it release its own
// successor (griddepcontrol.launch_dependents) and wait for its predecessor
// (griddepcontrol.wait).  Launched back to back with programmatic dependent
// launch, kernel i+1's weights therefore stream in while kernel i computes:
// what is left on the step's dependency chain is reading x, the dot products
// out of shared memory and the stores.  The slice budget takes most of an
// SM's shared memory (one such CTA per SM); the weights of the GEMV two
// launches ahead are pulled into L2 meanwhile, so the next slice copies come
// out of L2.
//
// Arithmetic per row as the streaming GEMV: lanes stride K (16-byte groups),
// f32 FMAs, one warp reduction; INT8 bytes dequantised exactly (byte into the
// mantissa of 2^23, one subtraction) and the row scale applied after the sum.
#include <cuda_bf16.h>

#include <atomic>

#include "vb_kernels.cuh"
#include "vb_pipe.cuh"

namespace vb {
namespace {

constexpr int kPfThreads = 256;
constexpr int kPfWarps = kPfThreads / 32;
constexpr int kPfChunk = 32768;  // bytes per bulk copy
constexpr int kPfMaxK = 4096;

// Bounded wait (thread 0) for the slice; no error word on this path's
// arguments is required: a timeout is reported through a.err when present.
__device__ __noinline__ bool pf_wait_slice(unsigned a) {
    const unsigned long long t0 = now_ns();
    for (unsigned it = 1;; it++) {
        if (mbar_try(a, 0u)) return true;
        if ((it & 255u) == 0 && now_ns() - t0 > kWaitNs) return false;
    }
}

// This CTA's rows of a GEMV: units (rows, or gate/up row pairs) are split
// evenly over the G CTAs.
struct PfSlice {
    int r0, rows;
    size_t row_bytes, bytes;
};
template <bool Q8>
__device__ __forceinline__ PfSlice pf_slice(const GemvArgs& a, int epi, int c, int G) {
    const int unit = (epi == kEpiSwiGLU) ? 2 : 1;  // gate/up rows stay together
    const int units = a.N / unit;
    const int u0 = (int)((long long)c * units / G), u1 = (int)((long long)(c + 1) * units / G);
    PfSlice sl;
    sl.r0 = u0 * unit;
    sl.rows = (u1 - u0) * unit;
    sl.row_bytes = (size_t)a.K * (Q8 ? 1 : 4);
    sl.bytes = (size_t)sl.rows * sl.row_bytes;
    return sl;
}

// Thread 0: the slice into shared memory (bulk copies completing on `bar`).
__device__ __forceinline__ void pf_issue_slice(const GemvArgs& a, const PfSlice& sl, unsigned char* dst, unsigned bar) {
    if (!sl.bytes) return;
    unsigned long long pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    mbar_expect_tx(bar, (unsigned)sl.bytes);
    const char* src = static_cast<const char*>(a.W) + (size_t)sl.r0 * sl.row_bytes;
    for (size_t off = 0; off < sl.bytes; off += kPfChunk) {
        const unsigned n = (unsigned)(sl.bytes - off < (size_t)kPfChunk ? sl.bytes - off : (size_t)kPfChunk);
        bulk_g2s(smem_addr(dst + off), src + off, n, bar, pol);
    }
}

// One thread: this CTA's 1/G share of [base, base + total) into L2.
__device__ __forceinline__ void pf_l2_share(const void* base_, size_t total, int c, int G) {
    if (!base_ || !total) return;
    const size_t share = (total / G + 15) & ~size_t(15);
    const size_t b0 = share * c;
    const size_t b1 = b0 + share < total ? b0 + share : total;
    const char* base = static_cast<const char*>(base_);
    for (size_t off = b0; off + 16 <= b1; off += kPfChunk) {
        const size_t n = (b1 - off < (size_t)kPfChunk ? b1 - off : (size_t)kPfChunk) & ~size_t(15);
        if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"((unsigned)n) : "memory");
    }
}

// One thread: the attention's cached K / V rows into L2 -- span s = (head, K
// or V) of pos * 512 bytes, split into G / (2 heads) pieces.
__device__ __forceinline__ void pf_kv_share(const GemvArgs& a, int c, int G) {
    if (!a.kv_k || a.kv_heads <= 0) return;
    const int spans = 2 * a.kv_heads;
    const int pieces = G / spans > 0 ? G / spans : 1;
    const int sp = c % spans, pc = c / spans;
    const int pos = *a.kv_pos;  // written before this step (positions already cached)
    if (pc < pieces && pos > 0) {
        const size_t span = (size_t)pos * 512;
        const size_t share = (span / pieces + 15) & ~size_t(15);
        const size_t b0 = share * pc, b1 = b0 + share < span ? b0 + share : span;
        const float* h = ((sp & 1) ? a.kv_v : a.kv_k) + (size_t)(sp >> 1) * a.kv_stride_h;
        const char* base = reinterpret_cast<const char*>(h);
        for (size_t off = b0; off + 16 <= b1; off += kPfChunk) {
            const size_t n = (b1 - off < (size_t)kPfChunk ? b1 - off : (size_t)kPfChunk) & ~size_t(15);
            if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"((unsigned)n) : "memory");
        }
    }
}

// x into shared memory (normalised when PRO is kProRms, merged from the
// attention's split partials when kProMerge), laid out for conflict-free reads.
template <bool Q8, int PRO>
__device__ __forceinline__ void pf_load_x(const GemvArgs& a, float* xs, double* red, int tid, int warp, int lane) {
    const int K = a.K;
    const float* x = a.x;
    if (a.x_tok) x += (size_t)(*a.x_tok) * (size_t)K;
    float sc = 1.0f;
    if (PRO == kProMerge) {
        // half-warp per head, lane l of it dims 8l .. 8l + 7: M = max_s m_s,
        // L = sum_s l_s e^(m_s - M), A = sum_s acc_s e^(m_s - M) in split order
        // (an empty split has m = -inf, l = 0, acc = 0), x = A / L
        const int S = a.attn_splits, H = K >> 7;
        const int hl = lane & 15;
        for (int h0 = 2 * warp; h0 < H; h0 += 2 * kPfWarps) {
            const int h = h0 + (lane >> 4);
            const bool act = h < H;
            const float* base = a.attn_parts + (size_t)(act ? h : 0) * S * kAttnPart;
            float M = -INFINITY;
            if (act)
                for (int sp = hl; sp < S; sp += 16) M = fmaxf(M, base[(size_t)sp * kAttnPart]);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.0f;
            f2 A[4] = {0ull, 0ull, 0ull, 0ull};
            if (act && M != -INFINITY) {
#pragma unroll 4
                for (int sp = 0; sp < S; sp++) {
                    const float* pp = base + (size_t)sp * kAttnPart;
                    const float f = expf(pp[0] - M);
                    const f2 f2v = f2pack(f, f);
                    L = fmaf(pp[1], f, L);
                    const float4 v0 = *reinterpret_cast<const float4*>(pp + 4 + 8 * hl);
                    const float4 v1 = *reinterpret_cast<const float4*>(pp + 8 + 8 * hl);
                    A[0] = f2fma(f2pack(v0.x, v0.y), f2v, A[0]);
                    A[1] = f2fma(f2pack(v0.z, v0.w), f2v, A[1]);
                    A[2] = f2fma(f2pack(v1.x, v1.y), f2v, A[2]);
                    A[3] = f2fma(f2pack(v1.z, v1.w), f2v, A[3]);
                }
            }
            if (act) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float lo, hi;
                    f2unpack(A[e], lo, hi);
                    const int i = h * 128 + 8 * hl + 2 * e;
                    xs[xs_index<Q8>(i)] = L > 0.0f ? lo / L : 0.0f;
                    xs[xs_index<Q8>(i + 1)] = L > 0.0f ? hi / L : 0.0f;
                }
            }
        }
    }
    if (PRO == kProRms) {
        double ss = 0.0;
        for (int i = tid; i < K; i += kPfThreads) {
            const float v = x[i];
            ss += (double)v * (double)v;
        }
        sc = rms_scale(block_sum_d<kPfThreads>(ss, red), K, a.eps);
    }
    if (PRO != kProMerge) {
        for (int i = tid; i < K; i += kPfThreads) {
            float v = x[i];
            if (PRO == kProRms) v = __fmul_rn(__fmul_rn(v, sc), a.norm_w[i]);
            xs[xs_index<Q8>(i)] = v;
        }
    }

}

// The slice's dot products (row pairs, or single rows, round-robin over the
// warps) and the epilogue.
template <bool Q8, int EPI>
__device__ __forceinline__ void pf_rows(const GemvArgs& a, const PfSlice& sl, const unsigned char* wsm, const float* xs,
                                        int warp, int lane) {
    const int K = a.K, r0 = sl.r0, rows = sl.rows;
    const size_t row_bytes = sl.row_bytes;
    constexpr int R = 2;
    for (int rg = warp * R; rg < rows; rg += kPfWarps * R) {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.0f;
        const int nr = rows - rg < R ? rows - rg : R;
        if (!Q8) {
            const int K4 = K >> 2;
            for (int k4 = lane; k4 < K4; k4 += 32) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + 4 * k4);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    if (r < nr) {
                        const float4 w = *reinterpret_cast<const float4*>(wsm + (size_t)(rg + r) * row_bytes + 16 * k4);
                        acc[r] = fmaf(w.x, xv.x, acc[r]);
                        acc[r] = fmaf(w.y, xv.y, acc[r]);
                        acc[r] = fmaf(w.z, xv.z, acc[r]);
                        acc[r] = fmaf(w.w, xv.w, acc[r]);
                    }
                }
            }
        } else {
            const int G16 = K >> 4;
            for (int gi = lane; gi < G16; gi += 32) {
                const float* xc = xs + ((gi >> 5) << 9) + 4 * lane;
                const float4 x0 = *reinterpret_cast<const float4*>(xc);
                const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
                const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
                const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    if (r < nr) {
                        const uint4 w = *reinterpret_cast<const uint4*>(wsm + (size_t)(rg + r) * row_bytes + 16 * gi);
                        const f4 a0 = i8x4_to_f32(w.x), a1 = i8x4_to_f32(w.y);
                        const f4 a2 = i8x4_to_f32(w.z), a3 = i8x4_to_f32(w.w);
                        float s = acc[r];
                        s = fmaf(a0.v[0], x0.x, s); s = fmaf(a0.v[1], x0.y, s);
                        s = fmaf(a0.v[2], x0.z, s); s = fmaf(a0.v[3], x0.w, s);
                        s = fmaf(a1.v[0], x1.x, s); s = fmaf(a1.v[1], x1.y, s);
                        s = fmaf(a1.v[2], x1.z, s); s = fmaf(a1.v[3], x1.w, s);
                        s = fmaf(a2.v[0], x2.x, s); s = fmaf(a2.v[1], x2.y, s);
                        s = fmaf(a2.v[2], x2.z, s); s = fmaf(a2.v[3], x2.w, s);
                        s = fmaf(a3.v[0], x3.x, s); s = fmaf(a3.v[1], x3.y, s);
                        s = fmaf(a3.v[2], x3.z, s); s = fmaf(a3.v[3], x3.w, s);
                        acc[r] = s;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            acc[r] = warp_sum(acc[r]);
            if (Q8 && r < nr) acc[r] *= a.scales[r0 + rg + r];
        }
        if (lane == 0) {
            const int row = r0 + rg;
            if (EPI == kEpiSwiGLU) {
                a.y[row >> 1] = silu_f(acc[0]) * acc[1];  // gate row 2j, up row 2j + 1
            } else {
#pragma unroll
                for (int r = 0; r < R; r++) {
                    if (r < nr) {
                        if (EPI == kEpiResidual) a.y[row + r] = a.y[row + r] + acc[r];
                        else a.y[row + r] = acc[r];
                    }
                }
            }
        }
    }
}

template <bool Q8, int PRO, int EPI>
__global__ void __launch_bounds__(kPfThreads) gemv_pf_kernel(GemvArgs a) {
    extern __shared__ __align__(128) unsigned char pf_smem[];
    __shared__ __align__(8) unsigned long long full;
    __shared__ double red[kPfWarps];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const PfSlice sl = pf_slice<Q8>(a, EPI, c, G);
    unsigned char* wsm = pf_smem;
    float* xs = reinterpret_cast<float*>(pf_smem + a.pf_xs_off);

    // 1. the slice: requested before anything else (it depends on no kernel);
    //    a later kernel's weights into L2 (this CTA's share), so the HBM stream
    //    runs ahead of the kernels that consume it; the attention's cached K / V
    //    rows into L2
    if (tid == 0) {
        mbar_init(smem_addr(&full), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        pf_issue_slice(a, sl, wsm, smem_addr(&full));
    }
    if (tid == 32) pf_l2_share(a.l2_ahead, a.l2_ahead_bytes, c, G);
    if (tid == 64) pf_kv_share(a, c, G);
    // 2. let the next kernel start prefetching its own slice, then wait for
    //    the kernels this one reads from
    pdl_trigger();
    pdl_wait();
    // 3. x
    pf_load_x<Q8, PRO>(a, xs, red, tid, warp, lane);
    // 4. the slice has landed (thread 0 waits; every thread then observes the
    //    completed phase itself, which orders its reads after the copies)
    int ok = 1;
    if (tid == 0 && sl.bytes) ok = pf_wait_slice(smem_addr(&full)) ? 1 : 0;
    if (!__syncthreads_and(ok)) {
        // a copy that never completed: record it, give the copies in flight
        // their bound to land (the shared memory goes to the next CTA), leave
        if (tid == 0) {
            if (a.err) atomicCAS(a.err, 0, kErrPipeTimeout);
            mbar_drain(smem_addr(&full), 0u);
        }
        return;
    }
    if (sl.bytes) (void)mbar_try(smem_addr(&full), 0u);
    // 5. dot products and epilogue
    pf_rows<Q8, EPI>(a, sl, wsm, xs, warp, lane);
}

template <bool Q8, int PRO>
cudaError_t pf_dispatch(const GemvArgs& a, int epi, int grid, size_t smem, cudaStream_t s) {
    switch (epi) {
        case kEpiStore: return launch_pdl(gemv_pf_kernel<Q8, PRO, kEpiStore>, grid, kPfThreads, smem, s, a);
        case kEpiResidual: return launch_pdl(gemv_pf_kernel<Q8, PRO, kEpiResidual>, grid, kPfThreads, smem, s, a);
        default: return launch_pdl(gemv_pf_kernel<Q8, PRO, kEpiSwiGLU>, grid, kPfThreads, smem, s, a);
    }
}

template <bool Q8, int PRO, int EPI>
cudaError_t pf_attr() {
    return cudaFuncSetAttribute(gemv_pf_kernel<Q8, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(kPfSliceBytes + sizeof(float) * kPfMaxK));
}

}  // namespace

int gemv_pf_parts(int N, int K, bool q8, int epi) {
    const int unit = epi == kEpiSwiGLU ? 2 : 1;
    const size_t row_bytes = (size_t)K * (q8 ? 1 : 4);
    const size_t units = (size_t)N / unit;
    // the smallest part count whose largest per-CTA slice fits the budget
    for (int parts = 1; parts <= 8; parts++) {
        const size_t units_part = (units + parts - 1) / parts;
        const size_t per_cta = (units_part + kPfCtas - 1) / kPfCtas * unit * row_bytes;
        if (per_cta <= kPfSliceBytes) return parts;
    }
    return 0;
}

vb_status launch_gemv_pf(const GemvArgs& a, bool q8, int pro, int epi, cudaStream_t s) {
    if (a.N <= 0 || a.K <= 0) return fail(VB_ERR_ARG, "gemv: empty shape");
    if (q8 ? (a.K % 16) : (a.K % 4)) return fail(VB_ERR_UNSUPPORTED, "gemv: K alignment");
    if (a.K > kPfMaxK) return fail(VB_ERR_UNSUPPORTED, "prefetching gemv: K > 4096");
    if (epi != kEpiStore && epi != kEpiResidual && epi != kEpiSwiGLU)
        return fail(VB_ERR_UNSUPPORTED, "prefetching gemv: epilogue");
    if (epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "gemv: swiglu needs even N");
    if ((reinterpret_cast<uintptr_t>(a.W) & 15u) != 0) return fail(VB_ERR_UNSUPPORTED, "gemv: W must be 16-byte aligned");
    if (pro == kProMerge &&
        (epi != kEpiResidual || a.K % 128 || !a.attn_parts || a.attn_splits < 1 || a.x_tok ||
         (reinterpret_cast<uintptr_t>(a.attn_parts) & 15u) != 0))
        return fail(VB_ERR_UNSUPPORTED, "prefetching gemv: merge prologue needs K = heads * 128, partials, residual");
    const int parts = gemv_pf_parts(a.N, a.K, q8, epi);
    if (parts == 0) return fail(VB_ERR_UNSUPPORTED, "prefetching gemv: weights too large for the slices");
    {
        static std::atomic<unsigned long long> done{0};
        int dev = 0;
        cudaGetDevice(&dev);
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(done.load() & bit)) {
            cudaError_t ce = cudaSuccess;
            if (ce == cudaSuccess) ce = pf_attr<false, kProNone, kEpiStore>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProNone, kEpiResidual>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProNone, kEpiSwiGLU>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProRms, kEpiStore>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProRms, kEpiResidual>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProRms, kEpiSwiGLU>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProNone, kEpiStore>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProNone, kEpiResidual>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProNone, kEpiSwiGLU>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProRms, kEpiStore>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProRms, kEpiResidual>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProRms, kEpiSwiGLU>();
            if (ce == cudaSuccess) ce = pf_attr<false, kProMerge, kEpiResidual>();
            if (ce == cudaSuccess) ce = pf_attr<true, kProMerge, kEpiResidual>();
            if (ce != cudaSuccess) return cuda_fail(ce, "prefetching gemv: shared memory attribute");
            done.fetch_or(bit);
        }
    }
    const int unit = epi == kEpiSwiGLU ? 2 : 1;
    const int units = a.N / unit;
    const size_t es = q8 ? 1 : 4;
    const size_t xs_bytes = sizeof(float) * (size_t)(q8 ? ((a.K + 511) / 512) * 512 : a.K);
    for (int p = 0; p < parts; p++) {
        const int uu0 = (int)((long long)p * units / parts), uu1 = (int)((long long)(p + 1) * units / parts);
        GemvArgs g = a;
        const int n0 = uu0 * unit;
        g.N = (uu1 - uu0) * unit;
        if (g.N == 0) continue;
        g.W = static_cast<const char*>(a.W) + (size_t)n0 * a.K * es;
        if (q8) g.scales = a.scales + n0;
        g.y = a.y + (epi == kEpiSwiGLU ? n0 / 2 : n0);
        if (p > 0) g.kv_k = nullptr;           // the cache rows once, by the first part
        if (a.l2_ahead && a.l2_ahead_bytes) {  // each part pulls its share of the look-ahead
            const size_t share = (a.l2_ahead_bytes / parts + 15) & ~size_t(15);
            const size_t b0 = share * p;
            g.l2_ahead = static_cast<const char*>(a.l2_ahead) + b0;
            g.l2_ahead_bytes = b0 < a.l2_ahead_bytes ? (a.l2_ahead_bytes - b0 < share ? a.l2_ahead_bytes - b0 : share) : 0;
        }
        const int grid = g.N / unit < kPfCtas ? g.N / unit : kPfCtas;
        // f32: shared memory sized to this launch's largest slice, so the o
        // and down CTAs (56 / 85 KB) share an SM with the next kernel's
        // (f32 per-op step 1182 -> 1198 tok/s); INT8: the whole budget, one
        // CTA per SM -- its 14-42 KB slices let up to eight kernels' CTAs in
        // at once, measured 1190 -> 921
        size_t slice = kPfSliceBytes;
        if (!q8) {
            const size_t max_units = ((size_t)(g.N / unit) + grid - 1) / grid;
            slice = (max_units * unit * (size_t)a.K * es + 127) & ~size_t(127);
        }
        g.pf_xs_off = (unsigned)slice;
        const size_t smem = slice + xs_bytes;
        cudaError_t ce;
        if (pro == kProMerge)
            ce = q8 ? launch_pdl(gemv_pf_kernel<true, kProMerge, kEpiResidual>, grid, kPfThreads, smem, s, g)
                    : launch_pdl(gemv_pf_kernel<false, kProMerge, kEpiResidual>, grid, kPfThreads, smem, s, g);
        else if (q8)
            ce = pro == kProRms ? pf_dispatch<true, kProRms>(g, epi, grid, smem, s)
                                : pf_dispatch<true, kProNone>(g, epi, grid, smem, s);
        else
            ce = pro == kProRms ? pf_dispatch<false, kProRms>(g, epi, grid, smem, s)
                                : pf_dispatch<false, kProNone>(g, epi, grid, smem, s);
        if (ce != cudaSuccess) return cuda_fail(ce, "gemv_pf_kernel launch");
    }
    return VB_OK;
}

}  // namespace vb
