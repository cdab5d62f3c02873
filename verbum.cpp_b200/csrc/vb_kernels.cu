// vb_kernels.cu -- one-op-per-kernel sm_100a building blocks of the decode
// step: streaming GEMV (f32 / INT8 with fused dequant), split-K SIMT GEMM for
// small batches, per-row quantisation, RMSNorm, per-head q/k norm + RoPE + KV
// append, split-K GQA decode attention, argmax, embedding.
//
// These kernels back the C ABI's kernel entry points (the counterparts of the
// reference launchers in kernels/cuda_ops.cu:181-292), the graph-captured
// per-op step path, and the batched engine.
#include <float.h>
#include <limits.h>
#include <math.h>

#include <cuda_bf16.h>

#include "vb_kernels.cuh"
#include "vb_tail.cuh"

namespace vb {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kNumSMs = 148;

// better() (argmax order, lowest index on ties) and silu_f() (model.cpp:15-18:
// x / (1 + exp(-x)), IEEE division, accurate expf) come from vb_pipe.cuh.


// The 16-byte groups lane and lane + 32 of INT8 rows r0 .. r0 + R - 1 (zero
// past the matrix or the row), streamed past L1.
template <int R>
__device__ __forceinline__ void q8_load_group(const int8_t* W, int r0, int N, int K, int lane, uint4 (&w)[R][2]) {
    const int G16 = K >> 4;
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int gi = 32 * u + lane;
#pragma unroll
        for (int r = 0; r < R; r++)
            w[r][u] = (gi < G16 && r0 + r < N) ? ld_stream_u4(W + (size_t)(r0 + r) * K + 16 * (size_t)gi)
                                                : make_uint4(0u, 0u, 0u, 0u);
    }
}

// ---------------------------------------------------------------------------
// GEMV: y = W . x with W [N, K] row-major (f32 or int8 + per-row scale).
// One warp owns R consecutive rows at a time; lanes stride K with 16-byte
// streaming loads, all of a row group's loads issued before the FMAs.
// ---------------------------------------------------------------------------
// Two CTAs per SM (INT8 lm_head shape: 4.9 TB/s; three CTAs spill, 3.4 TB/s;
// two rows per warp, 4.4 TB/s).
template <bool Q8, int R, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(GemvArgs a) {
    pdl_trigger();
    {
        // The weights do not depend on the previous kernel: while it drains,
        // pull this warp's first row group into L2 (one bulk prefetch per row).
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int g0 = blockIdx.x * kGemvWarps + warp;
        const size_t row_bytes = (size_t)a.K * (Q8 ? 1 : 4);
        if (lane < R && g0 * R + lane < a.N && (row_bytes & 15) == 0) {
            const char* row = static_cast<const char*>(a.W) + (size_t)(g0 * R + lane) * row_bytes;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row), "r"((unsigned)row_bytes) : "memory");
        }
    }
    pdl_wait();
    extern __shared__ __align__(16) float xs[];
    __shared__ double red[kGemvWarps];
    __shared__ float sbv[kGemvWarps];
    __shared__ int sbi[kGemvWarps];

    const int K = a.K;
    const float* x = a.x;
    if (a.x_tok) x += (size_t)(*a.x_tok) * (size_t)K;

    float sc = 1.0f;
    if (PRO == kProRms) {
        double ss = 0.0;
        for (int i = threadIdx.x; i < K; i += kGemvThreads) {
            const float v = x[i];
            ss += (double)v * (double)v;
        }
        sc = rms_scale(block_sum_d<kGemvThreads>(ss, red), K, a.eps);
    }
    for (int i = threadIdx.x; i < K; i += kGemvThreads) {
        float v = x[i];
        if (PRO == kProRms) v = __fmul_rn(__fmul_rn(v, sc), a.norm_w[i]);
        xs[xs_index<Q8>(i)] = v;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = a.N;
    const int ngroups = (N + R - 1) / R;
    float best_v = -INFINITY;
    int best_i = INT_MAX;

    // INT8 rows of at most 1024 bytes: each lane holds two 16-byte groups of
    // every row of a group; the next group's loads are issued before this
    // group's dot products, and dequantisation and FMAs run on f32 pairs
    const bool q8_short = Q8 && K <= 1024;
    uint4 wn[R][2];
    const int gstride = gridDim.x * kGemvWarps;
    if (q8_short) {
        const int g = blockIdx.x * kGemvWarps + warp;
        if (g < ngroups) q8_load_group<R>(static_cast<const int8_t*>(a.W), g * R, N, K, lane, wn);
    }
    for (int g = blockIdx.x * kGemvWarps + warp; g < ngroups; g += gstride) {
        const int r0 = g * R;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.0f;

        if (q8_short) {
            uint4 w[R][2];
#pragma unroll
            for (int r = 0; r < R; r++) { w[r][0] = wn[r][0]; w[r][1] = wn[r][1]; }
            if (g + gstride < ngroups)
                q8_load_group<R>(static_cast<const int8_t*>(a.W), (g + gstride) * R, N, K, lane, wn);
            f2 A[R], B[R];
#pragma unroll
            for (int r = 0; r < R; r++) { A[r] = 0ull; B[r] = 0ull; }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int gi = 32 * u + lane;
                if (gi < (K >> 4)) {
                    const float* xc = xs + ((gi >> 5) << 9) + 4 * lane;
                    const float4 x0 = *reinterpret_cast<const float4*>(xc);
                    const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
                    const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
                    const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
                    const f2 x0l = f2pack(x0.x, x0.y), x0h = f2pack(x0.z, x0.w);
                    const f2 x1l = f2pack(x1.x, x1.y), x1h = f2pack(x1.z, x1.w);
                    const f2 x2l = f2pack(x2.x, x2.y), x2h = f2pack(x2.z, x2.w);
                    const f2 x3l = f2pack(x3.x, x3.y), x3h = f2pack(x3.z, x3.w);
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        f2 lo, hi;
                        i8x4_to_f2(w[r][u].x, lo, hi);
                        A[r] = f2fma(lo, x0l, A[r]);
                        B[r] = f2fma(hi, x0h, B[r]);
                        i8x4_to_f2(w[r][u].y, lo, hi);
                        A[r] = f2fma(lo, x1l, A[r]);
                        B[r] = f2fma(hi, x1h, B[r]);
                        i8x4_to_f2(w[r][u].z, lo, hi);
                        A[r] = f2fma(lo, x2l, A[r]);
                        B[r] = f2fma(hi, x2h, B[r]);
                        i8x4_to_f2(w[r][u].w, lo, hi);
                        A[r] = f2fma(lo, x3l, A[r]);
                        B[r] = f2fma(hi, x3h, B[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; r++) acc[r] = f2sum(A[r]) + f2sum(B[r]);
        } else if (!Q8) {
            const float* W = static_cast<const float*>(a.W);
            const int K4 = K >> 2;
            constexpr int U = 8;
            for (int kb = 0; kb < K4; kb += 32 * U) {
                float4 w[R][U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int k4 = kb + 32 * u + lane;
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        if (k4 < K4 && r0 + r < N)
                            w[r][u] = ld_stream_f4(W + (size_t)(r0 + r) * K + 4 * (size_t)k4);
                        else
                            w[r][u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int k4 = kb + 32 * u + lane;
                    if (k4 < K4) {
                        const float4 xv = *reinterpret_cast<const float4*>(xs + 4 * k4);
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            acc[r] = fmaf(w[r][u].x, xv.x, acc[r]);
                            acc[r] = fmaf(w[r][u].y, xv.y, acc[r]);
                            acc[r] = fmaf(w[r][u].z, xv.z, acc[r]);
                            acc[r] = fmaf(w[r][u].w, xv.w, acc[r]);
                        }
                    }
                }
            }
        } else {
            // INT8 rows longer than 1024 bytes
            const int8_t* W = static_cast<const int8_t*>(a.W);
            const int G16 = K >> 4;  // 16-byte groups per row
            constexpr int U = 4;
            for (int gb = 0; gb < G16; gb += 32 * U) {
                uint4 w[R][U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int gi = gb + 32 * u + lane;
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        if (gi < G16 && r0 + r < N)
                            w[r][u] = ld_stream_u4(W + (size_t)(r0 + r) * K + 16 * (size_t)gi);
                        else
                            w[r][u] = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int gi = gb + 32 * u + lane;
                    if (gi < G16) {
                        const float* xc = xs + ((gi >> 5) << 9) + 4 * lane;
                        const float4 x0 = *reinterpret_cast<const float4*>(xc);
                        const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
                        const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
                        const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            f4 a0 = i8x4_to_f32(w[r][u].x);
                            f4 a1 = i8x4_to_f32(w[r][u].y);
                            f4 a2 = i8x4_to_f32(w[r][u].z);
                            f4 a3 = i8x4_to_f32(w[r][u].w);
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
        }

#pragma unroll
        for (int r = 0; r < R; r++) {
            acc[r] = warp_sum(acc[r]);
            if (Q8 && r0 + r < N) acc[r] = acc[r] * a.scales[r0 + r];
        }

        if (EPI == kEpiSwiGLU) {
#pragma unroll
            for (int p = 0; p < R / 2; p++) {
                const int rg = r0 + 2 * p;
                if (lane == p && rg + 1 < N) a.y[rg >> 1] = silu_f(acc[2 * p]) * acc[2 * p + 1];
            }
        } else {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = r0 + r;
                if (row < N) {
                    if (lane == r) {
                        if (EPI == kEpiResidual) a.y[row] = a.y[row] + acc[r];
                        else a.y[row] = acc[r];
                    }
                    if (EPI == kEpiArgmax && better(acc[r], row, best_v, best_i)) {
                        best_v = acc[r];
                        best_i = row;
                    }
                }
            }
        }
    }

    if (EPI == kEpiArgmax) {
        if (lane == 0) {
            sbv[warp] = best_v;
            sbi[warp] = best_i;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = sbv[0];
            int bi = sbi[0];
            for (int w = 1; w < kGemvWarps; w++)
                if (better(sbv[w], sbi[w], bv, bi)) { bv = sbv[w]; bi = sbi[w]; }
            a.part_val[blockIdx.x] = bv;
            a.part_idx[blockIdx.x] = bi;
        }
    }
}

__global__ void argmax_parts_kernel(const float* pv, const int* pi, int parts, int* out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < parts; i += blockDim.x)
        if (better(pv[i], pi[i], bv, bi)) { bv = pv[i]; bi = pi[i]; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        bv = sv[0]; bi = si[0];
        for (int i = 1; i < nw; i++)
            if (better(sv[i], si[i], bv, bi)) { bv = sv[i]; bi = si[i]; }
        *out = (bi == INT_MAX) ? 0 : bi;
    }
}

// One block per row of logits.
__global__ void argmax_rows_kernel(const float* logits, int64_t n, int* out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float* row = logits + (size_t)blockIdx.x * (size_t)n;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        if (better(row[i], (int)i, bv, bi)) { bv = row[i]; bi = (int)i; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        bv = sv[0]; bi = si[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); i++)
            if (better(sv[i], si[i], bv, bi)) { bv = sv[i]; bi = si[i]; }
        out[blockIdx.x] = (bi == INT_MAX) ? 0 : bi;
    }
}

// quant.cpp:9-41 with IEEE-exact device ops: the row max is order-free, the
// division, reciprocal and product are correctly rounded, and
// __float2int_rn is round-half-even like lrintf under the default mode.
__global__ void quantize_rows_kernel(const float* W, int64_t rows, int64_t cols, int8_t* q,
                                     float* scales) {
    __shared__ float red[32];
    __shared__ float s_inv;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* row = W + r * cols;
        float amax = 0.0f;
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
            const float v = fabsf(row[c]);
            amax = (amax < v) ? v : amax;
        }
        amax = warp_max(amax);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = 0.0f;
            for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = (m < red[i]) ? red[i] : m;
            const float scale = (m > 0.0f) ? __fdiv_rn(m, 127.0f) : 1.0f;
            scales[r] = scale;
            s_inv = __fdiv_rn(1.0f, scale);
        }
        __syncthreads();
        const float inv = s_inv;
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
            int v = __float2int_rn(__fmul_rn(row[c], inv));
            v = v > 127 ? 127 : (v < -127 ? -127 : v);
            q[r * cols + c] = (int8_t)v;
        }
        __syncthreads();
    }
}

// nn.cpp:8-42, one block per row.
// Also writes the bf16 split of the output (hi + lo = out) when hi is set:
// the tensor-core GEMM's activation operand, rows of `dim`.
__global__ void rmsnorm_rows_kernel(const float* x, const float* w, float* out, int dim, float eps,
                                    __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_trigger();
    pdl_wait();
    __shared__ double red[8];
    const float* xr = x + (size_t)blockIdx.x * dim;
    double ss = 0.0;
    for (int i = threadIdx.x; i < dim; i += 256) {
        const float v = xr[i];
        ss += (double)v * (double)v;
    }
    const float sc = rms_scale(block_sum_d<256>(ss, red), dim, eps);
    for (int i = threadIdx.x; i < dim; i += 256) {
        const float y = __fmul_rn(__fmul_rn(xr[i], sc), w[i]);
        if (out) out[(size_t)blockIdx.x * dim + i] = y;  // (null: the bf16 split only)
        if (hi) {
            const __nv_bfloat16 h = __float2bfloat16_rn(y);
            hi[(size_t)blockIdx.x * dim + i] = h;
            lo[(size_t)blockIdx.x * dim + i] = __float2bfloat16_rn(y - __bfloat162float(h));
        }
    }
}

// Split-K reduce of a residual projection fused with the following RMSNorm
// (residual_norm_row, vb_tail.cuh).  grid rows, block 256.
__global__ void reduce_residual_norm_kernel(float* x, const float* parts, int splits, const float* scales,
                                            const float* w, float* out, int rows, int dim, float eps,
                                            __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_trigger();
    pdl_wait();
    __shared__ double red[8];
    residual_norm_row<256>(x, parts, splits, scales, w, out, hi, lo, rows, dim, eps, blockIdx.x, red);
}

// Many rows (a prompt chunk): a warp per row, 8 rows per CTA; dim % 128 == 0,
// dim <= 2048.  Lane l holds elements 4l + 128j as float4s.
__global__ void __launch_bounds__(256) rmsnorm_rows_warp_kernel(const float* x, const float* w, float* out, int rows,
                                                                int dim, float eps, __nv_bfloat16* hi,
                                                                __nv_bfloat16* lo) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int nj = dim >> 7;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * dim);
    float4 v[16];
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 16; j++)
        if (j < nj) v[j] = xr[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < 16; j++)
        if (j < nj)
            ss += (double)v[j].x * v[j].x + (double)v[j].y * v[j].y + (double)v[j].z * v[j].z +
                  (double)v[j].w * v[j].w;
    const float sc = rms_scale(warp_sum_d(ss), dim, eps);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        if (j >= nj) break;
        const int i = 4 * lane + 128 * j;
        const float4 wv = *reinterpret_cast<const float4*>(w + i);
        const float y0 = __fmul_rn(__fmul_rn(v[j].x, sc), wv.x), y1 = __fmul_rn(__fmul_rn(v[j].y, sc), wv.y);
        const float y2 = __fmul_rn(__fmul_rn(v[j].z, sc), wv.z), y3 = __fmul_rn(__fmul_rn(v[j].w, sc), wv.w);
        const size_t o = (size_t)row * dim + i;
        if (out) *reinterpret_cast<float4*>(out + o) = make_float4(y0, y1, y2, y3);
        if (hi) {
            const __nv_bfloat162 h01 = __floats2bfloat162_rn(y0, y1), h23 = __floats2bfloat162_rn(y2, y3);
            const __nv_bfloat162 l01 = __floats2bfloat162_rn(y0 - __low2float(h01), y1 - __high2float(h01));
            const __nv_bfloat162 l23 = __floats2bfloat162_rn(y2 - __low2float(h23), y3 - __high2float(h23));
            uint2 hv, lv;
            hv.x = *reinterpret_cast<const uint32_t*>(&h01);
            hv.y = *reinterpret_cast<const uint32_t*>(&h23);
            lv.x = *reinterpret_cast<const uint32_t*>(&l01);
            lv.y = *reinterpret_cast<const uint32_t*>(&l23);
            *reinterpret_cast<uint2*>(hi + o) = hv;
            *reinterpret_cast<uint2*>(lo + o) = lv;
        }
    }
}

// Many rows (a prompt chunk): 8 rows per CTA, its 8 warps taking the rows'
// (row, head) pairs in turn (fewer, longer CTAs than one CTA per 8 heads).
__global__ void __launch_bounds__(256) qk_norm_rope_rows_kernel(QkNormArgs a) {
    pdl_trigger();
    pdl_wait();
    const int nh = a.H + a.KVH;
    const int r0 = blockIdx.x * 8;
    const int tasks = min(8, a.B - r0) * nh;
    for (int t = threadIdx.x >> 5; t < tasks; t += 8) qk_norm_one(a, r0 + t / nh, t % nh, threadIdx.x & 31);
}

__global__ void __launch_bounds__(256) qk_norm_rope_kernel(QkNormArgs a) {
    pdl_trigger();
    pdl_wait();
    const int hd = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (hd >= a.H + a.KVH) return;
    qk_norm_one(a, blockIdx.x, hd, threadIdx.x & 31);
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention (flash-decoding).  grid (splits, KVH, B),
// 8 warps.  Each CTA takes one contiguous slice of one sequence's cache for
// one KV head and serves all G query heads of that group from a single read
// of each K/V row.  Each warp runs an online softmax over every 8th block of
// 4 positions; warps merge in shared memory and the CTA writes (m, l, acc).
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = 8;
constexpr int kAttnPB = 4;  // positions per warp iteration (8 measured slower)

// Three CTAs per SM (at most 85 registers): measured 5.97 TB/s at 64 sequences
// x 2063 positions against 4.84 with 96 registers (two CTAs) and 5.70 with four
// CTAs (64 registers, spills).  (GQA group 4 keeps two CTAs: its larger
// state would spill at three.)
template <int G, bool PRE>
__global__ void __launch_bounds__(kAttnThreads, (G >= 4 || PRE) ? 2 : 3) attn_split_kernel(AttnArgs a) {
    pdl_trigger();
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* kb = a.k + (size_t)b * a.stride_b + (size_t)kvh * a.stride_h + 4 * lane;
    const float* vb = a.v + (size_t)b * a.stride_b + (size_t)kvh * a.stride_h + 4 * lane;
    // Stable positions: read them, pull the rope row and norm weights into L1
    // and load this warp's first block of cached rows (those before this
    // step's position) while the predecessor is still running.
    float4 kpre[kAttnPB], vpre[kAttnPB];
    bool pre = false;
    if constexpr (PRE) {
        int n0 = a.lens ? a.lens[b] : a.pos[b] + 1;
        n0 = n0 < 0 ? 0 : (n0 > a.n_max ? a.n_max : n0);
        const int c0 = (n0 + a.splits - 1) / a.splits;
        const int q0 = split * c0, q1 = min(n0, q0 + c0);
        const int base = q0 + warp * kAttnPB;
        if (base < q1) {
            pre = true;
#pragma unroll
            for (int u = 0; u < kAttnPB; u++) {
                const int p = base + u;
                if (p < q1 && p < n0 - 1) {
                    kpre[u] = ld_stream_f4(kb + (size_t)p * a.stride_pos);
                    vpre[u] = ld_stream_f4(vb + (size_t)p * a.stride_pos);
                } else {
                    kpre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    vpre[u] = kpre[u];
                }
            }
        }
        if (a.fuse_qk && warp <= G && n0 >= 1 && n0 - 1 < a.qk.rope_positions) {
            const size_t r = (size_t)(n0 - 1) * 128 + lane;
            const float* nw = warp < G ? a.qk.q_norm : a.qk.k_norm;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                asm volatile("prefetch.global.L1 [%0];" ::"l"(a.qk.cos_tab + r + 32 * e));
                asm volatile("prefetch.global.L1 [%0];" ::"l"(a.qk.sin_tab + r + 32 * e));
                asm volatile("prefetch.global.L1 [%0];" ::"l"(nw + lane + 32 * e));
            }
        }
    }
    pdl_wait();
    int n = a.lens ? a.lens[b] : a.pos[b] + 1;
    n = n < 0 ? 0 : (n > a.n_max ? a.n_max : n);
    const int chunk = (n + a.splits - 1) / a.splits;
    const int p0 = split * chunk;
    const int p1 = min(n, p0 + chunk);
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)a.D));

    float4 q[G];
    // fused q/k norm + RoPE (+ cache append): warps 0..G-1 the G query heads,
    // warp G the KV head; the new k, v serve position `pos` from shared memory
    __shared__ __align__(16) float qs[G][128];
    __shared__ __align__(16) float kvs[2][128];
    const int pos = n - 1;
    const bool has_pos = a.fuse_qk && pos >= p0 && pos < p1;
    if (a.fuse_qk) {
        int ok = 1;
        if (warp <= G) {
            float o[4], v[4];
            ok = qk_head(a.qk, b, warp < G ? kvh * G + warp : a.H + kvh, lane, o, v) ? 1 : 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                if (warp < G) {
                    qs[warp][lane + 32 * e] = o[e];
                } else {
                    kvs[0][lane + 32 * e] = o[e];
                    kvs[1][lane + 32 * e] = v[e];
                }
            }
            if (warp == G && has_pos && ok) {
                const size_t off = (size_t)b * a.stride_b + (size_t)pos * a.stride_pos + (size_t)kvh * a.stride_h;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    a.qk.kc[off + lane + 32 * e] = o[e];
                    a.qk.vc[off + lane + 32 * e] = v[e];
                }
            }
        }
        if (!__syncthreads_and(ok)) return;  // the position is outside the rope table (error word set)
#pragma unroll
        for (int g = 0; g < G; g++) q[g] = *reinterpret_cast<const float4*>(&qs[g][4 * lane]);
    } else {
#pragma unroll
        for (int g = 0; g < G; g++)
            q[g] = *reinterpret_cast<const float4*>(a.q + ((size_t)b * a.H + kvh * G + g) * 128 + 4 * lane);
    }
    // scores in base 2: q is pre-scaled by log2(e) / sqrt(D) and the
    // exponentials are ex2; the running max m is in the same units and is
    // converted back to natural units for the split partial
    constexpr float kLog2e = 1.4426950408889634f;
    const float qscale = inv_sqrt_d * kLog2e;
    f2 qa[G], qb[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        qa[g] = f2pack(q[g].x * qscale, q[g].y * qscale);
        qb[g] = f2pack(q[g].z * qscale, q[g].w * qscale);
    }
    float m[G], l[G];
    f2 acca[G], accb[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
        acca[g] = f2pack(0.f, 0.f);
        accb[g] = acca[g];
    }
    // K / V rows of the block of kAttnPB positions at `base` (this step's row
    // from shared memory: just computed, not read back)
    auto load_block = [&](int base, float4 (&kk)[kAttnPB], float4 (&vv)[kAttnPB]) {
#pragma unroll
        for (int u = 0; u < kAttnPB; u++) {
            const int p = base + u;
            if (has_pos && p == pos) {
                kk[u] = *reinterpret_cast<const float4*>(&kvs[0][4 * lane]);
                vv[u] = *reinterpret_cast<const float4*>(&kvs[1][4 * lane]);
            } else if (p < p1) {
                kk[u] = ld_stream_f4(kb + (size_t)p * a.stride_pos);
                vv[u] = ld_stream_f4(vb + (size_t)p * a.stride_pos);
            } else {
                kk[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv[u] = kk[u];
            }
        }
    };
    constexpr int NV = G * kAttnPB;                           // dot products per block
    constexpr int kShift = NV >= 16 ? 1 : (NV >= 8 ? 2 : 3);  // 5 - log2(NV)
    for (int base = p0 + warp * kAttnPB; base < p1; base += kAttnWarps * kAttnPB) {
        // (issuing the next block's loads first measured slower: 118 registers,
        // two CTAs per SM instead of three)
        float4 kk[kAttnPB], vv[kAttnPB];
        if (PRE && pre) {  // the first block, loaded before the wait (this step's row from shared memory)
            pre = false;
#pragma unroll
            for (int u = 0; u < kAttnPB; u++) {
                const bool mine = has_pos && base + u == pos;
                kk[u] = mine ? *reinterpret_cast<const float4*>(&kvs[0][4 * lane]) : kpre[u];
                vv[u] = mine ? *reinterpret_cast<const float4*>(&kvs[1][4 * lane]) : vpre[u];
            }
        } else {
            load_block(base, kk, vv);
        }
        // this lane's share of the G x kAttnPB dot products, summed over the
        // warp together; value g * kAttnPB + u is then read from lane
        // (g * kAttnPB + u) << kShift
        float d[NV];
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int u = 0; u < kAttnPB; u++)
                d[g * kAttnPB + u] = f2sum(f2fma(qb[g], f2pack(kk[u].z, kk[u].w),
                                                 f2mul(qa[g], f2pack(kk[u].x, kk[u].y))));
        const float r = warp_sum_scatter<NV>(d, lane);
#pragma unroll
        for (int g = 0; g < G; g++) {
            float s[kAttnPB];
            float mx = m[g];
#pragma unroll
            for (int u = 0; u < kAttnPB; u++) {
                const float x = __shfl_sync(0xffffffffu, r, (g * kAttnPB + u) << kShift);
                s[u] = (u == 0 || base + u < p1) ? x : -INFINITY;
                mx = fmaxf(mx, s[u]);
            }
            // (the block's first position is always valid, so mx is finite;
            // ex2(-inf) = 0 covers the first block and the masked positions)
            const float corr = ex2_approx(m[g] - mx);
            const f2 c2 = f2pack(corr, corr);
            float lg = l[g] * corr;
            f2 aa = f2mul(acca[g], c2), ab = f2mul(accb[g], c2);
#pragma unroll
            for (int u = 0; u < kAttnPB; u++) {
                const float e = ex2_approx(s[u] - mx);
                const f2 e2 = f2pack(e, e);
                lg += e;
                aa = f2fma(e2, f2pack(vv[u].x, vv[u].y), aa);
                ab = f2fma(e2, f2pack(vv[u].z, vv[u].w), ab);
            }
            l[g] = lg;
            acca[g] = aa;
            accb[g] = ab;
            m[g] = mx;
        }
    }

    __shared__ float sm_m[kAttnWarps][G], sm_l[kAttnWarps][G];
    __shared__ float4 sm_acc[kAttnWarps][G][32];
#pragma unroll
    for (int g = 0; g < G; g++) {
        if (lane == 0) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
        float4 o;
        f2unpack(acca[g], o.x, o.y);
        f2unpack(accb[g], o.z, o.w);
        sm_acc[warp][g][lane] = o;
    }
    __syncthreads();
    // thread -> (g, float index); G*128 values per CTA
    const int S = a.splits;
    for (int t = threadIdx.x; t < G * 128; t += kAttnThreads) {
        const int g = t >> 7, di = t & 127;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, sm_m[w][g]);
        float L = 0.0f, A = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; w++) {
                if (sm_m[w][g] == -INFINITY) continue;
                const float f = ex2_approx(sm_m[w][g] - M);
                L = fmaf(sm_l[w][g], f, L);
                const float* av = reinterpret_cast<const float*>(&sm_acc[w][g][0]);
                A = fmaf(av[di], f, A);
            }
        }
        const int h = kvh * G + g;
        float* part = a.ws + (((size_t)b * a.H + h) * S + split) * kAttnPart;
        part[4 + di] = A;
        if (di == 0) { part[0] = M * (1.0f / kLog2e); part[1] = L; }  // M back to natural units
    }
}

// grid (H, B), 256 threads: merges the S split partials of one (b, h):
// M = max_s m_s, L = sum_s l_s e^(m_s - M), A = sum_s acc_s e^(m_s - M),
// out = A / L.  Every thread takes a share of the maxima; then warp w sums
// splits w, w + 8, ... (each lane 4 of the 128 dims, four splits' loads in
// flight at once) and the 8 warp sums are added in warp order.
constexpr int kMergeThreads = 256;
__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NW = kMergeThreads / 32;
    const int S = a.splits;
    const float* base = a.ws + ((size_t)b * a.H + h) * S * kAttnPart;
    __shared__ float s_m[NW], s_l[NW];
    __shared__ float4 s_a[NW][32];
    float M = -INFINITY;
    for (int sp = threadIdx.x; sp < S; sp += kMergeThreads) M = fmaxf(M, base[(size_t)sp * kAttnPart]);
    M = warp_max(M);
    if (lane == 0) s_m[warp] = M;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, s_m[w]);
    float L = 0.0f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
        constexpr int U = 4;
        for (int s0 = warp; s0 < S; s0 += NW * U) {
            float ms[U], ls[U];
            float4 av[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int sp = s0 + NW * u;
                if (sp < S) {
                    const float* pp = base + (size_t)sp * kAttnPart;
                    ms[u] = pp[0];
                    ls[u] = pp[1];
                    av[u] = *reinterpret_cast<const float4*>(pp + 4 + 4 * lane);
                } else {
                    ms[u] = -INFINITY;
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (ms[u] == -INFINITY) continue;
                const float f = expf(ms[u] - M);
                L = fmaf(ls[u], f, L);
                A.x = fmaf(av[u].x, f, A.x);
                A.y = fmaf(av[u].y, f, A.y);
                A.z = fmaf(av[u].z, f, A.z);
                A.w = fmaf(av[u].w, f, A.w);
            }
        }
    }
    if (lane == 0) s_l[warp] = L;
    s_a[warp][lane] = A;
    __syncthreads();
    if (warp == 0) {
        float Lt = 0.0f;
        float4 At = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NW; w++) {
            Lt += s_l[w];
            const float4 v = s_a[w][lane];
            At.x += v.x; At.y += v.y; At.z += v.z; At.w += v.w;
        }
        const float c[4] = {At.x, At.y, At.z, At.w};
        const size_t o = ((size_t)b * a.H + h) * 128 + 4 * lane;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float y = (Lt > 0.0f) ? c[e] / Lt : 0.0f;
            a.out[o + e] = y;
            if (a.out_hi) {
                const __nv_bfloat16 hv = __float2bfloat16_rn(y);
                static_cast<__nv_bfloat16*>(a.out_hi)[o + e] = hv;
                static_cast<__nv_bfloat16*>(a.out_lo)[o + e] = __float2bfloat16_rn(y - __bfloat162float(hv));
            }
        }
    }
}

__global__ void embed_kernel(const float* E, const int* tokens, int dim, int vocab, float* out,
                             int* err) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && err) atomicExch(err, kErrBadToken);
        tok = 0;
    }
    const float4* src = reinterpret_cast<const float4*>(E + (size_t)tok * dim);
    float4* dst = reinterpret_cast<float4*>(out + (size_t)b * dim);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) dst[i] = src[i];
}

// (value, index) -> a key whose unsigned order is better()'s order: the
// value's bits mapped to an unsigned order (-0 taken as +0), then the index
// complemented so that the lower index wins a tie
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    unsigned u = __float_as_uint(v + 0.0f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxChunks = 16;  // CTAs per row

// grid (kArgmaxChunks, rows): a contiguous slice of one row, 16-byte loads
// where the row allows them
__global__ void __launch_bounds__(kArgmaxThreads) argmax_keys_kernel(const float* logits, int64_t n,
                                                                     unsigned long long* keys) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long sk[kArgmaxThreads / 32];
    const float* row = logits + (size_t)blockIdx.y * (size_t)n;
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * per < n ? (int64_t)blockIdx.x * per : n;
    const int64_t i1 = i0 + per < n ? i0 + per : n;
    unsigned long long best = 0ull;
    auto take = [&](float v, int64_t i) {
        if (v == v) {  // NaN is never picked
            const unsigned long long k = argmax_key(v, (int)i);
            best = k > best ? k : best;
        }
    };
    // aligned float4 body when the row start and slice start are 16-byte aligned
    const bool vec = ((reinterpret_cast<uintptr_t>(row + i0) & 15u) == 0);
    int64_t i = i0;
    if (vec) {
        const int64_t nv = (i1 - i0) / 4;
        const float4* r4 = reinterpret_cast<const float4*>(row + i0);
        for (int64_t j = threadIdx.x; j < nv; j += kArgmaxThreads) {
            const float4 v = __ldcg(r4 + j);
            const int64_t b = i0 + 4 * j;
            take(v.x, b); take(v.y, b + 1); take(v.z, b + 2); take(v.w, b + 3);
        }
        i = i0 + 4 * nv;
    }
    for (int64_t j = i + threadIdx.x; j < i1; j += kArgmaxThreads) take(__ldcg(row + j), j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
        best = ok > best ? ok : best;
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sk[w] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < kArgmaxThreads / 32; k++) best = sk[k] > best ? sk[k] : best;
        if (best) atomicMax(keys + blockIdx.y, best);
    }
}

__global__ void advance_keys_kernel(int* pos, int* tokens, int* next, unsigned long long* keys, int B) {
    pdl_trigger();
    pdl_wait();
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        const unsigned long long k = keys[b];
        const int idx = k ? (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull)) : 0;
        next[b] = idx;
        tokens[b] = idx;
        pos[b] += 1;
        keys[b] = 0ull;
    }
}

__global__ void advance_kernel(int* pos, int* tokens, const int* next, int B) {
    pdl_trigger();
    pdl_wait();
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        pos[b] += 1;
        if (tokens && next) tokens[b] = next[b];
    }
}

__global__ void rope_kernel(float* x, const float* c, const float* s, int pos, int heads, int D) {
    const int half = D / 2;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= heads * half) return;
    const int h = t / half, i = t % half;
    float* row = x + (size_t)h * D;
    const float* cr = c + (size_t)pos * D;
    const float* sr = s + (size_t)pos * D;
    const float av = row[i], bv = row[i + half];
    row[i] = __fsub_rn(__fmul_rn(av, cr[i]), __fmul_rn(bv, sr[i]));
    row[i + half] = __fadd_rn(__fmul_rn(bv, cr[i + half]), __fmul_rn(av, sr[i + half]));
}

__global__ void silu_mul_kernel(float* g, const float* u, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) g[i] = silu_f(g[i]) * u[i];
}

__global__ void add_kernel(float* a, const float* b, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = a[i] + b[i];
}

__global__ void cache_append_kernel(float* kc, float* vc, const float* kn, const float* vn,
                                    int pos, int width) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < width) {
        kc[(size_t)pos * width + i] = kn[i];
        vc[(size_t)pos * width + i] = vn[i];
    }
}

// ---------------------------------------------------------------------------
// Batched SIMT GEMM with split-K partials: P[s, m, n] = sum_k A[m,k] W[n,k]
// over split s's K range.  64x64 output tile, 256 threads, 4x4 per thread.
// ---------------------------------------------------------------------------
constexpr int kGM = 64, kGN = 64, kGK = 32;

template <bool Q8>
__global__ void __launch_bounds__(256) gemm_partial_kernel(GemmArgs a, int kper) {
    __shared__ __align__(16) float As[kGK][kGM + 4];
    __shared__ __align__(16) float Ws[kGK][kGN + 4];
    const int n0 = blockIdx.x * kGN, split = blockIdx.y;
    const int kbeg = split * kper, kend = min(a.K, kbeg + kper);
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int M = a.M, N = a.N, K = a.K;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    for (int k0 = kbeg; k0 < kend; k0 += kGK) {
#pragma unroll
        for (int it = 0; it < 2; it++) {
            const int idx = tid + 256 * it;
            const int m = idx >> 3, kq = idx & 7;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < M) v = *reinterpret_cast<const float4*>(a.A + (size_t)m * K + k0 + 4 * kq);
            As[4 * kq + 0][m] = v.x; As[4 * kq + 1][m] = v.y;
            As[4 * kq + 2][m] = v.z; As[4 * kq + 3][m] = v.w;
        }
        if (!Q8) {
            const float* W = static_cast<const float*>(a.W);
#pragma unroll
            for (int it = 0; it < 2; it++) {
                const int idx = tid + 256 * it;
                const int n = idx >> 3, kq = idx & 7;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (n0 + n < N) v = ld_stream_f4(W + (size_t)(n0 + n) * K + k0 + 4 * kq);
                Ws[4 * kq + 0][n] = v.x; Ws[4 * kq + 1][n] = v.y;
                Ws[4 * kq + 2][n] = v.z; Ws[4 * kq + 3][n] = v.w;
            }
        } else if (tid < 128) {
            const int8_t* W = static_cast<const int8_t*>(a.W);
            const int n = tid >> 1, hf = tid & 1;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (n0 + n < N) v = ld_stream_u4(W + (size_t)(n0 + n) * K + k0 + 16 * hf);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const f4 f = i8x4_to_f32(wv[j]);
#pragma unroll
                for (int e = 0; e < 4; e++) Ws[16 * hf + 4 * j + e][n] = f.v[e];
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kGK; kk++) {
            const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
            const float ar[4] = {av.x, av.y, av.z, av.w};
            const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(ar[i], wr[j], acc[i][j]);
        }
        __syncthreads();
    }
    float* P = a.ws + (size_t)split * M * N;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx * 4 + j;
            if (n < N) P[(size_t)m * N + n] = acc[i][j];
        }
    }
}

// Sums the split partials in fixed order and applies the epilogue.
template <bool Q8, int EPI>
__global__ void gemm_reduce_kernel(GemmArgs a, int splits) {
    pdl_trigger();
    pdl_wait();
    const int M = a.M, N = a.N;
    const int outN = (EPI == kEpiSwiGLU) ? N / 2 : N;
    const size_t total = (size_t)M * outN;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(t / outN), j = (int)(t % outN);
        if (EPI == kEpiSwiGLU) {
            float gsum = 0.f, usum = 0.f;
            for (int s = 0; s < splits; s++) {
                const float* P = a.ws + (size_t)s * M * N + (size_t)m * N;
                gsum += P[2 * j];
                usum += P[2 * j + 1];
            }
            if (Q8) { gsum *= a.scales[2 * j]; usum *= a.scales[2 * j + 1]; }
            const float hv = silu_f(gsum) * usum;
            a.C[(size_t)m * a.ldc + j] = hv;
            if (a.out_hi) {
                const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
                static_cast<__nv_bfloat16*>(a.out_hi)[(size_t)m * a.ldc + j] = hb;
                static_cast<__nv_bfloat16*>(a.out_lo)[(size_t)m * a.ldc + j] = __float2bfloat16_rn(hv - __bfloat162float(hb));
            }
        } else {
            float v = 0.f;
            for (int s = 0; s < splits; s++) v += a.ws[(size_t)s * M * N + (size_t)m * N + j];
            if (Q8) v *= a.scales[j];
            float* dst = a.C + (size_t)m * a.ldc + j;
            if (EPI == kEpiResidual) *dst = *dst + v;
            else *dst = v;
        }
    }
}

template <bool Q8>
int gemm_splits(int N, int K) {
    const int tiles = (N + kGN - 1) / kGN;
    int s = (2 * kNumSMs + tiles - 1) / tiles;
    const int maxs = K / kGK;
    if (s > maxs) s = maxs;
    if (s > 16) s = 16;
    if (s < 1) s = 1;
    return s;
}

}  // namespace

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------

static int gemv_rows_per_warp(int N, bool q8, int epi) {
    if (epi == kEpiSwiGLU) return q8 ? 4 : 2;
    if (q8) return N >= 4096 ? 4 : 2;
    return N >= 4096 ? 2 : 1;
}

int gemv_grid(int N, bool q8, int epi) {
    const int R = gemv_rows_per_warp(N, q8, epi);
    const int groups = (N + R - 1) / R;
    int blocks = (groups + kGemvWarps - 1) / kGemvWarps;
    const int cap = kNumSMs * 8;
    return blocks < cap ? blocks : cap;
}

template <bool Q8, int R, int PRO>
static void gemv_dispatch_epi(const GemvArgs& a, int epi, int grid, size_t smem,
                              cudaStream_t s) {
    switch (epi) {
        case kEpiStore: launch_pdl(gemv_kernel<Q8, R, PRO, kEpiStore>, grid, kGemvThreads, smem, s, a); break;
        case kEpiResidual: launch_pdl(gemv_kernel<Q8, R, PRO, kEpiResidual>, grid, kGemvThreads, smem, s, a); break;
        case kEpiSwiGLU:  // launch_gemv only picks even R for this epilogue
            launch_pdl(gemv_kernel<Q8, (R % 2 == 0 ? R : 2), PRO, kEpiSwiGLU>, grid, kGemvThreads, smem, s, a);
            break;
        default: launch_pdl(gemv_kernel<Q8, R, PRO, kEpiArgmax>, grid, kGemvThreads, smem, s, a); break;
    }
}

template <bool Q8, int R>
static void gemv_dispatch_pro(const GemvArgs& a, int pro, int epi, int grid, size_t smem,
                              cudaStream_t s) {
    if (pro == kProRms) gemv_dispatch_epi<Q8, R, kProRms>(a, epi, grid, smem, s);
    else gemv_dispatch_epi<Q8, R, kProNone>(a, epi, grid, smem, s);
}

vb_status launch_gemv(const GemvArgs& a, bool q8, int pro, int epi, cudaStream_t s,
                      int* grid_out) {
    if (a.N <= 0 || a.K <= 0) return fail(VB_ERR_ARG, "gemv: empty shape");
    if (q8 ? (a.K % 16) : (a.K % 4)) return fail(VB_ERR_UNSUPPORTED, "gemv: K alignment");
    if (a.K > 8192) return fail(VB_ERR_UNSUPPORTED, "gemv: K > 8192");
    if (epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "gemv: swiglu needs even N");
    const int R = gemv_rows_per_warp(a.N, q8, epi);
    const int grid = gemv_grid(a.N, q8, epi);
    const size_t smem = sizeof(float) * (size_t)(q8 ? ((a.K + 511) / 512) * 512 : a.K);
    if (q8) {
        if (R == 4) gemv_dispatch_pro<true, 4>(a, pro, epi, grid, smem, s);
        else gemv_dispatch_pro<true, 2>(a, pro, epi, grid, smem, s);
    } else {
        if (R == 2) gemv_dispatch_pro<false, 2>(a, pro, epi, grid, smem, s);
        else gemv_dispatch_pro<false, 1>(a, pro, epi, grid, smem, s);
    }
    if (grid_out) *grid_out = grid;
    VB_LAUNCH_CHECK("gemv_kernel");
    return VB_OK;
}

vb_status launch_argmax_parts(const float* pv, const int* pi, int parts, int* out,
                              cudaStream_t s) {
    launch_pdl(argmax_parts_kernel, 1, 1024, 0, s, pv, pi, parts, out);
    VB_LAUNCH_CHECK("argmax_parts_kernel");
    return VB_OK;
}

vb_status launch_argmax_rows(const float* logits, int rows, int64_t n, int* out,
                             cudaStream_t s) {
    if (rows <= 0 || n <= 0) return fail(VB_ERR_ARG, "argmax: empty input");
    launch_pdl(argmax_rows_kernel, rows, 1024, 0, s, logits, n, out);
    VB_LAUNCH_CHECK("argmax_rows_kernel");
    return VB_OK;
}

vb_status launch_argmax_rows_keys(const float* logits, int rows, int64_t n, unsigned long long* keys,
                                  cudaStream_t s) {
    if (rows <= 0 || n <= 0 || rows > 65535) return fail(VB_ERR_ARG, "argmax: bad shape");
    if (n > INT_MAX) return fail(VB_ERR_UNSUPPORTED, "argmax: row longer than INT_MAX");
    launch_pdl(argmax_keys_kernel, dim3(kArgmaxChunks, rows), kArgmaxThreads, 0, s, logits, n, keys);
    VB_LAUNCH_CHECK("argmax_keys_kernel");
    return VB_OK;
}

vb_status launch_advance_keys(int* pos, int* tokens, int* next, unsigned long long* keys, int B, cudaStream_t s) {
    launch_pdl(advance_keys_kernel, 1, 128, 0, s, pos, tokens, next, keys, B);
    VB_LAUNCH_CHECK("advance_keys_kernel");
    return VB_OK;
}

vb_status launch_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q,
                               float* scales, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return fail(VB_ERR_ARG, "quantize_rows: empty shape");
    const int grid = (int)(rows < 4096 ? rows : 4096);
    quantize_rows_kernel<<<grid, 256, 0, s>>>(W, rows, cols, q, scales);
    VB_LAUNCH_CHECK("quantize_rows_kernel");
    return VB_OK;
}

vb_status launch_rmsnorm_rows(const float* x, const float* w, float* out, int rows, int dim,
                              float eps, cudaStream_t s, void* hi, void* lo) {
    if (rows <= 0 || dim <= 0) return fail(VB_ERR_ARG, "rmsnorm: empty shape");
    if (!out && !hi) return fail(VB_ERR_ARG, "rmsnorm: no output");
    const uintptr_t al16 = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                           reinterpret_cast<uintptr_t>(out);
    const uintptr_t al8 = reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo);
    if (rows >= 1024 && dim % 128 == 0 && dim <= 2048 && (al16 & 15) == 0 && (al8 & 7) == 0) {
        launch_pdl(rmsnorm_rows_warp_kernel, (rows + 7) / 8, 256, 0, s, x, w, out, rows, dim, eps,
                   static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo));
        VB_LAUNCH_CHECK("rmsnorm_rows_warp_kernel");
        return VB_OK;
    }
    launch_pdl(rmsnorm_rows_kernel, rows, 256, 0, s, x, w, out, dim, eps, static_cast<__nv_bfloat16*>(hi),
               static_cast<__nv_bfloat16*>(lo));
    VB_LAUNCH_CHECK("rmsnorm_rows_kernel");
    return VB_OK;
}

vb_status launch_reduce_residual_norm(float* x, const float* parts, int splits, const float* scales,
                                      const float* w, float* out, void* hi, void* lo, int rows, int dim,
                                      float eps, cudaStream_t s) {
    if (rows <= 0 || dim <= 0 || splits <= 0) return fail(VB_ERR_ARG, "reduce_residual_norm: bad shape");
    const cudaError_t ce = launch_pdl(reduce_residual_norm_kernel, rows, 256, 0, s, x, parts, splits, scales, w, out,
                                      rows, dim, eps, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo));
    if (ce != cudaSuccess) return cuda_fail(ce, "reduce_residual_norm_kernel launch");
    return VB_OK;
}

vb_status launch_qk_norm_rope_append(const QkNormArgs& a, cudaStream_t s) {
    if (a.D != 128) return fail(VB_ERR_UNSUPPORTED, "head_dim must be 128");
    if (a.B >= 4096) {
        launch_pdl(qk_norm_rope_rows_kernel, (a.B + 7) / 8, 256, 0, s, a);
        VB_LAUNCH_CHECK("qk_norm_rope_rows_kernel");
        return VB_OK;
    }
    dim3 grid(a.B, (a.H + a.KVH + 7) / 8);  // rows on x: a prompt chunk has up to 2^31 - 1
    launch_pdl(qk_norm_rope_kernel, grid, 256, 0, s, a);
    VB_LAUNCH_CHECK("qk_norm_rope_kernel");
    return VB_OK;
}

int attn_splits_for(int B, int KVH, int n_max) {
    // Measured on B200 (decode attention alone, GB/s of K/V reads):
    //  - many (sequence, KV head) pairs (>= 512): ~16 CTAs per SM -- at 64
    //    sequences x 8 KV heads x 2063 positions 5 splits give 93% of the HBM
    //    copy peak (4 and 6 the same within 1%), 3 and 8 splits 88%;
    //  - fewer pairs: ~8 CTAs per SM -- 32 x 8 at 2048 positions: 5 splits
    //    5.77 TB/s against 10 splits 5.38; 1 x 8 at 32768: 148 splits 4.87
    //    against 296 splits 4.16;
    //  - splits of >= 64 positions (>= 128 from 4096 positions on: 1 x 8 at
    //    8192, 64 splits 3.84 TB/s against 128 splits 3.51).
    const int pairs = B * KVH;
    const int min_split = n_max >= 4096 ? 128 : kAttnMinSplit;
    const int target = kNumSMs * (pairs >= 512 ? 16 : 8);
    int by_len = (n_max + min_split - 1) / min_split;
    int by_grid = (target + pairs - 1) / pairs;
    int s = by_len < by_grid ? by_len : by_grid;
    return s < 1 ? 1 : s;
}

size_t attn_ws_bytes(int B, int H, int splits) {
    return sizeof(float) * (size_t)B * H * splits * kAttnPart;
}

vb_status launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.D != 128) return fail(VB_ERR_UNSUPPORTED, "attention: head_dim must be 128");
    if (a.H % a.KVH) return fail(VB_ERR_ARG, "attention: heads % kv_heads != 0");
    const int G = a.H / a.KVH;
    if (a.fuse_qk && (G + 1 > kAttnWarps || a.lens || !a.pos))
        return fail(VB_ERR_ARG, "attention: the fused q/k norm needs positions and G < warps");
    dim3 grid(a.splits, a.KVH, a.B);
    // the pre-wait form (positions stable: a decode step's graph) keeps its
    // first block in registers and runs two CTAs per SM; the other form three
    const bool pre = a.pos_stable != 0;
    switch (G) {
        case 1: pre ? launch_pdl(attn_split_kernel<1, true>, grid, kAttnThreads, 0, s, a)
                    : launch_pdl(attn_split_kernel<1, false>, grid, kAttnThreads, 0, s, a); break;
        case 2: pre ? launch_pdl(attn_split_kernel<2, true>, grid, kAttnThreads, 0, s, a)
                    : launch_pdl(attn_split_kernel<2, false>, grid, kAttnThreads, 0, s, a); break;
        case 4: pre ? launch_pdl(attn_split_kernel<4, true>, grid, kAttnThreads, 0, s, a)
                    : launch_pdl(attn_split_kernel<4, false>, grid, kAttnThreads, 0, s, a); break;
        default: return fail(VB_ERR_UNSUPPORTED, "attention: GQA group must be 1, 2 or 4");
    }
    VB_LAUNCH_CHECK("attn_split_kernel");
    if (a.no_merge) return VB_OK;
    launch_pdl(attn_merge_kernel, dim3(a.H, a.B), kMergeThreads, 0, s, a);
    VB_LAUNCH_CHECK("attn_merge_kernel");
    return VB_OK;
}

vb_status launch_embed(const float* E, const int* tokens, int B, int dim, int vocab,
                       float* out, int* err, cudaStream_t s) {
    if (dim % 4) return fail(VB_ERR_UNSUPPORTED, "embed: dim % 4");
    launch_pdl(embed_kernel, B, 256, 0, s, E, tokens, dim, vocab, out, err);
    VB_LAUNCH_CHECK("embed_kernel");
    return VB_OK;
}

vb_status launch_advance(int* pos, int* tokens, const int* next, int B, cudaStream_t s) {
    launch_pdl(advance_kernel, 1, 128, 0, s, pos, tokens, next, B);
    VB_LAUNCH_CHECK("advance_kernel");
    return VB_OK;
}

vb_status launch_rope(float* x, const float* c, const float* sn, int pos, int heads, int D,
                      cudaStream_t s) {
    if (D % 2 || heads <= 0) return fail(VB_ERR_ARG, "rope: bad shape");
    const int pairs = heads * (D / 2);
    rope_kernel<<<(pairs + 255) / 256, 256, 0, s>>>(x, c, sn, pos, heads, D);
    VB_LAUNCH_CHECK("rope_kernel");
    return VB_OK;
}

vb_status launch_silu_mul(float* g, const float* u, int n, cudaStream_t s) {
    if (n <= 0) return fail(VB_ERR_ARG, "silu_mul: n <= 0");
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, s>>>(g, u, n);
    VB_LAUNCH_CHECK("silu_mul_kernel");
    return VB_OK;
}

vb_status launch_add(float* a, const float* b, int n, cudaStream_t s) {
    if (n <= 0) return fail(VB_ERR_ARG, "add: n <= 0");
    add_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, b, n);
    VB_LAUNCH_CHECK("add_kernel");
    return VB_OK;
}

vb_status launch_cache_append(float* kc, float* vc, const float* kn, const float* vn, int pos,
                              int width, cudaStream_t s) {
    if (width <= 0 || pos < 0) return fail(VB_ERR_ARG, "cache_append: bad args");
    cache_append_kernel<<<(width + 255) / 256, 256, 0, s>>>(kc, vc, kn, vn, pos, width);
    VB_LAUNCH_CHECK("cache_append_kernel");
    return VB_OK;
}

size_t gemm_ws_floats(int M, int N, int K, bool q8) {
    const int s = q8 ? gemm_splits<true>(N, K) : gemm_splits<false>(N, K);
    return (size_t)s * M * N;
}

vb_status launch_gemm(const GemmArgs& a, bool q8, int epi, cudaStream_t s) {
    if (a.M <= 0 || a.M > kGM) return fail(VB_ERR_UNSUPPORTED, "gemm: M must be 1..64");
    if (a.K % kGK) return fail(VB_ERR_UNSUPPORTED, "gemm: K must be a multiple of 32");
    if (epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "gemm: swiglu needs even N");
    const int splits = q8 ? gemm_splits<true>(a.N, a.K) : gemm_splits<false>(a.N, a.K);
    if ((size_t)splits * a.M * a.N > a.ws_floats) return fail(VB_ERR_ARG, "gemm: workspace too small");
    int kper = (a.K + splits - 1) / splits;
    kper = (kper + kGK - 1) / kGK * kGK;
    dim3 grid((a.N + kGN - 1) / kGN, splits);
    if (q8) gemm_partial_kernel<true><<<grid, 256, 0, s>>>(a, kper);
    else gemm_partial_kernel<false><<<grid, 256, 0, s>>>(a, kper);
    VB_LAUNCH_CHECK("gemm_partial_kernel");
    return launch_gemm_reduce(a, splits, q8, epi, s);
}

vb_status launch_gemm_reduce(const GemmArgs& a, int splits, bool q8, int epi, cudaStream_t s) {
    if (epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "gemm: swiglu needs even N");
    const int outN = epi == kEpiSwiGLU ? a.N / 2 : a.N;
    const size_t total = (size_t)a.M * outN;
    int rb = (int)((total + 255) / 256);
    if (rb > kNumSMs * 8) rb = kNumSMs * 8;
#define VB_RED(Q, E) launch_pdl(gemm_reduce_kernel<Q, E>, rb, 256, 0, s, a, splits)
    if (q8) {
        if (epi == kEpiResidual) VB_RED(true, kEpiResidual);
        else if (epi == kEpiSwiGLU) VB_RED(true, kEpiSwiGLU);
        else VB_RED(true, kEpiStore);
    } else {
        if (epi == kEpiResidual) VB_RED(false, kEpiResidual);
        else if (epi == kEpiSwiGLU) VB_RED(false, kEpiSwiGLU);
        else VB_RED(false, kEpiStore);
    }
#undef VB_RED
    VB_LAUNCH_CHECK("gemm_reduce_kernel");
    return VB_OK;
}

}  // namespace vb
