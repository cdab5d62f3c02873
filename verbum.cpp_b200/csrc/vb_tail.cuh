// vb_tail.cuh -- consumers of split-K partials: the q/k norm + RoPE + cache
// append of one (row, head) and the residual add + RMSNorm + bf16 split of one
// row.  Partials are laid out [split][row][col] and summed in split order,
// read with ld.global.cg (another kernel's output).
#pragma once
#include <cuda_bf16.h>

#include "vb_kernels.cuh"
#include "vb_pipe.cuh"

namespace vb {

// The per-head RMSNorm (q_norm / k_norm, double sum of squares) and split-half
// RoPE from the host table (generate.cpp:52-64) of one head held by one warp:
// x[e] is dim lane + 32e, o[e] gets the normed, rotated value.
static __device__ __forceinline__ void qk_finish(const QkNormArgs& a, bool isq, int pos, const float* x, int lane,
                                                 float* o) {
    constexpr int D = 128;
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 4; e++) ss += (double)x[e] * (double)x[e];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float sc = rms_scale(ss, D, a.eps);
    const float* nw = isq ? a.q_norm : a.k_norm;
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; e++) y[e] = __fmul_rn(__fmul_rn(x[e], sc), nw[lane + 32 * e]);
    const float* c = a.cos_tab + (size_t)pos * D;
    const float* s = a.sin_tab + (size_t)pos * D;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const int d = lane + 32 * e;
        o[e] = e < 2 ? __fsub_rn(__fmul_rn(y[e], c[d]), __fmul_rn(y[e + 2], s[d]))
                     : __fadd_rn(__fmul_rn(y[e], c[d]), __fmul_rn(y[e - 2], s[d]));
    }
}

// generate.cpp:52-64 for one (row b, head hd) by one warp: per-head RMSNorm
// (q_norm / k_norm) and split-half RoPE from the host table; o[e] gets dim
// lane + 32e of the normed, rotated q or k, v[e] (k heads) the v value.  Lane
// l holds dims l, l + 32, l + 64, l + 96, so the RoPE pairs (d, d + 64) sit in
// one lane.  False (and the error word set) for a position outside the table.
static __device__ __forceinline__ bool qk_head(const QkNormArgs& a, int b, int hd, int lane, float* o, float* v) {
    const int D = 128;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.rope_positions) {
        if (lane == 0 && a.err) atomicExch(a.err, kErrCacheFull);
        return false;
    }
    const int QW = a.H * D, KW = a.KVH * D, RW = QW + 2 * KW;
    const bool isq = hd < a.H;
    const int h = isq ? hd : hd - a.H;
    const int col0 = isq ? h * D : QW + h * D;  // first column of this head's q or k
    const int vcol0 = QW + KW + h * D;
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = 0.f;
    if (a.parts) {
#pragma unroll
        for (int e = 0; e < 4; e++) x[e] = 0.f;
#pragma unroll 4
        for (int q = 0; q < a.splits; q++) {
            const float* pr = a.parts + ((size_t)q * a.B + b) * RW;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                x[e] += __ldcg(pr + col0 + lane + 32 * e);
                if (!isq) v[e] += __ldcg(pr + vcol0 + lane + 32 * e);
            }
        }
        if (a.scales) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                x[e] *= a.scales[col0 + lane + 32 * e];
                if (!isq) v[e] *= a.scales[vcol0 + lane + 32 * e];
            }
        }
    } else {
        const float* row = a.qkv + (size_t)b * RW;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            x[e] = row[col0 + lane + 32 * e];
            if (!isq) v[e] = row[vcol0 + lane + 32 * e];
        }
    }
    qk_finish(a, isq, pos, x, lane, o);
    return true;
}

// qk_head for (row b, head hd) plus its writes: q to q_out (when set), k and v into the
// cache at pos[b] of the row's sequence, and the optional bf16 copies.
static __device__ __forceinline__ void qk_norm_one(const QkNormArgs& a, int b, int hd, int lane) {
    const int D = 128;
    float o[4], v[4];
    if (!qk_head(a, b, hd, lane, o, v)) return;
    const int pos = a.pos[b];
    const bool isq = hd < a.H;
    const int h = isq ? hd : hd - a.H;
    __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(isq ? a.q_hi : a.k_hi);
    __nv_bfloat16* lo = static_cast<__nv_bfloat16*>(isq ? a.q_lo : a.k_lo);
    size_t bf = 0;
    if (isq) {
        const size_t qo = ((size_t)b * a.H + h) * D;
        bf = qo;
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (a.q_out) a.q_out[qo + lane + 32 * e] = o[e];
    } else {
        const int seq = a.rows_per_seq > 0 ? b / a.rows_per_seq : b;
        const size_t off = (size_t)seq * a.stride_b + (size_t)pos * a.stride_pos + (size_t)h * a.stride_h;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            a.kc[off + lane + 32 * e] = o[e];
            a.vc[off + lane + 32 * e] = v[e];
        }
        bf = ((size_t)(seq * a.KVH + h) * a.kbf_rows + pos) * D;
    }
    if (hi) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const __nv_bfloat16 oh = __float2bfloat16_rn(o[e]);
            hi[bf + lane + 32 * e] = oh;
            lo[bf + lane + 32 * e] = __float2bfloat16_rn(o[e] - __bfloat162float(oh));
        }
    }
}

// Residual projection's partials into row b (nn.cpp:8-42 for the norm):
// x[b][i] += (sum_s parts[s][b][i]) * scale[i]; out[b] = RMSNorm(x[b]) . w and
// its bf16 split.  NT threads, dim % NT == 0, dim / NT <= 16; red holds NT/32
// doubles.
template <int NT>
__device__ __forceinline__ void residual_norm_row(float* x, const float* parts, int splits, const float* scales,
                                                  const float* w, float* out, __nv_bfloat16* hi, __nv_bfloat16* lo,
                                                  int rows, int dim, float eps, int b, double* red) {
    float* xr = x + (size_t)b * dim;
    float xv[16];
    double ss = 0.0;
    // Four elements per thread at a time, with every split's load of all four
    // (and their residuals) in flight before any is summed (in split order) or
    // stored: a store to x between elements would hold the next element's loads
    // back behind it (it may alias them).
    constexpr int JB = 4;
#pragma unroll
    for (int j0 = 0; j0 < 16; j0 += JB) {
        if (threadIdx.x + NT * j0 >= dim) break;
        float v[JB], xo[JB];
#pragma unroll
        for (int jj = 0; jj < JB; jj++) {
            const int i = threadIdx.x + NT * (j0 + jj);
            v[jj] = 0.f;
            xo[jj] = i < dim ? __ldcg(xr + i) : 0.f;
        }
        for (int q0 = 0; q0 < splits; q0 += 16) {
            float t[JB][16];
#pragma unroll
            for (int jj = 0; jj < JB; jj++) {
                const int i = threadIdx.x + NT * (j0 + jj);
#pragma unroll
                for (int u = 0; u < 16; u++)
                    t[jj][u] = (i < dim && q0 + u < splits) ? __ldcg(parts + ((size_t)(q0 + u) * rows + b) * dim + i) : 0.f;
            }
#pragma unroll
            for (int jj = 0; jj < JB; jj++)
#pragma unroll
                for (int u = 0; u < 16; u++)
                    if (q0 + u < splits) v[jj] += t[jj][u];
        }
#pragma unroll
        for (int jj = 0; jj < JB; jj++) {
            const int i = threadIdx.x + NT * (j0 + jj);
            if (i >= dim) break;
            if (scales) v[jj] *= scales[i];
            xv[j0 + jj] = xo[jj] + v[jj];
            xr[i] = xv[j0 + jj];
            ss += (double)xv[j0 + jj] * (double)xv[j0 + jj];
        }
    }
    const float sc = rms_scale(block_sum_d<NT>(ss, red), dim, eps);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int i = threadIdx.x + NT * j;
        if (i >= dim) break;
        const float y = __fmul_rn(__fmul_rn(xv[j], sc), w[i]);
        out[(size_t)b * dim + i] = y;
        if (hi) {
            const __nv_bfloat16 h = __float2bfloat16_rn(y);
            hi[(size_t)b * dim + i] = h;
            lo[(size_t)b * dim + i] = __float2bfloat16_rn(y - __bfloat162float(h));
        }
    }
}

}  // namespace vb
