// vb_prefill.cu -- causal attention for a prompt chunk processed as a whole
// (the prefill of B sequences by GEMMs instead of one decode step per
// position).
//
// For every sequence b and query position p0 + c (c < C) of the chunk, and
// every query head h (GQA: KV head h / (H / KVH)), the same arithmetic as the
// reference's decode attention (generate.cpp:73-105) over keys 0..p0 + c:
//   s_j = (q . k_j) * (1/sqrt(D)),  ctx = sum_j softmax(s)_j v_j,
// computed as a flash-attention pass (online softmax over 32-key tiles) so a
// K/V tile read from the cache serves 64 query rows (32 positions x the 2
// query heads of the KV head) instead of one.  Different summation order from
// the reference's sequential sums: f32 rounding-level differences only.
//
// Layouts: q and out are [B*C][H*D] (row b*C + c); the cache of sequence b,
// KV head g, position p sits at k + b*stride_b + g*stride_h + p*D (the K/V
// rows of the chunk are appended before this kernel runs).
#include <cuda_bf16.h>

#include "vb_kernels.cuh"

namespace vb {
namespace {

constexpr int kPQ = 32;        // query positions per CTA (x 2 heads = 64 query rows)
constexpr int kPRows = 2 * kPQ;
constexpr int kPKT = 32;       // keys per tile
constexpr int kPLd = 132;      // padded shared row of a q / k vector (floats)
constexpr int kPPt = 68;       // padded row of the probability tile Pt[key][query row]
constexpr int kPThreads = 128;
constexpr size_t kPSmem = sizeof(float) * ((size_t)kPRows * kPLd + (size_t)kPKT * kPLd + (size_t)kPKT * 128 +
                                           (size_t)kPKT * kPPt);

// grid (ceil(C / 32), KVH, B), 128 threads.  Query row r = hh * 32 + c of the
// CTA is position c0 + c of query head 2 * kvh + hh.  Thread (tq, tk):
// tq = warp * 2 + lane / 16 owns query rows 8 tq .. 8 tq + 7 throughout;
// for the scores it takes keys tk and tk + 16 of the tile, for P.V the output
// dims 4 tk .. 4 tk + 3 and 64 + 4 tk .. 64 + 4 tk + 3.
__global__ void __launch_bounds__(kPThreads) prefill_attn_kernel(const PrefillAttnArgs a) {
    extern __shared__ __align__(16) float psm[];
    float* Qs = psm;                    // [64][kPLd]
    float* Ks = Qs + kPRows * kPLd;     // [32][kPLd]
    float* Vs = Ks + kPKT * kPLd;       // [32][128]
    float* Pt = Vs + kPKT * 128;        // [32][kPPt]
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int tk = lane & 15, tq = warp * 2 + (lane >> 4);
    const int c0 = blockIdx.x * kPQ, kvh = blockIdx.y, b = blockIdx.z;
    const int nq = min(kPQ, a.C - c0);
    const int QW = a.H * 128;
    const size_t row0 = (size_t)b * a.C + c0;
    for (int i = t; i < kPRows * 32; i += kPThreads) {
        const int r = i >> 5, d4 = (i & 31) * 4;
        const int hh = r / kPQ, c = r % kPQ;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < nq) v = *reinterpret_cast<const float4*>(a.q + (row0 + c) * QW + (kvh * 2 + hh) * 128 + d4);
        *reinterpret_cast<float4*>(Qs + r * kPLd + d4) = v;
    }
    const float* kb = a.k + (size_t)b * a.stride_b + (size_t)kvh * a.stride_h;
    const float* vb = a.v + (size_t)b * a.stride_b + (size_t)kvh * a.stride_h;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    const int nkeys = a.p0 + c0 + nq;  // keys 0 .. last query position of the CTA
    float m[8], l[8], o[8][8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        m[j] = -INFINITY;
        l[j] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) o[j][e] = 0.f;
    }
    for (int k0 = 0; k0 < nkeys; k0 += kPKT) {
        __syncthreads();  // the previous tile is no longer read (and Qs is written)
        for (int i = t; i < kPKT * 32; i += kPThreads) {
            const int kr = i >> 5, d4 = (i & 31) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + kr < nkeys) {
                kv = __ldg(reinterpret_cast<const float4*>(kb + (size_t)(k0 + kr) * 128 + d4));
                vv = __ldg(reinterpret_cast<const float4*>(vb + (size_t)(k0 + kr) * 128 + d4));
            }
            *reinterpret_cast<float4*>(Ks + kr * kPLd + d4) = kv;
            *reinterpret_cast<float4*>(Vs + kr * 128 + d4) = vv;
        }
        __syncthreads();
        float s[8][2];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = 0.f;
#pragma unroll 2
        for (int d = 0; d < 128; d += 4) {
            const float4 ka = *reinterpret_cast<const float4*>(Ks + tk * kPLd + d);
            const float4 kc = *reinterpret_cast<const float4*>(Ks + (tk + 16) * kPLd + d);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 qv = *reinterpret_cast<const float4*>(Qs + (tq * 8 + j) * kPLd + d);
                s[j][0] = fmaf(qv.x, ka.x, fmaf(qv.y, ka.y, fmaf(qv.z, ka.z, fmaf(qv.w, ka.w, s[j][0]))));
                s[j][1] = fmaf(qv.x, kc.x, fmaf(qv.y, kc.y, fmaf(qv.z, kc.z, fmaf(qv.w, kc.w, s[j][1]))));
            }
        }
        // causal mask, scale, online softmax (the 16 lanes of a half-warp share rows)
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int r = tq * 8 + j, c = r % kPQ;
            const int qpos = a.p0 + c0 + c;
            float s0 = (c < nq && k0 + tk <= qpos) ? s[j][0] * scale : -INFINITY;
            float s1 = (c < nq && k0 + tk + 16 <= qpos) ? s[j][1] * scale : -INFINITY;
            float mx = fmaxf(s0, s1);
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[j], mx);
            const float alpha = (m[j] == -INFINITY) ? 0.f : expf(m[j] - mn);
            const float e0 = (s0 == -INFINITY) ? 0.f : expf(s0 - mn);
            const float e1 = (s1 == -INFINITY) ? 0.f : expf(s1 - mn);
            float sum = e0 + e1;
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[j] = l[j] * alpha + sum;
            m[j] = mn;
#pragma unroll
            for (int e = 0; e < 8; e++) o[j][e] *= alpha;
            Pt[tk * kPPt + r] = e0;
            Pt[(tk + 16) * kPPt + r] = e1;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kPKT; kk++) {
            const float4 pa = *reinterpret_cast<const float4*>(Pt + kk * kPPt + tq * 8);
            const float4 pb = *reinterpret_cast<const float4*>(Pt + kk * kPPt + tq * 8 + 4);
            const float4 va = *reinterpret_cast<const float4*>(Vs + kk * 128 + 4 * tk);
            const float4 vc = *reinterpret_cast<const float4*>(Vs + kk * 128 + 64 + 4 * tk);
            const float pj[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                o[j][0] = fmaf(pj[j], va.x, o[j][0]);
                o[j][1] = fmaf(pj[j], va.y, o[j][1]);
                o[j][2] = fmaf(pj[j], va.z, o[j][2]);
                o[j][3] = fmaf(pj[j], va.w, o[j][3]);
                o[j][4] = fmaf(pj[j], vc.x, o[j][4]);
                o[j][5] = fmaf(pj[j], vc.y, o[j][5]);
                o[j][6] = fmaf(pj[j], vc.z, o[j][6]);
                o[j][7] = fmaf(pj[j], vc.w, o[j][7]);
            }
        }
    }
    __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(a.out_hi);
    __nv_bfloat16* lo = static_cast<__nv_bfloat16*>(a.out_lo);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int r = tq * 8 + j, hh = r / kPQ, c = r % kPQ;
        if (c >= nq) continue;
        const size_t base = (row0 + c) * QW + (size_t)(kvh * 2 + hh) * 128;
        const float lsum = l[j];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int d = e < 4 ? 4 * tk + e : 64 + 4 * tk + (e - 4);
            const float y = o[j][e] / lsum;
            a.out[base + d] = y;
            if (hi) {
                const __nv_bfloat16 h = __float2bfloat16_rn(y);
                hi[base + d] = h;
                lo[base + d] = __float2bfloat16_rn(y - __bfloat162float(h));
            }
        }
    }
}

}  // namespace

size_t prefill_attention_smem() { return kPSmem; }

vb_status launch_prefill_attention(const PrefillAttnArgs& a, cudaStream_t s) {
    if (a.D != 128) return fail(VB_ERR_UNSUPPORTED, "prefill attention: head_dim must be 128");
    if (a.KVH <= 0 || a.H != 2 * a.KVH) return fail(VB_ERR_UNSUPPORTED, "prefill attention: needs H == 2 * KVH");
    if (a.B <= 0 || a.C <= 0 || a.p0 < 0 || a.B > 65535) return fail(VB_ERR_ARG, "prefill attention: bad shape");
    static bool attr_done = false;
    if (!attr_done) {
        const cudaError_t ce =
            cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
        if (ce != cudaSuccess) return cuda_fail(ce, "prefill attention: shared memory attribute");
        attr_done = true;
    }
    const dim3 grid((a.C + kPQ - 1) / kPQ, a.KVH, a.B);
    prefill_attn_kernel<<<grid, kPThreads, kPSmem, s>>>(a);
    VB_LAUNCH_CHECK("prefill_attn_kernel");
    return VB_OK;
}

}  // namespace vb
