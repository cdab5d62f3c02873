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
#include "vb_tc.cuh"

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

// ---------------------------------------------------------------------------
// Tensor-core form for a prompt that starts at position 0 (the whole prompt in
// one chunk).  Operands are bf16 hi + lo pairs of the f32 values (q, the
// chunk's K rows, and V transposed so its positions run along K of the P.V
// product): S = Q_hi K_hi + Q_hi K_lo + Q_lo K_hi and O += P_hi V_hi +
// P_lo V_hi + P_hi V_lo, products exact in f32, dropped terms ~2^-16.
//
// CTA = 64 query positions x the 2 query heads of one KV head = 128 query rows
// (MMA M, tensor-memory lanes).  256 threads: threads r and 128 + r share row r,
// the first taking keys 0-31 of a tile and output dims 0-63, the second keys
// 32-63 and dims 64-127.  Per 64-key tile: TMA (double-buffered) -> S MMA into
// tensor memory (64 columns) -> each thread reads its half row of S, the two
// halves combine the row maximum and sum through shared memory (online
// softmax, causal mask), each writes its half of P_hi / P_lo into the row's
// 128-byte swizzled shared-memory line -> P.V MMA into tensor memory (128
// columns) -> each thread folds its 64 dims into its output registers.
constexpr int kAQ = 64;                         // query positions per CTA
constexpr int kAK = 64;                         // keys per tile
constexpr int kQT = 128 * 128;                  // [128 rows][64 bf16] swizzled tile, 16 KB
constexpr int kKT = 64 * 128;                   // [64 keys][64 bf16], 8 KB
constexpr int kVT = 128 * 128;                  // [128 dims][64 keys], 16 KB
constexpr int kOffQ = 0;                        // [hi/lo][d half] 4 x 16 KB
constexpr int kOffKV = 4 * kQT;                 // [buf] {K [hi/lo][d half] 4 x 8 KB, Vt [hi/lo] 2 x 16 KB}
constexpr int kKVBuf = 4 * kKT + 2 * kVT;       // 64 KB
constexpr int kOffP = kOffKV + 2 * kKVBuf;      // [hi/lo] 2 x 16 KB
constexpr size_t kTASmem = (size_t)kOffP + 2 * kQT + 1024;
constexpr uint32_t kIdS = idesc_bf16(128, kAK);
constexpr uint32_t kIdPV = idesc_bf16(128, 128);

struct TcAttnParams {
    int P, KVH, QW;          // prompt length, KV heads, H * 128
    __nv_bfloat16* out_hi;   // [B*P][QW] split of the output
    __nv_bfloat16* out_lo;
    float* out;              // optional f32 output
    int* err;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// bf16 hi / lo split of a pair: hi = rn(a) | rn(b), lo = rn(a - hi) | rn(b - hi)
// (the widened hi values are the packed word's halves shifted into place)
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = pack_bf16(a, b);
    lo = pack_bf16(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
}

__global__ void __launch_bounds__(256, 1)
    tc_prefill_attn_kernel(const __grid_constant__ CUtensorMap mq_hi, const __grid_constant__ CUtensorMap mq_lo,
                           const __grid_constant__ CUtensorMap mk_hi, const __grid_constant__ CUtensorMap mk_lo,
                           const __grid_constant__ CUtensorMap mv_hi, const __grid_constant__ CUtensorMap mv_lo,
                           const TcAttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) unsigned long long q_full, kv_full[2], s_done, pv_done;
    __shared__ unsigned tmem_slot;
    __shared__ float xch[2][128];  // the row halves' maximum per key tile, their sums at the end
    const unsigned sb = (smem_addr(smem_raw) + 1023u) & ~1023u;
    uint8_t* sg = smem_raw + (sb - smem_addr(smem_raw));
    const int t = threadIdx.x, warp = t >> 5;
    const int c0 = blockIdx.x * kAQ, kvh = blockIdx.y, b = blockIdx.z;
    const int nq = min(kAQ, p.P - c0);
    const int nt = (c0 + nq - 1) / kAK + 1;  // key tiles up to the last query position
    const int kv_row = (b * p.KVH + kvh);
    if (t == 0) {
        mbar_init(smem_addr(&q_full), 1);
        mbar_init(smem_addr(&kv_full[0]), 1);
        mbar_init(smem_addr(&kv_full[1]), 1);
        mbar_init(smem_addr(&s_done), 1);
        mbar_init(smem_addr(&pv_done), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(256)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tS = tmem_slot, tPV = tmem_slot + 128;
    auto issue_kv = [&](int tile, int buf) {
        const unsigned fb = smem_addr(&kv_full[buf]);
        const unsigned base = sb + kOffKV + (unsigned)buf * kKVBuf;
        mbar_expect_tx(fb, (unsigned)kKVBuf);
#pragma unroll
        for (int hl = 0; hl < 2; hl++)
#pragma unroll
            for (int dh = 0; dh < 2; dh++)
                tma_load_2d(base + (hl * 2 + dh) * kKT, hl ? &mk_lo : &mk_hi, dh * 64, kv_row * p.P + tile * kAK, fb);
        tma_load_2d(base + 4 * kKT, &mv_hi, tile * kAK, kv_row * 128, fb);
        tma_load_2d(base + 4 * kKT + kVT, &mv_lo, tile * kAK, kv_row * 128, fb);
    };
    if (t == 0) {
        const unsigned qb = smem_addr(&q_full);
        mbar_expect_tx(qb, (unsigned)(4 * kQT));
#pragma unroll
        for (int hl = 0; hl < 2; hl++)
#pragma unroll
            for (int dh = 0; dh < 2; dh++)
#pragma unroll
                for (int hh = 0; hh < 2; hh++)
                    tma_load_2d(sb + kOffQ + (hl * 2 + dh) * kQT + hh * (kQT / 2), hl ? &mq_lo : &mq_hi,
                                (2 * kvh + hh) * 128 + dh * 64, b * p.P + c0, qb);
        issue_kv(0, 0);
        if (nt > 1) issue_kv(1, 1);
    }
    const int r = t & 127, hf = t >> 7;  // query row: position c0 + (r & 63) of head 2 kvh + (r >> 6)
    const int qpos = c0 + (r & 63);
    const bool rvalid = (r & 63) < nq;
    // logits in base 2: exp(s / sqrt(D) - m) = 2^(s log2(e) / sqrt(D) - m')
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f)) * 1.44269504088896341f;
    const unsigned lane_off = (unsigned)(32 * (warp & 3)) << 16;  // warp w reads lanes 32 (w % 4) ..
    float o[64];
#pragma unroll
    for (int d = 0; d < 64; d++) o[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int issued = nt > 1 ? 2 : 1;  // key tiles requested so far
    int s_issued = -1, s_seen = -1;  // last S product issued (thread 32) / waited for (all)
    int pv_committed = -1;           // last P.V commit (thread 32)
    // thread 32: S = Q K^T of key tile `tile` into tS (false: its copies never came)
    auto issue_s = [&](int tile) -> bool {
        const int bf = tile & 1;
        const bool w = (tile > 0 || mbar_wait(smem_addr(&q_full), 0u, p.err, nullptr, kSiteFull, -1)) &&
                       mbar_wait(smem_addr(&kv_full[bf]), (unsigned)(tile >> 1) & 1u, p.err, nullptr, kSiteFull, tile);
        if (w) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned kb = sb + kOffKV + (unsigned)bf * kKVBuf;
#pragma unroll
            for (int dh = 0; dh < 2; dh++)
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t qh = sw128_desc(sb + kOffQ + dh * kQT + 32u * kk);
                    const uint64_t ql = sw128_desc(sb + kOffQ + (2 + dh) * kQT + 32u * kk);
                    const uint64_t kh = sw128_desc(kb + dh * kKT + 32u * kk);
                    const uint64_t kl = sw128_desc(kb + (2 + dh) * kKT + 32u * kk);
                    mma_f16(tS, qh, kh, kIdS, dh > 0 || kk > 0);
                    mma_f16(tS, qh, kl, kIdS, true);
                    mma_f16(tS, ql, kh, kIdS, true);
                }
        }
        // commit even after a failed wait so the waiters are released
        mma_commit(smem_addr(&s_done));
        s_issued = tile;
        return w;
    };
    for (int it = 0; it < nt; it++) {
        const int buf = it & 1;
        if (t == 32 && it == 0 && !issue_s(0)) ok = false;
        ok = mbar_wait(smem_addr(&s_done), (unsigned)it & 1u, p.err, nullptr, kSiteFull, it) && ok;
        s_seen = it;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float sv[32];
        tmem_ld32(tS + lane_off + 32u * (unsigned)hf, sv);
        const int k0 = it * kAK + 32 * hf;
        float mx = -INFINITY;
        if (rvalid && k0 + 31 <= qpos) {  // every key of this half tile is visible
#pragma unroll
            for (int j = 0; j < 32; j++) {
                sv[j] *= scale;
                mx = fmaxf(mx, sv[j]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                sv[j] = (rvalid && k0 + j <= qpos) ? sv[j] * scale : -INFINITY;
                mx = fmaxf(mx, sv[j]);
            }
        }
        // the two halves of a row sit in warps w and w + 4: a barrier of that pair only
        xch[hf][r] = mx;
        asm volatile("bar.sync %0, 64;" ::"r"(1 + (warp & 3)) : "memory");
        mx = fmaxf(xch[0][r], xch[1][r]);
        const float mn = fmaxf(m, mx);
        const float mb = mn == -INFINITY ? 0.f : mn;  // a row with no key yet: every weight 0
        const float alpha = ex2_approx(m - mb);
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            sv[j] = ex2_approx(sv[j] - mb);
            sum += sv[j];
        }
        // this half's share of the row sum (alpha is the same for both halves)
        l = l * alpha + sum;
        m = mn;
        // P_hi / P_lo: this thread's half row, chunks 4 hf .. 4 hf + 3 of 8 keys, 128-byte swizzle
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
            const int c = 4 * hf + cc;
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int q = 0; q < 4; q++) split_pair(sv[8 * cc + 2 * q], sv[8 * cc + 2 * q + 1], hv[q], lv[q]);
            const int off = r * 128 + ((c ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(sg + kOffP + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4*>(sg + kOffP + kQT + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        // One barrier per key tile: it orders this tile's P writes before its P.V, every
        // read of S before the next S product, the previous fold before this P.V, and the
        // row-maximum exchange before the next one; and it carries the failure verdict.
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        if (t == 32) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (ok) {
                const unsigned vb = sb + kOffKV + (unsigned)buf * kKVBuf + 4 * kKT;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t ph = sw128_desc(sb + kOffP + 32u * kk);
                    const uint64_t pl = sw128_desc(sb + kOffP + kQT + 32u * kk);
                    const uint64_t vh = sw128_desc(vb + 32u * kk);
                    const uint64_t vl = sw128_desc(vb + kVT + 32u * kk);
                    mma_f16(tPV, ph, vh, kIdPV, kk > 0);
                    mma_f16(tPV, pl, vh, kIdPV, true);
                    mma_f16(tPV, ph, vl, kIdPV, true);
                }
            }
            mma_commit(smem_addr(&pv_done));
            pv_committed = it;
            // the next key tile's S runs while the threads fold this P.V in (every thread
            // read this tile's S before the barrier above)
            if (it + 1 < nt && !issue_s(it + 1)) ok = false;
        }
        ok = mbar_wait(smem_addr(&pv_done), (unsigned)it & 1u, p.err, nullptr, kSiteFull, it) && ok;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // buffer `buf` is free again: request key tile it + 2 into it
        if (t == 0 && it + 2 < nt) {
            issue_kv(it + 2, buf);
            issued = it + 3;
        }
        {
            float pv[64];
            tmem_ld64(tPV + lane_off + 64u * (unsigned)hf, pv);
#pragma unroll
            for (int d = 0; d < 64; d++) o[d] = fmaf(o[d], alpha, pv[d]);
        }
    }
    // the row sum from its two halves (every thread has passed the last tile's barrier)
    xch[hf][r] = l;
    ok = __syncthreads_and(ok);
    l = xch[0][r] + xch[1][r];
    if (t == 32) {
        // never release tensor memory with an MMA in flight: a failed pass can
        // leave the next S product and the last P.V unobserved (these waits
        // end only when the products land, or at the time bound)
        if (s_issued > s_seen) mbar_drain(smem_addr(&s_done), (unsigned)s_issued & 1u);
        if (pv_committed >= 0) mbar_drain(smem_addr(&pv_done), (unsigned)pv_committed & 1u);
    }
    if (t == 0) {
        // never leave with copies in flight (the last two requested tiles)
        for (int i = issued > 2 ? issued - 2 : 0; i < issued; i++)
            mbar_drain(smem_addr(&kv_full[i & 1]), (unsigned)(i >> 1) & 1u);
        mbar_drain(smem_addr(&q_full), 0u);
    }
    if (ok && rvalid) {
        const int hh = r >> 6;
        const size_t base = (size_t)(b * p.P + qpos) * p.QW + (size_t)(2 * kvh + hh) * 128 + 64 * hf;
#pragma unroll
        for (int d = 0; d < 64; d += 8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; e++) y[e] = o[d + e] / l;
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int q = 0; q < 4; q++) split_pair(y[2 * q], y[2 * q + 1], hv[q], lv[q]);
            *reinterpret_cast<uint4*>(p.out_hi + base + d) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4*>(p.out_lo + base + d) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
            if (p.out) {
                *reinterpret_cast<float4*>(p.out + base + d) = make_float4(y[0], y[1], y[2], y[3]);
                *reinterpret_cast<float4*>(p.out + base + d + 4) = make_float4(y[4], y[5], y[6], y[7]);
            }
        }
    } else if (!ok && t == 0) {
        atomicCAS(p.err, 0, kErrPipeTimeout);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_slot), "r"(256) : "memory");
}

// bf16 hi / lo copies of the prompt's K rows ([B*KVH*P][128]) and of V
// transposed ([B*KVH*128][Ppad], positions along the row).  grid
// (ceil(P / 32), KVH, B), 256 threads.
__global__ void __launch_bounds__(256) prompt_kv_split_kernel(const float* k, const float* v, int64_t stride_b,
                                                              int64_t stride_h, int P, int Ppad, int KVH,
                                                              __nv_bfloat16* k_hi, __nv_bfloat16* k_lo,
                                                              __nv_bfloat16* vt_hi, __nv_bfloat16* vt_lo) {
    __shared__ float vs[32][129];
    const int p0 = blockIdx.x * 32, kvh = blockIdx.y, b = blockIdx.z, t = threadIdx.x;
    const size_t src = (size_t)b * stride_b + (size_t)kvh * stride_h;
    const size_t krow = (size_t)(b * KVH + kvh) * P;
    for (int i = t; i < 32 * 128; i += 256) {
        const int pp = i >> 7, d = i & 127;
        if (p0 + pp >= P) continue;
        const float kx = k[src + (size_t)(p0 + pp) * 128 + d];
        const __nv_bfloat16 kh = __float2bfloat16_rn(kx);
        k_hi[(krow + p0 + pp) * 128 + d] = kh;
        k_lo[(krow + p0 + pp) * 128 + d] = __float2bfloat16_rn(kx - __bfloat162float(kh));
        vs[pp][d] = v[src + (size_t)(p0 + pp) * 128 + d];
    }
    __syncthreads();
    // thread: dim d = t / 2, positions 16 * (t & 1) .. + 15 of the tile
    const int d = t >> 1, q0 = 16 * (t & 1);
    const size_t vrow = ((size_t)(b * KVH + kvh) * 128 + d) * Ppad + p0 + q0;
#pragma unroll
    for (int q = 0; q < 16; q++) {
        if (p0 + q0 + q >= P) break;
        const float vx = vs[q0 + q][d];
        const __nv_bfloat16 vh = __float2bfloat16_rn(vx);
        vt_hi[vrow + q] = vh;
        vt_lo[vrow + q] = __float2bfloat16_rn(vx - __bfloat162float(vh));
    }
}

// bf16 hi / lo copies of V transposed ([B*KVH*128][Ppad], positions along the
// row) for 64 positions per CTA: coalesced float4 reads, a padded
// shared-memory transpose, 16-byte stores of 8 positions.  grid
// (ceil(P / 64), KVH, B), 256 threads.
__global__ void __launch_bounds__(256) prompt_vt_kernel(const float* v, int64_t stride_b, int64_t stride_h, int P,
                                                        int Ppad, int KVH, __nv_bfloat16* vt_hi,
                                                        __nv_bfloat16* vt_lo) {
    __shared__ float vs[128][65];
    const int p0 = blockIdx.x * 64, kvh = blockIdx.y, b = blockIdx.z, t = threadIdx.x;
    const float* src = v + (size_t)b * stride_b + (size_t)kvh * stride_h;
    for (int i = t; i < 64 * 32; i += 256) {
        const int pp = i >> 5, d4 = (i & 31) * 4;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p0 + pp < P) x = __ldg(reinterpret_cast<const float4*>(src + (size_t)(p0 + pp) * 128 + d4));
        vs[d4][pp] = x.x;
        vs[d4 + 1][pp] = x.y;
        vs[d4 + 2][pp] = x.z;
        vs[d4 + 3][pp] = x.w;
    }
    __syncthreads();
    const size_t row0 = (size_t)(b * KVH + kvh) * 128;
    for (int i = t; i < 128 * 8; i += 256) {
        const int d = i >> 3, c = i & 7;
        uint32_t hv[4], lv[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float a = vs[d][8 * c + 2 * q], bb = vs[d][8 * c + 2 * q + 1];
            const __nv_bfloat16 ah = __float2bfloat16_rn(a), bh = __float2bfloat16_rn(bb);
            hv[q] = pack_bf16(__bfloat162float(ah), __bfloat162float(bh));
            lv[q] = pack_bf16(a - __bfloat162float(ah), bb - __bfloat162float(bh));
        }
        // positions past P are written as zeros (the padding of the last tile)
        const size_t o = (row0 + d) * Ppad + p0 + 8 * c;
        *reinterpret_cast<uint4*>(vt_hi + o) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4*>(vt_lo + o) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
}

}  // namespace

size_t prefill_attention_smem() { return kPSmem; }

vb_status launch_prefill_attention(const PrefillAttnArgs& a, cudaStream_t s) {
    if (a.D != 128) return fail(VB_ERR_UNSUPPORTED, "prefill attention: head_dim must be 128");
    if (a.KVH <= 0 || a.H != 2 * a.KVH) return fail(VB_ERR_UNSUPPORTED, "prefill attention: needs H == 2 * KVH");
    if (a.B <= 0 || a.C <= 0 || a.p0 < 0 || a.B > 65535) return fail(VB_ERR_ARG, "prefill attention: bad shape");
    {
        static std::atomic<unsigned long long> done{0};
        const cudaError_t ce = smem_attr_once(prefill_attn_kernel, (int)kPSmem, done);
        if (ce != cudaSuccess) return cuda_fail(ce, "prefill attention: shared memory attribute");
    }
    const dim3 grid((a.C + kPQ - 1) / kPQ, a.KVH, a.B);
    prefill_attn_kernel<<<grid, kPThreads, kPSmem, s>>>(a);
    VB_LAUNCH_CHECK("prefill_attn_kernel");
    return VB_OK;
}

size_t prompt_attention_tc_bytes(int B, int P, int H, int KVH) {
    const size_t Ppad = (size_t)(P + 63) / 64 * 64;
    return 2 * ((size_t)B * P * H * 128 + (size_t)B * KVH * P * 128 + (size_t)B * KVH * 128 * Ppad) * 2;
}

PromptCopies prompt_attention_copies(void* scratch, int B, int P, int H, int KVH) {
    const int QW = H * 128, Ppad = (P + 63) / 64 * 64;
    PromptCopies c;
    __nv_bfloat16* base = static_cast<__nv_bfloat16*>(scratch);
    c.q_hi = base;
    c.q_lo = base + (size_t)B * P * QW;
    c.k_hi = base + 2 * (size_t)B * P * QW;
    c.k_lo = static_cast<__nv_bfloat16*>(c.k_hi) + (size_t)B * KVH * P * 128;
    c.vt_hi = static_cast<__nv_bfloat16*>(c.k_lo) + (size_t)B * KVH * P * 128;
    c.vt_lo = static_cast<__nv_bfloat16*>(c.vt_hi) + (size_t)B * KVH * 128 * Ppad;
    return c;
}

vb_status launch_prompt_attention_tc(const PrefillAttnArgs& a, const float* q, void* scratch, cudaStream_t s,
                                     bool qk_ready) {
    if (a.D != 128 || a.H != 2 * a.KVH || a.p0 != 0 || a.C <= 0 || a.B <= 0)
        return fail(VB_ERR_UNSUPPORTED, "prompt attention (tensor cores): needs D 128, H 2*KVH, a prompt from 0");
    if (!a.out_hi || !a.out_lo) return fail(VB_ERR_ARG, "prompt attention (tensor cores): split output missing");
    const int B = a.B, P = a.C, KVH = a.KVH, QW = a.H * 128;
    const int Ppad = (P + 63) / 64 * 64;
    if ((size_t)B * P > (size_t)1 << 30 || (size_t)B * KVH * 128 > (size_t)1 << 30)
        return fail(VB_ERR_UNSUPPORTED, "prompt attention (tensor cores): too many rows");
    const PromptCopies cp = prompt_attention_copies(scratch, B, P, a.H, KVH);
    __nv_bfloat16 *q_hi = static_cast<__nv_bfloat16*>(cp.q_hi), *q_lo = static_cast<__nv_bfloat16*>(cp.q_lo);
    __nv_bfloat16 *k_hi = static_cast<__nv_bfloat16*>(cp.k_hi), *k_lo = static_cast<__nv_bfloat16*>(cp.k_lo);
    __nv_bfloat16 *vt_hi = static_cast<__nv_bfloat16*>(cp.vt_hi), *vt_lo = static_cast<__nv_bfloat16*>(cp.vt_lo);
    vb_status st;
    if (qk_ready) {
        // q and K copies were written by the q/k-norm kernel; V^T here (zero padding included)
        prompt_vt_kernel<<<dim3(Ppad / 64, KVH, B), 256, 0, s>>>(a.v, a.stride_b, a.stride_h, P, Ppad, KVH, vt_hi,
                                                                 vt_lo);
        VB_LAUNCH_CHECK("prompt_vt_kernel");
    } else {
        if (Ppad != P) {
            // padding columns of V^T are read by the last key tile (with zero weights): keep them finite
            VB_CUDA_TRY(cudaMemsetAsync(vt_hi, 0, (size_t)B * KVH * 128 * Ppad * 2 * 2, s));
        }
        if ((st = launch_split_bf16(q, B * P, QW, QW, q_hi, q_lo, s, false))) return st;
        prompt_kv_split_kernel<<<dim3((P + 31) / 32, KVH, B), 256, 0, s>>>(a.k, a.v, a.stride_b, a.stride_h, P, Ppad,
                                                                          KVH, k_hi, k_lo, vt_hi, vt_lo);
        VB_LAUNCH_CHECK("prompt_kv_split_kernel");
    }
    CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
    if ((st = tc_make_map(&mqh, q_hi, B * P, QW, 64)) || (st = tc_make_map(&mql, q_lo, B * P, QW, 64)) ||
        (st = tc_make_map(&mkh, k_hi, B * KVH * P, 128, 64)) || (st = tc_make_map(&mkl, k_lo, B * KVH * P, 128, 64)) ||
        (st = tc_make_map(&mvh, vt_hi, B * KVH * 128, Ppad, 128)) ||
        (st = tc_make_map(&mvl, vt_lo, B * KVH * 128, Ppad, 128)))
        return st;
    {
        static std::atomic<unsigned long long> done{0};
        const cudaError_t ce = smem_attr_once(tc_prefill_attn_kernel, (int)kTASmem, done);
        if (ce != cudaSuccess) return cuda_fail(ce, "prompt attention: shared memory attribute");
    }
    TcAttnParams p{};
    p.P = P;
    p.KVH = KVH;
    p.QW = QW;
    p.out_hi = static_cast<__nv_bfloat16*>(a.out_hi);
    p.out_lo = static_cast<__nv_bfloat16*>(a.out_lo);
    p.out = a.out;
    p.err = a.err;
    tc_prefill_attn_kernel<<<dim3((P + kAQ - 1) / kAQ, KVH, B), 256, kTASmem, s>>>(mqh, mql, mkh, mkl, mvh, mvl, p);
    VB_LAUNCH_CHECK("tc_prefill_attn_kernel");
    return VB_OK;
}

}  // namespace vb
