// vb_mega2.cu -- batch-1 decode step, persistent, TWO grid barriers per layer.
//
// Grid = 8 thread-block clusters x 8 CTAs (one CTA per SM, 64 SMs: a 12-stage
// TMA ring per CTA already saturates HBM from 64 SMs).  Cluster k owns KV
// head k.  Per layer:
//
//   phase A  (cluster k, CTA r)
//     x += sum_c D-partials of the previous layer (fixed order), RMSNorm
//     rows [64r, 64r+64) of the kv-head-k block of Wqkv  (q head 2k, 2k+1, k, v)
//     cluster barrier; gather the 512 q/k/v values from the 8 CTAs (DSMEM)
//     q/k RMSNorm + RoPE, KV append (r = 0), attention over this CTA's
//     32-position chunks (chunk c on CTA c % 8) with an online softmax
//     cluster barrier; merge the 8 CTA partials (DSMEM) -> ctx of heads 2k,2k+1
//     split-K o_proj: rows [128r, 128r+128) of Wo[:, 256k:256k+256] . ctx
//       -> partial_o[k]
//   grid barrier
//   phase B  (every CTA b)
//     x += sum_k partial_o[k] (fixed order), RMSNorm
//     its slice of gate/up pairs -> h slice (SwiGLU fused)
//     split-K down: sum_{i in slice} h_i * Wd^T[i, :] -> 1024-wide partial
//     cluster barrier; CTA r reduces elements [128r, 128r+128) over the 8
//     CTAs of its cluster (DSMEM) -> partial_d[cluster]
//   grid barrier
// then LM (all CTAs): x += sum partial_d, final RMSNorm, logits rows + argmax.
//
// Every CTA keeps its own copy of the residual stream x in shared memory; all
// copies are bit-identical (same inputs summed in the same order).  Weights
// are stored in layouts made for this schedule (a row permutation of Wqkv,
// column blocks of Wo, the transpose of Wd); INT8 values and per-row scales are
// the same numbers, placed differently, so quantisation stays bit-exact.
//
// A producer warp streams every byte the CTA needs for the whole token through
// the shared-memory ring (cp.async.bulk + mbarriers) and never waits for
// activations.  All waits are bounded (2 s of %globaltimer) and record where
// they gave up.  Cluster barriers are mbarriers arrived on remotely at cluster
// scope by each CTA's consumer thread 0, so the producer never joins them.
#include <limits.h>
#include <math.h>

#include <string>
#include <vector>

#include "vb_engine.cuh"
#include "vb_pipe.cuh"

namespace vb {
namespace {

constexpr int kCS = 8;              // CTAs per cluster
constexpr int kStageBytes = 16384;
constexpr int kStages = 11;
constexpr int kCW = 8;              // consumer warps
constexpr int kCT = kCW * 32;       // consumer threads
constexpr int kThreads = kCT + 32;  // + producer warp
constexpr int kChunk = 32;
constexpr int kHid = 1024;          // hidden size this kernel is laid out for
constexpr int kXs = 4096;           // normalised-input capacity (floats)
constexpr int kPer = kXs / kCT;     // 16
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kXs * sizeof(float);

struct M2Layer {
    const void* wqkv;  // [KVH][512][hidden]
    const float* sqkv; // [KVH][512]
    const void* wo;    // [KVH][hidden][256]
    const float* so;   // [hidden]
    const void* wgu;   // [2*ffn][hidden], gate/up rows interleaved
    const float* sgu;  // [2*ffn]
    const void* wdt;   // [ffn][hidden]  (Wd transposed)
    const float* sd;   // [hidden]
    const float* in_norm;
    const float* post_norm;
    const float* q_norm;
    const float* k_norm;
};

struct M2Params {
    const M2Layer* layers;
    const float* embed;
    const float* final_norm;
    const float* rope_cos;
    const float* rope_sin;
    float* kc;  // [L][KVH][max_seq][128]
    float* vc;
    float* logits;
    float* part_o;  // [KVH][hidden]
    float* part_d;  // [nclusters][hidden]
    float* am_val;
    int* am_idx;
    int* am_ticket;
    unsigned* bar;
    int* tok;
    int* pos;
    int* next;
    int* hist;
    int* step;
    int* err;
    int* dbg;
    unsigned long long* trace;  // optional: per CTA, kTraceMarks stamps per layer
    int hidden, nlayers, kvh, ffn, vocab, max_seq, nclusters;
    float eps;
};

// Trace: word 0 = start, then per layer kTraceMarks %globaltimer stamps of
// consumer thread 0: A residual+norm, A qkv rows, A gather, A attention,
// A merge, A o_proj, A release, B residual+norm, B gate/up, B down,
// B cluster reduce, B release.
constexpr int kTraceStride2 = 1024;
constexpr int kTraceMarks = 12;
__device__ __forceinline__ void tmark(const M2Params& p, int l, int i) {
    if (p.trace && threadIdx.x == 0 && 1 + kTraceMarks * (l + 1) < kTraceStride2)
        p.trace[(size_t)blockIdx.x * kTraceStride2 + 1 + kTraceMarks * l + i] = now_ns();
}

struct __align__(16) S2 {
    float xr[kHid];       // residual stream (identical in every CTA)
    float accd[kHid];     // split-K down partial of this CTA
    float qkv_part[64];   // this CTA's 64 rows of its kv-head block
    float qkv[512];       // gathered q(2 heads) | k | v
    float q[2][128];
    float tq[2][128];
    float kn[128];
    float tk[128];
    float vn[128];
    float att_acc[2][128];  // this CTA's attention partial
    float att_m[2], att_l[2];
    float sc[2][kChunk];
    float e[2][kChunk];
    float cm[2], cl[2];
    float h[64];
    double red[16];
    float bv[kCW];
    int bi[kCW];
    int gflag;
    int wflag;
    unsigned long long full[kStages];
    unsigned long long empty[kStages];
    unsigned long long cbar;  // cluster barrier: kCS remote arrivals per phase
    volatile int seq[kStages];
};

__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cluster_id() {
    unsigned r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned mapa(unsigned local, unsigned rank) {
    unsigned r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_dsmem(unsigned addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Cluster-wide barrier over the consumer threads of the kCS CTAs.
__device__ bool cluster_sync(const M2Params& p, S2& S, unsigned& cphase) {
    consumers_sync<kCT>();
    if (threadIdx.x == 0) {
        const unsigned la = smem_addr(&S.cbar);
        for (unsigned r = 0; r < kCS; r++) {
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mapa(la, r))
                         : "memory");
        }
        bool ok = true;
        const unsigned par = cphase & 1u;
        const unsigned long long t0 = now_ns();
        for (unsigned it = 0;; it++) {
            unsigned done;
            asm volatile(
                "{ .reg .pred q; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 q, [%1], %2; "
                "selp.u32 %0, 1, 0, q; }"
                : "=r"(done)
                : "r"(la), "r"(par)
                : "memory");
            if (done) break;
            if ((it & 255u) == 255u) {
                if (err_read(p.err)) { ok = false; break; }
                if (now_ns() - t0 > kWaitNs) {
                    record_fail(p.err, p.dbg, kErrPipeTimeout, 6, (int)cphase, 0);
                    ok = false;
                    break;
                }
            }
        }
        S.wflag = ok ? 1 : 0;
    }
    cphase++;
    consumers_sync<kCT>();
    return S.wflag != 0;
}

__device__ bool grid_barrier2(const M2Params& p, unsigned target, S2& S, bool ok_in) {
    if (!consumers_sync_and<kCT>(ok_in)) {
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kErrPipeTimeout);
        return false;
    }
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p.bar), "r"(1u) : "memory");
        bool ok = true;
        if (ld_acquire(p.bar) < target) {
            const unsigned long long t0 = now_ns();
            for (unsigned it = 1;; it++) {
                if (ld_acquire(p.bar) >= target) break;
                if ((it & 63u) == 0) {
                    if (err_read(p.err)) { ok = false; break; }
                    if (now_ns() - t0 > kWaitNs) {
                        record_fail(p.err, p.dbg, kErrBarrierTimeout, kSiteGrid, (int)target,
                                    (int)ld_acquire(p.bar));
                        ok = false;
                        break;
                    }
                }
            }
        }
        S.gflag = ok ? 1 : 0;
    }
    consumers_sync<kCT>();
    return S.gflag != 0;
}

// ------------------------------------------------------------------ plans
struct Plan {
    const char* w;     // first byte of this CTA's rows
    int row_bytes;
    int rps;           // rows per stage
    int r0, r1;        // rows of the CTA's range (relative to the matrix)
    int K;
    bool q8;
    int nstages;
};

__device__ __forceinline__ Plan make_plan(const void* W, int K, bool q8, int r0, int r1, int unit) {
    Plan g;
    g.K = K;
    g.q8 = q8;
    g.row_bytes = K * (q8 ? 1 : 4);
    g.rps = kStageBytes / g.row_bytes;
    if (unit == 2) g.rps &= ~1;
    g.r0 = r0;
    g.r1 = r1;
    g.w = static_cast<const char*>(W) + (size_t)r0 * g.row_bytes;
    g.nstages = (r1 - r0 + g.rps - 1) / g.rps;
    return g;
}

__device__ __forceinline__ void split(int units, int part, int parts, int unit, int& r0, int& r1) {
    r0 = (int)((long long)part * units / parts) * unit;
    r1 = (int)((long long)(part + 1) * units / parts) * unit;
}

// Phase plans, identical on the producer and consumer side.
__device__ __forceinline__ Plan plan_qkv(const M2Params& p, int l, bool q8, int k, int r) {
    const M2Layer& L = p.layers[l];
    const size_t blk = (size_t)512 * p.hidden * (q8 ? 1 : 4);
    return make_plan(static_cast<const char*>(L.wqkv) + k * blk, p.hidden, q8, 64 * r, 64 * r + 64, 1);
}
__device__ __forceinline__ Plan plan_o(const M2Params& p, int l, bool q8, int k, int r) {
    const M2Layer& L = p.layers[l];
    const int rows = p.hidden / kCS;
    const size_t blk = (size_t)p.hidden * 256 * (q8 ? 1 : 4);
    return make_plan(static_cast<const char*>(L.wo) + k * blk, 256, q8, rows * r, rows * r + rows, 1);
}
__device__ __forceinline__ Plan plan_gu(const M2Params& p, int l, bool q8, int b, int G) {
    int r0, r1;
    split(p.ffn, b, G, 2, r0, r1);
    return make_plan(p.layers[l].wgu, p.hidden, q8, r0, r1, 2);
}
__device__ __forceinline__ Plan plan_dt(const M2Params& p, int l, bool q8, int b, int G) {
    int r0, r1;
    split(p.ffn, b, G, 1, r0, r1);
    return make_plan(p.layers[l].wdt, p.hidden, q8, r0, r1, 1);
}
__device__ __forceinline__ Plan plan_lm(const M2Params& p, int b, int G) {
    int r0, r1;
    split(p.vocab, b, G, 1, r0, r1);
    return make_plan(p.embed, p.hidden, false, r0, r1, 1);
}

// --------------------------------------------------------------- consumers
__device__ __forceinline__ float dot_f32(const float* wrow, const float* xs, int K, int lane) {
    const float4* w4 = reinterpret_cast<const float4*>(wrow);
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    float a0 = 0.f, a1 = 0.f;
    for (int k = lane; k < (K >> 2); k += 64) {
        const float4 w = w4[k], x = x4[k];
        a0 = fmaf(w.x, x.x, a0); a0 = fmaf(w.y, x.y, a0); a0 = fmaf(w.z, x.z, a0); a0 = fmaf(w.w, x.w, a0);
        if (k + 32 < (K >> 2)) {
            const float4 w2 = w4[k + 32], x2 = x4[k + 32];
            a1 = fmaf(w2.x, x2.x, a1); a1 = fmaf(w2.y, x2.y, a1); a1 = fmaf(w2.z, x2.z, a1); a1 = fmaf(w2.w, x2.w, a1);
        }
    }
    return warp_sum(a0 + a1);
}

__device__ __forceinline__ float dot_i8(const int8_t* wrow, const float* xs, int K, int lane) {
    float a0 = 0.f, a1 = 0.f;
    for (int gi = lane; gi < (K >> 4); gi += 32) {
        const uint4 w = *reinterpret_cast<const uint4*>(wrow + 16 * gi);
        const float* xc = xs + ((gi >> 5) << 9) + 4 * lane;
        const float4 x0 = *reinterpret_cast<const float4*>(xc);
        const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
        const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
        const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
        const f4 b0 = i8x4_to_f32(w.x), b1 = i8x4_to_f32(w.y);
        const f4 b2 = i8x4_to_f32(w.z), b3 = i8x4_to_f32(w.w);
        a0 = fmaf(b0.v[0], x0.x, a0); a0 = fmaf(b0.v[1], x0.y, a0);
        a1 = fmaf(b0.v[2], x0.z, a1); a1 = fmaf(b0.v[3], x0.w, a1);
        a0 = fmaf(b1.v[0], x1.x, a0); a0 = fmaf(b1.v[1], x1.y, a0);
        a1 = fmaf(b1.v[2], x1.z, a1); a1 = fmaf(b1.v[3], x1.w, a1);
        a0 = fmaf(b2.v[0], x2.x, a0); a0 = fmaf(b2.v[1], x2.y, a0);
        a1 = fmaf(b2.v[2], x2.z, a1); a1 = fmaf(b2.v[3], x2.w, a1);
        a0 = fmaf(b3.v[0], x3.x, a0); a0 = fmaf(b3.v[1], x3.y, a0);
        a1 = fmaf(b3.v[2], x3.z, a1); a1 = fmaf(b3.v[3], x3.w, a1);
    }
    return warp_sum(a0 + a1);
}

__device__ __forceinline__ int perm_index(int i) {
    const int c = i >> 9, r = i & 511;
    return (c << 9) + (((r >> 2) & 3) << 7) + ((r >> 4) << 2) + (r & 3);
}

// Stage wait shared by all consumer modes.  in_order: every warp takes every
// stage (no slot-order gate needed); otherwise warps take every 8th stage and
// wait for the slot's previous round first.
__device__ bool stage_wait(const M2Params& p, S2& S, int gs, bool in_order) {
    const int lane = threadIdx.x & 31;
    const int slot = gs % kStages;
    const unsigned par = (unsigned)(gs / kStages) & 1u;
    const unsigned a = smem_addr(&S.full[slot]);
    int ok = 1;
    if (lane == 0) {
        ok = ((in_order || seq_wait(S.seq, slot, gs, kStages, p.err, p.dbg)) &&
              mbar_wait(a, par, p.err, p.dbg, kSiteFull, gs)) ? 1 : 0;
        if (ok) S.seq[slot] = gs;
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok && lane != 0)
        for (int i = 0; i < 1024 && !mbar_try(a, par); i++) {
        }
    return ok != 0;
}

// Epilogues of the row-dot phases (lane 0 of the warp that computed the row
// stores; every lane sees the same reduced values).
struct EpiQkvPart {  // phase A: this CTA's rows of its kv-head block
    float* dst;
    int base;
    __device__ void operator()(int row, float a, float) const {
        if ((threadIdx.x & 31) == 0) dst[row - base] = a;
    }
};
struct EpiStore {  // phase A: o_proj partial of the cluster's kv head
    float* dst;
    __device__ void operator()(int row, float a, float) const {
        if ((threadIdx.x & 31) == 0) dst[row] = a;
    }
};
struct EpiSwiGLU {  // phase B: h slice
    float* h;
    int p0;
    __device__ void operator()(int row, float g, float u) const {
        if ((threadIdx.x & 31) == 0) h[(row >> 1) - p0] = silu_f(g) * u;
    }
};
struct EpiLogits {  // LM: logits + running argmax of this lane
    float* logits;
    float* bv;
    int* bi;
    __device__ void operator()(int row, float a, float) const {
        if ((threadIdx.x & 31) == 0) logits[row] = a;
        if (a > *bv || (a == *bv && row < *bi)) {
            *bv = a;
            *bi = row;
        }
    }
};

// Row-dot GEMV phase: result of row r (absolute) goes to epi(r, value).
// warp mode (f32, rows per stage < 8): warp w takes stages w, w+8, ...
// coop mode: every warp takes every stage, rows dealt out across warps.
template <class Epi>
__device__ bool gemv_rows(const M2Params& p, const Plan& g, int gbase, const char* ring, S2& S,
                          const float* xs, const float* scales, bool coop, int pair, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = coop ? 0 : warp; j < g.nstages; j += coop ? 1 : kCW) {
        const int gs = gbase + j;
        if (!stage_wait(p, S, gs, coop)) return false;
        const char* st = ring + (size_t)(gs % kStages) * kStageBytes;
        const int rA = g.r0 + j * g.rps;
        const int nr = min(g.rps, g.r1 - rA);
        const int step = pair ? 2 : 1;
        const int first = coop ? warp * step : 0, stride = coop ? kCW * step : step;
        for (int r = first; r + step - 1 < nr; r += stride) {
            float a = g.q8 ? dot_i8(reinterpret_cast<const int8_t*>(st + (size_t)r * g.row_bytes), xs, g.K, lane)
                           : dot_f32(reinterpret_cast<const float*>(st + (size_t)r * g.row_bytes), xs, g.K, lane);
            if (g.q8) a *= __ldg(scales + rA + r);
            float b = 0.f;
            if (pair) {
                b = g.q8 ? dot_i8(reinterpret_cast<const int8_t*>(st + (size_t)(r + 1) * g.row_bytes), xs, g.K, lane)
                         : dot_f32(reinterpret_cast<const float*>(st + (size_t)(r + 1) * g.row_bytes), xs, g.K, lane);
                if (g.q8) b *= __ldg(scales + rA + r + 1);
            }
            epi(rA + r, a, b);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&S.empty[gs % kStages]), coop ? 1u : (unsigned)kCW);
    }
    return true;
}

// x += sum of `n` partial vectors (fixed order), then RMSNorm with the
// pre-loaded norm registers into xs (lane-interleaved layout for INT8).
__device__ void residual_norm(const M2Params& p, S2& S, float* xs, const float* parts, int n,
                              const float* emb_row, const float (&nw)[kPer], bool perm) {
    const int t = threadIdx.x;
    const int H = p.hidden;
    double ss = 0.0;
    float v[kHid / kCT];
#pragma unroll
    for (int k = 0; k < kHid / kCT; k++) {
        const int i = t + k * kCT;
        float x = 0.f;
        if (i < H) {
            if (emb_row) {
                x = emb_row[i];
            } else {
                float add = 0.f;
                for (int c = 0; c < n; c++) add += __ldcg(parts + (size_t)c * H + i);
                x = S.xr[i] + add;
            }
            S.xr[i] = x;
            ss += (double)x * (double)x;
        }
        v[k] = x;
    }
    ss = warp_sum_d(ss);
    if ((t & 31) == 0) S.red[t >> 5] = ss;
    consumers_sync<kCT>();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kCW; w++) tot += S.red[w];
    const float sc = rms_scale(tot, H, p.eps);
#pragma unroll
    for (int k = 0; k < kHid / kCT; k++) {
        const int i = t + k * kCT;
        if (i < H) xs[perm ? perm_index(i) : i] = __fmul_rn(__fmul_rn(v[k], sc), nw[k]);
    }
    consumers_sync<kCT>();
}

__device__ __forceinline__ void load_norm(const float* w, int K, float (&nw)[kPer]) {
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int i = threadIdx.x + k * kCT;
        nw[k] = (w && i < K) ? __ldg(w + i) : 0.f;
    }
}

__device__ __forceinline__ float rope1(const float* y, int d, const float* cr, const float* sr) {
    return d < 64 ? __fsub_rn(__fmul_rn(y[d], cr[d]), __fmul_rn(y[d + 64], sr[d]))
                  : __fadd_rn(__fmul_rn(y[d], cr[d]), __fmul_rn(y[d - 64], sr[d]));
}

// Phase A for the cluster owning kv head k.
template <bool Q8>
__device__ bool phase_a(const M2Params& p, S2& S, const char* ring, float* xs, int l, int k,
                        int rank, int pos, int nchunks, int& g, unsigned& cphase) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const M2Layer& L = p.layers[l];
    // 1. this CTA's 64 rows of the kv-head block of Wqkv
    {
        const Plan pl = plan_qkv(p, l, Q8, k, rank);
        const float* sc = Q8 ? L.sqkv + k * 512 : nullptr;
        bool ok = gemv_rows(p, pl, g, ring, S, xs, sc, Q8, 0, EpiQkvPart{S.qkv_part, 64 * rank});
        g += pl.nstages;
        if (!consumers_sync_and<kCT>(ok)) return false;
        tmark(p, l, 1);
    }
    // 2. gather the kv head's q/k/v from the 8 CTAs of the cluster
    if (!cluster_sync(p, S, cphase)) return false;
    {
        const unsigned la = smem_addr(&S.qkv_part[0]);
        for (int i = t; i < 512; i += kCT) S.qkv[i] = ld_dsmem(mapa(la + 4 * (i & 63), i >> 6));
    }
    consumers_sync<kCT>();
    tmark(p, l, 2);
    // 3. q/k RMSNorm + RoPE (generate.cpp:52-64), v as is
    {
        const int hs = t >> 7, d = t & 127;
        const float qv = S.qkv[hs * 128 + d];
        const float kv = t < 128 ? S.qkv[256 + d] : 0.f;
        const double sq = warp_sum_d((double)qv * qv), sk = warp_sum_d((double)kv * kv);
        if (lane == 0) {
            S.red[warp] = sq;
            S.red[8 + warp] = sk;
        }
        consumers_sync<kCT>();
        const double tq = S.red[hs * 4] + S.red[hs * 4 + 1] + S.red[hs * 4 + 2] + S.red[hs * 4 + 3];
        S.tq[hs][d] = __fmul_rn(__fmul_rn(qv, rms_scale(tq, 128, p.eps)), L.q_norm[d]);
        if (t < 128) {
            const double tk = S.red[8] + S.red[9] + S.red[10] + S.red[11];
            S.tk[d] = __fmul_rn(__fmul_rn(kv, rms_scale(tk, 128, p.eps)), L.k_norm[d]);
            S.vn[d] = S.qkv[384 + d];
        }
        consumers_sync<kCT>();
        const float* cr = p.rope_cos + (size_t)pos * 128;
        const float* sr = p.rope_sin + (size_t)pos * 128;
        S.q[hs][d] = rope1(S.tq[hs], d, cr, sr);
        if (t < 128) S.kn[d] = rope1(S.tk, d, cr, sr);
        consumers_sync<kCT>();
        if (rank == 0 && t < 128) {
            const size_t off = ((size_t)(l * p.kvh + k) * p.max_seq + pos) * 128 + t;
            p.kc[off] = S.kn[t];
            p.vc[off] = S.vn[t];
        }
    }
    // 4. attention over this CTA's chunks, online softmax across chunks
    {
        const int hs = t >> 7, d = t & 127;
        float M = -INFINITY, Lsum = 0.f, acc = 0.f;
        const int n = pos + 1;
        const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
        for (int c = rank; c < nchunks; c += kCS) {
            const int ks = g, vs = g + 1;
            g += 2;
            if (t == 0) {
                S.wflag = mbar_wait(smem_addr(&S.full[ks % kStages]), (unsigned)(ks / kStages) & 1u,
                                    p.err, p.dbg, kSiteAttFull, ks) &&
                          mbar_wait(smem_addr(&S.full[vs % kStages]), (unsigned)(vs / kStages) & 1u,
                                    p.err, p.dbg, kSiteAttFull, vs);
                if (S.wflag) {
                    S.seq[ks % kStages] = ks;
                    S.seq[vs % kStages] = vs;
                }
            }
            consumers_sync<kCT>();
            if (!S.wflag) return false;
            for (int i = 0; i < 1024 && !mbar_try(smem_addr(&S.full[ks % kStages]), (unsigned)(ks / kStages) & 1u); i++) {
            }
            for (int i = 0; i < 1024 && !mbar_try(smem_addr(&S.full[vs % kStages]), (unsigned)(vs / kStages) & 1u); i++) {
            }
            const float* Kt = reinterpret_cast<const float*>(ring + (size_t)(ks % kStages) * kStageBytes);
            const float* Vt = reinterpret_cast<const float*>(ring + (size_t)(vs % kStages) * kStageBytes);
            const int p0 = c * kChunk;
            {
                const float4 q0 = *reinterpret_cast<const float4*>(&S.q[0][4 * lane]);
                const float4 q1 = *reinterpret_cast<const float4*>(&S.q[1][4 * lane]);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int pl = 4 * warp + u, pa = p0 + pl;
                    const float4 k4 = (pa == pos) ? *reinterpret_cast<const float4*>(&S.kn[4 * lane])
                                                  : *reinterpret_cast<const float4*>(Kt + pl * 128 + 4 * lane);
                    float d0 = q0.x * k4.x, d1 = q1.x * k4.x;
                    d0 = fmaf(q0.y, k4.y, d0); d0 = fmaf(q0.z, k4.z, d0); d0 = fmaf(q0.w, k4.w, d0);
                    d1 = fmaf(q1.y, k4.y, d1); d1 = fmaf(q1.z, k4.z, d1); d1 = fmaf(q1.w, k4.w, d1);
                    d0 = warp_sum(d0) * inv_sqrt_d;
                    d1 = warp_sum(d1) * inv_sqrt_d;
                    if (lane == 0) {
                        S.sc[0][pl] = pa < n ? d0 : -INFINITY;
                        S.sc[1][pl] = pa < n ? d1 : -INFINITY;
                    }
                }
            }
            consumers_sync<kCT>();
            if (warp < 2) {
                const float s = S.sc[warp][lane];
                const float m = warp_max(s);
                const float e = (s == -INFINITY) ? 0.f : expf(s - m);
                const float lsum = warp_sum(e);
                S.e[warp][lane] = e;
                if (lane == 0) {
                    S.cm[warp] = m;
                    S.cl[warp] = lsum;
                }
            }
            consumers_sync<kCT>();
            float ac = 0.f;
            const int nv = min(kChunk, n - p0);
            for (int pl = 0; pl < nv; pl++) {
                const float v = (p0 + pl == pos) ? S.vn[d] : Vt[pl * 128 + d];
                ac = fmaf(S.e[hs][pl], v, ac);
            }
            const float mc = S.cm[hs], lc = S.cl[hs];
            const float Mn = fmaxf(M, mc);
            const float fo = (M == -INFINITY) ? 0.f : expf(M - Mn);
            const float fc = expf(mc - Mn);
            acc = acc * fo + ac * fc;
            Lsum = Lsum * fo + lc * fc;
            M = Mn;
            consumers_sync<kCT>();
            if (t == 0) {
                mbar_arrive(smem_addr(&S.empty[ks % kStages]), kCW);
                mbar_arrive(smem_addr(&S.empty[vs % kStages]), kCW);
            }
        }
        S.att_acc[hs][d] = acc;
        if (d == 0) {
            S.att_m[hs] = M;
            S.att_l[hs] = Lsum;
        }
    }
    tmark(p, l, 3);
    // 5. merge the 8 CTA partials of the cluster -> ctx of heads 2k, 2k+1
    if (!cluster_sync(p, S, cphase)) return false;
    {
        const int hs = t >> 7, d = t & 127;
        const unsigned am = smem_addr(&S.att_m[hs]), al = smem_addr(&S.att_l[hs]);
        const unsigned aa = smem_addr(&S.att_acc[hs][d]);
        float mr[kCS];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kCS; r++) {
            mr[r] = ld_dsmem(mapa(am, r));
            M = fmaxf(M, mr[r]);
        }
        float Lsum = 0.f, A = 0.f;
#pragma unroll
        for (int r = 0; r < kCS; r++) {
            if (mr[r] == -INFINITY) continue;
            const float f = expf(mr[r] - M);
            Lsum = fmaf(ld_dsmem(mapa(al, r)), f, Lsum);
            A = fmaf(ld_dsmem(mapa(aa, r)), f, A);
        }
        const float cval = (Lsum > 0.f) ? A / Lsum : 0.f;
        const int i = hs * 128 + d;
        xs[Q8 ? perm_index(i) : i] = cval;
    }
    consumers_sync<kCT>();
    tmark(p, l, 4);
    // 6. split-K o_proj: rows [128r, 128r+128) of Wo[:, 256k:256k+256]
    {
        const Plan pl = plan_o(p, l, Q8, k, rank);
        bool ok = gemv_rows(p, pl, g, ring, S, xs, L.so, true, 0,
                            EpiStore{p.part_o + (size_t)k * p.hidden});
        g += pl.nstages;
        tmark(p, l, 5);
        return ok;
    }
}

template <bool Q8>
__global__ void __launch_bounds__(kThreads, 1) mega2_kernel(const __grid_constant__ M2Params p) {
    extern __shared__ __align__(1024) char dsmem[];
    __shared__ S2 S;
    char* ring = dsmem;
    float* xs = reinterpret_cast<float*>(dsmem + (size_t)kStages * kStageBytes);
    const int b = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cid = (int)cluster_id(), rank = (int)cluster_rank();

    if (p.trace)
        for (int i = threadIdx.x; i < kTraceStride2; i += kThreads)
            p.trace[(size_t)blockIdx.x * kTraceStride2 + i] = 0ull;
    if (threadIdx.x == 0) {
        if (p.trace) p.trace[(size_t)blockIdx.x * kTraceStride2] = now_ns();
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_addr(&S.full[s]), 1);
            mbar_init(smem_addr(&S.empty[s]), kCW);
            S.seq[s] = s - kStages;
        }
        mbar_init(smem_addr(&S.cbar), kCS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // every CTA of the cluster has initialised its barriers before any remote arrive
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");

    const int pos = *p.pos;
    const int n = pos + 1;
    const int nchunks = (n + kChunk - 1) / kChunk;
    const bool owns_kv = cid < p.kvh;

    if (warp == kCW) {
        // ------------------------------------------------------------ producer
        // every thread of the cluster arrives once at the closing cluster
        // barrier before it leaves (see the end of the kernel)
        if (lane != 0) {
            asm volatile("barrier.cluster.arrive.release;" ::: "memory");
            return;
        }
        unsigned long long pol;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        int g = 0;
        bool ok = true;
        auto issue = [&](const void* src, unsigned bytes) {
            const int slot = g % kStages;
            if (!mbar_wait(smem_addr(&S.empty[slot]), ((unsigned)(g / kStages) & 1u) ^ 1u, p.err,
                           p.dbg, kSiteEmpty, g)) {
                ok = false;
                return;
            }
            mbar_expect_tx(smem_addr(&S.full[slot]), bytes);
            bulk_g2s(smem_addr(ring + (size_t)slot * kStageBytes), src, bytes,
                     smem_addr(&S.full[slot]), pol);
            g++;
        };
        auto issue_plan = [&](const Plan& pl) {
            for (int j = 0; j < pl.nstages && ok; j++) {
                const int rows = min(pl.rps, pl.r1 - pl.r0 - j * pl.rps);
                issue(pl.w + (size_t)j * pl.rps * pl.row_bytes, (unsigned)(rows * pl.row_bytes));
            }
        };
        for (int l = 0; l < p.nlayers && ok; l++) {
            if (owns_kv) {
                issue_plan(plan_qkv(p, l, Q8, cid, rank));
                for (int c = rank; c < nchunks && ok; c += kCS) {
                    const int rows = min(kChunk, p.max_seq - c * kChunk);
                    const size_t off = ((size_t)(l * p.kvh + cid) * p.max_seq + (size_t)c * kChunk) * 128;
                    issue(p.kc + off, (unsigned)(rows * 512));
                    if (ok) issue(p.vc + off, (unsigned)(rows * 512));
                }
                if (ok) issue_plan(plan_o(p, l, Q8, cid, rank));
            }
            if (ok) issue_plan(plan_gu(p, l, Q8, b, G));
            if (ok) issue_plan(plan_dt(p, l, Q8, b, G));
        }
        if (ok) issue_plan(plan_lm(p, b, G));
        const int first = g > kStages ? g - kStages : 0;
        for (int gs = first; gs < g; gs++) {
            const unsigned a = smem_addr(&S.full[gs % kStages]);
            const unsigned par = (unsigned)(gs / kStages) & 1u;
            const unsigned long long t0 = now_ns();
            while (!mbar_try(a, par) && now_ns() - t0 < kWaitNs) {
            }
        }
        asm volatile("barrier.cluster.arrive.release;" ::: "memory");
        return;
    }

    // -------------------------------------------------------------- consumers
    {
    const int tok = *p.tok;
    const float* emb_row = p.embed + (size_t)tok * p.hidden;
    int g = 0;
    unsigned nbar = 0, cphase = 0;
    bool ok = true;
    float nw[kPer];
    load_norm(p.layers[0].in_norm, p.hidden, nw);
    for (int l = 0; l < p.nlayers && ok; l++) {
        const M2Layer& L = p.layers[l];
        // ---- phase A
        bool r = true;
        if (owns_kv) {
            residual_norm(p, S, xs, p.part_d, p.nclusters, l == 0 ? emb_row : nullptr, nw, Q8);
            tmark(p, l, 0);
            r = phase_a<Q8>(p, S, ring, xs, l, cid, rank, pos, nchunks, g, cphase);
        }
        load_norm(L.post_norm, p.hidden, nw);
        ok = grid_barrier2(p, (++nbar) * G, S, r);
        tmark(p, l, 6);
        if (!ok) break;
        // ---- phase B
        if (!owns_kv && l == 0) {
            // CTAs outside the kv clusters start their residual copy here
            for (int i = threadIdx.x; i < p.hidden; i += kCT) S.xr[i] = emb_row[i];
            consumers_sync<kCT>();
        } else if (!owns_kv) {
            // catch up with the previous layer's D partials
            for (int i = threadIdx.x; i < p.hidden; i += kCT) {
                float add = 0.f;
                for (int c = 0; c < p.nclusters; c++) add += __ldcg(p.part_d + (size_t)c * p.hidden + i);
                S.xr[i] += add;
            }
            consumers_sync<kCT>();
        }
        residual_norm(p, S, xs, p.part_o, p.kvh, nullptr, nw, Q8);
        tmark(p, l, 7);
        {
            const Plan pl = plan_gu(p, l, Q8, b, G);
            const int P0 = pl.r0 >> 1;
            r = gemv_rows(p, pl, g, ring, S, xs, L.sgu, Q8 || pl.rps >= 8, 1, EpiSwiGLU{S.h, P0});
            g += pl.nstages;
        }
        if (!consumers_sync_and<kCT>(r)) { ok = false; break; }
        tmark(p, l, 8);
        {   // split-K down: accd[j] = sum_i h_i * WdT[i][j]; thread t owns j = 4t..4t+3
            const Plan pl = plan_dt(p, l, Q8, b, G);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            const int t = threadIdx.x;
            for (int j = 0; j < pl.nstages && r; j++) {
                const int gs = g + j;
                if (!stage_wait(p, S, gs, true)) { r = false; break; }
                const char* st = ring + (size_t)(gs % kStages) * kStageBytes;
                const int rA = pl.r0 + j * pl.rps;
                const int nr = min(pl.rps, pl.r1 - rA);
                for (int rr = 0; rr < nr; rr++) {
                    const float hv = S.h[rA + rr - pl.r0];
                    if (Q8) {
                        const uint32_t wv = *reinterpret_cast<const uint32_t*>(st + (size_t)rr * pl.row_bytes + 4 * t);
                        const f4 f = i8x4_to_f32(wv);
                        acc.x = fmaf(hv, f.v[0], acc.x); acc.y = fmaf(hv, f.v[1], acc.y);
                        acc.z = fmaf(hv, f.v[2], acc.z); acc.w = fmaf(hv, f.v[3], acc.w);
                    } else {
                        const float4 w4 = *reinterpret_cast<const float4*>(st + (size_t)rr * pl.row_bytes + 16 * t);
                        acc.x = fmaf(hv, w4.x, acc.x); acc.y = fmaf(hv, w4.y, acc.y);
                        acc.z = fmaf(hv, w4.z, acc.z); acc.w = fmaf(hv, w4.w, acc.w);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_addr(&S.empty[gs % kStages]), 1u);
            }
            g += pl.nstages;
            *reinterpret_cast<float4*>(&S.accd[4 * t]) = acc;
        }
        if (!consumers_sync_and<kCT>(r)) { ok = false; break; }
        tmark(p, l, 9);
        if (!cluster_sync(p, S, cphase)) { ok = false; break; }
        {   // reduce the cluster's 8 partials: CTA rank reduces [128 rank, +128)
            const int t = threadIdx.x;
            const int per = p.hidden / kCS;
            if (t < per) {
                const int j = rank * per + t;
                const unsigned a = smem_addr(&S.accd[j]);
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < kCS; q++) v += ld_dsmem(mapa(a, q));
                if (Q8) v *= __ldg(L.sd + j);
                p.part_d[(size_t)cid * p.hidden + j] = v;
            }
        }
        load_norm(l + 1 < p.nlayers ? p.layers[l + 1].in_norm : p.final_norm, p.hidden, nw);
        tmark(p, l, 10);
        ok = grid_barrier2(p, (++nbar) * G, S, true);
        tmark(p, l, 11);
    }
    if (!ok) goto consumer_exit;
    // ---- LM: final norm + lm_head + argmax
    residual_norm(p, S, xs, p.part_d, p.nclusters, nullptr, nw, false);
    float best_v = -INFINITY;
    int best_i = INT_MAX;
    {
        const Plan pl = plan_lm(p, b, G);
        const bool r = gemv_rows(p, pl, g, ring, S, xs, nullptr, false, 0,
                                 EpiLogits{p.logits, &best_v, &best_i});
        if (!consumers_sync_and<kCT>(r)) goto consumer_exit;
    }
    if (lane == 0) {
        S.bv[warp] = best_v;
        S.bi[warp] = best_i;
    }
    consumers_sync<kCT>();
    if (threadIdx.x == 0) {
        float bv = S.bv[0];
        int bi = S.bi[0];
        for (int w = 1; w < kCW; w++)
            if (better(S.bv[w], S.bi[w], bv, bi)) { bv = S.bv[w]; bi = S.bi[w]; }
        p.am_val[b] = bv;
        p.am_idx[b] = bi;
        __threadfence();
        const int old = atomicAdd(p.am_ticket, 1);
        if (old == G - 1) {
            __threadfence();
            for (int c = 0; c < G; c++) {
                const float v = __ldcg(p.am_val + c);
                const int i = __ldcg(p.am_idx + c);
                if (better(v, i, bv, bi)) { bv = v; bi = i; }
            }
            const int pick = (bi == INT_MAX) ? 0 : bi;
            *p.next = pick;
            const int s = *p.step;
            if (s >= 0 && s < p.max_seq) p.hist[s] = pick;
            *p.step = s + 1;
            *p.tok = pick;
            *p.pos = pos + 1;
            *p.bar = 0u;
            *p.am_ticket = 0;
        }
    }
    }
consumer_exit:
    // No CTA leaves while a peer of its cluster may still read its shared
    // memory: all consumer threads meet here on every path (the producer
    // warp arrived on its way out).
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// --------------------------------------------------------- weight re-layout
template <class T>
__global__ void transpose_kernel(const T* src, T* dst, int rows, int cols) {
    __shared__ T tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = src[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int r = bx + j, c = by + threadIdx.x;  // dst is [cols][rows]
        if (r < cols && c < rows) dst[(size_t)r * rows + c] = tile[threadIdx.x][j];
    }
}

struct Mega2State {
    M2Params params;
    unsigned long long* trace = nullptr;
    M2Layer* d_layers = nullptr;
    std::vector<void*> bufs;
    char* ws = nullptr;
    char* counters = nullptr;
    size_t counters_bytes = 0;
    int grid = 0;
};

}  // namespace

vb_status mega2_prepare(vb_engine* e) {
    const vb_config& c = e->cfg;
    if (c.heads != 2 * c.kv_heads || c.head_dim != 128 || c.hidden != kHid || c.ffn % 512 ||
        c.kv_heads * kCS > 148)
        return fail(VB_ERR_UNSUPPORTED, "two-barrier step: needs hidden 1024, GQA 2, head_dim 128");
    if (!e->kc) return fail(VB_ERR_NO_CACHE, "call reset_cache() first");
    const bool q8 = e->quantized;
    auto kern = q8 ? mega2_kernel<true> : mega2_kernel<false>;
    VB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c.kv_heads * kCS);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kCS;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int nc = 0;
        VB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&nc, kern, &cfg));
        if (nc < c.kv_heads) return fail(VB_ERR_UNSUPPORTED, "two-barrier step: clusters do not fit");
    }
    Mega2State* m = new Mega2State();
    cudaStream_t s = e->stream;
    const size_t es = q8 ? 1 : 4;
    const size_t hd = c.hidden, D = 128;
    auto alloc = [&](size_t bytes) -> void* {
        void* ptr = nullptr;
        if (cudaMalloc(&ptr, bytes) != cudaSuccess) return nullptr;
        m->bufs.push_back(ptr);
        return ptr;
    };
    std::vector<M2Layer> hl(c.layers);
    cudaError_t ce = cudaSuccess;
    for (int l = 0; l < c.layers && ce == cudaSuccess; l++) {
        const vb_layer_dev& Ld = e->L[l];
        M2Layer& M = hl[l];
        const char* wqkv = static_cast<const char*>(q8 ? (const void*)Ld.qqkv : (const void*)Ld.wqkv);
        const char* wo = static_cast<const char*>(q8 ? (const void*)Ld.qo : (const void*)Ld.wo);
        const char* wd = static_cast<const char*>(q8 ? (const void*)Ld.qd : (const void*)Ld.wd);
        char* nqkv = static_cast<char*>(alloc((size_t)c.kv_heads * 512 * hd * es));
        char* no = static_cast<char*>(alloc(hd * e->q_width * es));
        char* ndt = static_cast<char*>(alloc((size_t)c.ffn * hd * es));
        float* nsq = q8 ? static_cast<float*>(alloc((size_t)c.kv_heads * 512 * 4)) : nullptr;
        if (!nqkv || !no || !ndt || (q8 && !nsq)) {
            ce = cudaErrorMemoryAllocation;
            break;
        }
        const size_t rowb = hd * es;
        for (int k = 0; k < c.kv_heads && ce == cudaSuccess; k++) {
            // block k rows: q head 2k, q head 2k+1, k head k, v head k (128 rows each)
            const int src_rows[4] = {(2 * k) * 128, (2 * k + 1) * 128, (c.heads + k) * 128,
                                     (c.heads + c.kv_heads + k) * 128};
            for (int q = 0; q < 4 && ce == cudaSuccess; q++) {
                ce = cudaMemcpyAsync(nqkv + ((size_t)k * 512 + q * 128) * rowb,
                                     wqkv + (size_t)src_rows[q] * rowb, 128 * rowb,
                                     cudaMemcpyDeviceToDevice, s);
                if (q8 && ce == cudaSuccess)
                    ce = cudaMemcpyAsync(nsq + k * 512 + q * 128, Ld.sqkv + src_rows[q], 128 * 4,
                                         cudaMemcpyDeviceToDevice, s);
            }
            // Wo columns [256k, 256k+256) -> block k [hidden][256]
            if (ce == cudaSuccess)
                ce = cudaMemcpy2DAsync(no + (size_t)k * hd * 256 * es, 256 * es, wo + (size_t)k * 256 * es,
                                       (size_t)e->q_width * es, 256 * es, hd, cudaMemcpyDeviceToDevice, s);
        }
        if (ce != cudaSuccess) break;
        dim3 tb(32, 8), tg((c.ffn + 31) / 32, (c.hidden + 31) / 32);
        if (q8)
            transpose_kernel<int8_t><<<tg, tb, 0, s>>>(reinterpret_cast<const int8_t*>(wd),
                                                       reinterpret_cast<int8_t*>(ndt), c.hidden, c.ffn);
        else
            transpose_kernel<float><<<tg, tb, 0, s>>>(reinterpret_cast<const float*>(wd),
                                                      reinterpret_cast<float*>(ndt), c.hidden, c.ffn);
        ce = cudaGetLastError();
        M.wqkv = nqkv;
        M.sqkv = nsq;
        M.wo = no;
        M.so = Ld.so;
        M.wgu = q8 ? (const void*)Ld.qgu : (const void*)Ld.wgu;
        M.sgu = Ld.sgu;
        M.wdt = ndt;
        M.sd = Ld.sd;
        M.in_norm = Ld.in_norm;
        M.post_norm = Ld.post_norm;
        M.q_norm = Ld.q_norm;
        M.k_norm = Ld.k_norm;
    }
    const int G = c.kv_heads * kCS;
    m->grid = G;
    if (ce == cudaSuccess) {
        m->d_layers = static_cast<M2Layer*>(alloc(sizeof(M2Layer) * c.layers));
        if (!m->d_layers) ce = cudaErrorMemoryAllocation;
    }
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(m->d_layers, hl.data(), sizeof(M2Layer) * c.layers, cudaMemcpyHostToDevice, s);
    const size_t po = sizeof(float) * (size_t)c.kv_heads * hd;
    const size_t pd = sizeof(float) * (size_t)c.kv_heads * hd;
    const size_t am = sizeof(float) * (size_t)G * 2;
    const size_t cnt = 256 * sizeof(int);
    if (ce == cudaSuccess) {
        m->ws = static_cast<char*>(alloc(po + pd + am + cnt));
        if (!m->ws) ce = cudaErrorMemoryAllocation;
    }
    if (ce == cudaSuccess) {
        m->counters = m->ws + po + pd + am;
        m->counters_bytes = cnt;
        ce = cudaMemsetAsync(m->ws, 0, po + pd + am + cnt, s);
    }
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) {
        for (void* ptr : m->bufs) cudaFree(ptr);
        delete m;
        return cuda_fail(ce, "two-barrier step set-up");
    }
    M2Params& P = m->params;
    P.layers = m->d_layers;
    P.embed = e->embed;
    P.final_norm = e->final_norm;
    P.rope_cos = e->rope_cos;
    P.rope_sin = e->rope_sin;
    P.kc = e->kc;
    P.vc = e->vc;
    P.logits = e->logits;
    P.part_o = reinterpret_cast<float*>(m->ws);
    P.part_d = reinterpret_cast<float*>(m->ws + po);
    P.am_val = reinterpret_cast<float*>(m->ws + po + pd);
    P.am_idx = reinterpret_cast<int*>(m->ws + po + pd + am / 2);
    int* cn = reinterpret_cast<int*>(m->counters);
    P.bar = reinterpret_cast<unsigned*>(cn);
    P.am_ticket = cn + 32;
    P.dbg = cn + 128;
    P.tok = e->d_tok;
    P.pos = e->d_pos;
    P.next = e->d_next;
    P.hist = e->d_hist;
    P.step = e->d_step;
    P.err = e->d_err;
    P.hidden = c.hidden;
    P.nlayers = c.layers;
    P.kvh = c.kv_heads;
    P.ffn = c.ffn;
    P.vocab = c.vocab;
    P.max_seq = e->max_seq;
    P.nclusters = c.kv_heads;
    P.eps = c.eps;
    P.trace = nullptr;
    if (e->trace_on) {
        const size_t tb = (size_t)G * kTraceStride2 * sizeof(unsigned long long);
        if (cudaMalloc(&m->trace, tb) == cudaSuccess) {
            m->bufs.push_back(m->trace);
            cudaMemsetAsync(m->trace, 0, tb, s);
            cudaStreamSynchronize(s);
            P.trace = m->trace;
        }
    }
    e->mega2 = m;
    return VB_OK;
}

vb_status mega2_enqueue_step(vb_engine* e, cudaStream_t s) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (!m) return fail(VB_ERR_STATE, "two-barrier step not prepared");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kCS;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t ce = e->quantized ? cudaLaunchKernelEx(&cfg, mega2_kernel<true>, m->params)
                                  : cudaLaunchKernelEx(&cfg, mega2_kernel<false>, m->params);
    if (ce != cudaSuccess) return cuda_fail(ce, "two-barrier step launch");
    return VB_OK;
}

void mega2_release(vb_engine* e) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (m) {
        cudaStreamSynchronize(e->stream);
        for (void* ptr : m->bufs) cudaFree(ptr);
        delete m;
    }
    e->mega2 = nullptr;
}

int mega2_read_trace(vb_engine* e, unsigned long long* host, int cap) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (!m || !m->trace) return 0;
    const int total = m->grid * kTraceStride2;
    const int n = cap < total ? cap : total;
    cudaStreamSynchronize(e->stream);
    if (cudaMemcpy(host, m->trace, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return n;
}

void mega2_reset_counters(vb_engine* e) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (m) {
        cudaMemsetAsync(m->counters, 0, m->counters_bytes, e->stream);
        cudaStreamSynchronize(e->stream);
    }
}

}  // namespace vb
