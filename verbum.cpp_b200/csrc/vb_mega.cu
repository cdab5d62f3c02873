// vb_mega.cu -- the whole batch-1 decode step in one persistent kernel.
//
// One cooperative launch per token, one CTA per SM.  Each CTA owns a fixed
// contiguous slice of the rows of every projection (and a fixed set of
// attention units), so the bytes it must stream for the whole token are known
// at launch.  A producer warp streams them -- weights and K/V tiles -- through
// a 12-stage x 16 KB shared-memory ring with cp.async.bulk (TMA, L2
// evict-first) completing on mbarriers, and never waits for the activations:
// it runs ahead across phase boundaries as far as the ring allows.  Eight
// consumer warps do the math phase by phase; between phases the CTAs meet at a
// grid barrier (an L2 counter with bounded spinning), so HBM keeps streaming
// the next phase's weights while the barrier resolves.
//
// Phases per layer (model.cpp:235-254 with attention_step, generate.cpp:24-108):
//   QKV  rmsnorm(x) . Wqkv^T                    -> qkv        (fused norm prologue)
//   ATT  per (kv head, 32-position chunk) unit: q/k RMSNorm + RoPE, KV append,
//        scores, chunk softmax, P.V; the last unit of each kv head merges the
//        chunks (atomic ticket)                  -> ctx
//   O    x + ctx . Wo^T                         -> x          (fused residual)
//   GU   silu(g) * u, [g;u] = rmsnorm(x).Wgu^T   -> h          (fused SwiGLU)
//   D    x + h . Wd^T                           -> x          (fused residual)
// then LM: rmsnorm(x) . E^T -> logits with per-CTA argmax; the last CTA picks
// the token (strict '>' ties: lowest index), advances pos/token for the next
// launch and resets the barrier counter.
//
// Every wait (mbarrier, grid barrier) gives up after 2 s of %globaltimer,
// records an error word and lets the kernel exit; the producer then waits
// (bounded) for its copies in flight before returning.
#include <limits.h>
#include <math.h>

#include <string>
#include <vector>

#include "vb_engine.cuh"
#include "vb_pipe.cuh"

namespace vb {
namespace {

constexpr int kStageBytes = 16384;
constexpr int kStages = 12;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;  // 256
constexpr int kThreads = kConsumers + 32;        // + 1 producer warp
constexpr int kChunk = 32;                       // attention positions per unit
constexpr int kXsFloats = 4096;                  // activation vector capacity
constexpr int kTraceStride = 1024;  // trace words per CTA
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kXsFloats * sizeof(float);

enum Phase : int { kQKV = 0, kATT = 1, kO = 2, kGU = 3, kD = 4, kLM = 5 };

struct MegaLayer {
    const void* wqkv;
    const void* wo;
    const void* wgu;
    const void* wd;
    const float* sqkv;
    const float* so;
    const float* sgu;
    const float* sd;
    const float* in_norm;
    const float* post_norm;
    const float* q_norm;
    const float* k_norm;
};

struct MegaParams {
    const MegaLayer* layers;
    const float* embed;
    const float* final_norm;
    const float* rope_cos;
    const float* rope_sin;
    float* kc;  // [L][KVH][max_seq][128]
    float* vc;
    float* x;
    float* qkv;
    float* ctx;
    float* h;
    float* logits;
    float* att_part;  // [H][max_chunks][130]
    int* att_ticket;  // [KVH]
    float* am_val;    // [grid]
    int* am_idx;      // [grid]
    int* am_ticket;
    unsigned* bar;
    int* tok;
    int* pos;
    int* next;
    int* hist;
    int* step;
    int* err;
    int* dbg;  // where a bounded wait gave up: {code, cta, site, index, extra}
    unsigned long long* trace;  // optional: per CTA, start + (arrive, leave) of every grid barrier
    int hidden, nlayers, heads, kvh, ffn, vocab, qkv_rows, q_width, max_seq, max_chunks;
    float eps;
};

// Trace words of phase b (1-based, the phase closed by grid barrier b) for
// this CTA, 6 per phase: 0 activation loaded, 1 first stage observed,
// 2 arrival, 3 release (consumer thread 0), 4 first and 5 last stage issued
// (producer).
constexpr int kTraceWords = 6;
__device__ __forceinline__ void trace_at(const MegaParams& p, int b, int w) {
    if (p.trace && kTraceWords * b < kTraceStride)
        p.trace[(size_t)blockIdx.x * kTraceStride + kTraceWords * (b - 1) + 1 + w] = now_ns();
}
__device__ __forceinline__ void trace_mark(const MegaParams& p, int b, int w) {
    if (threadIdx.x == 0) trace_at(p, b, w);
}
__device__ __forceinline__ void trace_first(const MegaParams& p, int b) {
    if (p.trace && kTraceWords * b < kTraceStride) {
        unsigned long long* q =
            p.trace + (size_t)blockIdx.x * kTraceStride + kTraceWords * (b - 1) + 2;
        if (*q == 0) *q = now_ns();
    }
}

// ------------------------------------------------------------- the schedule
// Rows of a GEMV phase owned by CTA c of G: contiguous, balanced, in units of
// `unit` rows (2 for the interleaved gate/up pairs).
struct GemvPlan {
    const char* w;       // row 0 of this CTA's slice
    int row_bytes;
    int rps;             // rows per ring stage
    int r0, r1;          // absolute rows
    int K;
    bool q8;
    int nstages;
};

__device__ __forceinline__ GemvPlan plan_gemv(const MegaParams& p, int layer, int kind, bool q8,
                                              int cta, int G) {
    GemvPlan g;
    int rows, unit = 1;
    const void* W;
    bool wq8 = q8;
    switch (kind) {
        case kQKV: W = p.layers[layer].wqkv; g.K = p.hidden; rows = p.qkv_rows; break;
        case kO: W = p.layers[layer].wo; g.K = p.q_width; rows = p.hidden; break;
        case kGU: W = p.layers[layer].wgu; g.K = p.hidden; rows = 2 * p.ffn; unit = 2; break;
        case kD: W = p.layers[layer].wd; g.K = p.ffn; rows = p.hidden; break;
        default: W = p.embed; g.K = p.hidden; rows = p.vocab; wq8 = false; break;
    }
    g.q8 = wq8;
    g.row_bytes = g.K * (wq8 ? 1 : 4);
    g.rps = kStageBytes / g.row_bytes;
    if (unit == 2) g.rps &= ~1;
    const int units = rows / unit;
    g.r0 = (int)((long long)cta * units / G) * unit;
    g.r1 = (int)((long long)(cta + 1) * units / G) * unit;
    g.w = static_cast<const char*>(W) + (size_t)g.r0 * g.row_bytes;
    g.nstages = (g.r1 - g.r0 + g.rps - 1) / g.rps;
    return g;
}

// Attention units of CTA c: u = c, c+G, ... < KVH * nchunks; kv head u % KVH,
// chunk u / KVH.
__device__ __forceinline__ int att_units(int total, int cta, int G) {
    return total > cta ? (total - cta - 1) / G + 1 : 0;
}

// ------------------------------------------------------------- consumer side
struct __align__(16) Smem {
    float q[2][128];
    float kn[128];
    float vn[128];
    float tq[2][128];
    float tk[128];
    float sc[2][kChunk];
    float e[2][kChunk];
    float m[2], l[2];
    double red[16];
    float bv[kConsumerWarps];
    int bi[kConsumerWarps];
    int gflag;  // grid-barrier outcome
    int tflag;  // attention merge ticket outcome
    int wflag;  // attention stage wait outcome
    unsigned long long full[kStages];
    unsigned long long empty[kStages];
    // seq[slot] = global index of the last stage whose data a consumer has
    // observed in that slot.  Consumers take stages out of order (warp w takes
    // w, w+8, ...), and a parity wait cannot tell round r from round r-2; a
    // consumer therefore waits for stage s only once seq[slot] == s - kStages,
    // i.e. once the slot's previous round is known to have completed.
    volatile int seq[kStages];
    int cur_b;  // index of the grid barrier that closes the current phase (tracing)
};

// Loads an activation vector (written by other CTAs this launch: read via L2)
// into shared memory, optionally RMS-normalised (nn.cpp:8-42 arithmetic),
// laid out lane-interleaved per 512 elements for INT8 phases.
constexpr int kMaxPer = kXsFloats / kConsumers;  // 16 vector elements per consumer thread

// Loads the norm weight elements this thread will need into registers; issued
// before a grid barrier so the (HBM) latency hides under the wait.
__device__ __forceinline__ void prefetch_norm(const float* w, int K, float (&nw)[kMaxPer]) {
    const int t = threadIdx.x;
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
        const int i = t + k * kConsumers;
        nw[k] = (w && i < K) ? __ldg(w + i) : 0.f;
    }
}

__device__ void load_act(const float* src, const float* norm_w, const float (&nw)[kMaxPer],
                         float eps, int K, bool perm, float* xs, Smem& S, bool l2) {
    // one read of the vector into registers (K <= kXsFloats = 16 per thread)
    const int t = threadIdx.x;
    float v[kMaxPer];
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
        const int i = t + k * kConsumers;
        v[k] = 0.f;
        if (i < K) {
            v[k] = l2 ? __ldcg(src + i) : src[i];
            ss += (double)v[k] * (double)v[k];
        }
    }
    float sc = 1.0f;
    if (norm_w) {
        ss = warp_sum_d(ss);
        if ((t & 31) == 0) S.red[t >> 5] = ss;
        consumers_sync<kConsumers>();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) tot += S.red[w];
        sc = rms_scale(tot, K, eps);
    }
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
        const int i = t + k * kConsumers;
        if (i < K) {
            float x = v[k];
            if (norm_w) x = __fmul_rn(__fmul_rn(x, sc), nw[k]);
            int dst = i;
            if (perm) {
                const int c = i >> 9, r = i & 511;
                dst = (c << 9) + (((r >> 2) & 3) << 7) + ((r >> 4) << 2) + (r & 3);
            }
            xs[dst] = x;
        }
    }
    consumers_sync<kConsumers>();
}

__device__ __forceinline__ float dot_row_f32(const float* wrow, const float* xs, int K, int lane) {
    const float4* w4 = reinterpret_cast<const float4*>(wrow);
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    float a0 = 0.f, a1 = 0.f;
    const int K4 = K >> 2;
    int k = lane;
    for (; k + 32 < K4; k += 64) {
        const float4 w = w4[k], x = x4[k];
        const float4 w2 = w4[k + 32], x2 = x4[k + 32];
        a0 = fmaf(w.x, x.x, a0); a0 = fmaf(w.y, x.y, a0); a0 = fmaf(w.z, x.z, a0); a0 = fmaf(w.w, x.w, a0);
        a1 = fmaf(w2.x, x2.x, a1); a1 = fmaf(w2.y, x2.y, a1); a1 = fmaf(w2.z, x2.z, a1); a1 = fmaf(w2.w, x2.w, a1);
    }
    if (k < K4) {
        const float4 w = w4[k], x = x4[k];
        a0 = fmaf(w.x, x.x, a0); a0 = fmaf(w.y, x.y, a0); a0 = fmaf(w.z, x.z, a0); a0 = fmaf(w.w, x.w, a0);
    }
    return warp_sum(a0 + a1);
}

__device__ __forceinline__ float dot_row_i8(const int8_t* wrow, const float* xs, int K, int lane) {
    float a0 = 0.f, a1 = 0.f;
    const int G16 = K >> 4;
    for (int gi = lane; gi < G16; gi += 32) {
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

// Consumer side of one GEMV phase.  Warp w takes stages w, w+8, ... of the
// phase; rows inside a stage are reduced with warp shuffles.
template <int KIND>
__device__ bool gemv_phase(const MegaParams& p, const GemvPlan& g, int layer, int gbase,
                           const char* ring, Smem& S, const float* xs, const float* emb_row,
                           float& best_v, int& best_i) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* scales = nullptr;
    if (g.q8) {
        const MegaLayer& L = p.layers[layer];
        scales = KIND == kQKV ? L.sqkv : KIND == kO ? L.so : KIND == kGU ? L.sgu : L.sd;
    }
    for (int j = warp; j < g.nstages; j += kConsumerWarps) {
        const int gs = gbase + j;
        const int slot = gs % kStages;
        if (!warp_wait(smem_addr(&S.full[slot]), (unsigned)(gs / kStages) & 1u, p.err, p.dbg, gs,
                       S.seq, slot, kStages))
            return false;
        if (lane == 0) trace_first(p, S.cur_b);
        const char* st = ring + (size_t)slot * kStageBytes;
        const int rA = g.r0 + j * g.rps;
        const int nr = min(g.rps, g.r1 - rA);
        float gate = 0.f;
        for (int r = 0; r < nr; r++) {
            const char* wrow = st + (size_t)r * g.row_bytes;
            float acc = g.q8 ? dot_row_i8(reinterpret_cast<const int8_t*>(wrow), xs, g.K, lane)
                             : dot_row_f32(reinterpret_cast<const float*>(wrow), xs, g.K, lane);
            const int row = rA + r;
            if (g.q8) acc *= __ldg(scales + row);
            if (KIND == kQKV) {
                if (lane == 0) p.qkv[row] = acc;
            } else if (KIND == kO || KIND == kD) {
                if (lane == 0) {
                    const float base = (KIND == kO && layer == 0) ? emb_row[row] : __ldcg(p.x + row);
                    p.x[row] = base + acc;
                }
            } else if (KIND == kGU) {
                if ((r & 1) == 0) {
                    gate = acc;
                } else if (lane == 0) {
                    p.h[row >> 1] = silu_f(gate) * acc;
                }
            } else {  // kLM
                if (lane == 0) p.logits[row] = acc;
                if (better(acc, row, best_v, best_i)) {
                    best_v = acc;
                    best_i = row;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&S.empty[slot]), kConsumerWarps);
    }
    return true;
}

// Cooperative variant for INT8 weights: every warp takes every stage (in
// order, so no slot-order gate is needed) and the stage's rows are dealt out
// across the warps -- an INT8 stage holds 5-16 rows, too much dequantisation
// work for one warp.  Each warp releases the slot with one arrival.
template <int KIND>
__device__ bool gemv_phase_coop(const MegaParams& p, const GemvPlan& g, int layer, int gbase,
                                const char* ring, Smem& S, const float* xs, const float* emb_row) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const MegaLayer& L = p.layers[layer];
    const float* scales = KIND == kQKV ? L.sqkv : KIND == kO ? L.so : KIND == kGU ? L.sgu : L.sd;
    for (int j = 0; j < g.nstages; j++) {
        const int gs = gbase + j;
        const int slot = gs % kStages;
        const unsigned par = (unsigned)(gs / kStages) & 1u;
        int ok = 1;
        if (lane == 0) {
            ok = mbar_wait(smem_addr(&S.full[slot]), par, p.err, p.dbg, kSiteFull, gs) ? 1 : 0;
            if (ok) {
                S.seq[slot] = gs;
                trace_first(p, S.cur_b);
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        if (lane != 0)
            for (int i = 0; i < 1024 && !mbar_try(smem_addr(&S.full[slot]), par); i++) {
            }
        const char* st = ring + (size_t)slot * kStageBytes;
        const int rA = g.r0 + j * g.rps;
        const int nr = min(g.rps, g.r1 - rA);
        if (KIND == kGU) {
            for (int pr = warp; 2 * pr + 1 < nr; pr += kConsumerWarps) {
                const int8_t* w0 = reinterpret_cast<const int8_t*>(st + (size_t)(2 * pr) * g.row_bytes);
                const float gsum = dot_row_i8(w0, xs, g.K, lane) * __ldg(scales + rA + 2 * pr);
                const float usum = dot_row_i8(w0 + g.row_bytes, xs, g.K, lane) *
                                   __ldg(scales + rA + 2 * pr + 1);
                if (lane == 0) p.h[(rA >> 1) + pr] = silu_f(gsum) * usum;
            }
        } else {
            for (int r = warp; r < nr; r += kConsumerWarps) {
                const int row = rA + r;
                const float acc = dot_row_i8(reinterpret_cast<const int8_t*>(st + (size_t)r * g.row_bytes),
                                             xs, g.K, lane) * __ldg(scales + row);
                if (lane == 0) {
                    if (KIND == kQKV) {
                        p.qkv[row] = acc;
                    } else {
                        const float base = (KIND == kO && layer == 0) ? emb_row[row] : __ldcg(p.x + row);
                        p.x[row] = base + acc;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&S.empty[slot]), 1);
    }
    return true;
}

template <int KIND>
__device__ __forceinline__ bool run_gemv(const MegaParams& p, const GemvPlan& g, int layer,
                                         int gbase, const char* ring, Smem& S, const float* xs,
                                         const float* emb_row, float& bv, int& bi) {
    if (KIND != kLM && g.q8) return gemv_phase_coop<KIND>(p, g, layer, gbase, ring, S, xs, emb_row);
    return gemv_phase<KIND>(p, g, layer, gbase, ring, S, xs, emb_row, bv, bi);
}

// One attention unit (kv head kvh, chunk c) by all consumer warps; K tile in
// ring stage `ks`, V tile in `vs`.
__device__ bool att_unit(const MegaParams& p, int layer, int kvh, int c, int pos, int nchunks,
                         int ks, int vs, const char* ring, Smem& S) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int hs = t >> 7, d = t & 127;
    const int QW = p.q_width, KW = p.kvh * 128;
    const MegaLayer& L = p.layers[layer];
    // q (2 heads) and new k / v of this kv head: RMSNorm + RoPE (generate.cpp:52-64)
    const float qv = __ldcg(p.qkv + (2 * kvh + hs) * 128 + d);
    const float kv = (t < 128) ? __ldcg(p.qkv + QW + kvh * 128 + d) : 0.f;
    double sq = warp_sum_d((double)qv * qv), sk = warp_sum_d((double)kv * kv);
    if (lane == 0) {
        S.red[warp] = sq;
        S.red[8 + warp] = sk;
    }
    consumers_sync<kConsumers>();
    const double tq = S.red[hs * 4] + S.red[hs * 4 + 1] + S.red[hs * 4 + 2] + S.red[hs * 4 + 3];
    const float scq = rms_scale(tq, 128, p.eps);
    S.tq[hs][d] = __fmul_rn(__fmul_rn(qv, scq), L.q_norm[d]);
    if (t < 128) {
        const double tk = S.red[8] + S.red[9] + S.red[10] + S.red[11];
        const float sck = rms_scale(tk, 128, p.eps);
        S.tk[d] = __fmul_rn(__fmul_rn(kv, sck), L.k_norm[d]);
        S.vn[d] = __ldcg(p.qkv + QW + KW + kvh * 128 + d);
    }
    consumers_sync<kConsumers>();
    {
        const float* cr = p.rope_cos + (size_t)pos * 128;
        const float* sr = p.rope_sin + (size_t)pos * 128;
        float o;
        if (d < 64) o = __fsub_rn(__fmul_rn(S.tq[hs][d], cr[d]), __fmul_rn(S.tq[hs][d + 64], sr[d]));
        else o = __fadd_rn(__fmul_rn(S.tq[hs][d], cr[d]), __fmul_rn(S.tq[hs][d - 64], sr[d]));
        S.q[hs][d] = o;
        if (t < 128) {
            float ok;
            if (d < 64) ok = __fsub_rn(__fmul_rn(S.tk[d], cr[d]), __fmul_rn(S.tk[d + 64], sr[d]));
            else ok = __fadd_rn(__fmul_rn(S.tk[d], cr[d]), __fmul_rn(S.tk[d - 64], sr[d]));
            S.kn[d] = ok;
        }
    }
    const int kslot = ks % kStages, vslot = vs % kStages;
    const unsigned kpar = (unsigned)(ks / kStages) & 1u, vpar = (unsigned)(vs / kStages) & 1u;
    if (t == 0) {
        S.wflag = seq_wait(S.seq, kslot, ks, kStages, p.err, p.dbg) &&
                  mbar_wait(smem_addr(&S.full[kslot]), kpar, p.err, p.dbg, kSiteAttFull, ks) &&
                  seq_wait(S.seq, vslot, vs, kStages, p.err, p.dbg) &&
                  mbar_wait(smem_addr(&S.full[vslot]), vpar, p.err, p.dbg, kSiteAttFull, vs);
        if (S.wflag) {
            S.seq[kslot] = ks;
            S.seq[vslot] = vs;
            __threadfence_block();
            trace_first(p, S.cur_b);
        }
    }
    consumers_sync<kConsumers>();
    if (!S.wflag) return false;  // same value in every consumer thread
    for (int i = 0; i < 1024 && !mbar_try(smem_addr(&S.full[kslot]), kpar); i++) {
    }
    for (int i = 0; i < 1024 && !mbar_try(smem_addr(&S.full[vslot]), vpar); i++) {
    }
    const float* Kt = reinterpret_cast<const float*>(ring + (size_t)kslot * kStageBytes);
    const float* Vt = reinterpret_cast<const float*>(ring + (size_t)vslot * kStageBytes);
    const int n = pos + 1;
    const int p0 = c * kChunk;
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    // scores: warp w takes positions 4w..4w+3
    {
        const float4 q0 = *reinterpret_cast<const float4*>(&S.q[0][4 * lane]);
        const float4 q1 = *reinterpret_cast<const float4*>(&S.q[1][4 * lane]);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int pl = 4 * warp + u, pa = p0 + pl;
            float4 k4 = (pa == pos) ? *reinterpret_cast<const float4*>(&S.kn[4 * lane])
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
    consumers_sync<kConsumers>();
    if (warp < 2) {
        const float s = S.sc[warp][lane];
        const float m = warp_max(s);
        const float e = (s == -INFINITY) ? 0.0f : expf(s - m);
        const float l = warp_sum(e);
        S.e[warp][lane] = e;
        if (lane == 0) {
            S.m[warp] = m;
            S.l[warp] = l;
        }
    }
    consumers_sync<kConsumers>();
    {
        float acc = 0.f;
        const int nv = min(kChunk, n - p0);
        for (int pl = 0; pl < nv; pl++) {
            const float v = (p0 + pl == pos) ? S.vn[d] : Vt[pl * 128 + d];
            acc = fmaf(S.e[hs][pl], v, acc);
        }
        float* part = p.att_part + ((size_t)(2 * kvh + hs) * p.max_chunks + c) * 130;
        part[2 + d] = acc;
        if (d == 0) {
            part[0] = S.m[hs];
            part[1] = S.l[hs];
        }
    }
    if (pos >= p0 && pos < p0 + kChunk && t < 128) {
        const size_t off = ((size_t)(layer * p.kvh + kvh) * p.max_seq + pos) * 128 + t;
        p.kc[off] = S.kn[t];
        p.vc[off] = S.vn[t];
    }
    consumers_sync<kConsumers>();
    if (t == 0) {
        mbar_arrive(smem_addr(&S.empty[kslot]), kConsumerWarps);
        mbar_arrive(smem_addr(&S.empty[vslot]), kConsumerWarps);
        __threadfence();
        const int old = atomicAdd(p.att_ticket + kvh, 1);
        S.tflag = (old == nchunks - 1);
        __threadfence();
    }
    consumers_sync<kConsumers>();
    if (S.tflag) {  // last unit of this kv head: merge the chunks
        const float* base = p.att_part + (size_t)(2 * kvh + hs) * p.max_chunks * 130;
        float M = -INFINITY;
        for (int cc = 0; cc < nchunks; cc++) M = fmaxf(M, __ldcg(base + cc * 130));
        float Lsum = 0.f, A = 0.f;
        for (int cc = 0; cc < nchunks; cc++) {
            const float mc = __ldcg(base + cc * 130);
            if (mc == -INFINITY) continue;
            const float f = expf(mc - M);
            Lsum = fmaf(__ldcg(base + cc * 130 + 1), f, Lsum);
            A = fmaf(__ldcg(base + cc * 130 + 2 + d), f, A);
        }
        p.ctx[(2 * kvh + hs) * 128 + d] = (Lsum > 0.f) ? A / Lsum : 0.f;
        consumers_sync<kConsumers>();
        if (t == 0) p.att_ticket[kvh] = 0;
    }
    consumers_sync<kConsumers>();  // the shared scratch is reused by the next unit
    return true;
}

// Grid-wide barrier across the consumer groups of all CTAs.  Called by all
// consumer threads; thread 0 arrives and spins (bounded) on the counter.
__device__ bool grid_barrier(const MegaParams& p, unsigned target, Smem& S, bool ok_in) {
    if (!consumers_sync_and<kConsumers>(ok_in)) {
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kErrPipeTimeout);
        return false;
    }
    if (threadIdx.x == 0) {
        const int bi = (int)(target / gridDim.x);
        trace_mark(p, bi, 2);
        // one-way release arrival; the CTA barrier above orders every consumer
        // thread's writes before it (release is cumulative)
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
        trace_mark(p, bi, 3);
    }
    consumers_sync<kConsumers>();
    return S.gflag != 0;
}

template <bool Q8>
__global__ void __launch_bounds__(kThreads, 1) mega_step_kernel(const __grid_constant__ MegaParams p) {
    extern __shared__ __align__(1024) char dsmem[];
    __shared__ Smem S;
    char* ring = dsmem;
    float* xs = reinterpret_cast<float*>(dsmem + (size_t)kStages * kStageBytes);
    const int cta = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (p.trace)  // this CTA's trace words restart at zero every step
        for (int i = threadIdx.x; i < kTraceStride; i += kThreads)
            p.trace[(size_t)blockIdx.x * kTraceStride + i] = 0ull;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_addr(&S.full[s]), 1);
            mbar_init(smem_addr(&S.empty[s]), kConsumerWarps);  // one arrival per consumer warp
            S.seq[s] = s - kStages;  // "stage s - kStages" = before the first round
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int pos = *p.pos;
    const int n = pos + 1;
    const int nchunks = (n + kChunk - 1) / kChunk;
    const int att_total = p.kvh * nchunks;
    const int my_units = att_units(att_total, cta, G);

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
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
        int pb = 1;  // phase being issued (= index of the barrier that closes it)
        auto issue_gemv = [&](const GemvPlan& pl) {
            for (int j = 0; j < pl.nstages && ok; j++) {
                const int rows = min(pl.rps, pl.r1 - pl.r0 - j * pl.rps);
                issue(pl.w + (size_t)j * pl.rps * pl.row_bytes, (unsigned)(rows * pl.row_bytes));
                if (j == 0) trace_at(p, pb, 4);
            }
            trace_at(p, pb, 5);
            pb++;
        };
        for (int l = 0; l < p.nlayers && ok; l++) {
            issue_gemv(plan_gemv(p, l, kQKV, Q8, cta, G));
            for (int i = 0; i < my_units && ok; i++) {
                const int u = cta + i * G, kvh = u % p.kvh, c = u / p.kvh;
                const int rows = min(kChunk, p.max_seq - c * kChunk);
                const size_t off = ((size_t)(l * p.kvh + kvh) * p.max_seq + (size_t)c * kChunk) * 128;
                issue(p.kc + off, (unsigned)(rows * 512));
                if (i == 0) trace_at(p, pb, 4);
                if (ok) issue(p.vc + off, (unsigned)(rows * 512));
            }
            trace_at(p, pb, 5);
            pb++;
            if (ok) issue_gemv(plan_gemv(p, l, kO, Q8, cta, G));
            if (ok) issue_gemv(plan_gemv(p, l, kGU, Q8, cta, G));
            if (ok) issue_gemv(plan_gemv(p, l, kD, Q8, cta, G));
        }
        if (ok) issue_gemv(plan_gemv(p, 0, kLM, Q8, cta, G));
        // Drain on every path: a ring slot is refilled only after its previous
        // stage was released, so only the last kStages copies can still be in
        // flight; the CTA must not exit (on an early consumer exit included)
        // while any of them is writing its shared memory.
        const int first = g > kStages ? g - kStages : 0;
        for (int gs = first; gs < g; gs++) {
            const unsigned a = smem_addr(&S.full[gs % kStages]);
            const unsigned par = (unsigned)(gs / kStages) & 1u;
            const unsigned long long t0 = now_ns();
            while (!mbar_try(a, par) && now_ns() - t0 < kWaitNs) {
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    if (p.trace && threadIdx.x == 0) p.trace[(size_t)cta * kTraceStride] = now_ns();
    if (threadIdx.x == 0) S.cur_b = 1;
    const int tok = *p.tok;
    const float* emb_row = p.embed + (size_t)tok * p.hidden;
    int g = 0;
    unsigned nbar = 0;
    float best_v = -INFINITY;
    int best_i = INT_MAX;
    bool ok = true;
    float nw[kMaxPer];
    prefetch_norm(p.layers[0].in_norm, p.hidden, nw);
    for (int l = 0; l < p.nlayers && ok; l++) {
        const MegaLayer& L = p.layers[l];
        {   // QKV
            const GemvPlan pl = plan_gemv(p, l, kQKV, Q8, cta, G);
            if (threadIdx.x == 0) S.cur_b = nbar + 1;
            load_act(l == 0 ? emb_row : p.x, L.in_norm, nw, p.eps, p.hidden, Q8, xs, S, l != 0);
            trace_mark(p, nbar + 1, 0);
            const bool r = run_gemv<kQKV>(p, pl, l, g, ring, S, xs, emb_row, best_v, best_i);
            g += pl.nstages;
            ok = grid_barrier(p, (++nbar) * G, S, r);
            if (!ok) break;
        }
        {   // ATT
            bool r = true;
            if (threadIdx.x == 0) S.cur_b = nbar + 1;
            consumers_sync<kConsumers>();
            trace_mark(p, nbar + 1, 0);
            for (int i = 0; i < my_units && r; i++) {
                const int u = cta + i * G;
                r = att_unit(p, l, u % p.kvh, u / p.kvh, pos, nchunks, g + 2 * i, g + 2 * i + 1,
                             ring, S);
            }
            g += 2 * my_units;
            ok = grid_barrier(p, (++nbar) * G, S, r);
            if (!ok) break;
        }
        {   // O + residual
            const GemvPlan pl = plan_gemv(p, l, kO, Q8, cta, G);
            if (threadIdx.x == 0) S.cur_b = nbar + 1;
            load_act(p.ctx, nullptr, nw, p.eps, p.q_width, Q8, xs, S, true);
            trace_mark(p, nbar + 1, 0);
            const bool r = run_gemv<kO>(p, pl, l, g, ring, S, xs, emb_row, best_v, best_i);
            g += pl.nstages;
            prefetch_norm(L.post_norm, p.hidden, nw);
            ok = grid_barrier(p, (++nbar) * G, S, r);
            if (!ok) break;
        }
        {   // gate/up + SwiGLU
            const GemvPlan pl = plan_gemv(p, l, kGU, Q8, cta, G);
            if (threadIdx.x == 0) S.cur_b = nbar + 1;
            load_act(p.x, L.post_norm, nw, p.eps, p.hidden, Q8, xs, S, true);
            trace_mark(p, nbar + 1, 0);
            const bool r = run_gemv<kGU>(p, pl, l, g, ring, S, xs, emb_row, best_v, best_i);
            g += pl.nstages;
            ok = grid_barrier(p, (++nbar) * G, S, r);
            if (!ok) break;
        }
        {   // down + residual
            const GemvPlan pl = plan_gemv(p, l, kD, Q8, cta, G);
            if (threadIdx.x == 0) S.cur_b = nbar + 1;
            load_act(p.h, nullptr, nw, p.eps, p.ffn, Q8, xs, S, true);
            trace_mark(p, nbar + 1, 0);
            const bool r = run_gemv<kD>(p, pl, l, g, ring, S, xs, emb_row, best_v, best_i);
            g += pl.nstages;
            prefetch_norm(l + 1 < p.nlayers ? p.layers[l + 1].in_norm : p.final_norm, p.hidden, nw);
            ok = grid_barrier(p, (++nbar) * G, S, r);
            if (!ok) break;
        }
    }
    if (!ok) return;  // uniform: every consumer thread saw the same barrier outcome
    {   // final norm + lm_head + argmax
        const GemvPlan pl = plan_gemv(p, 0, kLM, Q8, cta, G);
        load_act(p.x, p.final_norm, nw, p.eps, p.hidden, false, xs, S, true);
        const bool r = gemv_phase<kLM>(p, pl, 0, g, ring, S, xs, emb_row, best_v, best_i);
        if (!consumers_sync_and<kConsumers>(r)) return;
    }
    if (lane == 0) {
        S.bv[warp] = best_v;
        S.bi[warp] = best_i;
    }
    consumers_sync<kConsumers>();
    if (threadIdx.x == 0) {
        float bv = S.bv[0];
        int bi = S.bi[0];
        for (int w = 1; w < kConsumerWarps; w++)
            if (better(S.bv[w], S.bi[w], bv, bi)) { bv = S.bv[w]; bi = S.bi[w]; }
        p.am_val[cta] = bv;
        p.am_idx[cta] = bi;
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

struct MegaState {
    MegaParams params;
    unsigned long long* trace = nullptr;
    MegaLayer* d_layers = nullptr;
    char* ws = nullptr;
    size_t counters_bytes = 0;
    char* counters = nullptr;
    int grid = 0;
};

}  // namespace

vb_status mega_prepare(vb_engine* e) {
    const vb_config& c = e->cfg;
    if (e->lm_int8) return fail(VB_ERR_UNSUPPORTED, "fused step: f32 lm_head only");
    if (c.heads != 2 * c.kv_heads || c.head_dim != 128)
        return fail(VB_ERR_UNSUPPORTED, "fused step: needs GQA group 2 and head_dim 128");
    const int ks[3] = {c.hidden, e->q_width, c.ffn};
    for (int k : ks) {
        if (k > kXsFloats || k % 512 || 4 * k > kStageBytes)
            return fail(VB_ERR_UNSUPPORTED, "fused step: K must be a multiple of 512 and <= 4096");
    }
    if (!e->kc) return fail(VB_ERR_NO_CACHE, "call reset_cache() first");
    int dev = e->device, sms = 0, coop = 0;
    VB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    VB_CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    if (!coop) return fail(VB_ERR_UNSUPPORTED, "fused step: cooperative launch unsupported");
    auto kern = e->quantized ? mega_step_kernel<true> : mega_step_kernel<false>;
    VB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes));
    int per_sm = 0;
    VB_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, kSmemBytes));
    if (per_sm < 1) return fail(VB_ERR_UNSUPPORTED, "fused step: does not fit on an SM");

    MegaState* m = new MegaState();
    MegaParams& P = m->params;
    m->grid = sms;
    std::vector<MegaLayer> hl(c.layers);
    for (int l = 0; l < c.layers; l++) {
        const vb_layer_dev& L = e->L[l];
        MegaLayer& M = hl[l];
        M.wqkv = e->quantized ? (const void*)L.qqkv : (const void*)L.wqkv;
        M.wo = e->quantized ? (const void*)L.qo : (const void*)L.wo;
        M.wgu = e->quantized ? (const void*)L.qgu : (const void*)L.wgu;
        M.wd = e->quantized ? (const void*)L.qd : (const void*)L.wd;
        M.sqkv = L.sqkv; M.so = L.so; M.sgu = L.sgu; M.sd = L.sd;
        M.in_norm = L.in_norm; M.post_norm = L.post_norm; M.q_norm = L.q_norm; M.k_norm = L.k_norm;
    }
    cudaError_t ce = cudaMalloc(&m->d_layers, sizeof(MegaLayer) * c.layers);
    if (ce == cudaSuccess)
        ce = cudaMemcpy(m->d_layers, hl.data(), sizeof(MegaLayer) * c.layers, cudaMemcpyHostToDevice);
    const int max_chunks = (e->max_seq + kChunk - 1) / kChunk;
    const size_t part_bytes = sizeof(float) * (size_t)c.heads * max_chunks * 130;
    const size_t am_bytes = sizeof(float) * (size_t)sms * 2;
    const size_t cnt_bytes = 256 * sizeof(int);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->ws, part_bytes + am_bytes + cnt_bytes);
    if (ce != cudaSuccess) {
        if (m->d_layers) cudaFree(m->d_layers);
        delete m;
        return cuda_fail(ce, "fused step workspace");
    }
    m->counters = m->ws + part_bytes + am_bytes;
    m->counters_bytes = cnt_bytes;
    // on the engine's stream: it does not order with the legacy default stream
    ce = cudaMemsetAsync(m->counters, 0, cnt_bytes, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    if (ce != cudaSuccess) {
        cudaFree(m->d_layers);
        cudaFree(m->ws);
        delete m;
        return cuda_fail(ce, "fused step counters");
    }
    P.layers = m->d_layers;
    P.embed = e->embed;
    P.final_norm = e->final_norm;
    P.rope_cos = e->rope_cos;
    P.rope_sin = e->rope_sin;
    P.kc = e->kc;
    P.vc = e->vc;
    P.x = e->x;
    P.qkv = e->qkv;
    P.ctx = e->ctx;
    P.h = e->h;
    P.logits = e->logits;
    P.att_part = reinterpret_cast<float*>(m->ws);
    P.am_val = reinterpret_cast<float*>(m->ws + part_bytes);
    P.am_idx = reinterpret_cast<int*>(m->ws + part_bytes + am_bytes / 2);
    int* cnt = reinterpret_cast<int*>(m->counters);
    P.bar = reinterpret_cast<unsigned*>(cnt);
    P.am_ticket = cnt + 32;
    P.att_ticket = cnt + 64;
    P.dbg = cnt + 128;
    P.trace = nullptr;
    if (e->trace_on) {
        const size_t tb = (size_t)sms * kTraceStride * sizeof(unsigned long long);
        if (cudaMalloc(&m->trace, tb) == cudaSuccess) {
            cudaMemsetAsync(m->trace, 0, tb, e->stream);
            cudaStreamSynchronize(e->stream);
            P.trace = m->trace;
        }
    }
    P.tok = e->d_tok;
    P.pos = e->d_pos;
    P.next = e->d_next;
    P.hist = e->d_hist;
    P.step = e->d_step;
    P.err = e->d_err;
    P.hidden = c.hidden;
    P.nlayers = c.layers;
    P.heads = c.heads;
    P.kvh = c.kv_heads;
    P.ffn = c.ffn;
    P.vocab = c.vocab;
    P.qkv_rows = e->qkv_rows;
    P.q_width = e->q_width;
    P.max_seq = e->max_seq;
    P.max_chunks = max_chunks;
    P.eps = c.eps;
    e->mega = m;
    return VB_OK;
}

vb_status mega_enqueue_step(vb_engine* e, cudaStream_t s) {
    MegaState* m = static_cast<MegaState*>(e->mega);
    if (!m) return fail(VB_ERR_STATE, "fused step not prepared");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t ce = e->quantized ? cudaLaunchKernelEx(&cfg, mega_step_kernel<true>, m->params)
                                  : cudaLaunchKernelEx(&cfg, mega_step_kernel<false>, m->params);
    if (ce != cudaSuccess) return cuda_fail(ce, "fused step launch");
    return VB_OK;
}

void mega_release(vb_engine* e) {
    MegaState* m = static_cast<MegaState*>(e->mega);
    if (m) {
        cudaStreamSynchronize(e->stream);
        if (m->d_layers) cudaFree(m->d_layers);
        if (m->ws) cudaFree(m->ws);
        if (m->trace) cudaFree(m->trace);
        delete m;
    }
    e->mega = nullptr;
}

int mega_read_trace(vb_engine* e, unsigned long long* host, int cap) {
    MegaState* m = static_cast<MegaState*>(e->mega);
    if (!m || !m->trace) return 0;
    const int total = m->grid * kTraceStride;
    const int n = cap < total ? cap : total;
    cudaStreamSynchronize(e->stream);
    if (cudaMemcpy(host, m->trace, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        return 0;
    return n;
}

std::string mega_debug(vb_engine* e) {
    MegaState* m = static_cast<MegaState*>(e->mega);
    if (!m) return "";
    int d[5] = {0, 0, 0, 0, 0};
    if (cudaMemcpy(d, m->params.dbg, sizeof d, cudaMemcpyDeviceToHost) != cudaSuccess) return "";
    if (!d[0]) return "";
    static const char* sites[] = {"?", "producer empty-slot wait", "consumer stage wait",
                                  "attention stage wait", "grid barrier", "slot order wait"};
    return std::string(" [code ") + std::to_string(d[0]) + ", cta " + std::to_string(d[1]) + ", " +
           sites[(d[2] >= 1 && d[2] <= 5) ? d[2] : 0] + ", index " + std::to_string(d[3]) +
           ", extra " + std::to_string(d[4]) + "]";
}

void mega_reset_counters(vb_engine* e) {
    MegaState* m = static_cast<MegaState*>(e->mega);
    if (m) {
        cudaMemsetAsync(m->counters, 0, m->counters_bytes, e->stream);
        cudaStreamSynchronize(e->stream);
    }
}

}  // namespace vb
