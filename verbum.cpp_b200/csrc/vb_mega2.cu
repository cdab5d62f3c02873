// vb_mega2.cu -- batch-1 decode step as one persistent kernel with no grid
// barrier: every cross-CTA dependency is carried by tagged data words.
//
// Grid = every co-resident thread-block cluster of 8 CTAs (one CTA per SM;
// 15 clusters on a B200 at this shared-memory size).  Cluster k < kv_heads
// owns KV head k; the other clusters sit phase A out.  Per layer:
//
//   phase A  (cluster k, CTA r)
//     x += sum_c down partials of the previous layer (fixed order), RMSNorm
//     rows [64r, 64r+64) of the kv-head-k block of Wqkv (q head 2k, 2k+1, k,
//       v), each value pushed into all 8 CTAs' shared memory
//     q/k RMSNorm + RoPE, KV append (r = 0), attention over this CTA's
//     32-position chunks (chunk c on CTA c % 8) with an online softmax; the
//     partial (acc, max, sum) pushed to all 8 CTAs, merged in rank order
//     split-K o_proj: rows [128r, 128r+128) of Wo[:, 256k:256k+256] . ctx
//       -> o partial of head k (global)
//   phase B  (every CTA b)
//     x += sum_k o partials (fixed order), RMSNorm
//     its slice of gate/up pairs -> h slice (SwiGLU fused)
//     split-K down: sum_{i in slice} h_i * Wd^T[i, :]; outputs [128q, +128)
//       pushed to CTA q of the cluster, which sums the 8 in rank order
//       -> down partial of the cluster (global)
// then LM (all CTAs): x += sum of down partials, final RMSNorm, logits rows +
// argmax (the last CTA to finish picks the token).
//
// Exchange words are 64 bits: the f32 value and a tag naming the launch, the
// layer and the exchange.  Producers store them (into a peer CTA's shared
// memory, or global memory); consumers poll until the tag is the expected one.
// The data is its own flag, so a consumer proceeds one memory round trip
// after the last producer's store, with no barrier, fence or counter between.
// Global partials alternate between two buffers by layer parity, which is
// enough for no producer to overwrite a word some consumer has yet to read.
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
// they gave up.
#include <limits.h>
#include <math.h>
#include <stdlib.h>

#include <algorithm>
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
constexpr int kThreads = kCT + 32;  // + ring producer warp
constexpr int kChunk = 32;
constexpr int kHid = 1024;          // hidden size this kernel is laid out for
constexpr int kXs = kHid;           // normalised-input capacity (floats)
constexpr int kPer = kXs / kCT;     // 4
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kXs * sizeof(float);

struct M2Layer {
    const void* wqkv;  // [KVH][512][hidden]: kv block k rows = q head 2k, 2k+1, k head k, v head k
    const float* sqkv; // [KVH][512]
    const void* wo;    // [KVH][hidden][256]: Wo columns 256k..256k+255
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
    const int8_t* lm_q8;   // opt-in INT8 lm_head rows (else the f32 embedding)
    const float* lm_sc;
    const float* final_norm;
    const float* rope_cos;
    const float* rope_sin;
    float* kc;  // [L][KVH][max_seq][128]
    float* vc;
    float* logits;
    unsigned long long* xo;  // [2][KVH][hidden] tagged o_proj partials (by layer parity)
    unsigned long long* xd;  // [2][nclusters][hidden] tagged down-proj partials
    int* epoch;              // launches so far (tags of this launch use epoch + 1)
    float* am_val;
    int* am_idx;
    int* am_ticket;
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
// consumer thread 0 after: A partials arrived, A norm, A qkv rows, A gather,
// A attention, A merge, A o_proj, B partials arrived, B norm, B gate/up,
// B down + push, B reduce.
constexpr int kTraceStride2 = 2048;
constexpr int kTraceMarks = 12;
// The phase trace and cycle profile are compiled in only with VB_STEP_TRACE=1
// (a profiling build): the product kernel carries none of their code.
#ifndef VB_STEP_TRACE
#define VB_STEP_TRACE 0
#endif
__device__ __forceinline__ long long tclk() {
#if VB_STEP_TRACE
    return clock64();
#else
    return 0;
#endif
}
__device__ __forceinline__ void tmark(const M2Params& p, int l, int i) {
    if (VB_STEP_TRACE && p.trace && threadIdx.x == 0 && 1 + kTraceMarks * (l + 1) < kTraceStride2)
        p.trace[(size_t)blockIdx.x * kTraceStride2 + 1 + kTraceMarks * l + i] = now_ns();
}

// Cycle profile (tracing only, consumer thread 0): per layer kProfWords words
// at kProfBase: [0..7] wait/total clock64 cycles of the qkv, o_proj, gate/up
// and down phases, [8..10] cycles in the gather, merge and reduce exchanges,
// [11] attention stage-wait cycles and [12] chunks of warp 0, [13] attention
// cycles, [14] clock64 and [15] %globaltimer at the layer's start; [16 + 3i]
// first-stage compute, [17 + 3i] dot+reduce, [18 + 3i] epilogue cycles of
// gemv i (qkv, o, gate/up).
constexpr int kProfBase = 400;
constexpr int kProfWords = 40;
__device__ __forceinline__ long long* prof_ptr(const M2Params& p, int l) {
    if (!VB_STEP_TRACE || !p.trace || threadIdx.x != 0 || kProfBase + kProfWords * (l + 1) > kTraceStride2) return nullptr;
    return reinterpret_cast<long long*>(p.trace + (size_t)blockIdx.x * kTraceStride2 + kProfBase + kProfWords * l);
}

// Exchange words: {value bits, tag} in one 64-bit word, written by the
// producing CTA (into a peer's shared memory, or global memory) and polled by
// the consumer until the tag is the expected one -- the data is its own flag,
// so no barrier, fence or counter sits between producer and consumer.
// tag = (epoch + 1) << 8 | layer << 2 | kind.
enum XKind : unsigned { kXQkv = 0, kXAtt = 1, kXRed = 2, kXGlobal = 3 };
constexpr int kAttWords = 264;  // 256 acc + m[2] + l[2] (+ pad)

struct __align__(16) S2 {
    unsigned long long qkv64[512];          // pushed by the 8 CTAs: 64 rows each
    union {
        unsigned long long att64[kCS][kAttWords];  // attention partials of the 8 CTAs
        unsigned long long red64[kCS][128];        // down partials for my 128 outputs
    } xu;
    float xr[kHid];       // residual stream (identical in every CTA)
    float qkv[512];       // gathered q(2 heads) | k | v
    float q[2][128];
    float tq[2][128];
    float kn[128];
    float tk[128];
    float vn[128];
    float att_acc[2][128];  // this CTA's attention partial
    float att_m[2], att_l[2];
    float wacc[kCW][2][128];  // per-warp attention partials
    float wm[kCW][2], wl[kCW][2];
    float h[64];
    float sc_qkv[64];     // INT8 row scales of this CTA's phase-A rows
    float sc_o[128];
    float sc_gu[128];     // ... of its phase-B gate/up rows
    float sc_d[128];      // ... of the down-proj outputs it reduces
    double red[16];
    float bv[kCW];
    int bi[kCW];
    int wflag;
    unsigned long long full[kStages];
    unsigned long long empty[kStages];
    volatile int seq[kStages];
};

// Functions below that take S2& / shared pointers and are not inlined tell
// the compiler the pointers are shared-memory ones, so it keeps
// shared-memory instructions; several are kept out of line on purpose: the
// whole per-layer code path has to stay small enough for the instruction
// caches, since every layer runs all of it once.
#define VB_SHARED(ptr) __builtin_assume(__isShared(ptr))

// One out-of-line copy of the double-precision norm scale (three call sites).
__device__ __noinline__ float rms_scale_ool(double sumsq, int dim, float eps) { return rms_scale(sumsq, dim, eps); }

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

__device__ __forceinline__ unsigned xtag(unsigned ep1, int l, unsigned kind) {
    return (ep1 << 8) | ((unsigned)l << 2) | kind;
}
__device__ __forceinline__ unsigned long long xpack(float v, unsigned tag) {
    return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ unsigned xtag_of(unsigned long long w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float xval(unsigned long long w) { return __uint_as_float((unsigned)w); }

__device__ __forceinline__ void st_peer(unsigned addr, unsigned long long v) {
    asm volatile("st.relaxed.cluster.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ void st_gpu(unsigned long long* ptr, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_gpu(const unsigned long long* ptr) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr));
    return v;
}
__device__ __forceinline__ unsigned long long ld_own(unsigned saddr) {
    unsigned long long v;
    asm volatile("ld.relaxed.cluster.shared::cta.u64 %0, [%1];" : "=l"(v) : "r"(saddr));
    return v;
}

// Slow path of wait_own: bounded spin until the word at shared address
// `saddr` carries `tag`.  Returns the word, or 0 (tag 0 is never live) after
// the time bound (error recorded) or when another CTA has failed.
__device__ __noinline__ unsigned long long spin_own(const M2Params& p, unsigned saddr, unsigned tag, int site) {
    const unsigned long long t0 = now_ns();
    for (unsigned it = 1;; it++) {
        const unsigned long long v = ld_own(saddr);
        if (xtag_of(v) == tag) return v;
        if ((it & 63u) == 0) {
            if (err_read(p.err)) return 0ull;
            if (now_ns() - t0 > kWaitNs) {
                record_fail(p.err, p.dbg, kErrPipeTimeout, site, (int)blockIdx.x, (int)xtag_of(v));
                return 0ull;
            }
        }
    }
}
__device__ __forceinline__ bool wait_own(const M2Params& p, const unsigned long long* w, unsigned tag, int site,
                                         float& out) {
    const unsigned sa = smem_addr(w);
    unsigned long long v = ld_own(sa);
    if (xtag_of(v) != tag) {
        v = spin_own(p, sa, tag, site);
        if (xtag_of(v) != tag) return false;
    }
    out = xval(v);
    return true;
}

// Sum over c < n (in c order) of the tagged partials parts[c][t + k*kCT],
// k = 0..3, polling global memory until every word of a group of 8 partials
// carries `tag` (all loads of a group in flight together).  A failed wait
// leaves the error word set (the caller checks it).
__device__ __noinline__ float4 sum_parts_tagged(const M2Params& p, const unsigned long long* parts, int n,
                                                unsigned tag) {
    const int t = threadIdx.x, H = p.hidden;
    float add[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c0 = 0; c0 < n; c0 += 8) {
        unsigned long long w[4][8];
        unsigned long long t0 = 0;
        for (unsigned it = 0;; it++) {
            bool ready = true;
#pragma unroll
            for (int cc = 0; cc < 8; cc++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int c = c0 + cc;
                    w[k][cc] = c < n ? ld_gpu(parts + (size_t)c * H + t + k * kCT) : xpack(0.f, tag);
                }
#pragma unroll
            for (int cc = 0; cc < 8; cc++)
#pragma unroll
                for (int k = 0; k < 4; k++) ready &= xtag_of(w[k][cc]) == tag;
            if (ready) break;
            if (it == 0) {
                t0 = now_ns();
            } else if ((it & 7u) == 0) {
                if (err_read(p.err)) return make_float4(0.f, 0.f, 0.f, 0.f);
                if (now_ns() - t0 > kWaitNs) {
                    record_fail(p.err, p.dbg, kErrBarrierTimeout, kSiteGrid, (int)tag, c0);
                    return make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int cc = 0; cc < 8; cc++) add[k] += xval(w[k][cc]);
    }
    return make_float4(add[0], add[1], add[2], add[3]);
}

// ------------------------------------------------------------------ plans
struct Plan {
    const char* w;     // first byte of this CTA's rows
    int row_bytes;
    int rps;           // rows per stage
    int r0, r1;        // rows of the CTA's range (relative to the matrix)
    int nstages;
};

__device__ __forceinline__ Plan make_plan(const void* W, int K, bool q8, int r0, int r1, int unit) {
    Plan g;
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
    return p.lm_q8 ? make_plan(p.lm_q8, p.hidden, true, r0, r1, 1) : make_plan(p.embed, p.hidden, false, r0, r1, 1);
}

// --------------------------------------------------------------- consumers
__device__ __forceinline__ int perm_index(int i) {
    const int c = i >> 9, r = i & 511;
    return (c << 9) + (((r >> 2) & 3) << 7) + ((r >> 4) << 2) + (r & 3);
}

// Stage wait shared by all consumer modes.  in_order: every warp takes every
// stage (no slot-order gate needed); otherwise warps take stages out of order
// and wait for the slot's previous round first.
__device__ __forceinline__ bool stage_wait(const M2Params& p, S2& S, int gs, bool in_order) {
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
__device__ __forceinline__ void stage_release(S2& S, int gs, unsigned count) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(smem_addr(&S.empty[gs % kStages]), count);
}

// Epilogue of the row-dot phases, run by the lane that owns the row (or the
// gate/up pair) with the reduced, scaled values.
enum EpiKind : int { kEpiQkvPush = 0, kEpiStoreTagged = 1, kEpiSwiGLU = 2, kEpiLogits = 3 };
struct Epi {
    int kind;
    unsigned base;            // qkv push: shared address of qkv64
    unsigned tag;
    unsigned long long* dst;  // store: tagged o partial row 0
    float* h;                 // swiglu: h slice, first pair p0
    int p0;
    float* logits;
};

// Dot products of NR rows of one stage with xs, all rows in flight at once
// (rows past the stage's valid ones read stale shared memory; their results
// are never used).  f32: every lane takes float4 columns lane, lane+32, ...
template <int NR, int K>
__device__ __forceinline__ void dot_rows_f32(const char* st, int row_bytes, int cnt, const float* xs,
                                             int lane, float (&acc)[NR]) {
    static_assert(K % 128 == 0, "f32 rows: K multiple of 128");
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    f2 a[NR], b[NR];
#pragma unroll
    for (int r = 0; r < NR; r++) a[r] = b[r] = 0ull;
#pragma unroll 2
    for (int it = 0; it < K / 128; it++) {
        const int k = lane + 32 * it;
        const float4 x = x4[k];
        const f2 xlo = f2pack(x.x, x.y), xhi = f2pack(x.z, x.w);
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const float4 w = reinterpret_cast<const float4*>(st + (size_t)r * row_bytes)[k];
            a[r] = f2fma(f2pack(w.x, w.y), xlo, a[r]);
            b[r] = f2fma(f2pack(w.z, w.w), xhi, b[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = f2sum(a[r]) + f2sum(b[r]);
#pragma unroll
    for (int off = 16; off; off >>= 1)
#pragma unroll
        for (int r = 0; r < NR; r++) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
}

// 16 int8 of one row against 16 x values: two pair accumulators.
__device__ __forceinline__ void dot16_i8(uint4 w, float4 x0, float4 x1, float4 x2, float4 x3, f2& a, f2& b) {
    f2 lo, hi;
    i8x4_to_f2(w.x, lo, hi);
    a = f2fma(lo, f2pack(x0.x, x0.y), a);
    b = f2fma(hi, f2pack(x0.z, x0.w), b);
    i8x4_to_f2(w.y, lo, hi);
    a = f2fma(lo, f2pack(x1.x, x1.y), a);
    b = f2fma(hi, f2pack(x1.z, x1.w), b);
    i8x4_to_f2(w.z, lo, hi);
    a = f2fma(lo, f2pack(x2.x, x2.y), a);
    b = f2fma(hi, f2pack(x2.z, x2.w), b);
    i8x4_to_f2(w.w, lo, hi);
    a = f2fma(lo, f2pack(x3.x, x3.y), a);
    b = f2fma(hi, f2pack(x3.z, x3.w), b);
}

// INT8 rows against the lane-interleaved xs.  K % 512 == 0: the whole warp on
// each row; K == 256: two rows at a time, one per half-warp.
template <int NR, int K>
__device__ __forceinline__ void dot_rows_i8(const char* st, int row_bytes, int cnt, const float* xs,
                                            int lane, float (&acc)[NR]) {
    static_assert(K % 512 == 0 || K == 256, "INT8 rows: K multiple of 512, or 256");
    if constexpr (K >= 512) {
        f2 a[NR], b[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) a[r] = b[r] = 0ull;
#pragma unroll 1
        for (int it = 0; it < K / 512; it++) {
            const int gi = lane + 32 * it;
            const float* xc = xs + ((gi >> 5) << 9) + 4 * lane;
            const float4 x0 = *reinterpret_cast<const float4*>(xc);
            const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
            const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
            const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
#pragma unroll
            for (int r = 0; r < NR; r++)
                dot16_i8(*reinterpret_cast<const uint4*>(st + (size_t)r * row_bytes + 16 * gi), x0, x1, x2, x3,
                         a[r], b[r]);
        }
#pragma unroll
        for (int r = 0; r < NR; r++) acc[r] = f2sum(a[r]) + f2sum(b[r]);
#pragma unroll
        for (int off = 16; off; off >>= 1)
#pragma unroll
            for (int r = 0; r < NR; r++) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
    } else {  // K == 256: 16 groups per row
        const int h = lane >> 4, gi = lane & 15;
        const float* xc = xs + 4 * gi;
        const float4 x0 = *reinterpret_cast<const float4*>(xc);
        const float4 x1 = *reinterpret_cast<const float4*>(xc + 128);
        const float4 x2 = *reinterpret_cast<const float4*>(xc + 256);
        const float4 x3 = *reinterpret_cast<const float4*>(xc + 384);
        float ap[(NR + 1) / 2];
#pragma unroll
        for (int q = 0; q < (NR + 1) / 2; q++) {
            const int r = 2 * q + h;
            f2 a = 0ull, b = 0ull;
            dot16_i8(*reinterpret_cast<const uint4*>(st + (size_t)r * row_bytes + 16 * gi), x0, x1, x2, x3, a, b);
            ap[q] = f2sum(a) + f2sum(b);
        }
#pragma unroll
        for (int off = 8; off; off >>= 1)
#pragma unroll
            for (int q = 0; q < (NR + 1) / 2; q++) ap[q] += __shfl_xor_sync(0xffffffffu, ap[q], off);
#pragma unroll
        for (int q = 0; q < (NR + 1) / 2; q++) {
            acc[2 * q] = __shfl_sync(0xffffffffu, ap[q], 0);
            if (2 * q + 1 < NR) acc[2 * q + 1] = __shfl_sync(0xffffffffu, ap[q], 16);
        }
    }
}

// The epilogue for one row (or gate/up pair), run by the lane that owns it.
// Logits also fold the row into this lane's running best.
__device__ __noinline__ void epi_apply(const Epi& epi, int row, float a, float bval, float& best_v, int& best_i) {
    switch (epi.kind) {
    case kEpiQkvPush: {
        const unsigned long long w = xpack(a, epi.tag);
#pragma unroll 1
        for (unsigned q = 0; q < kCS; q++) st_peer(mapa(epi.base + 8u * (unsigned)row, q), w);
        break;
    }
    case kEpiStoreTagged:
        st_gpu(epi.dst + row, xpack(a, epi.tag));
        break;
    case kEpiSwiGLU:
        epi.h[(row >> 1) - epi.p0] = silu_f(a) * bval;
        break;
    default:
        epi.logits[row] = a;
        if (better(a, row, best_v, best_i)) {
            best_v = a;
            best_i = row;
        }
        break;
    }
}

template <int NR>
__device__ __forceinline__ float pick(const float (&v)[NR], int i) {
    float r = 0.f;
#pragma unroll
    for (int k = 0; k < NR; k++)
        if (k == i) r = v[k];
    return r;
}

// Row-dot GEMV phase: the value of row r (absolute) goes to the epilogue,
// scaled by scl[r - g.r0] (shared memory, INT8) when scl is set.
// Work items: each stage is cut into rps / NR parts of NR rows; warp w takes
// items w, w + 8, ... (item i: stage i / parts, part i % parts), so every
// warp has NR independent rows in flight and one interleaved reduction per
// item.  pair: rows come in gate/up pairs.  Logits: the best (value, row) of
// this warp lands in S.bv / S.bi.
template <bool Q8, int NR, int K>
__device__ __noinline__ bool gemv_rows(const M2Params& p, const Plan g, int gbase, const char* ring, S2& S,
                                       const float* xs, const float* scl, bool pair, const Epi epi,
                                       long long* prof, long long* prof2) {
    VB_SHARED(ring);
    VB_SHARED(&S);
    VB_SHARED(xs);
    if (scl) VB_SHARED(scl);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int parts = g.rps / NR;                 // 1, 2, 4 or 8
    const unsigned share = (unsigned)(kCW / parts);  // empty-barrier arrivals per item
    float best_v = -INFINITY;
    int best_i = INT_MAX;
    long long t_wait = 0, t_dot = 0, t_epi = 0, t_first = -1;
    const long long t_start = tclk();
    const int items = g.nstages * parts;
    for (int it = warp; it < items; it += kCW) {
        const int j = it / parts, part = it - j * parts;
        const int gs = gbase + j;
        const long long tw = tclk();
        if (!stage_wait(p, S, gs, false)) return false;
        t_wait += tclk() - tw;
        const char* st = ring + (size_t)(gs % kStages) * kStageBytes;
        const int rA = g.r0 + j * g.rps;
        const int nr = min(g.rps, g.r1 - rA);
        const int lo = part * NR;
        const int cnt = max(0, min(NR, nr - lo));
        float acc[NR];
        const long long td = tclk();
        if constexpr (Q8) dot_rows_i8<NR, K>(st + (size_t)lo * g.row_bytes, g.row_bytes, cnt, xs, lane, acc);
        else dot_rows_f32<NR, K>(st + (size_t)lo * g.row_bytes, g.row_bytes, cnt, xs, lane, acc);
        if (prof2) asm volatile("" : "+f"(acc[0]));
        const long long te = tclk();
        t_dot += te - td;
        stage_release(S, gs, share);
        const int row0 = rA + lo;
        const int mine = pair ? 2 * lane : lane;
        if (mine + (pair ? 1 : 0) < cnt) {
            float a = pick(acc, mine), bval = pair ? pick(acc, mine + 1) : 0.f;
            const int row = row0 + mine;
            if (scl) {
                a *= scl[row - g.r0];
                if (pair) bval *= scl[row + 1 - g.r0];
            }
            epi_apply(epi, row, a, bval, best_v, best_i);
        }
        const long long tf = tclk();
        t_epi += tf - te;
        if (t_first < 0) t_first = tf - td;
    }
    if (epi.kind == kEpiLogits) {
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, off);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
            if (better(ov, oi, best_v, best_i)) {
                best_v = ov;
                best_i = oi;
            }
        }
        if (lane == 0) {
            S.bv[warp] = best_v;
            S.bi[warp] = best_i;
        }
    }
    if (prof) {
        prof[0] += t_wait;
        prof[1] += tclk() - t_start;
    }
    if (prof2) {
        prof2[0] += t_first;
        prof2[1] += t_dot;
        prof2[2] += t_epi;
    }
    return true;
}

// x += sum of `n` tagged partial vectors (fixed order), then RMSNorm with the
// pre-loaded norm values into xs (lane-interleaved layout for INT8).  Trace
// mark `mk` is stamped once the partials have arrived.  Returns false
// (uniformly across the consumer threads) when a wait gave up.
__device__ __noinline__ bool residual_norm(const M2Params& p, S2& S, float* xs, const unsigned long long* parts,
                                           int n, unsigned tag, const float* emb_row, const float4 nw, bool perm,
                                           int l, int mk) {
    VB_SHARED(&S);
    VB_SHARED(xs);
    const int t = threadIdx.x;
    float4 add = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!emb_row) add = sum_parts_tagged(p, parts, n, tag);
    if (!consumers_sync_and<kCT>(err_read(p.err) == 0)) return false;
    if (mk >= 0) tmark(p, l, mk);
    const float av[4] = {add.x, add.y, add.z, add.w};
    const float wv[4] = {nw.x, nw.y, nw.z, nw.w};
    float v[4];
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = t + k * kCT;
        const float x = emb_row ? emb_row[i] : S.xr[i] + av[k];
        S.xr[i] = x;
        ss += (double)x * (double)x;
        v[k] = x;
    }
    ss = warp_sum_d(ss);
    if ((t & 31) == 0) S.red[t >> 5] = ss;
    consumers_sync<kCT>();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kCW; w++) tot += S.red[w];
    const float sc = rms_scale_ool(tot, p.hidden, p.eps);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = t + k * kCT;
        xs[perm ? perm_index(i) : i] = __fmul_rn(__fmul_rn(v[k], sc), wv[k]);
    }
    consumers_sync<kCT>();
    return true;
}

// Residual update without a norm (CTAs that sit out phase A keep their copy
// of x current while the kv clusters work).
__device__ __noinline__ bool residual_only(const M2Params& p, S2& S, const unsigned long long* parts, int n,
                                           unsigned tag, const float* emb_row) {
    VB_SHARED(&S);
    const int t = threadIdx.x;
    float4 add = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!emb_row) add = sum_parts_tagged(p, parts, n, tag);
    if (!consumers_sync_and<kCT>(err_read(p.err) == 0)) return false;
    const float av[4] = {add.x, add.y, add.z, add.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = t + k * kCT;
        S.xr[i] = emb_row ? emb_row[i] : S.xr[i] + av[k];
    }
    consumers_sync<kCT>();
    return true;
}

__device__ __forceinline__ float4 load_norm(const float* w) {
    const int t = threadIdx.x;
    return make_float4(__ldg(w + t), __ldg(w + t + kCT), __ldg(w + t + 2 * kCT), __ldg(w + t + 3 * kCT));
}

__device__ __forceinline__ float rope1(const float* y, int d, const float* cr, const float* sr) {
    return d < 64 ? __fsub_rn(__fmul_rn(y[d], cr[d]), __fmul_rn(y[d + 64], sr[d]))
                  : __fadd_rn(__fmul_rn(y[d], cr[d]), __fmul_rn(y[d - 64], sr[d]));
}

// Phase A step 2-3: wait for the kv head's 512 q/k/v values pushed by the 8
// CTAs of the cluster; q/k RMSNorm + RoPE (generate.cpp:52-64), v as is; the
// rank-0 CTA appends k, v to the cache.
__device__ __noinline__ bool qkv_finish(const M2Params& p, S2& S, int l, int k, int rank, int pos, unsigned ep1,
                                        long long* prof) {
    VB_SHARED(&S);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const M2Layer& L = p.layers[l];
    {
        const long long c0 = tclk();
        // (armed failure test: CTA 0 waits at layer 0 for a tag no CTA writes)
        const unsigned tag = (l == 0 && blockIdx.x == 0 && fault_armed()) ? 0xFFFFFFFFu : xtag(ep1, l, kXQkv);
        bool ok = true;
        for (int i = t; i < 512 && ok; i += kCT) ok = wait_own(p, &S.qkv64[i], tag, 7, S.qkv[i]);
        if (!consumers_sync_and<kCT>(ok)) return false;
        if (prof) prof[8] += tclk() - c0;
    }
    tmark(p, l, 3);
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
    S.tq[hs][d] = __fmul_rn(__fmul_rn(qv, rms_scale_ool(tq, 128, p.eps)), L.q_norm[d]);
    if (t < 128) {
        const double tk = S.red[8] + S.red[9] + S.red[10] + S.red[11];
        S.tk[d] = __fmul_rn(__fmul_rn(kv, rms_scale_ool(tk, 128, p.eps)), L.k_norm[d]);
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
    return true;
}

// Phase A step 4: attention over this CTA's 32-position chunks c = rank,
// rank + 8, ...; each half of local chunk j (16 positions) goes to warp
// (2 j + half) % 8, which keeps an online softmax over its half-chunks (lanes
// p and p + 16 score position p over the two dim halves with a column skew that
// keeps the K reads free of bank conflicts; for PV lane l owns dims 4l..4l+3).
// Two warps per chunk measured INT8 1224 -> 1237 tok/s, f32 889 -> 906; four
// (8 positions each) INT8 1241 -> 1207.
// The warps' partials are then merged (warp order) into S.att_*.
__device__ __noinline__ bool attention(const M2Params& p, S2& S, const char* ring, int l, int rank, int pos,
                                       int nchunks, int g, long long* prof) {
    VB_SHARED(&S);
    VB_SHARED(ring);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n = pos + 1;
    const int njl = rank < nchunks ? (nchunks - rank + kCS - 1) / kCS : 0;
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    f2 a0lo = 0ull, a0hi = 0ull, a1lo = 0ull, a1hi = 0ull;  // dims 4l..4l+3 of heads 0, 1
    bool ok = true;
    // item it = 2 j + half: local chunk j's positions [16 half, 16 half + 16),
    // so two warps share a chunk; lanes l and l + 16 score position l & 15
    // over dims [0, 64) and [64, 128)
    const int pl = lane & 15, dh = lane >> 4;
    for (int it = warp; it < 2 * njl && ok; it += kCW) {
        const int j = it >> 1, half = it & 1;
        const int c = rank + kCS * j;
        const int gk = g + 2 * j, gv = gk + 1;
        const long long tw = tclk();
        ok = stage_wait(p, S, gk, false) && stage_wait(p, S, gv, false);
        if (!ok) break;
        if (prof) {
            prof[11] += tclk() - tw;
            prof[12] += 1;
        }
        const float* Kt = reinterpret_cast<const float*>(ring + (size_t)(gk % kStages) * kStageBytes);
        const float* Vt = reinterpret_cast<const float*>(ring + (size_t)(gv % kStages) * kStageBytes);
        const int p0 = c * kChunk + 16 * half;
        const bool valid = p0 + pl < n;
        const float* krow = (p0 + pl == pos) ? S.kn : Kt + (16 * half + pl) * 128;
        f2 s0a = 0ull, s0b = 0ull, s1a = 0ull, s1b = 0ull;
#pragma unroll 4
        for (int i = 0; i < 16; i++) {
            const int c4 = 4 * (((i + pl) & 15) + 16 * dh);
            const float4 k4 = *reinterpret_cast<const float4*>(krow + c4);
            const float4 qa = *reinterpret_cast<const float4*>(&S.q[0][c4]);
            const float4 qb = *reinterpret_cast<const float4*>(&S.q[1][c4]);
            const f2 klo = f2pack(k4.x, k4.y), khi = f2pack(k4.z, k4.w);
            s0a = f2fma(f2pack(qa.x, qa.y), klo, s0a);
            s0b = f2fma(f2pack(qa.z, qa.w), khi, s0b);
            s1a = f2fma(f2pack(qb.x, qb.y), klo, s1a);
            s1b = f2fma(f2pack(qb.z, qb.w), khi, s1b);
        }
        float s0 = f2sum(s0a) + f2sum(s0b), s1 = f2sum(s1a) + f2sum(s1b);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 16);  // the two dim halves
        s1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        const float sc0 = valid ? s0 * inv_sqrt_d : -INFINITY;
        const float sc1 = valid ? s1 * inv_sqrt_d : -INFINITY;
        const float mn0 = fmaxf(m0, warp_max(sc0)), mn1 = fmaxf(m1, warp_max(sc1));
        const float f0 = (m0 == -INFINITY) ? 0.f : expf(m0 - mn0);
        const float f1 = (m1 == -INFINITY) ? 0.f : expf(m1 - mn1);
        const float e0 = valid ? expf(sc0 - mn0) : 0.f;
        const float e1 = valid ? expf(sc1 - mn1) : 0.f;
        // (each position sits in two lanes: sum one copy)
        l0 = l0 * f0 + warp_sum(dh ? 0.f : e0);
        l1 = l1 * f1 + warp_sum(dh ? 0.f : e1);
        const f2 ff0 = f2pack(f0, f0), ff1 = f2pack(f1, f1);
        a0lo = f2mul(a0lo, ff0);
        a0hi = f2mul(a0hi, ff0);
        a1lo = f2mul(a1lo, ff1);
        a1hi = f2mul(a1hi, ff1);
        m0 = mn0;
        m1 = mn1;
        const int nv = min(16, n - p0);
#pragma unroll 4
        for (int pp = 0; pp < 16; pp++) {
            const float* vrow = (p0 + pp == pos) ? S.vn : Vt + (16 * half + pp) * 128;
            float4 v4 = *reinterpret_cast<const float4*>(vrow + 4 * lane);
            if (pp >= nv) v4 = make_float4(0.f, 0.f, 0.f, 0.f);  // stale rows past the context
            const float w0 = __shfl_sync(0xffffffffu, e0, pp), w1 = __shfl_sync(0xffffffffu, e1, pp);
            const f2 vlo = f2pack(v4.x, v4.y), vhi = f2pack(v4.z, v4.w);
            const f2 ww0 = f2pack(w0, w0), ww1 = f2pack(w1, w1);
            a0lo = f2fma(ww0, vlo, a0lo);
            a0hi = f2fma(ww0, vhi, a0hi);
            a1lo = f2fma(ww1, vlo, a1lo);
            a1hi = f2fma(ww1, vhi, a1hi);
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(smem_addr(&S.empty[gk % kStages]), (unsigned)(kCW / 2));
            mbar_arrive(smem_addr(&S.empty[gv % kStages]), (unsigned)(kCW / 2));
        }
    }
    {
        float4 a0, a1;
        f2unpack(a0lo, a0.x, a0.y);
        f2unpack(a0hi, a0.z, a0.w);
        f2unpack(a1lo, a1.x, a1.y);
        f2unpack(a1hi, a1.z, a1.w);
        *reinterpret_cast<float4*>(&S.wacc[warp][0][4 * lane]) = a0;
        *reinterpret_cast<float4*>(&S.wacc[warp][1][4 * lane]) = a1;
    }
    if (lane == 0) {
        S.wm[warp][0] = m0;
        S.wm[warp][1] = m1;
        S.wl[warp][0] = l0;
        S.wl[warp][1] = l1;
    }
    if (!consumers_sync_and<kCT>(ok)) return false;
    const int hs = t >> 7, d = t & 127;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCW; w++) M = fmaxf(M, S.wm[w][hs]);
    float Lsum = 0.f, A = 0.f;
#pragma unroll 1
    for (int w = 0; w < kCW; w++) {
        const float mw = S.wm[w][hs];
        if (mw == -INFINITY) continue;
        const float f = expf(mw - M);
        Lsum = fmaf(S.wl[w][hs], f, Lsum);
        A = fmaf(S.wacc[w][hs][d], f, A);
    }
    S.att_acc[hs][d] = A;
    if (d == 0) {
        S.att_m[hs] = M;
        S.att_l[hs] = Lsum;
    }
    return true;
}

// Phase A step 5: push this CTA's attention partial to the 8 CTAs of the
// cluster, then merge the 8 partials (rank order) -> ctx of heads 2k, 2k+1
// into xs (lane-interleaved layout for INT8).
__device__ __noinline__ bool merge_ctx(const M2Params& p, S2& S, float* xs, int l, int rank, unsigned ep1,
                                       bool perm, long long* prof) {
    VB_SHARED(&S);
    VB_SHARED(xs);
    const int t = threadIdx.x;
    const long long c0 = tclk();
    const unsigned tag = xtag(ep1, l, kXAtt);
    const int hs = t >> 7, d = t & 127;
    const unsigned base = smem_addr(&S.xu.att64[rank][0]);
    // each thread pushes what it wrote itself at the end of the attention
    const unsigned long long wa = xpack(S.att_acc[hs][d], tag);
#pragma unroll 1
    for (unsigned q = 0; q < kCS; q++) st_peer(mapa(base + 8u * (unsigned)(hs * 128 + d), q), wa);
    if (d == 0) {
        const unsigned long long wm = xpack(S.att_m[hs], tag), wl = xpack(S.att_l[hs], tag);
#pragma unroll 1
        for (unsigned q = 0; q < kCS; q++) {
            st_peer(mapa(base + 8u * (unsigned)(256 + hs), q), wm);
            st_peer(mapa(base + 8u * (unsigned)(258 + hs), q), wl);
        }
    }
    bool ok = true;
    float M = -INFINITY;
#pragma unroll 1
    for (int r = 0; r < kCS && ok; r++) {
        float mr = 0.f;
        ok = wait_own(p, &S.xu.att64[r][256 + hs], tag, 8, mr);
        M = fmaxf(M, mr);
    }
    float Lsum = 0.f, A = 0.f;
#pragma unroll 1
    for (int r = 0; r < kCS && ok; r++) {
        float mr = 0.f, lr = 0.f, ar = 0.f;
        ok = wait_own(p, &S.xu.att64[r][256 + hs], tag, 8, mr) && wait_own(p, &S.xu.att64[r][258 + hs], tag, 8, lr) &&
             wait_own(p, &S.xu.att64[r][hs * 128 + d], tag, 8, ar);
        if (mr == -INFINITY) continue;
        const float f = expf(mr - M);
        Lsum = fmaf(lr, f, Lsum);
        A = fmaf(ar, f, A);
    }
    if (!consumers_sync_and<kCT>(ok)) return false;
    if (prof) prof[9] += tclk() - c0;
    const float cval = (Lsum > 0.f) ? A / Lsum : 0.f;
    const int i = hs * 128 + d;
    xs[perm ? perm_index(i) : i] = cval;
    consumers_sync<kCT>();
    return true;
}

// Phase B split-K down: thread t owns outputs j = 4t..4t+3 of
// sum_{i in slice} h_i * WdT[i][j]; the 4 values are pushed to the CTA of the
// cluster that reduces them (rank 4t / 128).
template <bool Q8>
__device__ __noinline__ bool down_push(const M2Params& p, S2& S, const char* ring, const Plan pl, int g, int l,
                                       int rank, unsigned ep1, long long* prof) {
    VB_SHARED(&S);
    VB_SHARED(ring);
    const int t = threadIdx.x;
    f2 alo = 0ull, ahi = 0ull;  // outputs 4t, 4t+1 | 4t+2, 4t+3
    const long long d0 = tclk();
    long long dw = 0;
    for (int j = 0; j < pl.nstages; j++) {
        const int gs = g + j;
        const long long tw = tclk();
        if (!stage_wait(p, S, gs, true)) return false;
        dw += tclk() - tw;
        const char* st = ring + (size_t)(gs % kStages) * kStageBytes;
        const int rA = pl.r0 + j * pl.rps;
        const int nr = min(pl.rps, pl.r1 - rA);
#pragma unroll 4
        for (int rr = 0; rr < nr; rr++) {
            const float hv = S.h[rA + rr - pl.r0];
            const f2 hh = f2pack(hv, hv);
            if constexpr (Q8) {
                f2 lo, hi;
                i8x4_to_f2(*reinterpret_cast<const uint32_t*>(st + (size_t)rr * pl.row_bytes + 4 * t), lo, hi);
                alo = f2fma(hh, lo, alo);
                ahi = f2fma(hh, hi, ahi);
            } else {
                const float4 w4 = *reinterpret_cast<const float4*>(st + (size_t)rr * pl.row_bytes + 16 * t);
                alo = f2fma(hh, f2pack(w4.x, w4.y), alo);
                ahi = f2fma(hh, f2pack(w4.z, w4.w), ahi);
            }
        }
        stage_release(S, gs, 1u);
    }
    if (prof) {
        prof[6] += dw;
        prof[7] += tclk() - d0;
    }
    const unsigned tag = xtag(ep1, l, kXRed);
    const int per = p.hidden / kCS;
    const int q = (4 * t) / per, o = 4 * t - q * per;
    const unsigned dst = mapa(smem_addr(&S.xu.red64[rank][o]), (unsigned)q);
    float4 acc;
    f2unpack(alo, acc.x, acc.y);
    f2unpack(ahi, acc.z, acc.w);
    st_peer(dst, xpack(acc.x, tag));
    st_peer(dst + 8u, xpack(acc.y, tag));
    st_peer(dst + 16u, xpack(acc.z, tag));
    st_peer(dst + 24u, xpack(acc.w, tag));
    return true;
}

// Phase B reduce: outputs [128 rank, +128) summed over the cluster's 8 CTAs
// in rank order (x the INT8 row scale) -> tagged down partial of the cluster.
__device__ __noinline__ bool reduce_store(const M2Params& p, S2& S, int l, int cid, int rank, unsigned ep1,
                                          bool q8, long long* prof) {
    VB_SHARED(&S);
    const long long c0 = tclk();
    const unsigned tag = xtag(ep1, l, kXRed);
    const int t = threadIdx.x;
    const int per = p.hidden / kCS;
    bool ok = true;
    if (t < per) {
        float v = 0.f;
#pragma unroll 1
        for (int q = 0; q < kCS && ok; q++) {
            float pv = 0.f;
            ok = wait_own(p, &S.xu.red64[q][t], tag, 9, pv);
            v += pv;
        }
        if (q8) v *= S.sc_d[t];
        if (ok)
            st_gpu(p.xd + ((size_t)(l & 1) * p.nclusters + cid) * p.hidden + rank * per + t,
                   xpack(v, xtag(ep1, l, kXGlobal)));
    }
    if (!consumers_sync_and<kCT>(ok)) return false;
    if (prof) prof[10] += tclk() - c0;
    return true;
}

// ------------------------------------------------------------ stage walk
// Every stage this CTA consumes in one token, in consumption order; f(src,
// bytes) per stage, stopping early when f returns false.
template <class F>
__device__ bool plan_stages(const Plan& pl, F& f) {
    for (int j = 0; j < pl.nstages; j++) {
        const int rows = min(pl.rps, pl.r1 - pl.r0 - j * pl.rps);
        if (!f(pl.w + (size_t)j * pl.rps * pl.row_bytes, (unsigned)(rows * pl.row_bytes))) return false;
    }
    return true;
}
template <bool Q8, class F>
__device__ void walk_stages(const M2Params& p, int b, int G, int cid, int rank, int nchunks, F& f) {
    const bool owns_kv = cid < p.kvh;
    for (int l = 0; l < p.nlayers; l++) {
        if (owns_kv) {
            if (!plan_stages(plan_qkv(p, l, Q8, cid, rank), f)) return;
            for (int c = rank; c < nchunks; c += kCS) {
                const int rows = min(kChunk, p.max_seq - c * kChunk);
                const size_t off = ((size_t)(l * p.kvh + cid) * p.max_seq + (size_t)c * kChunk) * 128;
                if (!f(p.kc + off, (unsigned)(rows * 512))) return;
                if (!f(p.vc + off, (unsigned)(rows * 512))) return;
            }
            if (!plan_stages(plan_o(p, l, Q8, cid, rank), f)) return;
        }
        if (!plan_stages(plan_gu(p, l, Q8, b, G), f)) return;
        if (!plan_stages(plan_dt(p, l, Q8, b, G), f)) return;
    }
    plan_stages(plan_lm(p, b, G), f);
}

// Ring producer: waits for the slot to be free, then one bulk copy into it.
struct RingIssue {
    const M2Params* p;
    S2* S;
    char* ring;
    unsigned long long pol;
    int g;
    bool ok;
    __device__ bool operator()(const void* src, unsigned bytes) {
        const int slot = g % kStages;
        if (!mbar_wait(smem_addr(&S->empty[slot]), ((unsigned)(g / kStages) & 1u) ^ 1u, p->err, p->dbg,
                       kSiteEmpty, g)) {
            ok = false;
            return false;
        }
        mbar_expect_tx(smem_addr(&S->full[slot]), bytes);
        bulk_g2s(smem_addr(ring + (size_t)slot * kStageBytes), src, bytes, smem_addr(&S->full[slot]), pol);
        g++;
        return true;
    }
};

// INT8 row scales of the next phase, loaded into registers before the wait
// for that phase's inputs (so their latency hides behind it) and stored to
// shared memory after it.
struct PreScales {
    float a, b;
};
__device__ __forceinline__ PreScales pre_scales_a(const M2Params& p, int l, int k, int rank) {
    const M2Layer& L = p.layers[l];
    const int t = threadIdx.x;
    PreScales v{0.f, 0.f};
    if (t < 64) v.a = __ldg(L.sqkv + k * 512 + 64 * rank + t);
    if (t < 128) v.b = __ldg(L.so + 128 * rank + t);
    return v;
}
__device__ __forceinline__ void put_scales_a(S2& S, const PreScales& v) {
    const int t = threadIdx.x;
    if (t < 64) S.sc_qkv[t] = v.a;
    if (t < 128) S.sc_o[t] = v.b;
}
__device__ __forceinline__ PreScales pre_scales_b(const M2Params& p, int l, int b, int G, int rank) {
    const M2Layer& L = p.layers[l];
    const int t = threadIdx.x;
    int r0, r1;
    split(p.ffn, b, G, 2, r0, r1);
    PreScales v{0.f, 0.f};
    if (t < r1 - r0) v.a = __ldg(L.sgu + r0 + t);
    if (t < 128) v.b = __ldg(L.sd + 128 * rank + t);
    return v;
}
__device__ __forceinline__ void put_scales_b(S2& S, const PreScales& v) {
    const int t = threadIdx.x;
    if (t < 128) {
        S.sc_gu[t] = v.a;
        S.sc_d[t] = v.b;
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

    if (VB_STEP_TRACE && p.trace)
        for (int i = threadIdx.x; i < kTraceStride2; i += kThreads)
            p.trace[(size_t)blockIdx.x * kTraceStride2 + i] = 0ull;
    // exchange words start with tag 0, which no launch uses; the cluster
    // barrier below orders this before any peer's push
    for (int i = threadIdx.x; i < 512; i += kThreads) S.qkv64[i] = 0ull;
    for (int i = threadIdx.x; i < kCS * kAttWords; i += kThreads) (&S.xu.att64[0][0])[i] = 0ull;
    if (threadIdx.x == 0) {
        if (VB_STEP_TRACE && p.trace) p.trace[(size_t)blockIdx.x * kTraceStride2] = now_ns();
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_addr(&S.full[s]), 1);
            mbar_init(smem_addr(&S.empty[s]), kCW);
            S.seq[s] = s - kStages;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // every CTA of the cluster has initialised its barriers and exchange
    // words before any remote access
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
        RingIssue f{&p, &S, ring, 0ull, 0, true};
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(f.pol));
        walk_stages<Q8>(p, b, G, cid, rank, nchunks, f);
        const int g = f.g;
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
    const unsigned ep1 = (unsigned)*p.epoch + 1u;
    int g = 0;
    bool ok = true;
    float4 nw = load_norm(p.layers[0].in_norm);
    PreScales psc{0.f, 0.f};
    if (Q8 && owns_kv) psc = pre_scales_a(p, 0, cid, rank);
    for (int l = 0; l < p.nlayers && ok; l++) {
        const M2Layer& L = p.layers[l];
        long long* prof = prof_ptr(p, l);
        if (prof) {
            prof[14] = tclk();
            prof[15] = (long long)now_ns();
        }
        const unsigned long long* xd_prev = p.xd + (size_t)((l + 1) & 1) * p.nclusters * p.hidden;
        const unsigned tag_prev = l > 0 ? xtag(ep1, l - 1, kXGlobal) : 0u;
        // ---- phase A (kv clusters): qkv rows -> gather -> attention -> merge -> o_proj
        if (owns_kv) {
            if (!residual_norm(p, S, xs, xd_prev, p.nclusters, tag_prev, l == 0 ? emb_row : nullptr, nw, Q8, l, 0)) {
                ok = false;
                break;
            }
            if (Q8) {
                put_scales_a(S, psc);
                consumers_sync<kCT>();
            }
            tmark(p, l, 1);
            {   // this CTA's 64 rows of kv block cid, each pushed to the 8 CTAs
                const Plan pl = plan_qkv(p, l, Q8, cid, rank);
                const Epi epi{kEpiQkvPush, smem_addr(&S.qkv64[0]), xtag(ep1, l, kXQkv), nullptr, nullptr, 0, nullptr};
                bool r;
                if constexpr (Q8) r = gemv_rows<true, 8, kHid>(p, pl, g, ring, S, xs, S.sc_qkv, false, epi, prof,
                                                             prof ? prof + 16 : nullptr);
                else r = gemv_rows<false, 4, kHid>(p, pl, g, ring, S, xs, nullptr, false, epi, prof,
                                                   prof ? prof + 16 : nullptr);
                g += pl.nstages;
                if (!consumers_sync_and<kCT>(r)) { ok = false; break; }
                tmark(p, l, 2);
            }
            if (!qkv_finish(p, S, l, cid, rank, pos, ep1, prof)) { ok = false; break; }
            {
                const long long t_att = tclk();
                const bool r = attention(p, S, ring, l, rank, pos, nchunks, g, prof);
                g += 2 * (rank < nchunks ? (nchunks - rank + kCS - 1) / kCS : 0);
                if (!r) { ok = false; break; }
                tmark(p, l, 4);
                if (prof) prof[13] += tclk() - t_att;
            }
            if (!merge_ctx(p, S, xs, l, rank, ep1, Q8, prof)) { ok = false; break; }
            tmark(p, l, 5);
            {   // split-K o_proj: hidden rows 128r.. of kv head cid's ctx columns
                const Plan pl = plan_o(p, l, Q8, cid, rank);
                const Epi epi{kEpiStoreTagged, 0u, xtag(ep1, l, kXGlobal),
                              p.xo + ((size_t)(l & 1) * p.kvh + cid) * p.hidden, nullptr, 0, nullptr};
                bool r;
                if constexpr (Q8) r = gemv_rows<true, 16, 256>(p, pl, g, ring, S, xs, S.sc_o, false, epi,
                                                              prof ? prof + 2 : nullptr, prof ? prof + 19 : nullptr);
                else r = gemv_rows<false, 16, 256>(p, pl, g, ring, S, xs, nullptr, false, epi,
                                                   prof ? prof + 2 : nullptr, prof ? prof + 19 : nullptr);
                g += pl.nstages;
                if (!r) { ok = false; break; }
                tmark(p, l, 6);
            }
        } else {
            // CTAs outside the kv clusters bring their x up to date here, so
            // that every read of the previous layer's down partials happens
            // before any of this layer's are produced.
            if (!residual_only(p, S, xd_prev, p.nclusters, tag_prev, l == 0 ? emb_row : nullptr)) {
                ok = false;
                break;
            }
        }
        nw = load_norm(L.post_norm);
        if (Q8) psc = pre_scales_b(p, l, b, G, rank);
        // ---- phase B (all CTAs): waits for the o_proj partials of all kv heads
        if (!residual_norm(p, S, xs, p.xo + (size_t)(l & 1) * p.kvh * p.hidden, p.kvh, xtag(ep1, l, kXGlobal),
                           nullptr, nw, Q8, l, 7)) { ok = false; break; }
        if (Q8) {
            put_scales_b(S, psc);
            consumers_sync<kCT>();
        }
        tmark(p, l, 8);
        {   // this CTA's gate/up pairs -> h slice (SwiGLU fused)
            const Plan pl = plan_gu(p, l, Q8, b, G);
            const Epi epi{kEpiSwiGLU, 0u, 0u, nullptr, S.h, pl.r0 >> 1, nullptr};
            bool r;
            if constexpr (Q8) r = gemv_rows<true, 8, kHid>(p, pl, g, ring, S, xs, S.sc_gu, true, epi,
                                                         prof ? prof + 4 : nullptr, prof ? prof + 22 : nullptr);
            else r = gemv_rows<false, 4, kHid>(p, pl, g, ring, S, xs, nullptr, true, epi,
                                               prof ? prof + 4 : nullptr, prof ? prof + 22 : nullptr);
            g += pl.nstages;
            if (!consumers_sync_and<kCT>(r)) { ok = false; break; }
        }
        tmark(p, l, 9);
        {
            const Plan pl = plan_dt(p, l, Q8, b, G);
            const bool r = down_push<Q8>(p, S, ring, pl, g, l, rank, ep1, prof);
            g += pl.nstages;
            if (!consumers_sync_and<kCT>(r)) { ok = false; break; }
        }
        tmark(p, l, 10);
        if (!reduce_store(p, S, l, cid, rank, ep1, Q8, prof)) { ok = false; break; }
        nw = load_norm(l + 1 < p.nlayers ? p.layers[l + 1].in_norm : p.final_norm);
        if (Q8 && owns_kv && l + 1 < p.nlayers) psc = pre_scales_a(p, l + 1, cid, rank);
        tmark(p, l, 11);
    }
    if (!ok) goto consumer_exit;
    // ---- LM: final norm + lm_head + argmax
    if (!residual_norm(p, S, xs, p.xd + (size_t)((p.nlayers - 1) & 1) * p.nclusters * p.hidden, p.nclusters,
                       xtag(ep1, p.nlayers - 1, kXGlobal), nullptr, nw, p.lm_q8 != nullptr, 0, -1))
        goto consumer_exit;
    {
        const Plan pl = plan_lm(p, b, G);
        const Epi epi{kEpiLogits, 0u, 0u, nullptr, nullptr, 0, p.logits};
        bool r;
        if (p.lm_q8) {
            // INT8 rows: this CTA's row scales into the exchange buffer, idle in this phase
            // (every push into it for the last layer has been consumed)
            float* sl = reinterpret_cast<float*>(&S.xu);
            for (int i = threadIdx.x; i < pl.r1 - pl.r0; i += kCT) sl[i] = p.lm_sc[pl.r0 + i];
            consumers_sync<kCT>();
            r = gemv_rows<true, 8, kHid>(p, pl, g, ring, S, xs, sl, false, epi, nullptr, nullptr);
        } else {
            r = gemv_rows<false, 4, kHid>(p, pl, g, ring, S, xs, nullptr, false, epi, nullptr, nullptr);
        }
        if (!consumers_sync_and<kCT>(r)) goto consumer_exit;
    }
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
            *p.epoch = (ep1 < (1u << 23)) ? (int)ep1 : 0;
            *p.am_ticket = 0;
        }
    }
    }
consumer_exit:
    // No CTA leaves while a peer of its cluster may still access its shared
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
        c.kv_heads * kCS > 148 || c.layers > 63)
        return fail(VB_ERR_UNSUPPORTED, "two-barrier step: needs hidden 1024, GQA 2, head_dim 128");
    if (!e->kc) return fail(VB_ERR_NO_CACHE, "call reset_cache() first");
    const bool q8 = e->quantized;
    auto kern = q8 ? mega2_kernel<true> : mega2_kernel<false>;
    int nclusters = c.kv_heads;
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
        // phase B and the lm_head run on every co-resident cluster; phase A
        // on the first kv_heads of them
        nclusters = nc;
        if (const char* v = getenv("VB_STEP_CLUSTERS")) {
            const int want = atoi(v);
            if (want >= c.kv_heads && want <= nc) nclusters = want;
        }
        if ((c.ffn + nclusters * kCS - 1) / (nclusters * kCS) > 64)
            return fail(VB_ERR_UNSUPPORTED, "two-barrier step: ffn slice too wide");
    }
    // the INT8 lm_head keeps a CTA's row scales in the exchange buffer
    if (e->lm_int8 && (size_t)(c.vocab + nclusters * kCS - 1) / (nclusters * kCS) * sizeof(float) > sizeof(S2::xu))
        return fail(VB_ERR_UNSUPPORTED, "clustered step: too few CTAs for the INT8 lm_head's scales");
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
    const int G = nclusters * kCS;
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
    m->grid = G;
    if (ce == cudaSuccess) {
        m->d_layers = static_cast<M2Layer*>(alloc(sizeof(M2Layer) * c.layers));
        if (!m->d_layers) ce = cudaErrorMemoryAllocation;
    }
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(m->d_layers, hl.data(), sizeof(M2Layer) * c.layers, cudaMemcpyHostToDevice, s);
    // tagged exchange buffers (two layer parities each), argmax slots and
    // counters: all zeroed together (tag 0 is never a live tag)
    const size_t po = sizeof(unsigned long long) * 2 * (size_t)c.kv_heads * hd;
    const size_t pd = sizeof(unsigned long long) * 2 * (size_t)nclusters * hd;
    const size_t am = sizeof(float) * (size_t)G * 2;
    const size_t cnt = 256 * sizeof(int);
    if (ce == cudaSuccess) {
        m->ws = static_cast<char*>(alloc(po + pd + am + cnt));
        if (!m->ws) ce = cudaErrorMemoryAllocation;
    }
    if (ce == cudaSuccess) {
        m->counters = m->ws;
        m->counters_bytes = po + pd + am + cnt;
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
    P.lm_q8 = e->lm_int8 ? e->lm_q8 : nullptr;
    P.lm_sc = e->lm_int8 ? e->lm_sc : nullptr;
    P.final_norm = e->final_norm;
    P.rope_cos = e->rope_cos;
    P.rope_sin = e->rope_sin;
    P.kc = e->kc;
    P.vc = e->vc;
    P.logits = e->logits;
    P.xo = reinterpret_cast<unsigned long long*>(m->ws);
    P.xd = reinterpret_cast<unsigned long long*>(m->ws + po);
    P.am_val = reinterpret_cast<float*>(m->ws + po + pd);
    P.am_idx = reinterpret_cast<int*>(m->ws + po + pd + am / 2);
    int* cn = reinterpret_cast<int*>(m->ws + po + pd + am);
    P.epoch = cn;
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
    P.nclusters = nclusters;
    P.eps = c.eps;
    P.trace = nullptr;
    if (VB_STEP_TRACE && e->trace_on) {
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

vb_status mega2_set_fault(int v, cudaStream_t s) {
    VB_CUDA_TRY(set_fault_word(v, s));
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

// Where the last failed step gave up, from the debug words the first failing
// wait recorded: " [code c, cta b, <site>, index i, extra x]" or "".
std::string mega2_debug(vb_engine* e) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (!m) return "";
    int d[5] = {0, 0, 0, 0, 0};
    if (cudaMemcpy(d, m->params.dbg, sizeof d, cudaMemcpyDeviceToHost) != cudaSuccess) return "";
    if (!d[0]) return "";
    static const char* sites[] = {"?",
                                  "producer empty-slot wait",
                                  "consumer stage wait",
                                  "attention stage wait",
                                  "global partials exchange",
                                  "slot order wait",
                                  "?",
                                  "cluster q/k/v gather",
                                  "cluster attention merge",
                                  "cluster down-proj reduce"};
    const int si = (d[2] >= 1 && d[2] <= 9) ? d[2] : 0;
    return std::string(" [code ") + std::to_string(d[0]) + ", cta " + std::to_string(d[1]) + ", " + sites[si] +
           ", index " + std::to_string(d[3]) + ", extra " + std::to_string(d[4]) + "]";
}

void mega2_reset_counters(vb_engine* e) {
    Mega2State* m = static_cast<Mega2State*>(e->mega2);
    if (m) {
        cudaMemsetAsync(m->counters, 0, m->counters_bytes, e->stream);
        cudaStreamSynchronize(e->stream);
    }
}

}  // namespace vb
