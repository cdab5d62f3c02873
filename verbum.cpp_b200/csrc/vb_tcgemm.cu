// vb_tcgemm.cu -- projections of the batched decode step on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory, operands staged in
// shared memory by TMA).
//
// C[m][n] = sum_k A[m][k] W[n][k] for the M <= 64 activation rows of a batched
// step against a weight matrix W [N][K] (the reference's matmul_nt,
// core/src/ops.cpp:42-70, and matmul_nt_q8, core/src/quant.cpp:43-70, with
// x holding M rows).  The MMA runs on bf16 operands with f32 accumulation:
//   * INT8 weights are stored once as bf16 (every value in [-127, 127] is exact
//     in bf16), the per-row scale is applied after the sum as the reference
//     does;
//   * f32 weights (the tied lm_head, and the f32 model) are stored as a bf16
//     pair W = W_hi + W_lo;
//   * the f32 activations are split the same way, A = A_hi + A_lo.
// The sum takes A_hi W + A_lo W (INT8) or A_hi W_hi + A_lo W_hi + A_hi W_lo
// (f32): products of bf16 values are exact in f32, and the dropped terms are
// ~2^-16 relative, so the result tracks the f32 reference closely.
//
// One CTA computes a 128-row weight tile (the MMA's M) against all 64
// activation rows (the MMA's N) over one K range (split-K).  With several
// splits each CTA stores its partial P[split][m][n] and the reduce kernel sums
// them in split order across the whole GPU (one CTA per tile summing 16
// splits was measured slower); a single split applies the epilogue itself.
// Either way the INT8 row scales are applied after the sum, as the reference
// does, then the epilogue (store, residual add, or SwiGLU with its bf16 split
// for the next GEMM).
//
// Warp 0 lane 0 issues TMA copies into a 3- or 4-stage ring, warp 1 lane 0 issues the
// MMAs (tcgen05.commit frees a stage when its MMAs are done), and all four warps
// read the 128 x 64 f32 accumulator tile out of tensor memory.  Every wait is
// bounded; on a timeout the error word is set, in-flight copies and MMAs are
// waited for (bounded), tensor memory is freed and the kernel returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "vb_engine.cuh"
#include "vb_pipe.cuh"
#include "vb_tail.cuh"
#include "vb_tc.cuh"

namespace vb {
namespace {

constexpr int kTSMs = 148;        // B200 SM count (split-K sizing)
constexpr int kTM = 128;         // weight rows per tile (MMA M)
constexpr int kTN = 64;          // activation rows (MMA N)
constexpr int kTK = 64;          // K per stage: one 128-byte swizzle row of bf16
constexpr int kTThreads = 128;
constexpr int kWTile = kTM * kTK * 2;   // 16 KB
constexpr int kATile = kTN * kTK * 2;   // 8 KB
// one stage: W_hi [, W_lo], A_hi, A_lo
__host__ __device__ constexpr int stage_bytes(int wp) { return wp * kWTile + 2 * kATile; }
__host__ __device__ constexpr size_t tc_smem(int wp, int ns) { return (size_t)ns * stage_bytes(wp) + 1024; }  // + alignment slack
// Ring depth and CTAs per SM: a weight pair (f32) keeps 4 stages of 48 KB, one
// CTA per SM; single bf16 weights (INT8) keep kQStages stages of 32 KB.
constexpr int kPStages = 4;
constexpr int kQStages = 4;
__host__ __device__ constexpr int ctas_per_sm(int wp) { return wp == 2 ? 1 : (2 * tc_smem(1, kQStages) + 2048 <= 228 * 1024 ? 2 : 1); }

struct TcParams {
    int M, N;       // activation rows, weight rows (blockIdx.z: 64-row activation tile)
    int chunks;     // K / kTK
    int per_split;  // chunks per split
    int splits;
    int partials;   // write P even for one split (a fused consumer reads it)
    float* P;       // [splits][M][N]
    const float* scales;
    float* C;
    int ldc;
    int epi;
    __nv_bfloat16* out_hi;
    __nv_bfloat16* out_lo;
    int* err;
    QkNormArgs qk;  // kEpiQkNorm
};

// ---------------------------------------------------------------------------
// Split-K summed inside a thread-block cluster (the q|k|v GEMM of the batched
// step, epilogue kEpiQkNorm): the S CTAs of a tile's splits
// form one cluster (cluster rank = split).  Each parks its 128 x 64 partial in
// its own shared memory as [64 rows][128 features]; after a cluster barrier,
// rank r reads rows [r R, r R + R) of all S partials over DSMEM, sums them in
// split order and applies the epilogue; a second barrier keeps every partial
// alive until all ranks have read it.
constexpr int kClusterMaxSplits = 8;  // portable cluster size

// Rows [b0, b1) of tile n0 (128 features = one head) from the S parked
// partials at shared::cluster addresses rq[0..S): the per-head q/k norm +
// RoPE + append, with the q/k-norm kernel's arithmetic (partials summed in
// split order from 0, INT8 scale after the sum).  The same in-cluster sum
// for the gate|up GEMM's SwiGLU measured slower than its reduce kernel
// (batched step 5.77 -> 5.93 ms with 2 splits, whose 48 clusters are all
// resident; 6.07 -> 6.22 ms with 3, which are not).
__device__ __forceinline__ void cluster_epilogue(const TcParams& p, const unsigned* rq, int S, int n0, int b0,
                                                 int b1, int warp, int lane) {
    const QkNormArgs& a = p.qk;
    const int hd = n0 / kTM;
    const bool isq = hd < a.H, isk = !isq && hd < a.H + a.KVH;
    const int h = isq ? hd : (isk ? hd - a.H : hd - a.H - a.KVH);
    for (int b = b0 + warp; b < b1; b += kTThreads / 32) {
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        const unsigned ro = 4u * (unsigned)(b * kTM + lane);
#pragma unroll
        for (int q = 0; q < kClusterMaxSplits; q++) {
            if (q < S) {
#pragma unroll
                for (int e = 0; e < 4; e++) x[e] += cl_ld(rq[q] + ro + 128u * (unsigned)e);
            }
        }
        if (p.scales) {
#pragma unroll
            for (int e = 0; e < 4; e++) x[e] *= p.scales[n0 + lane + 32 * e];
        }
        const int pos = a.pos[b];
        if (pos < 0 || pos >= a.rope_positions) {
            if (lane == 0 && a.err) atomicExch(a.err, kErrCacheFull);
            continue;
        }
        if (isq) {
            float o[4];
            qk_finish(a, true, pos, x, lane, o);
            const size_t qo = ((size_t)b * a.H + h) * kTM;
#pragma unroll
            for (int e = 0; e < 4; e++) a.q_out[qo + lane + 32 * e] = o[e];
        } else {
            const size_t off = (size_t)b * a.stride_b + (size_t)pos * a.stride_pos + (size_t)h * a.stride_h;
            if (isk) {
                float o[4];
                qk_finish(a, false, pos, x, lane, o);
#pragma unroll
                for (int e = 0; e < 4; e++) a.kc[off + lane + 32 * e] = o[e];
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++) a.vc[off + lane + 32 * e] = x[e];
            }
        }
    }
}

// Instruction descriptor, kind::f16: f32 accumulator [4,6) = 1, A bf16 [7,10) = 1,
// B bf16 [10,13) = 1, both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(unsigned tmem, uint64_t adesc, uint64_t bdesc, bool acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.u32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"((unsigned)acc)
        : "memory");
}

template <int WP, int NS, bool CL>
__global__ void __launch_bounds__(kTThreads, ctas_per_sm(WP))
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap tw_lo,
                   const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                   const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    constexpr int kTStages = NS;
    constexpr int kTStage = stage_bytes(WP);
    constexpr int kAOff = WP * kWTile;
    __shared__ __align__(8) unsigned long long full[kTStages], empty[kTStages], done;
    __shared__ unsigned tmem_slot;
    __shared__ int fail;
    __shared__ unsigned cl_ok;  // CL: this CTA's partial is parked
    const unsigned sbase = (smem_addr(smem_raw) + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTM;
    const int split = blockIdx.y;
    const int m0 = blockIdx.z * kTN;  // first activation row of this tile
    const int Mt = min(kTN, p.M - m0);
    const int c0 = split * p.per_split;
    const int nch = min(p.per_split, p.chunks - c0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTStages; s++) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        mbar_init(smem_addr(&done), 1);
        fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(kTN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = tmem_slot;
    pdl_trigger();

    if (warp == 0 && lane == 0 && nch > 0) {
        // ------------------------------------------------------ TMA producer
        // The weights do not depend on the previous kernel: the first stages'
        // weight tiles are requested before waiting for it, the activation
        // tiles after.
        const int pre = min(nch, kTStages);
        // (armed failure test: the first CTA never fills its first stage)
        const int withheld = (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && fault_armed()) ? 0 : -1;
        for (int i = 0; i < pre; i++) {
            if (i == withheld) continue;
            const unsigned st = sbase + (unsigned)i * kTStage;
            const unsigned fb = smem_addr(&full[i]);
            mbar_expect_tx(fb, (unsigned)(WP * kWTile + 2 * kATile));
            const int x = (c0 + i) * kTK;
            tma_load_2d(st, &tw_hi, x, n0, fb);
            if (WP == 2) tma_load_2d(st + kWTile, &tw_lo, x, n0, fb);
        }
        pdl_wait();
        int issued = 0;
        for (int i = 0; i < nch; i++) {
            const int s = i % kTStages;
            const unsigned st = sbase + (unsigned)s * kTStage;
            const unsigned fb = smem_addr(&full[s]);
            const int x = (c0 + i) * kTK;
            if (i >= pre) {
                if (!mbar_wait(smem_addr(&empty[s]), ((unsigned)(i / kTStages) & 1u) ^ 1u, p.err, nullptr, kSiteEmpty,
                               i)) {
                    fail = 1;
                    break;
                }
                mbar_expect_tx(fb, (unsigned)(WP * kWTile + 2 * kATile));
                tma_load_2d(st, &tw_hi, x, n0, fb);
                if (WP == 2) tma_load_2d(st + kWTile, &tw_lo, x, n0, fb);
            }
            if (i != withheld) {
                tma_load_2d(st + kAOff, &ta_hi, x, m0, fb);
                tma_load_2d(st + kAOff + kATile, &ta_lo, x, m0, fb);
            }
            issued = i + 1;
        }
        // a stage whose weights went out before a failure still has its copies in flight
        if (issued < pre) issued = pre;
        // never leave with copies in flight
        for (int i = issued > kTStages ? issued - kTStages : 0; i < issued; i++)
            if (i != withheld) mbar_drain(smem_addr(&full[i % kTStages]), (unsigned)(i / kTStages) & 1u);
    } else if (warp == 1 && lane == 0 && nch > 0) {
        // ------------------------------------------------------- MMA issuer
        int committed = 0;
        for (int i = 0; i < nch && !fail; i++) {
            const int s = i % kTStages;
            if (!mbar_wait(smem_addr(&full[s]), (unsigned)(i / kTStages) & 1u, p.err, nullptr, kSiteFull, i)) {
                fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned st = sbase + (unsigned)s * kTStage;
#pragma unroll
            for (int kk = 0; kk < kTK / 16; kk++) {
                const uint64_t wh = sw128_desc(st + 32u * kk);
                const uint64_t ah = sw128_desc(st + kAOff + 32u * kk);
                const uint64_t al = sw128_desc(st + kAOff + kATile + 32u * kk);
                mma_bf16(tmem, wh, ah, i > 0 || kk > 0);
                mma_bf16(tmem, wh, al, true);
                if (WP == 2) mma_bf16(tmem, sw128_desc(st + kWTile + 32u * kk), ah, true);
            }
            mma_commit(smem_addr(&empty[s]));
            committed = i + 1;
        }
        (void)committed;
        mma_commit(smem_addr(&done));
    }
    // -------------------------------------------------------------- epilogue
    __syncwarp();
    pdl_wait();  // partials and outputs are read / written by neighbouring kernels
    bool ok = nch > 0;
    if (ok) {
        // the MMA thread commits `done` after its last MMA, also after a
        // failed wait: once it completes no MMA is in flight
        ok = mbar_drain(smem_addr(&done), 0u);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    ok = __syncthreads_and(ok && !fail);
    if (ok) {
        float v[kTN];
        const unsigned taddr = tmem + ((unsigned)(32 * warp) << 16);
        unsigned* r = reinterpret_cast<unsigned*>(v);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
            "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
            "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
            "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
            "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
              "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
              "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
              "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]),
              "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
              "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]),
              "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
              "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int n = n0 + 32 * warp + lane;
        if constexpr (CL) {
            // park the partial [64 rows][128 features] in the drained ring
            float* T = reinterpret_cast<float*>(smem_raw + (sbase - smem_addr(smem_raw)));
#pragma unroll
            for (int m = 0; m < kTN; m++) T[m * kTM + 32 * warp + lane] = v[m];
        }
        bool mine = !CL;  // a single split applies the epilogue itself
        if (p.splits > 1 || p.partials) {  // (split-K runs with one activation tile)
            mine = false;
            float* P = p.P + (size_t)split * p.M * p.N + n;
            if (n < p.N)
#pragma unroll
                for (int m = 0; m < kTN; m++)
                    if (m < Mt) P[(size_t)m * p.N] = v[m];
        }
        if (mine) {
            const float sc = (p.scales && n < p.N) ? p.scales[n] : 1.f;
            if (p.epi == kEpiSwiGLU) {
                // gate row n (even) and up row n + 1 sit in adjacent lanes
#pragma unroll
                for (int m = 0; m < kTN; m++) {
                    const float val = v[m] * sc;
                    const float up = __shfl_down_sync(0xffffffffu, val, 1);
                    if (m < Mt && (lane & 1) == 0 && n + 1 < p.N) {
                        const float h = silu_f(val) * up;
                        const size_t o = (size_t)(m0 + m) * p.ldc + (n >> 1);
                        p.C[o] = h;
                        if (p.out_hi) {
                            const __nv_bfloat16 hb = __float2bfloat16_rn(h);
                            p.out_hi[o] = hb;
                            p.out_lo[o] = __float2bfloat16_rn(h - __bfloat162float(hb));
                        }
                    }
                }
            } else if (n < p.N) {
                float* c = p.C + (size_t)m0 * p.ldc + n;
                if (p.epi == kEpiResidual) {
#pragma unroll
                    for (int m = 0; m < kTN; m++) v[m] = (m < Mt ? c[(size_t)m * p.ldc] : 0.f) + v[m] * sc;
#pragma unroll
                    for (int m = 0; m < kTN; m++)
                        if (m < Mt) c[(size_t)m * p.ldc] = v[m];
                } else {
#pragma unroll
                    for (int m = 0; m < kTN; m++)
                        if (m < Mt) c[(size_t)m * p.ldc] = v[m] * sc;
                }
            }
        }
    } else if (threadIdx.x == 0 && nch > 0) {
        atomicCAS(p.err, 0, kErrPipeTimeout);
    }
    if constexpr (CL) {
        // every CTA of the cluster passes both barriers, a failed one too
        if (threadIdx.x == 0) cl_ok = ok ? 1u : 0u;
        cluster_sync_all();
        const int S = p.splits;
        const unsigned tb = sbase;
        unsigned rq[kClusterMaxSplits];
        bool all = true;
#pragma unroll
        for (int q = 0; q < kClusterMaxSplits; q++) {
            rq[q] = 0u;
            if (q < S) {
                rq[q] = cl_map(tb, (unsigned)q);
                all = all && cl_ld_u32(cl_map(smem_addr(&cl_ok), (unsigned)q)) != 0u;
            }
        }
        if (all) {
            const int r = (int)cl_rank();
            const int R = (Mt + S - 1) / S;
            const int b0 = r * R, b1 = min(Mt, b0 + R);
            cluster_epilogue(p, rq, S, n0, b0, b1, warp, lane);
        }
        cluster_sync_all();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTN) : "memory");
}

// ---------------------------------------------------------------------------
// Wide tiles for many activation rows (a prompt chunk): one CTA computes
// MB x 128 activation rows (the MMA's M, tensor-memory lanes; MB accumulators
// of 256 columns) x 256 weight rows (the MMA's N) over all of K: 96 KB in per
// 64-wide K step for a weight pair (MB = 1, 3 MMAs per product), 64 KB for
// single bf16 weights.  Same operands and accumulation as above; no split-K.
// The launcher runs it for weight pairs; single bf16 weights (the INT8 model)
// take the persistent form further below.
constexpr int kWM = 128;                 // activation rows per tile
constexpr int kWN = 256;                 // weight rows per tile
constexpr int kWA = kWM * kTK * 2;       // 16 KB per activation half
constexpr int kWW = kWN * kTK * 2;       // 32 KB per weight half
__host__ __device__ constexpr int wide_stage(int wp, int mb) { return mb * 2 * kWA + wp * kWW; }
__host__ __device__ constexpr int wide_stages(int wp, int mb) { return (wp == 1 && mb == 1) ? 3 : 2; }
__host__ __device__ constexpr size_t wide_smem(int wp, int mb) {
    return (size_t)wide_stages(wp, mb) * wide_stage(wp, mb) + 1024;
}
constexpr uint32_t kIdescWide = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kWN >> 3) << 17) |
                                ((uint32_t)(kWM >> 4) << 24);

__device__ __forceinline__ void mma_wide(unsigned tmem, uint64_t adesc, uint64_t bdesc, bool acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.u32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdescWide), "r"((unsigned)acc)
        : "memory");
}

// One warp's staged rows (T: up to 32 rows x 64 columns, row stride 68 floats)
// to the output rows mrow .. mrow + rows - 1, columns nb .. nb + 63: lane j takes
// columns nb + 2j and nb + 2j + 1, so each store instruction covers 256
// contiguous bytes of a row.  The residual form loads 16 rows' old values before
// it stores any of them (the stores could alias later loads, so the compiler
// would otherwise wait out one load latency per row).
__device__ __forceinline__ void wide_store_rows(const TcParams& p, const float* T, int mrow, int rows, int nb,
                                                int lane) {
    const int n = nb + 2 * lane;
    const bool c0ok = n < p.N, c1ok = n + 1 < p.N;
    const float s0 = (p.scales && c0ok) ? p.scales[n] : 1.f;
    const float s1 = (p.scales && c1ok) ? p.scales[n + 1] : 1.f;
    if (p.epi == kEpiResidual) {
        constexpr int kB = 16;
        for (int r0 = 0; r0 < rows; r0 += kB) {
            float2 old[kB];
#pragma unroll
            for (int q = 0; q < kB; q++) {
                old[q] = make_float2(0.f, 0.f);
                if (r0 + q < rows) {
                    const float* c = p.C + (size_t)(mrow + r0 + q) * p.ldc + n;
                    if (c1ok && ((reinterpret_cast<uintptr_t>(c) & 7) == 0)) {
                        old[q] = *reinterpret_cast<const float2*>(c);
                    } else {
                        if (c0ok) old[q].x = c[0];
                        if (c1ok) old[q].y = c[1];
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < kB; q++) {
                if (r0 + q >= rows) break;
                const float2 t2 = *reinterpret_cast<const float2*>(T + (r0 + q) * 68 + 2 * lane);
                const float2 o2 = make_float2(old[q].x + t2.x * s0, old[q].y + t2.y * s1);
                float* c = p.C + (size_t)(mrow + r0 + q) * p.ldc + n;
                if (c1ok && ((reinterpret_cast<uintptr_t>(c) & 7) == 0)) {
                    *reinterpret_cast<float2*>(c) = o2;
                } else {
                    if (c0ok) c[0] = o2.x;
                    if (c1ok) c[1] = o2.y;
                }
            }
        }
        return;
    }
    // 8 rows at a time: their staged values are read before any store (the
    // compiler cannot move shared-memory reads past global stores), so the rows'
    // arithmetic overlaps
    constexpr int kB = 8;
    for (int r0 = 0; r0 < rows; r0 += kB) {
        float2 t2[kB];
#pragma unroll
        for (int q = 0; q < kB; q++)
            t2[q] = r0 + q < rows ? *reinterpret_cast<const float2*>(T + (r0 + q) * 68 + 2 * lane)
                                  : make_float2(0.f, 0.f);
        if (p.epi == kEpiSwiGLU) {
            if (!c1ok) continue;  // gate row n, up row n + 1 -> output n / 2
            float h[kB];
#pragma unroll
            for (int q = 0; q < kB; q++) h[q] = silu_f(t2[q].x * s0) * (t2[q].y * s1);
#pragma unroll
            for (int q = 0; q < kB; q++) {
                if (r0 + q >= rows) break;
                const size_t o = (size_t)(mrow + r0 + q) * p.ldc + (n >> 1);
                if (p.C) p.C[o] = h[q];
                if (p.out_hi) {
                    const __nv_bfloat16 hb = __float2bfloat16_rn(h[q]);
                    p.out_hi[o] = hb;
                    p.out_lo[o] = __float2bfloat16_rn(h[q] - __bfloat162float(hb));
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < kB; q++) {
                if (r0 + q >= rows) break;
                const float g = t2[q].x * s0, u = t2[q].y * s1;
                float* c = p.C + (size_t)(mrow + r0 + q) * p.ldc + n;
                if (c1ok && ((reinterpret_cast<uintptr_t>(c) & 7) == 0)) {
                    *reinterpret_cast<float2*>(c) = make_float2(g, u);
                } else {
                    if (c0ok) c[0] = g;
                    if (c1ok) c[1] = u;
                }
            }
        }
    }
}

// grid (ceil(N / 256), ceil(M / (128 MB))); 128 threads: warp 0 lane 0 issues
// the TMA copies, warp 1 lane 0 the MMAs, all four warps the epilogue (thread =
// activation row m0 + 128 mb + 32 w + lane, 256 weight columns read out 64 at
// a time per row block).
template <int WP, int MB>
__global__ void __launch_bounds__(kTThreads, 1)
    tc_gemm_wide_kernel(const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap tw_lo,
                        const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                        const TcParams p) {
    constexpr int NS = wide_stages(WP, MB);
    constexpr int kStage = wide_stage(WP, MB);
    constexpr int kWOff = MB * 2 * kWA;  // weight tile offset within a stage
    constexpr unsigned kCols = (unsigned)(kWN * MB);
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) unsigned long long full[NS], empty[NS], done;
    __shared__ unsigned tmem_slot;
    __shared__ int fail;
    const unsigned sbase = (smem_addr(smem_raw) + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kWN, m0 = blockIdx.y * kWM * MB;
    const int nch = p.chunks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        mbar_init(smem_addr(&done), 1);
        fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = tmem_slot;
    if (warp == 0 && lane == 0) {
        int issued = 0;
        for (int i = 0; i < nch; i++) {
            const int s = i % NS;
            if (i >= NS &&
                !mbar_wait(smem_addr(&empty[s]), ((unsigned)(i / NS) & 1u) ^ 1u, p.err, nullptr, kSiteEmpty, i)) {
                fail = 1;
                break;
            }
            const unsigned st = sbase + (unsigned)s * kStage;
            const unsigned fb = smem_addr(&full[s]);
            mbar_expect_tx(fb, (unsigned)kStage);
            const int x = i * kTK;
#pragma unroll
            for (int mb = 0; mb < MB; mb++) {
                tma_load_2d(st + mb * 2 * kWA, &ta_hi, x, m0 + mb * kWM, fb);
                tma_load_2d(st + mb * 2 * kWA + kWA, &ta_lo, x, m0 + mb * kWM, fb);
            }
            tma_load_2d(st + kWOff, &tw_hi, x, n0, fb);
            if (WP == 2) tma_load_2d(st + kWOff + kWW, &tw_lo, x, n0, fb);
            issued = i + 1;
        }
        // never leave with copies in flight
        for (int i = issued > NS ? issued - NS : 0; i < issued; i++)
            mbar_drain(smem_addr(&full[i % NS]), (unsigned)(i / NS) & 1u);
    } else if (warp == 1 && lane == 0) {
        for (int i = 0; i < nch && !fail; i++) {
            const int s = i % NS;
            if (!mbar_wait(smem_addr(&full[s]), (unsigned)(i / NS) & 1u, p.err, nullptr, kSiteFull, i)) {
                fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned st = sbase + (unsigned)s * kStage;
#pragma unroll
            for (int kk = 0; kk < kTK / 16; kk++) {
                const uint64_t wh = sw128_desc(st + kWOff + 32u * kk);
#pragma unroll
                for (int mb = 0; mb < MB; mb++) {
                    const unsigned tm = tmem + (unsigned)(mb * kWN);
                    const uint64_t ah = sw128_desc(st + mb * 2 * kWA + 32u * kk);
                    const uint64_t al = sw128_desc(st + mb * 2 * kWA + kWA + 32u * kk);
                    mma_wide(tm, ah, wh, i > 0 || kk > 0);
                    mma_wide(tm, al, wh, true);
                    if (WP == 2) mma_wide(tm, ah, sw128_desc(st + kWOff + kWW + 32u * kk), true);
                }
            }
            mma_commit(smem_addr(&empty[s]));
        }
        mma_commit(smem_addr(&done));
    }
    __syncwarp();
    // committed after the last MMA, also after a failed wait
    bool ok = mbar_drain(smem_addr(&done), 0u);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    ok = __syncthreads_and(ok && !fail);
    if (ok) {
        // Each warp stages its 32 rows x 64 columns in shared memory (the
        // pipeline stages are free now), then writes row by row: lane j takes
        // columns 2j, 2j + 1, so every store instruction covers 256
        // consecutive bytes of one output row.
        float* T = reinterpret_cast<float*>(smem_raw + (sbase - smem_addr(smem_raw))) + warp * 32 * 68;
        for (int blk = 0; blk < MB * (kWN / 64); blk++) {
            const int mb = blk / (kWN / 64), cb = (blk % (kWN / 64)) * 64;
            const int nb = n0 + cb;
            if (nb >= p.N) continue;  // uniform across the CTA
            const int mrow0 = m0 + mb * kWM;
            float v[64];
            tmem_ld64(tmem + ((unsigned)(32 * warp) << 16) + (unsigned)(mb * kWN + cb), v);
#pragma unroll
            for (int j = 0; j < 64; j += 4)
                *reinterpret_cast<float4*>(T + lane * 68 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            __syncwarp();
            wide_store_rows(p, T, mrow0 + 32 * warp, min(32, p.M - (mrow0 + 32 * warp)), nb, lane);
            __syncwarp();
        }
    } else if (threadIdx.x == 0) {
        atomicCAS(p.err, 0, kErrPipeTimeout);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// ---------------------------------------------------------------------------
// Persistent form of the wide tiles (single bf16 weights): one CTA per SM loops
// over 128 x 256 tiles (weight tile fastest, so neighbouring CTAs share the
// activation tile in L2) with two accumulators in tensor memory, so the
// epilogue of one tile overlaps the MMAs of the next.  Warps 0-7: epilogue
// (warp w reads tensor-memory lane quarter w % 4 and the column blocks
// 64 (w / 4) + 128 i, staging in its own shared memory), warp 8 lane 0: TMA
// producer (a 2-stage ring), warp 9 lane 0: MMA issuer.
constexpr int kPersistEpiWarps = 8;
constexpr int kPersistThreads = 32 * (kPersistEpiWarps + 2);
constexpr int kPersistStages = 2;
constexpr int kPersistStage = 2 * kWA + kWW;                       // A_hi, A_lo, W: 64 KB
constexpr int kPersistStaging = kPersistEpiWarps * 32 * 68 * 4;    // epilogue rows, 68 KB
constexpr size_t kPersistSmem = (size_t)kPersistStages * kPersistStage + kPersistStaging + 1024;
static_assert(kPersistSmem + 256 <= 232448, "persistent gemm: shared memory");

// AND of a predicate over the epilogue threads (named barrier 1)
__device__ __forceinline__ bool epilogue_all(bool v) {
    unsigned r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, 1, %2, p; "
        "selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((unsigned)v), "r"(32 * kPersistEpiWarps)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kPersistThreads, 1)
    tc_gemm_persist_kernel(const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap ta_hi,
                           const __grid_constant__ CUtensorMap ta_lo, const TcParams p, int ntn, int ntiles) {
    constexpr int NS = kPersistStages;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) unsigned long long full[NS], empty[NS], acc_full[2], acc_empty[2], done;
    __shared__ unsigned tmem_slot;
    __shared__ int fail;
    const unsigned sbase = (smem_addr(smem_raw) + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.chunks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_addr(&acc_full[b]), 1);
            mbar_init(smem_addr(&acc_empty[b]), 1);
        }
        mbar_init(smem_addr(&done), 1);
        fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(2 * kWN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = tmem_slot;
    const int my_tiles = ntiles > (int)blockIdx.x ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    if (warp == kPersistEpiWarps) {
        if (lane == 0) {
            int g = 0;  // stage counter across tiles
            for (int j = 0; j < my_tiles && !fail; j++) {
                const int tile = (int)blockIdx.x + j * (int)gridDim.x;
                const int n0 = (tile % ntn) * kWN, m0 = (tile / ntn) * kWM;
                for (int i = 0; i < nch; i++, g++) {
                    const int s = g % NS;
                    if (g >= NS &&
                        !mbar_wait(smem_addr(&empty[s]), ((unsigned)(g / NS) & 1u) ^ 1u, p.err, nullptr, kSiteEmpty, g)) {
                        fail = 1;
                        break;
                    }
                    const unsigned st = sbase + (unsigned)s * kPersistStage;
                    const unsigned fb = smem_addr(&full[s]);
                    mbar_expect_tx(fb, (unsigned)kPersistStage);
                    const int x = i * kTK;
                    tma_load_2d(st, &ta_hi, x, m0, fb);
                    tma_load_2d(st + kWA, &ta_lo, x, m0, fb);
                    tma_load_2d(st + 2 * kWA, &tw_hi, x, n0, fb);
                }
            }
            // never leave with copies in flight
            for (int q = g > NS ? g - NS : 0; q < g; q++) mbar_drain(smem_addr(&full[q % NS]), (unsigned)(q / NS) & 1u);
        }
    } else if (warp == kPersistEpiWarps + 1) {
        if (lane == 0) {
            int g = 0;
            for (int j = 0; j < my_tiles && !fail; j++) {
                const int ab = j & 1;
                // the epilogue has read this accumulator's previous tile
                if (j >= 2 && !mbar_wait(smem_addr(&acc_empty[ab]), (unsigned)((j >> 1) - 1) & 1u, p.err, nullptr,
                                         kSiteEmpty, -j)) {
                    fail = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const unsigned tm = tmem + (unsigned)(ab * kWN);
                for (int i = 0; i < nch; i++, g++) {
                    const int s = g % NS;
                    if (!mbar_wait(smem_addr(&full[s]), (unsigned)(g / NS) & 1u, p.err, nullptr, kSiteFull, g)) {
                        fail = 1;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const unsigned st = sbase + (unsigned)s * kPersistStage;
#pragma unroll
                    for (int kk = 0; kk < kTK / 16; kk++) {
                        const uint64_t ah = sw128_desc(st + 32u * kk);
                        const uint64_t al = sw128_desc(st + kWA + 32u * kk);
                        const uint64_t wh = sw128_desc(st + 2 * kWA + 32u * kk);
                        mma_wide(tm, ah, wh, i > 0 || kk > 0);
                        mma_wide(tm, al, wh, true);
                    }
                    mma_commit(smem_addr(&empty[s]));
                }
                mma_commit(smem_addr(&acc_full[ab]));  // (also after a failed wait: releases the epilogue)
            }
            mma_commit(smem_addr(&done));  // completes once no MMA of this CTA is in flight
        }
    } else {
        // epilogue warps
        const int quarter = warp & 3;  // tensor-memory lanes 32 quarter .. + 31
        float* T = reinterpret_cast<float*>(smem_raw + (sbase - smem_addr(smem_raw)) + NS * kPersistStage) +
                   warp * 32 * 68;
        for (int j = 0; j < my_tiles; j++) {
            const int ab = j & 1;
            const bool ok = mbar_wait(smem_addr(&acc_full[ab]), (unsigned)(j >> 1) & 1u, p.err, nullptr, kSiteFull, j);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // one verdict for the epilogue warps (they meet at barrier 1 below)
            if (!epilogue_all(ok && !fail)) break;
            const int tile = (int)blockIdx.x + j * (int)gridDim.x;
            const int n0 = (tile % ntn) * kWN, m0 = (tile / ntn) * kWM;
            for (int cb = 64 * (warp >> 2); cb < kWN; cb += 64 * (kPersistEpiWarps / 4)) {
                const int nb = n0 + cb;
                if (nb >= p.N) break;  // uniform across the warp
                float v[64];
                tmem_ld64(tmem + ((unsigned)(32 * quarter) << 16) + (unsigned)(ab * kWN + cb), v);
#pragma unroll
                for (int q = 0; q < 64; q += 4)
                    *reinterpret_cast<float4*>(T + lane * 68 + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                __syncwarp();
                wide_store_rows(p, T, m0 + 32 * quarter, min(32, p.M - (m0 + 32 * quarter)), nb, lane);
                __syncwarp();
            }
            // this accumulator may take the tile after next
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            asm volatile("bar.sync 1, %0;" ::"r"(32 * kPersistEpiWarps) : "memory");
            if (threadIdx.x == 0) mbar_arrive(smem_addr(&acc_empty[ab]), 1u);
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (fail && threadIdx.x == 0) atomicCAS(p.err, 0, kErrPipeTimeout);
    if (warp == 0) {
        // no MMA may still write the accumulators being released
        if (lane == 0) mbar_drain(smem_addr(&done), 0u);
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kWN) : "memory");
    }
}

// A [M][lda] f32 -> A_hi, A_lo [rows][K] bf16 with A = A_hi + A_lo (rows >= M
// zero).
__global__ void split_bf16_kernel(const float* A, int M, int K, int lda, int rows, __nv_bfloat16* hi,
                                  __nv_bfloat16* lo) {
    const size_t total = (size_t)rows * K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / K), k = (int)(i % K);
        const float x = m < M ? A[(size_t)m * lda + k] : 0.f;
        const __nv_bfloat16 h = __float2bfloat16_rn(x);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(x - __bfloat162float(h));
    }
}

// W [N][K] (f32, or int8 when q8) -> bf16 copies: W_hi (= W exactly for int8)
// and, for f32, W_lo = W - W_hi.
__global__ void weights_bf16_kernel(const void* W, bool q8, size_t total, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        if (q8) {
            hi[i] = __float2bfloat16_rn((float)static_cast<const int8_t*>(W)[i]);
        } else {
            const float x = static_cast<const float*>(W)[i];
            const __nv_bfloat16 h = __float2bfloat16_rn(x);
            hi[i] = h;
            lo[i] = __float2bfloat16_rn(x - __bfloat162float(h));
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

vb_status make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    return tc_make_map(map, base, rows, K, box_rows);
}

}  // namespace

// 2-D bf16 tensor map over [rows][K], boxes of 64 (K) x box_rows, 128-byte swizzle.
vb_status tc_make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VB_ERR_CUDA, "tensor-core gemm: cuTensorMapEncodeTiled failed");
    return VB_OK;
}

int tc_gemm_tiles(int N) { return (N + kTM - 1) / kTM; }

int tc_gemm_splits(int N, int K, bool pair) {
    // as many (tile, split) CTAs as fit in one wave
    const int tiles = (N + kTM - 1) / kTM;
    const int chunks = K / kTK;
    // VB_TC_MAX_SPLITS caps the split-K factor (more splits: more partials to sum)
    static const int max_splits = [] {
        const char* v = getenv("VB_TC_MAX_SPLITS");
        const int m = v ? atoi(v) : 0;
        return m > 0 ? m : 1 << 20;
    }();
    int s = std::min(kTSMs * ctas_per_sm(pair ? 2 : 1) / tiles, max_splits);
    if (s > chunks) s = chunks;
    if (s < 1) s = 1;
    // every split gets at least one chunk
    const int per = (chunks + s - 1) / s;
    return (chunks + per - 1) / per;
}

int cluster_splits(int wp, int tiles, int chunks, int splits);

bool tc_gemm_cluster_reduce(int M, int N, int K, bool pair) {
    if (M < 1 || M > kTN || K % kTK || K <= 0 || N <= 0) return false;
    return cluster_splits(pair ? 2 : 1, (N + kTM - 1) / kTM, K / kTK, tc_gemm_splits(N, K, pair)) > 0;
}

size_t tc_gemm_ws_floats(int M, int N, int K) {
    const int s = std::max(tc_gemm_splits(N, K, false), tc_gemm_splits(N, K, true));
    return (size_t)s * M * N;
}

vb_status launch_split_bf16(const float* A, int M, int K, int lda, void* hi, void* lo, cudaStream_t s,
                            bool pad64) {
    if (M < 1 || K <= 0) return fail(VB_ERR_ARG, "split_bf16: bad shape");
    const int rows = pad64 ? std::max(M, kTN) : M;
    const size_t total = (size_t)rows * K;
    int blocks = (int)((total + 255) / 256);
    if (blocks > kTSMs * 16) blocks = kTSMs * 16;
    split_bf16_kernel<<<blocks, 256, 0, s>>>(A, M, K, lda, rows, static_cast<__nv_bfloat16*>(hi),
                                             static_cast<__nv_bfloat16*>(lo));
    VB_LAUNCH_CHECK("split_bf16_kernel");
    return VB_OK;
}

vb_status launch_weights_bf16(const void* W, bool q8, size_t count, void* hi, void* lo, cudaStream_t s) {
    int blocks = (int)((count + 255) / 256);
    if (blocks > kTSMs * 16) blocks = kTSMs * 16;
    weights_bf16_kernel<<<blocks, 256, 0, s>>>(W, q8, count, static_cast<__nv_bfloat16*>(hi),
                                               static_cast<__nv_bfloat16*>(lo));
    VB_LAUNCH_CHECK("weights_bf16_kernel");
    return VB_OK;
}

// How many (1, cs, 1) clusters of the decode GEMM are resident at once on
// this device (cached per device, weight form and cluster size).
int cluster_capacity(int wp, int cs) {
    static std::atomic<int> cache[8][2][kClusterMaxSplits + 1] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::atomic<int>* slot = dev < 8 ? &cache[dev][wp - 1][cs] : nullptr;
    if (slot) {
        const int v = slot->load();
        if (v) return v;
    }
    {
        // the occupancy query sees the kernel's dynamic shared memory limit
        static std::atomic<unsigned long long> done_pair{0}, done_single{0};
        const cudaError_t ce = wp == 2 ? smem_attr_once(tc_gemm_kernel<2, kPStages, true>, (int)tc_smem(2, kPStages),
                                                        done_pair)
                                       : smem_attr_once(tc_gemm_kernel<1, kQStages, true>, (int)tc_smem(1, kQStages),
                                                        done_single);
        if (ce != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, cs, 1);
    cfg.blockDim = dim3(kTThreads);
    cfg.dynamicSmemBytes = wp == 2 ? tc_smem(2, kPStages) : tc_smem(1, kQStages);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = cs;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t ce = wp == 2 ? cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<2, kPStages, true>, &cfg)
                                   : cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<1, kQStages, true>, &cfg);
    if (ce != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (slot) slot->store(n > 0 ? n : -1);
    return n;
}

// The largest split count <= min(splits, 8) whose clusters (one per tile) are
// all resident at once: a second wave of clusters would double the GEMM (one
// CTA per SM on a B200 holds 33 4-CTA clusters -- the q|k|v GEMM's 32 tiles x
// 4 splits fit -- 45 3-CTA and 15 8-CTA clusters).  Every split gets at least
// one chunk.  0: none fits.
int cluster_splits(int wp, int tiles, int chunks, int splits) {
    for (int cs = std::min(splits, kClusterMaxSplits); cs >= 1; cs--) {
        const int per = (chunks + cs - 1) / cs;
        const int eff = (chunks + per - 1) / per;
        if (cluster_capacity(wp, eff) >= tiles) return eff;
    }
    return 0;
}

vb_status launch_tc_gemm(const TcGemmArgs& a, cudaStream_t s) {
    if (a.M < 1) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: M must be >= 1");
    const int mtiles = (a.M + kTN - 1) / kTN;
    if (mtiles > 65535) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: M too large");
    if (mtiles > 1 && a.partials_only) return fail(VB_ERR_ARG, "tensor-core gemm: partials need M <= 64");
    if (a.K % kTK || a.K <= 0) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: K must be a multiple of 64");
    if (a.N <= 0) return fail(VB_ERR_ARG, "tensor-core gemm: N <= 0");
    const int wp = a.w_lo ? 2 : 1;
    // several activation tiles fill the GPU without split-K
    int splits = mtiles > 1 ? 1 : tc_gemm_splits(a.N, a.K, wp == 2);
    // the q/k norm sums its splits inside a cluster, with a split count whose
    // clusters are all resident at once
    int cl_s = 0;
    if (a.epi == kEpiQkNorm && mtiles == 1 && !a.partials_only)
        cl_s = cluster_splits(wp, (a.N + kTM - 1) / kTM, a.K / kTK, splits);
    const bool cl = cl_s > 0;
    if (cl) splits = cl_s;
    if (a.epi == kEpiQkNorm) {
        if (!cl) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: the q/k norm epilogue needs M <= 64");
        const QkNormArgs* q = a.qk;
        if (!q || q->D != kTM || q->B != a.M || q->rows_per_seq > 0 || q->q_hi || q->k_hi || !q->q_out || !q->pos ||
            !q->kc || !q->vc || a.N != (q->H + 2 * q->KVH) * kTM)
            return fail(VB_ERR_ARG, "tensor-core gemm: q/k norm epilogue arguments");
    }
    if (!cl && (splits > 1 || a.partials_only) && (size_t)splits * a.M * a.N > a.ws_floats)
        return fail(VB_ERR_ARG, "tensor-core gemm: workspace too small");
    {
        static std::atomic<unsigned long long> done_pair{0}, done_single{0}, done_pair_cl{0}, done_single_cl{0};
        cudaError_t ce = wp == 2 ? smem_attr_once(tc_gemm_kernel<2, kPStages, false>, (int)tc_smem(2, kPStages), done_pair)
                                 : smem_attr_once(tc_gemm_kernel<1, kQStages, false>, (int)tc_smem(1, kQStages),
                                                  done_single);
        if (ce == cudaSuccess && cl)
            ce = wp == 2 ? smem_attr_once(tc_gemm_kernel<2, kPStages, true>, (int)tc_smem(2, kPStages), done_pair_cl)
                         : smem_attr_once(tc_gemm_kernel<1, kQStages, true>, (int)tc_smem(1, kQStages), done_single_cl);
        if (ce != cudaSuccess) return cuda_fail(ce, "tensor-core gemm: shared memory attribute");
    }
    CUtensorMap mwh, mwl, mah, mal;
    vb_status st;
    if (a.M >= kWM && a.N >= kWN && !a.partials_only) {
        // many activation rows: wide tiles (boxes within the tensors), no split-K; SwiGLU
        // may write its bf16 split alone
        if (!a.C && !(a.epi == kEpiSwiGLU && a.out_hi && a.out_lo))
            return fail(VB_ERR_ARG, "tensor-core gemm: output missing");
        if (a.epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "tensor-core gemm: swiglu needs even N");
        if (a.M / kWM + 1 > 65535) return fail(VB_ERR_UNSUPPORTED, "tensor-core gemm: M too large");
        if (wp == 1) {
            // single bf16 weights: the persistent form
            static std::atomic<unsigned long long> done_persist{0};
            const cudaError_t ce = smem_attr_once(tc_gemm_persist_kernel, (int)kPersistSmem, done_persist);
            if (ce != cudaSuccess) return cuda_fail(ce, "tensor-core gemm: shared memory attribute");
            if ((st = make_map(&mwh, a.w_hi, a.N, a.K, kWN))) return st;
            if ((st = make_map(&mah, a.a_hi, a.M, a.K, kWM))) return st;
            if ((st = make_map(&mal, a.a_lo, a.M, a.K, kWM))) return st;
            TcParams p{};
            p.M = a.M;
            p.N = a.N;
            p.chunks = a.K / kTK;
            p.per_split = p.chunks;
            p.splits = 1;
            p.scales = a.scales;
            p.C = a.C;
            p.ldc = a.ldc;
            p.epi = a.epi;
            p.out_hi = static_cast<__nv_bfloat16*>(a.out_hi);
            p.out_lo = static_cast<__nv_bfloat16*>(a.out_lo);
            p.err = a.err;
            const int ntn = (a.N + kWN - 1) / kWN, ntm = (a.M + kWM - 1) / kWM;
            const int ntiles = ntn * ntm;
            const int grid = ntiles < kTSMs ? ntiles : kTSMs;
            tc_gemm_persist_kernel<<<grid, kPersistThreads, kPersistSmem, s>>>(mwh, mah, mal, p, ntn, ntiles);
            VB_LAUNCH_CHECK("tc_gemm_persist_kernel");
            return VB_OK;
        }
        // a weight pair (f32 weights as bf16 hi + lo): one CTA per tile
        static std::atomic<unsigned long long> done_wide{0};
        const cudaError_t ce = smem_attr_once(tc_gemm_wide_kernel<2, 1>, (int)wide_smem(2, 1), done_wide);
        if (ce != cudaSuccess) return cuda_fail(ce, "tensor-core gemm: shared memory attribute");
        if ((st = make_map(&mwh, a.w_hi, a.N, a.K, kWN))) return st;
        if ((st = make_map(&mwl, a.w_lo, a.N, a.K, kWN))) return st;
        if ((st = make_map(&mah, a.a_hi, a.M, a.K, kWM))) return st;
        if ((st = make_map(&mal, a.a_lo, a.M, a.K, kWM))) return st;
        TcParams p{};
        p.M = a.M;
        p.N = a.N;
        p.chunks = a.K / kTK;
        p.per_split = p.chunks;
        p.splits = 1;
        p.scales = a.scales;
        p.C = a.C;
        p.ldc = a.ldc;
        p.epi = a.epi;
        p.out_hi = static_cast<__nv_bfloat16*>(a.out_hi);
        p.out_lo = static_cast<__nv_bfloat16*>(a.out_lo);
        p.err = a.err;
        const dim3 grid((a.N + kWN - 1) / kWN, (a.M + kWM - 1) / kWM);
        tc_gemm_wide_kernel<2, 1><<<grid, kTThreads, wide_smem(2, 1), s>>>(mwh, mwl, mah, mal, p);
        VB_LAUNCH_CHECK("tc_gemm_wide_kernel");
        return VB_OK;
    }
    if ((st = make_map(&mwh, a.w_hi, a.N, a.K, kTM))) return st;
    if ((st = make_map(&mwl, wp == 2 ? a.w_lo : a.w_hi, a.N, a.K, kTM))) return st;
    // activations: [max(M, 64)][K] (rows past M of a single tile are read and dropped)
    const int arows = a.M > kTN ? a.M : kTN;
    if ((st = make_map(&mah, a.a_hi, arows, a.K, kTN))) return st;
    if ((st = make_map(&mal, a.a_lo, arows, a.K, kTN))) return st;
    if (!a.C && !a.partials_only && a.epi != kEpiQkNorm) return fail(VB_ERR_ARG, "tensor-core gemm: output missing");
    if (a.epi == kEpiSwiGLU && (a.N % 2)) return fail(VB_ERR_ARG, "tensor-core gemm: swiglu needs even N");
    TcParams p;
    p.M = a.M;
    p.N = a.N;
    p.chunks = a.K / kTK;
    p.per_split = (p.chunks + splits - 1) / splits;
    p.splits = splits;
    p.partials = a.partials_only ? 1 : 0;
    p.P = a.ws;
    p.scales = a.scales;
    p.C = a.C;
    p.ldc = a.ldc;
    p.epi = a.epi;
    p.out_hi = static_cast<__nv_bfloat16*>(a.out_hi);
    p.out_lo = static_cast<__nv_bfloat16*>(a.out_lo);
    p.err = a.err;
    p.qk = a.epi == kEpiQkNorm ? *a.qk : QkNormArgs{};
    const dim3 grid((a.N + kTM - 1) / kTM, splits, mtiles);
    // failure-path test: an armed launch (never one being captured) withholds
    // a stage; the hook word is written and complete before the launch
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    VB_CUDA_TRY(cudaStreamIsCapturing(s, &cs));
    const bool inject = cs == cudaStreamCaptureStatusNone && fault_take(kFaultGemmStage);
    if (inject) {
        VB_CUDA_TRY(set_fault_word(1, s));
        VB_CUDA_TRY(cudaStreamSynchronize(s));
    }
    cudaError_t ce;
    if (cl)
        ce = wp == 2 ? launch_pdl_cluster(tc_gemm_kernel<2, kPStages, true>, grid, kTThreads, tc_smem(2, kPStages),
                                          dim3(1, splits, 1), s, mwh, mwl, mah, mal, p)
                     : launch_pdl_cluster(tc_gemm_kernel<1, kQStages, true>, grid, kTThreads, tc_smem(1, kQStages),
                                          dim3(1, splits, 1), s, mwh, mwl, mah, mal, p);
    else
        ce = wp == 2 ? launch_pdl(tc_gemm_kernel<2, kPStages, false>, grid, kTThreads, tc_smem(2, kPStages), s, mwh,
                                  mwl, mah, mal, p)
                     : launch_pdl(tc_gemm_kernel<1, kQStages, false>, grid, kTThreads, tc_smem(1, kQStages), s, mwh,
                                  mwl, mah, mal, p);
    if (inject) VB_CUDA_TRY(set_fault_word(0, s));
    if (ce != cudaSuccess) return cuda_fail(ce, "tc_gemm_kernel launch");
    if (cl || splits == 1 || a.partials_only) return VB_OK;
    GemmArgs g{};
    g.scales = a.scales;
    g.C = a.C;
    g.M = a.M;
    g.N = a.N;
    g.K = a.K;
    g.ldc = a.ldc;
    g.ws = a.ws;
    g.ws_floats = a.ws_floats;
    g.out_hi = a.out_hi;
    g.out_lo = a.out_lo;
    return launch_gemm_reduce(g, splits, a.scales != nullptr, a.epi, s);
}

}  // namespace vb
