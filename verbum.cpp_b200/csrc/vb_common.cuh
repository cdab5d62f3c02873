// vb_common.cuh -- shared device/host helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "verbum_b200.h"

namespace vb {

// ---------------------------------------------------------------------------
// host-side error plumbing: every C-ABI call returns a vb_status; the message
// of the last failure on the calling thread is kept for vb_last_error().
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
vb_status fail(vb_status code, const std::string& msg);
vb_status cuda_fail(cudaError_t e, const char* what);

#define VB_CUDA_TRY(expr)                                         \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return ::vb::cuda_fail(_e, #expr); \
    } while (0)

#define VB_LAUNCH_CHECK(what)                                     \
    do {                                                          \
        cudaError_t _e = cudaGetLastError();                      \
        if (_e != cudaSuccess) return ::vb::cuda_fail(_e, what);  \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Failure-path test hook (vb_debug_arm_fault): the site armed for the next
// launch.  fault_take(site) returns true once -- for the first launch of that
// site after arming -- and disarms it.
enum FaultSite : int { kFaultNone = 0, kFaultStepExchange = 1, kFaultGemmStage = 2 };
bool fault_take(int site);

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 2^x by the PTX ex2.approx instruction (relative error ~2^-22, -inf -> +0)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Warp sums of NV values at once (NV a power of two <= 32): a transposed
// butterfly -- at each of the first log2(NV) xor steps a lane sends half of its
// values and keeps the other half -- then plain xor steps.  Returns, in every
// lane, the warp-wide sum of value lane >> (5 - log2(NV)): NV - 1 + 5 - log2(NV)
// shuffles in all instead of 5 * NV.
template <int NV>
__device__ __forceinline__ float warp_sum_scatter(float (&v)[NV], int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV: a power of two <= 32");
    int mask = 16;
#pragma unroll
    for (int n = NV; n > 1; n >>= 1, mask >>= 1) {
        const bool upper = lane & mask;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
    }
    float r = v[0];
#pragma unroll
    for (; mask > 0; mask >>= 1) r += __shfl_xor_sync(0xffffffffu, r, mask);
    return r;
}

// Thread-block cluster helpers: barrier over the cluster, this CTA's rank,
// and loads from a peer CTA's shared memory (distributed shared memory).
// (the non-.aligned barrier forms: no assumption that the warp has reconverged)
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ unsigned cl_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cl_map(unsigned local, unsigned rank) {
    unsigned r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ float cl_ld(unsigned addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ unsigned cl_ld_u32(unsigned addr) {
    unsigned v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// Streaming 16-byte global load that does not allocate in L1 (weights and KV
// rows are touched exactly once per step).
__device__ __forceinline__ float4 ld_stream_f4(const void* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Exact int8 -> f32 for the four signed bytes of `w` without I2F.
// Each biased byte u = b + 128 is dropped into the low mantissa bits of
// 2^23 (bit pattern 0x4B000000), giving the float 2^23 + u exactly; one
// subtraction of 2^23 + 128 then leaves b exactly.  This is the standard
// "magic number" integer-to-float construction (IEEE-754 binary32 has a
// 23-bit mantissa, so every integer below 2^24 is representable).
// Position of x[i] inside a GEMV's shared copy of its input.  INT8 lanes
// load 16 consecutive weights; storing the matching activations
// lane-interleaved per 512-element chunk makes every lane's float4 reads
// bank-conflict free.
template <bool Q8>
__device__ __forceinline__ int xs_index(int i) {
    if (!Q8) return i;
    const int c = i >> 9, r = i & 511;
    const int l = r >> 4, j = (r >> 2) & 3, e = r & 3;
    return (c << 9) + (j << 7) + (l << 2) + e;
}

struct f4 {
    float v[4];
};
__device__ __forceinline__ f4 i8x4_to_f32(uint32_t w) {
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;  // 2^23 + 128
    f4 r;
    r.v[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - bias;
    r.v[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - bias;
    r.v[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - bias;
    r.v[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - bias;
    return r;
}

// Packed f32x2 arithmetic (sm_100): two lanes of f32 math per instruction,
// each lane rounded exactly like the scalar operation.
typedef unsigned long long f2;
__device__ __forceinline__ f2 f2pack(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float f2sum(f2 v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}
__device__ __forceinline__ void f2unpack(f2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 f2fma(f2 a, f2 b, f2 c) {
    f2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f2 f2sub(f2 a, f2 b) {
    f2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2 f2mul(f2 a, f2 b) {
    f2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// 4 int8 -> two exact f32 pairs (q0, q1), (q2, q3): each byte is placed in
// the mantissa of 2^23 (after a bias of 128) and the offset subtracted.
__device__ __forceinline__ void i8x4_to_f2(uint32_t w, f2& lo, f2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const f2 bias = f2pack(8388736.0f, 8388736.0f);  // 2^23 + 128
    lo = f2sub(f2pack(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                      __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), bias);
    hi = f2sub(f2pack(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                      __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), bias);
}

// Block-wide double sum for blockDim.x == NT (multiple of 32). `red` holds
// NT/32 doubles. Every thread gets the total.
template <int NT>
__device__ __forceinline__ double block_sum_d(double v, double* red) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < NT / 32; i++) t += red[i];
    __syncthreads();
    return t;
}

// RMSNorm scale exactly as the reference computes it (nn.cpp:31-34):
// double sum of squares -> float mean + eps -> 1/sqrt in float.
__device__ __forceinline__ float rms_scale(double sumsq, int dim, float eps) {
    const float mean = (float)(sumsq / (double)dim);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// ---------------------------------------------------------------------------
// device-side error word: bounded waits record where they gave up instead of
// spinning forever; the host reads it after the step.
// ---------------------------------------------------------------------------
enum : int {
    kErrNone = 0,
    kErrBarrierTimeout = 1,
    kErrPipeTimeout = 2,
    kErrBadToken = 3,
    kErrCacheFull = 4,
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch: kernels on the decode paths are launched so
// that the next kernel can start (be scheduled, run its prologue) while its
// predecessor drains.  Each such kernel calls pdl_trigger() (lets its own
// successor launch once every CTA got here) and pdl_wait() before it touches
// anything an earlier kernel wrote; launched the ordinary way, both are
// no-ops.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// launch_pdl with thread-block clusters of the given shape
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, dim3 cluster,
                               cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = cluster.x;
    at[1].val.clusterDim.y = cluster.y;
    at[1].val.clusterDim.z = cluster.z;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace vb
