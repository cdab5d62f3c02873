// vb_tc.cuh -- the 5th-generation tensor-core building blocks shared by the
// GEMMs (vb_tcgemm.cu) and the prompt attention (vb_prefill.cu): 2-D TMA
// loads into shared memory, 128-byte-swizzle K-major shared-memory matrix
// descriptors, tcgen05.mma (kind::f16, bf16 in, f32 accumulate in tensor
// memory), commit to an mbarrier and the 32-lane x 64-column tensor-memory
// read-out.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "vb_pipe.cuh"

namespace vb {

__device__ __forceinline__ void tma_load_2d(unsigned dst, const CUtensorMap* map, int x, int y, unsigned mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 bytes,
// 8-row groups 1024 bytes apart (the canonical layout TMA's 128-byte swizzle
// writes).  Fields: start >> 4 [0,14), leading offset [16,30) (unused for
// swizzled K-major, 1), stride offset >> 4 [32,46), version 1 [46,48),
// layout type 2 = 128-byte swizzle [61,64).
__device__ __forceinline__ uint64_t sw128_desc(unsigned saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator [4,6) = 1, A bf16 [7,10) = 1,
// B bf16 [10,13) = 1, both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(unsigned tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.u32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((unsigned)acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(unsigned mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}

// 64 consecutive f32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld64(unsigned taddr, float* v) {
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
}

// 32 consecutive f32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld32(unsigned taddr, float* v) {
    unsigned* r = reinterpret_cast<unsigned*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D bf16 tensor map over [rows][cols], boxes of 64 columns x box_rows rows,
// 128-byte swizzle (vb_tcgemm.cu).
vb_status tc_make_map(CUtensorMap* map, const void* base, int rows, int cols, int box_rows);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) holds for the current
// device only: set it once per device (bit d of `done`) before the kernel's
// first launch there.
template <typename Kernel>
cudaError_t smem_attr_once(Kernel* kern, int bytes, std::atomic<unsigned long long>& done) {
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return ce;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (ce == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return ce;
}

}  // namespace vb
