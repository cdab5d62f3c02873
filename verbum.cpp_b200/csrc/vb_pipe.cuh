// vb_pipe.cuh -- PTX building blocks of the persistent decode kernels:
// mbarrier waits with a %globaltimer bound, TMA bulk copies, named barriers,
// error recording.  Included into one anonymous namespace per kernel file.
#pragma once

#include "vb_common.cuh"

namespace vb {
namespace {

constexpr unsigned long long kWaitNs = 2000000000ull;  // every wait gives up after 2 s

// Test hook for the failure paths, armed from the host for exactly one launch
// (vb_debug_arm_fault): non-zero makes the armed kernel wait for something
// nothing will produce -- an exchange word no CTA writes, a stage no copy
// fills -- so one of its bounded waits runs out, it records the timeout and
// returns, and the host reports VB_ERR_TIMEOUT.  Each kernel file has its own
// copy (this header is compiled into each); zero in normal operation.
__device__ int g_fault_arm = 0;
__device__ __forceinline__ bool fault_armed() { return *reinterpret_cast<volatile int*>(&g_fault_arm) != 0; }
// Host side: sets this file's hook word on `s` (ordered with the launch).
inline cudaError_t set_fault_word(int v, cudaStream_t s) {
    return cudaMemcpyToSymbolAsync(g_fault_arm, &v, sizeof(int), 0, cudaMemcpyHostToDevice, s);
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ unsigned smem_addr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(unsigned a, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned a, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned a, unsigned count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned a, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ int err_read(const int* err) {
    return *reinterpret_cast<const volatile int*>(err);
}
// Wait sites recorded in the debug words when a bounded wait gives up.
enum Site : int { kSiteEmpty = 1, kSiteFull = 2, kSiteAttFull = 3, kSiteGrid = 4 };

// First failure wins: sets the error word and, if it was the first, records
// where the kernel gave up.
__device__ __noinline__ void record_fail(int* err, int* dbg, int code, int site, int index, int extra) {
    if (atomicCAS(err, 0, code) == 0 && dbg) {
        dbg[1] = blockIdx.x;
        dbg[2] = site;
        dbg[3] = index;
        dbg[4] = extra;
        __threadfence();
        dbg[0] = code;
    }
}

// Bounded wait for the phase of parity `parity` of mbarrier `a` to complete.
// The spin loops are kept out of line: the persistent kernels run every wait
// site once per layer and their code has to stay small.
__device__ __noinline__ bool mbar_wait_slow(unsigned a, unsigned parity, int* err, int* dbg, int site, int index) {
    const unsigned long long t0 = now_ns();
    for (unsigned it = 1;; it++) {
        if (mbar_try(a, parity)) return true;
        if ((it & 255u) == 0) {
            if (err_read(err)) return false;
            if (now_ns() - t0 > kWaitNs) {
                record_fail(err, dbg, kErrPipeTimeout, site, index, (int)parity);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_wait(unsigned a, unsigned parity, int* err, int* dbg, int site, int index) {
    return mbar_try(a, parity) || mbar_wait_slow(a, parity, err, dbg, site, index);
}
// Bounded wait that does NOT give up when the error word is set: a CTA that
// is leaving (after its own or another CTA's failure) uses it to let the bulk
// copies and tensor-core operations it issued land first, since its shared
// and tensor memory go to the next CTA once it exits.  Only the time bound
// ends it early.
__device__ __noinline__ bool mbar_drain(unsigned a, unsigned parity) {
    const unsigned long long t0 = now_ns();
    for (unsigned it = 1;; it++) {
        if (mbar_try(a, parity)) return true;
        if ((it & 255u) == 0 && now_ns() - t0 > kWaitNs) return false;
    }
}
// Bounded wait until the previous round of `slot` (stage s - kStages) has been
// observed by a consumer (or this round already has, by another warp sharing
// the stage).
__device__ __noinline__ bool seq_wait_slow(volatile int* seq, int slot, int s, int stages, int* err, int* dbg) {
    const int want = s - stages;
    const unsigned long long t0 = now_ns();
    for (unsigned it = 1;; it++) {
        if (seq[slot] >= want) return true;
        if ((it & 255u) == 0) {
            if (err_read(err)) return false;
            if (now_ns() - t0 > kWaitNs) {
                record_fail(err, dbg, kErrPipeTimeout, 5, s, seq[slot]);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool seq_wait(volatile int* seq, int slot, int s, int stages, int* err, int* dbg) {
    return seq[slot] >= s - stages || seq_wait_slow(seq, slot, s, stages, err, dbg);
}

// Warp-uniform wait: lane 0 waits (bounded) and broadcasts the outcome; on
// success the other lanes observe the already-completed phase themselves so
// that each of them acquires the stage's contents.
__device__ bool warp_wait(unsigned a, unsigned parity, int* err, int* dbg, int index,
                          volatile int* seq, int slot, int stages) {
    const int lane = threadIdx.x & 31;
    int ok = 1;
    if (lane == 0) {
        ok = (seq_wait(seq, slot, index, stages, err, dbg) &&
              mbar_wait(a, parity, err, dbg, kSiteFull, index)) ? 1 : 0;
        if (ok) {
            seq[slot] = index;
            __threadfence_block();
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok && lane != 0) {
        for (int i = 0; i < 1024 && !mbar_try(a, parity); i++) {
        }
    }
    return ok != 0;
}

__device__ __forceinline__ void bulk_g2s(unsigned dst, const void* src, unsigned bytes,
                                         unsigned mbar, unsigned long long pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(mbar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
template <int NT = 256>
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}
// Named barrier over the consumer threads that also ANDs a per-thread flag,
// so every consumer thread leaves with the same decision.
template <int NT = 256>
__device__ __forceinline__ bool consumers_sync_and(bool v) {
    unsigned r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, 1, %2, p; selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((unsigned)v), "n"(NT)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}


}  // namespace
}  // namespace vb
