// common.cuh — shared device helpers for the sm_100a kernels.
//
// mbarrier + bulk-copy (TMA, non-tensor, this CTA's shared memory only) primitives written as
// inline PTX, bounded waits that report through an error word instead of
// trapping, and small math helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace leap {

// Error codes written to the context's device error word.
enum DeviceError : int {
    kDevOk = 0,
    kDevWaitTimeout = 1,   // an mbarrier wait gave up
    kDevBadIndex = 2,      // a bounds check failed
};

// A wait gives up after kMaxWaitPolls polls or kMaxWaitNs of elapsed time
// (GPU global timer), whichever comes first.  Each try_wait poll blocks for
// a hardware-chosen interval at most; no suspend-time hint is given (a hint
// of 1 us measured 1.6 % slower on the decode kernel: the thread may sleep
// past the phase completion).
constexpr uint32_t kMaxWaitPolls = 1u << 22;
constexpr unsigned long long kMaxWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch: wait until the preceding kernel of the
// stream has completed and its memory is visible (a no-op when this kernel
// was launched without the attribute) ...
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// ... and allow the next kernel of the stream to begin launching.
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Order generic-proxy global accesses with async-proxy (bulk copy) ones.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Atomic add with acquire-release semantics at GPU scope: publishes the
// writes ordered before it and observes the writes published by earlier
// release operations on the same counter.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                 : "=r"(old)
                 : "l"(p), "r"(v)
                 : "memory");
    return old;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
            smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// Wait until the phase with the given parity has completed.  Returns false
// (and the caller reports kDevWaitTimeout) after kMaxWaitPolls polls or
// kMaxWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    unsigned long long t0 = 0;
    for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255) == 0) {
            const unsigned long long t = global_ns();
            if (i == 0) t0 = t;
            else if (t - t0 > kMaxWaitNs) return false;
        }
    }
    return false;
}

// Non-blocking test: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// One-dimensional bulk copy global -> shared (TMA engine), completing
// `bytes` of transaction count on `bar`.  src/dst 16-byte aligned, bytes a
// multiple of 16.  The destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem,
                                         uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Report a device-side error once (first writer wins).
__device__ __forceinline__ void report_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// report_error, and the code also stored (plainly) to a host-mapped word
// when the caller waits on the host for this kernel (err_host non-null).
__device__ __forceinline__ void report_error(int *err, int *err_host, int code) {
    report_error(err, code);
    if (err_host) *reinterpret_cast<volatile int *>(err_host) = code;
}

constexpr float kLog2e = 1.4426950408889634f;

// Interleaved-pair RoPE rotation with separately rounded products, as the
// reference's AVX2 branch computes it (x*c, swap(x)*s, addsub;
// src/inference/FloatTransformer.cpp:461-464):
//   (x0*c - x1*s, x1*c + x0*s), no fused multiply-add.
__device__ __forceinline__ float2 rope_pair(float x0, float x1, float c, float s) {
    float2 r;
    r.x = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    r.y = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    return r;
}

}  // namespace leap
