// wf_ptx.cuh - inline-PTX wrappers for sm_100a used by the MoE kernels:
// mbarriers, bulk (TMA) copies global->shared, warp MMA, and the packed
// FP4 / FP8 conversions.  Every wait is bounded; see wf_wait().
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace wf {

// A device-side wait gives up after this many SM clock cycles (~1-2 s at
// B200 clocks) and reports kErrTimeout instead of hanging the GPU.  Waits on
// another role's progress take the limit the launch carries (this value unless
// the host lowered it, see wf_set_wait_limit); waits for a copy or MMA this
// thread issued itself (the drains before a CTA exits or frees TMEM) always
// take this one, so a CTA never leaves with its own operations in flight.
constexpr long long kWaitLimitCycles = 2000000000LL;

// bits of the device error word
constexpr int kErrTimeout = 1;
constexpr int kErrExpertId = 2;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of the phase with `parity`.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity` to complete.  On timeout sets
// kErrTimeout in *err and returns false.  With the default bound the thread
// blocks in try_wait between checks of the clock; a lowered bound is kept to
// the cycle by polling without blocking (try_wait may suspend the thread for
// longer than a short bound).
__device__ __forceinline__ bool wf_wait(uint64_t *bar, uint32_t parity, int *err,
                                        long long limit = kWaitLimitCycles) {
    if (limit < kWaitLimitCycles) {
        const long long t0 = clock64();
        while (!mbar_test_wait(bar, parity)) {
            if (clock64() - t0 > limit) {
                atomicOr(err, kErrTimeout);
                return false;
            }
        }
        return true;
    }
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) {
            atomicOr(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

// ---- bulk copy (TMA, non-tensor) global -> shared, completes on mbarrier --
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- programmatic dependent launch --------------------------------------
// Lets the next kernel on the stream start launching (its CTAs run their
// prologue) while this one drains.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Blocks until the previous kernel on the stream has completed and its memory
// writes are visible; returns at once when launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- named barrier among the consumer warps -----------------------------
__device__ __forceinline__ void bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- shared / global vector loads ----------------------------------------
__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ uint4 ldg128(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// L2-coherent load (skips L1) for data other CTAs of the same launch wrote.
__device__ __forceinline__ uint4 ldcg128(const void *p) {
    return __ldcg(reinterpret_cast<const uint4 *>(p));
}

// ---- warp MMA m16n8k16, f16 inputs, f32 accumulate -----------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- packed conversions ----------------------------------------------------
// 4 bytes of packed E2M1 (8 codes, low nibble first) -> 4 x f16x2; element
// 2i of the word lands in the low half of o[i].
__device__ __forceinline__ void fp4x8_to_f16x8(uint32_t w, uint32_t (&o)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w));
}

// 2 bytes of e4m3 (low byte = lower element) -> f16x2
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
    uint32_t o;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(o) : "h"(v));
    return o;
}

// two floats -> e4m3x2 (round to nearest even, saturating to +-448);
// `lo` lands in the low byte.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
    uint16_t o;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(o) : "f"(hi), "f"(lo));
    return o;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

// e8m0 byte -> float (2^(b-127); b = 0 gives the subnormal 2^-127)
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
    return __uint_as_float(b ? (b << 23) : 0x00400000u);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) {
    return __uint_as_float(b16 << 16);
}

}  // namespace wf
