// device_common.cuh -- sm_100a device helpers shared by the GEMV and
// dequantization kernels: shared-memory addressing, mbarrier + bulk-copy (TMA
// engine) primitives, programmatic dependent launch, bounded waits, and
// NexusLLM's fp16 decoder.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nexus_gpu {

// Device-side status word (one per loaded module and device).  Kernels OR
// error bits into it instead of trapping; the host reads and clears it with
// nexus_gpu_device_status().  The library is one translation unit
// (nexus_gpu.cu), so the definition lives here.
enum : unsigned {
    kStatusWaitTimeout = 1u,   // an mbarrier wait exceeded its time limit
};
__device__ unsigned g_device_status = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts16(uint32_t a, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(v) : "memory");
}

// N consecutive 32-bit words starting at a 2-byte-aligned shared address q.
// Reads N+1 aligned words from q & ~3 and realigns them with byte permutes
// (selector 0x3210 when q is 4-aligned, 0x5432 when it is 2 mod 4).  The
// caller guarantees that the word after the data is inside the allocation.
template <int N>
__device__ __forceinline__ void lds_words_2a(uint32_t q, uint32_t (&out)[N]) {
    const uint32_t base = q & ~3u;
    const uint32_t sel = (q & 2u) ? 0x5432u : 0x3210u;
    uint32_t w[N + 1];
#pragma unroll
    for (int k = 0; k <= N; ++k) w[k] = lds32(base + 4 * k);
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = __byte_perm(w[k], w[k + 1], sel);
}

// NexusLLM's fp16 -> fp32 decoder, bit for bit (include/quantization.hpp:59-70):
// bits = sign | (((h & 0x7fff) << 13) + (0x70 << 23)); exponent 0x1f -> +0.0.
// Zero and subnormal halves are not special-cased (0x0000 -> 2^-15).
__device__ __forceinline__ float nexus_fp16(uint32_t h) {
    const uint32_t v = (((h & 0x7fffu) << 13) + 0x38000000u) | ((h & 0x8000u) << 16);
    return ((h & 0x7c00u) == 0x7c00u) ? 0.0f : __uint_as_float(v);
}
// Same decoder applied to the high half of a 32-bit word (no shift needed
// for the sign, which is already in bit 31).
__device__ __forceinline__ float nexus_fp16_hi(uint32_t w) {
    const uint32_t v = (((w >> 3) & 0x0fffe000u) + 0x38000000u) | (w & 0x80000000u);
    return ((w & 0x7c000000u) == 0x7c000000u) ? 0.0f : __uint_as_float(v);
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking form: never suspends the thread (for loops that poll other
// work while they wait).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `ns` nanoseconds pass, instead of spinning on the issue
// slots its warp's scheduler shares with working warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase with the given parity, for at most `limit_ns`.  On
// timeout the status word records it and false is returned; the caller then
// stops issuing work and leaves.  No trap, no unbounded spin.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legal wait
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t k = 1;; ++k) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((k & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {  // the clock is read rarely
            atomicOr(&g_device_status, kStatusWaitTimeout);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared through the TMA engine, completing on an
// mbarrier transaction count.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// ------------------------------------------------ programmatic dependent launch
// Block until the grids this one depends on have completed and their writes
// are visible (a no-op when the launch had no programmatic dependency).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to begin launching.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ------------------------------------------------------------ int8 dot products
// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four weight bytes w (elements e..e+3) against int16 x pairs v0 = (x[e],
// x[e+1]) and v1 = (x[e+2], x[e+3]): two dp2a, full 16-bit x in one pass.
// _u: unsigned weight bytes; _s: signed.
__device__ __forceinline__ int dpx_u(uint32_t w, uint32_t v0, uint32_t v1, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(v0), "r"(w), "r"(c));
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(v1), "r"(w), "r"(d));
    return d;
}
__device__ __forceinline__ int dpx_s(uint32_t w, uint32_t v0, uint32_t v1, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(v0), "r"(w), "r"(c));
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(v1), "r"(w), "r"(d));
    return d;
}

}  // namespace nexus_gpu
