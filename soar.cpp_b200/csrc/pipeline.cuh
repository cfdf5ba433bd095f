// Device helpers shared by the streaming kernels: bf16 conversions, mbarrier
// waits with a time limit, 1D bulk async copies (cp.async.bulk, never with
// cluster multicast), and the consumer-only named barrier.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace soarb {
namespace {

// ------------------------------------------------------------ bf16 helpers --

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Two fp32 -> packed bf16x2, round to nearest even (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// -------------------------------------------------- mbarrier / bulk copies --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// Bounded wait for the phase of `bar` with the given parity to complete. Gives
// up after limit_ns of %globaltimer (setting *s_err), or as soon as another
// thread has set *s_err.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* s_err,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 1023u) == 0) {
            if (global_timer_ns() - t0 > limit_ns) {
                atomicOr(s_err, 1);
                return false;
            }
            if (*reinterpret_cast<volatile int*>(s_err)) return false;  // another thread gave up
        }
    }
}
// global -> shared, completes `bytes` of transaction on `bar`
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// shared -> global, tracked by the issuing thread's bulk groups
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// all but the newest N committed groups have finished reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// System-scope release store / acquire load (peer flags over NVLink).
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_f64(double* p, double v) {
    asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ double ld_relaxed_sys_f64(const double* p) {
    double v;
    asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until flags[q] >= epoch for every q < n (local memory written
// by peers). Returns false, setting *err, after limit_ns.
__device__ __forceinline__ bool wait_flags(const uint64_t* flags, int n, uint64_t epoch, int* err,
                                           uint64_t limit_ns = kWaitLimitNs) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        bool all = true;
        for (int q = 0; q < n; ++q) all = all && (ld_acquire_sys(flags + q) >= epoch);
        if (all) return true;
        if (i == 0) t0 = global_timer_ns();
        if ((i & 255u) == 255u && global_timer_ns() - t0 > limit_ns) {
            atomicOr(err, 1);
            return false;
        }
    }
}

// Programmatic dependent launch (griddepcontrol, sm_90+). Every kernel of the
// step is launched with programmatic stream serialization (launch_pdl), so it
// may be scheduled while the kernel before it on the stream drains; it calls
// pdl_wait() before touching global memory, which returns once that kernel
// has completed and its writes are visible (immediately when there is none).
// pdl_trigger() lets the next kernel be scheduled as this one's CTAs retire.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier 1 over the kThreadsN consumer threads only.
template <int kThreadsN>
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kThreadsN) : "memory");
}

}  // namespace
}  // namespace soarb
