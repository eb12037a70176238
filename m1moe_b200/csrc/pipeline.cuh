// pipeline.cuh — sm_100a primitives for the shared-memory weight pipelines:
// 1-D bulk async copies (cp.async.bulk, the TMA engine's linear mode) that
// complete on an mbarrier, bounded mbarrier waits, L2 eviction hints and
// Programmatic Dependent Launch (griddepcontrol).
//
// Every CTA fetches its own tiles from this GPU's memory; no copy is shared
// between CTAs.
#pragma once

#include <stdint.h>

namespace m1 {

// Device error word bits (m1moe_cuda_synchronize reports them as M1MOE_ERR_DEVICE).
constexpr int kErrWaitTimeout = 1;   // an mbarrier wait exceeded its iteration limit
constexpr int kErrBadIndex = 2;      // a token id or a KV position was out of range (dense step)
constexpr int kErrRange = 4;         // a value left the fp16 range of the tensor-core operands

// A wait gives up after this many try_wait polls (each poll may suspend the
// thread for a hardware-defined interval), i.e. far longer than any copy.
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  On timeout
// the CTA's abort flag and the device error word are set and false returned;
// callers then stop consuming and unwind.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          int *err) {
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    if (err) atomicOr(err, kErrWaitTimeout);
    return false;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Linear bulk copy global -> this CTA's shared memory; completes `bytes` of
// transaction count on `bar`.  dst, src 16-byte aligned; bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (no data is consumed, so it
// is safe ahead of any dependency wait).  src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic Dependent Launch: wait until the preceding grid in the stream
// has completed and its memory is visible (a no-op without a PDL predecessor);
// allow the following grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Phase tracing: when `trace` is non-null, slot [cta][event] receives the SM
// cycle counter (exact within a CTA), and slots 20/21 the global nanosecond
// timer at events 0 and 10, which places each CTA on a common time axis and
// gives the cycle length (off by default; m1moe_cuda_set_trace).
constexpr int kTraceEvents = 20;
constexpr int kTraceSlots = 32;
constexpr int kTraceCtas = 160;
__device__ __forceinline__ void trace_event(unsigned long long *trace, int kernel, int event) {
    if (trace == nullptr || blockIdx.x >= kTraceCtas) return;
    unsigned long long *row = trace + ((size_t)kernel * kTraceCtas + blockIdx.x) * kTraceSlots;
    const unsigned long long c = clock64();
    row[event] = c;
    if (event == 0 || event == 10) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        row[event == 0 ? 20 : 21] = t;
    }
}

// A value (not a time) into trace slot `slot` of this CTA's row.
__device__ __forceinline__ void trace_value(unsigned long long *trace, int kernel, int slot,
                                            unsigned long long v) {
    if (trace == nullptr || blockIdx.x >= kTraceCtas) return;
    trace[((size_t)kernel * kTraceCtas + blockIdx.x) * kTraceSlots + slot] = v;
}

// Named barrier `id` for `nthreads` threads (a multiple of 32), whichever
// warps they are.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrive at named barrier `id` without waiting (the waiting side calls
// named_sync with the same thread count).
__device__ __forceinline__ void named_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// floor(n / d) for 0 <= n < 2^31 and a divisor d >= 1 known on the host:
// n * m >> k with m = ceil(2^k / d), k = 31 + ceil(log2 d) (the round-up
// multiplier of Granlund and Montgomery, "Division by invariant integers
// using multiplication", PLDI 1994: the error m*n/2^k - n/d < 1/d never
// reaches the next integer).  A runtime integer division is a long
// dependent instruction chain; this is one wide multiply.
struct FastDiv {
    unsigned long long m;
    int k;
};

__device__ __forceinline__ int fdiv(int n, const FastDiv &f) {
    return (int)(((unsigned long long)(unsigned)n * f.m) >> f.k);
}

inline FastDiv make_fastdiv(int d) {
    int l = 0;
    while ((1LL << l) < d) ++l;
    const int k = 31 + l;
    return FastDiv{((1ULL << k) + (unsigned long long)d - 1) / (unsigned long long)d, k};
}

// Named barrier that also ANDs a predicate over the participating threads.
__device__ __forceinline__ bool named_sync_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, %3, p; "
        "selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// A [begin, end) byte range rounded out to 16-byte boundaries for a bulk copy;
// `skew` is the offset of the wanted bytes inside the copied range.
struct Span16 {
    const uint8_t *src;
    uint32_t bytes;
    uint32_t skew;
};

__device__ __forceinline__ Span16 span16(const uint8_t *p, size_t n) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t a0 = a & ~uintptr_t(15), a1 = (a + n + 15) & ~uintptr_t(15);
    return {reinterpret_cast<const uint8_t *>(a0), static_cast<uint32_t>(a1 - a0),
            static_cast<uint32_t>(a - a0)};
}

}  // namespace m1
