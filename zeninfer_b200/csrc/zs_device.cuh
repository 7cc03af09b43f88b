// zs_device.cuh -- sm_100a building blocks of the sampler kernels.
//
// Keys.  A candidate (value v, token id i) is packed into one uint64:
//     key = ord(v) << 32 | ~i
// ord() maps floats to uint32 monotonically with -0 == +0 and NaN below -inf,
// so "key a > key b" is exactly "a ranks before b" in the shortlist order
// value-descending, id-ascending.  Keys of real tokens are never 0, so 0 is the
// "accept everything" threshold and the empty/removed marker.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace zs {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t ord_of(float v) {
    if (v != v) return 0u;
    if (v == 0.0f) v = 0.0f;
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float value_of_ord(uint32_t o) {
    if (o == 0u) return __int_as_float(0x7fc00000);
    uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t make_key(float v, int32_t id) {
    return ((uint64_t)ord_of(v) << 32) | (uint64_t)(~(uint32_t)id);
}

__device__ __forceinline__ int32_t key_id(uint64_t k) { return (int32_t)(~(uint32_t)k); }
__device__ __forceinline__ float key_value(uint64_t k) { return value_of_ord((uint32_t)(k >> 32)); }

// ---- xorshift64* (zen::Rng, src/sample.cpp:15-22) ----
__device__ __forceinline__ uint64_t rng_next(uint64_t& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 2685821657736338717ull;
}
__device__ __forceinline__ double rng_uniform(uint64_t& s) {
    return (double)(rng_next(s) >> 11) * (1.0 / 9007199254740992.0);
}

// ---- programmatic dependent launch ----
// A kernel launched with programmatic stream serialization may start while the
// kernel before it in the stream is still running; grid_dep_wait() returns once
// that kernel has completed and its memory writes are visible.  Without that launch
// attribute it returns at once.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Lets the next kernel in the stream (if launched as above) be scheduled now; it
// still reads nothing of this kernel's before its grid_dep_wait().
__device__ __forceinline__ void grid_dep_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- shared-memory addresses, mbarriers and the bulk-copy engine ----
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every wait in these kernels gives up after this long and reports
// ZS_ERR_DEVICE_TIMEOUT instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// try_wait that may suspend the thread for up to hint_ns before returning false.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for an mbarrier phase; false when the limit ran out.  Meant for
// one thread per CTA (others sleep on a named barrier meanwhile).  Backs off
// with nanosleep so a waiting thread does not take issue slots from the warps
// doing the work.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    uint32_t ns = 32;
    while (!mbar_try_wait(bar, parity)) {
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// 1-D bulk copy global -> shared (no tensor map, no multicast), completion
// signalled as transaction bytes on `bar`.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before its
// later async-proxy ones (a bulk copy into a buffer the warp has just read).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// L2 policy for data read exactly once: evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier over the consumer warps only (the producer warp never joins).
// bar.sync is the .aligned form: every lane of a warp must execute it together.
// The compiler does not see inline asm as a barrier and does not reconverge a
// warp before it, so __syncwarp() does that first; without it, lanes leaving a
// divergent branch (or a bounded wait) at different times would arrive
// separately and the barrier's count would go wrong.
template <int NT>
__device__ __forceinline__ void consumer_sync() {
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// consumer_sync that also ORs a predicate over the consumer threads; every
// thread gets the same result.  A decision taken from shared state that other
// threads may still be changing (a counter that later appends bump) must come
// through here, never from each thread reading the state on its own after a
// plain barrier: fast threads would act on a value slow threads never see.
template <int NT>
__device__ __forceinline__ bool consumer_sync_or(bool pred) {
    __syncwarp();
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(NT)
        : "memory");
    return r != 0;
}

// Asks L2 for the 128-byte line holding p (no register, no wait).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace zs
