// Device helpers for sm_100a: streaming loads, bulk async copies, mbarriers
// with bounded waits, fp16 unpacking and the SiLU activation.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace swb {

// Upper bound for any wait on an mbarrier. A legitimate wait lasts at most the
// latency of one bulk copy (microseconds); past this the kernel records
// SWB_DEVERR_TIMEOUT in the device error word and stops instead of hanging.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Device error word of the translation unit that includes this header (one per
// shared library); read and cleared by swb_device_error().
static __device__ int g_device_error = 0;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Timeline points of the streaming kernels, called by one thread of a CTA:
// 0 entry, 1 first ring stage landed, 2 last stage consumed, 3 results written,
// 4 the producer's last copy issued. A profiling build defines SWB_TIMELINE to
// record when each CTA passes each point; the library leaves it empty.
#ifndef SWB_TIMELINE
#define SWB_TIMELINE(point) ((void)0)
#endif

// ---------------------------------------------------------------- loads

// 128-bit read-only streaming load: weights are read exactly once, so skip L1.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_stream_b32(const void* p) {
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = bits;
    return __half22float2(h);
}

// ------------------------------------------------------------- mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of `bar` with the given parity to complete. Gives up
// after kWaitLimitNs, raising SWB_DEVERR_TIMEOUT, and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, 1);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------- bulk async copy

// L2 policy for data read exactly once (weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Global -> shared bulk copy completing on an mbarrier (non-multicast).
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// Programmatic dependent launch. launch_dependents lets the next kernel in the
// stream (launched with the programmatic-serialization attribute) start early;
// wait blocks until every kernel this one depends on has completed and its
// memory is visible. Both are no-ops when no programmatic dependency exists.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------- cluster launch control
// Work stealing on sm_100: try_cancel asks the hardware to cancel a CTA of this
// grid that has not started yet and writes a 16-byte response into shared memory,
// completing `bar` with 16 transaction bytes. The response says whether a CTA was
// cancelled and, if so, its blockIdx -- whose work the caller then does itself.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
    asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];"
                 ::"r"(resp), "r"(bar) : "memory");
}

// Orders generic-proxy accesses to shared memory against async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Decodes a try_cancel response: returns the cancelled CTA's x index, or -1 when
// no CTA was left to cancel.
__device__ __forceinline__ int clc_decode(const uint4& r) {
    const unsigned long long lo = (unsigned long long)r.x | ((unsigned long long)r.y << 32);
    const unsigned long long hi = (unsigned long long)r.z | ((unsigned long long)r.w << 32);
    uint32_t ok, x;
    asm volatile(
        "{\n\t.reg .b128 rr;\n\t.reg .pred p;\n\t"
        "mov.b128 rr, {%2, %3};\n\t"
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, rr;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, rr;\n\t}"
        : "=r"(ok), "=r"(x)
        : "l"(lo), "l"(hi)
        : "memory");
    return ok ? int(x) : -1;
}

// Named barrier among the first `threads` threads of the CTA (id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------ peer-memory signals
// Upper bound for waiting on another GPU's flag (a peer that died or never
// launched): the kernel records SWB_DEVERR_PEER_TIMEOUT and skips its output.
constexpr uint64_t kPeerWaitLimitNs = 1000000000ull;

// Release store at system scope: every store this CTA made before the preceding
// barrier is visible to whoever acquires this flag, on any GPU.
// One exchange slot: an fp32 value and the call epoch that wrote it, stored as one
// aligned 64-bit word. An aligned scalar 64-bit access is single-copy atomic, so a
// reader that sees the epoch also sees the value: no fence or separate flag is
// needed, on this GPU or across NVLink.
__device__ __forceinline__ void st_slot_sys(unsigned long long* p, float v, uint32_t epoch) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_slot_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Waits (bounded) until the slot holds the value written in `epoch`. On time-out it
// records SWB_DEVERR_PEER_TIMEOUT and returns false.
__device__ __forceinline__ bool wait_slot(const unsigned long long* p, uint32_t epoch, float& v) {
    unsigned long long w = ld_slot_sys(p);
    if (uint32_t(w >> 32) != epoch) {
        const uint64_t t0 = global_timer_ns();
        do {
            if (global_timer_ns() - t0 > kPeerWaitLimitNs) {
                atomicOr(&g_device_error, 2);
                return false;
            }
            w = ld_slot_sys(p);
        } while (uint32_t(w >> 32) != epoch);
    }
    v = __uint_as_float(uint32_t(w));
    return true;
}

// ----------------------------------------------------------- activation

// SiLU(v) = v / (1 + exp(-v)), written in two branches so exp never overflows
// (the same stable form as include/kernels.cuh:18-21 of the reference).
__device__ __forceinline__ float silu(float v) {
    if (v >= 0.f) return v / (1.f + expf(-v));
    const float e = expf(v);
    return v * e / (1.f + e);
}

__device__ __forceinline__ float round_half(float v) { return __half2float(__float2half_rn(v)); }

}  // namespace swb
