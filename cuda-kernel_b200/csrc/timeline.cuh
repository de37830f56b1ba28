// Timeline measurement build (make timeline -> lib/libswiglu_b200_timeline.so).
// Force-included ahead of swiglu_b200.cu: it defines SWB_TIMELINE so that each
// CTA of the streaming kernels records %globaltimer at the points device.cuh
// lists, and appends a ring-depth sweep around the tuned geometries to the
// registry (ids 150-162). The product library is built without this file.
//
// Records: one per CTA, in the order CTAs start (a ticket taken at entry).
// words 0-6: globaltimer (ns) at points 0-6 (0 if the CTA never passed it);
// word 7: blockIdx.x | gridDim.x << 16 | %smid << 32 | blockDim.x << 48.
// Capacity: kTimelineCap CTAs; later CTAs are not recorded.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define SWB_EXTRA_CONFIGS(X)                     \
    X(151, SWB_FAM_RBULK, 8, 2, 8, 8, 16384, 3)  \
    X(152, SWB_FAM_RBULK, 16, 1, 8, 4, 32768, 3) \
    X(154, SWB_FAM_RBULK, 16, 1, 8, 4, 32768, 5) \
    X(156, SWB_FAM_SBULK, 8, 2, 8, 8, 16384, 2)  \
    X(157, SWB_FAM_SBULK, 16, 1, 8, 4, 32768, 4) \
    X(159, SWB_FAM_BULK, 8, 2, 8, 1, 2048, 12)   \
    X(160, SWB_FAM_RBULK, 4, 2, 8, 8, 8192, 8)   \
    X(162, SWB_FAM_BULK, 4, 2, 8, 1, 4096, 2)

namespace swb_timeline {
constexpr unsigned kTimelineCap = 65536;
constexpr unsigned kTimelineWords = 8;
__device__ unsigned long long g_records[kTimelineCap * kTimelineWords];
__device__ unsigned int g_ticket;

// The CTA's record slot, taken by the thread that passes point 0.
__device__ __forceinline__ unsigned int& cta_slot() {
    __shared__ unsigned int slot;
    return slot;
}

__device__ __forceinline__ void point(int pt) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (pt == 0) {
        unsigned int smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        const unsigned int s = atomicAdd(&g_ticket, 1u);
        cta_slot() = s;
        if (s < kTimelineCap)
            g_records[size_t(s) * kTimelineWords + 7] =
                (unsigned long long)blockIdx.x | ((unsigned long long)gridDim.x << 16) |
                ((unsigned long long)smid << 32) | ((unsigned long long)blockDim.x << 48);
    }
    const unsigned int s = cta_slot();
    if (s < kTimelineCap && pt >= 0 && pt < 7) g_records[size_t(s) * kTimelineWords + pt] = t;
}
}  // namespace swb_timeline

#define SWB_TIMELINE(pt) ::swb_timeline::point(pt)

// Host side: clear the records, and copy them out (after a device synchronise).
extern "C" __attribute__((visibility("default"))) int swb_timeline_reset(void) {
    static unsigned long long zeros[swb_timeline::kTimelineCap * swb_timeline::kTimelineWords];
    const unsigned int z = 0;
    if (cudaMemcpyToSymbol(swb_timeline::g_ticket, &z, sizeof z) != cudaSuccess) return 1;
    if (cudaMemcpyToSymbol(swb_timeline::g_records, zeros, sizeof zeros) != cudaSuccess) return 1;
    return 0;
}

extern "C" __attribute__((visibility("default"))) int swb_timeline_read(void* out, unsigned int* count) {
    if (cudaDeviceSynchronize() != cudaSuccess) return 1;
    if (cudaMemcpyFromSymbol(count, swb_timeline::g_ticket, sizeof(unsigned int)) != cudaSuccess) return 1;
    if (cudaMemcpyFromSymbol(out, swb_timeline::g_records, sizeof(swb_timeline::g_records)) != cudaSuccess)
        return 1;
    return 0;
}

extern "C" __attribute__((visibility("default"))) int swb_timeline_capacity(void) {
    return int(swb_timeline::kTimelineCap);
}
