// The whole SwiGLU layer in one persistent kernel.
//
// Phase 1 computes h = SiLU(Wg x + bg) * (Wu x + bu) for this CTA's rows of the
// intermediate dimension; a grid barrier makes all of h visible; phase 2 computes
// y = Wd h + bd + x for this CTA's rows of the hidden dimension (or, tensor
// parallel, sums the ranks' partials over NVLink first). One producer thread per
// CTA streams Wg/Wu rows and then Wd rows through the same ring of shared-memory
// stages without a break, so while the barrier waits for the slowest CTA the
// ring is already filling with phase-2 weights; and there is one launch per
// layer instead of two. Each phase keeps its consumer threads' slice of x (x,
// then h) in registers, as rbulk_kernel does.
#pragma once

#include "kernels.cuh"

namespace swb {

constexpr int kLayerMaxCtas = 1024;
constexpr int kLayerMaxJ = 8;  // 16-byte vectors of a row per consumer thread, each phase

struct LayerParams {
    const __half* wg;
    const __half* wu;
    const __half* wd;
    const __half* x;
    const __half* bg;
    const __half* bu;
    const __half* bd;
    __half* h;
    float* y;
    uint32_t* sync;  // [0]: grid-barrier word (zero before the first call; see layer_kernel)
    int hidden;      // phase 1: inter rows x hidden cols; phase 2: hidden rows x inter cols
    int inter;
    int rs1, rs2;    // whole rows per ring stage in each phase
    int stages;
    int stage_bytes;
};

struct LayerLayout {
    size_t ring, full, empty, part1, part2, total;
};

__host__ __device__ inline LayerLayout layer_layout(int stage_bytes, int stages, int cw, int rpc1, int rpc2) {
    LayerLayout L;
    L.ring = 0;
    L.full = align_up(size_t(stages) * stage_bytes, 16);
    L.empty = L.full + size_t(stages) * 8;
    L.part1 = align_up(L.empty + size_t(stages) * 8, 16);
    L.part2 = align_up(L.part1 + size_t(rpc1) * cw * 2 * 4, 16);
    L.total = align_up(L.part2 + size_t(rpc2) * cw * 4, 16);
    return L;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Loads the vectors t + j*CT (j < kLayerMaxJ) of a length-`cols` fp16 vector into
// registers as fp32; zero beyond the end. `cached_l2_only` reads through L2
// (for data other CTAs wrote during this kernel).
template <int CT>
__device__ __forceinline__ void load_slice(const __half* v, int cols, int t, bool cached_l2_only,
                                           float (&xr)[kLayerMaxJ][8]) {
    const int nv = cols / 8;
    const bool v16 = (reinterpret_cast<uintptr_t>(v) & 15) == 0;
#pragma unroll
    for (int j = 0; j < kLayerMaxJ; ++j) {
        const int q = t + j * CT;
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[j][e] = 0.f;
        if (q < nv) {
            if (v16) {
                const uint4 w = cached_l2_only ? __ldcg(reinterpret_cast<const uint4*>(v) + q)
                                               : *(reinterpret_cast<const uint4*>(v) + q);
                const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = half2_bits_to_float2(w4[k]);
                    xr[j][2 * k] = f.x;
                    xr[j][2 * k + 1] = f.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    xr[j][e] = cached_l2_only ? __half2float(__ldcg(v + size_t(q) * 8 + e)) : __half2float(v[size_t(q) * 8 + e]);
            }
        }
    }
}

template <int CW, int CPS, bool TP>
__global__ void __launch_bounds__((CW + 1) * 32, CPS) layer_kernel(const LayerParams L, const TpParams tp) {
    constexpr int CT = CW * 32;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_failed;
    __shared__ int s_ok;

    const int G = gridDim.x, b = blockIdx.x;
    const int a0 = int((long long)b * L.inter / G), a1 = int((long long)(b + 1) * L.inter / G);
    const int d0 = int((long long)b * L.hidden / G), d1 = int((long long)(b + 1) * L.hidden / G);
    const int nA = a1 - a0, nD = d1 - d0;
    const int units1 = (nA + L.rs1 - 1) / L.rs1, units2 = (nD + L.rs2 - 1) / L.rs2;
    const int rpc1 = (L.inter + G - 1) / G, rpc2 = (L.hidden + G - 1) / G;
    const int stages = L.stages;
    const LayerLayout Y = layer_layout(L.stage_bytes, stages, CW, rpc1, rpc2);
    unsigned char* ring = smem + Y.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Y.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + Y.empty);
    float* part1 = reinterpret_cast<float*>(smem + Y.part1);
    float* part2 = reinterpret_cast<float*>(smem + Y.part2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_failed = 0;
        s_ok = 1;
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), CW);
        }
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch_dependents();

    if (warp == CW) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first_policy();
        int s = 0, issued = 0;
        uint32_t ph = 0;
        for (int k = 0; k < units1 + units2; ++k) {
            if (k >= stages && !mbar_wait(smem_u32(empty + s), ph ^ 1u)) break;
            const uint32_t fb = smem_u32(full + s);
            unsigned char* dst = ring + size_t(s) * L.stage_bytes;
            if (k < units1) {
                const int row = a0 + k * L.rs1;
                const int ru = min(L.rs1, a1 - row);
                const uint32_t bytes = uint32_t(ru) * uint32_t(L.hidden) * 2u;
                mbar_arrive_expect_tx(fb, 2u * bytes);
                const size_t goff = size_t(row) * L.hidden;
                bulk_copy_g2s(smem_u32(dst), L.wg + goff, bytes, fb, pol);
                bulk_copy_g2s(smem_u32(dst + size_t(L.rs1) * L.hidden * 2), L.wu + goff, bytes, fb, pol);
            } else {
                const int row = d0 + (k - units1) * L.rs2;
                const int ru = min(L.rs2, d1 - row);
                const uint32_t bytes = uint32_t(ru) * uint32_t(L.inter) * 2u;
                mbar_arrive_expect_tx(fb, bytes);
                bulk_copy_g2s(smem_u32(dst), L.wd + size_t(row) * L.inter, bytes, fb, pol);
            }
            ++issued;
            if (++s == stages) { s = 0; ph ^= 1u; }
        }
        const int drain = issued < stages ? issued : stages;
        for (int j = 1; j <= drain; ++j) {
            const int k = issued - j;
            if (!mbar_wait(smem_u32(full + (k % stages)), uint32_t((k / stages) & 1))) break;
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int t = threadIdx.x;
    griddep_wait();  // x may be the previous kernel's output
    // Tensor parallel: every CTA reads this call's exchange epoch before it reaches
    // the grid barrier; CTA 0 stores it after the barrier.
    const uint32_t xe0 = (TP && t == 0) ? *reinterpret_cast<volatile const uint32_t*>(tp.ctr) : 0u;
    float xr[kLayerMaxJ][8];
    int s = 0;
    uint32_t ph = 0;

    // ---- phase 1: gate rows [a0, a1)
    load_slice<CT>(L.x, L.hidden, t, false, xr);
    // Both phases reduce RG rows at once (stage_rows); RG is chosen from the
    // vectors per thread, once per phase, so each loop keeps only the part of
    // xr it reads in registers.
    auto phase = [&](auto nm, auto rg, auto jv, int units, int base, int first, int last, int rsx, int cols,
                     float* part) {
        constexpr int NM = decltype(nm)::value, RG = decltype(rg)::value, J = decltype(jv)::value;
        const int nv = cols / 8;
        for (int k = 0; k < units; ++k) {
            if (!mbar_wait(smem_u32(full + s), ph)) { s_failed = 1; break; }
            const int row0 = first + k * rsx;
            const int ru = min(rsx, last - row0);
            const __half* sw = reinterpret_cast<const __half*>(ring + size_t(s) * L.stage_bytes);
            stage_rows<CW, kLayerMaxJ, NM, RG, J>(sw, ru, rsx, cols, nv, xr, part, row0 - base);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(empty + s));
            if (++s == stages) { s = 0; ph ^= 1u; }
        }
    };
    using I1 = std::integral_constant<int, 1>;
    using I2 = std::integral_constant<int, 2>;
    using I4 = std::integral_constant<int, 4>;
    using I8 = std::integral_constant<int, 8>;
    using IJ = std::integral_constant<int, kLayerMaxJ>;
    {
        const int jn = (L.hidden / 8 + CT - 1) / CT;
        if (jn <= 1) phase(I2{}, I4{}, I1{}, units1, a0, a0, a1, L.rs1, L.hidden, part1);
        else if (jn <= 2) phase(I2{}, I2{}, I2{}, units1, a0, a0, a1, L.rs1, L.hidden, part1);
        else phase(I2{}, I1{}, IJ{}, units1, a0, a0, a1, L.rs1, L.hidden, part1);
    }
    named_barrier_sync(1, CT);
    if (s_failed) return;
    for (int i = t; i < nA; i += CT) {
        float ga = 0.f, ub = 0.f;
        for (int j = 0; j < CW; ++j) {
            ga += part1[(size_t(i) * CW + j) * 2];
            ub += part1[(size_t(i) * CW + j) * 2 + 1];
        }
        if (L.bg) ga += __half2float(L.bg[a0 + i]);
        if (L.bu) ub += __half2float(L.bu[a0 + i]);
        L.h[a0 + i] = __float2half_rn(silu(ga) * ub);
    }

    // ---- grid barrier: all of h written and visible (bounded wait). One word:
    // CTA 0 adds 2^31 - (G - 1), every other CTA adds 1, so the adds of one
    // barrier sum to 2^31 and the word's top bit flips exactly when the last CTA
    // arrives (its low 31 bits stay zero between barriers, whatever the grid).
    // Each CTA waits for the top bit to differ from the one it saw on arrival: a
    // single L2 round trip per poll, instead of one per CTA of the grid.
    named_barrier_sync(1, CT);
    if (t == 0) {
        __threadfence();  // this CTA's h (ordered before by the CTA barrier) visible at gpu scope
        const uint32_t add = b == 0 ? 0x80000000u - uint32_t(G - 1) : 1u;
        const uint32_t seen = atomicAdd(L.sync, add) & 0x80000000u;
        const uint64_t t0 = global_timer_ns();
        while ((ld_acquire_gpu(L.sync) & 0x80000000u) == seen) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_device_error, 1);
                s_ok = 0;
                break;
            }
        }
        __threadfence();
    }
    const uint32_t xe = xe0 + 1u;  // this call's epoch (read before the barrier, used after it)
    if (TP && b == 0 && t == 0) *reinterpret_cast<volatile uint32_t*>(tp.ctr) = xe;
    named_barrier_sync(1, CT);
    if (!s_ok) return;

    // ---- phase 2: down rows [d0, d1) against h
    load_slice<CT>(L.h, L.inter, t, true, xr);
    {
        const int jn = (L.inter / 8 + CT - 1) / CT;
        if (jn <= 1) phase(I1{}, I8{}, I1{}, units2, d0, d0, d1, L.rs2, L.inter, part2);
        else if (jn <= 2) phase(I1{}, I4{}, I2{}, units2, d0, d0, d1, L.rs2, L.inter, part2);
        else phase(I1{}, I1{}, IJ{}, units2, d0, d0, d1, L.rs2, L.inter, part2);
    }
    named_barrier_sync(1, CT);
    if (s_failed) return;

    if constexpr (!TP) {
        for (int i = t; i < nD; i += CT) {
            float a = 0.f;
            for (int j = 0; j < CW; ++j) a += part2[size_t(i) * CW + j];
            if (L.bd) a += __half2float(L.bd[d0 + i]);
            a += __half2float(L.x[d0 + i]);
            L.y[d0 + i] = a;
        }
    } else {
        // The exchange of rbulk_allreduce_kernel: partial rows to every rank, rank-ordered sum.
        __shared__ uint32_t s_xe;
        if (t == 0) s_xe = xe;
        named_barrier_sync(1, CT);
        tp_exchange_rows<CT>(tp, s_xe, L.hidden, d0, nD, L.y, [&](int i) {
            float a = 0.f;
            for (int j = 0; j < CW; ++j) a += part2[size_t(i) * CW + j];
            return a;
        });
    }
}

}  // namespace swb
