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
    uint32_t* sync;  // [0]: grid-barrier word (zero before the first call; see layer_kernel);
                     // stream_layer_kernel: [1] CTAs done, [kStreamCountBase + c] rows of h block c
    int hidden;      // phase 1: inter rows x hidden cols; phase 2: hidden rows x inter cols
    int inter;
    int rs1, rs2;    // whole rows per ring stage in each phase (stream_layer_kernel: rs1 only)
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


// ====================================================== streaming whole layer
//
// stream_layer_kernel (layer ids 220+): the whole layer in one persistent kernel
// with no grid barrier. Phase 1 gives CTA b the gate rows b, b + G, b + 2G, ... so
// that the grid writes h in ascending order; phase 2 gives CTA b the contiguous
// rows [d0, d1) of y and streams them block by block: a ring stage holds the
// block's CB columns of each of the CTA's rows (CB = 8 * CT / RSPLIT elements of h).
// Warps: CW consumers; one producer thread streaming Wg/Wu rows, then Wd blocks,
// through one ring without a break; and two warps that keep every global round
// trip off the ring's path. The signal warp takes each finished gate stage's row
// sums (shared memory), writes the stage's h rows and counts them in the words of
// their blocks -- a fence, then a relaxed add, one stage later, once the stores
// have landed, so the fence costs little. The loader warp, from the kernel's start,
// waits (bounded) for each block's word to say all its h elements are written and
// copies the block into this CTA's shared copy of h, releasing a one-shot mbarrier
// per block; the consumers of a block wait on that barrier only.
// A CTA therefore waits only for the blocks the slowest CTAs are still producing,
// while it streams and multiplies the others. Consumer thread t owns vector
// t mod (CT / RSPLIT) of a block and rows t div (CT / RSPLIT) + RSPLIT * i, each
// accumulated in a register across blocks; at the end each row is reduced over
// its threads in a fixed order, so the result is deterministic. The last CTA to
// finish resets the block words (and, tensor parallel, advances the exchange epoch
// every CTA read at its start), so calls need no clearing; after a device error
// zero the words again. Launched cooperatively, or programmatically after the
// kernel before it in the stream (SWB_PREFETCH_WEIGHTS): then the grid is no larger
// than what fits at once, and a CTA that is not yet resident only makes others wait.
constexpr int kLayerWorkspaceWords = 2048;  // SWB_LAYER_WORKSPACE_BYTES / 4
constexpr int kStreamCountBase = 64;       // first block word in LayerParams::sync
constexpr int kStreamMaxBlocks = kLayerWorkspaceWords - kStreamCountBase;
constexpr int kStreamMaxInter = 16384;     // h held whole in shared memory (fp16)

struct StreamLayout {
    size_t ring, full, empty, gdone, hready, hsm, bias, part1, part2, total;
};

// rpc1 / rpc2: most gate rows / y rows of one CTA; units1: most gate stages of one CTA;
// nblk: blocks of h; inter: elements of h.
__host__ __device__ inline StreamLayout stream_layout(int stage_bytes, int stages, int cw, int rpc1, int rpc2,
                                                      int units1, int nblk, int inter) {
    StreamLayout Y;
    Y.ring = 0;
    Y.full = align_up(size_t(stages) * stage_bytes, 16);
    Y.empty = Y.full + size_t(stages) * 8;
    Y.gdone = Y.empty + size_t(stages) * 8;                 // one per gate stage: its CW warps are done
    Y.hready = Y.gdone + size_t(units1) * 8;                // one per block: copied into hsm (loader warp)
    Y.hsm = align_up(Y.hready + size_t(nblk) * 8, 16);      // [inter] fp16: this CTA's copy of h
    Y.bias = align_up(Y.hsm + size_t(inter) * 2, 16);       // [row][bg, bu] of the gate rows
    Y.part1 = align_up(Y.bias + size_t(rpc1) * 2 * 4, 16);        // [row][warp][gate, up]
    Y.part2 = align_up(Y.part1 + size_t(rpc1) * cw * 2 * 4, 16);  // [row][warp]
    Y.total = align_up(Y.part2 + size_t(rpc2) * cw * 4, 16);
    return Y;
}

// Waits (bounded) until *p >= target. On time-out records SWB_DEVERR_TIMEOUT, returns false.
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t target) {
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(p) < target) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, 1);
            return false;
        }
    }
    return true;
}

template <int CW, int CPS, int RSPLIT, int MAXR, bool TP>
__global__ void __launch_bounds__((CW + 3) * 32, CPS) stream_layer_kernel(const LayerParams L, const TpParams tp) {
    constexpr int CT = CW * 32;
    constexpr int VPB = CT / RSPLIT;  // 16-byte vectors of a block row = threads per row slot
    constexpr int CB = VPB * 8;       // h elements (Wd columns) per block
    static_assert(VPB % 32 == 0, "a row slot is whole warps");
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_failed;

    const int G = gridDim.x, b = blockIdx.x;
    const int H = L.hidden, I = L.inter;
    const int nA = b < I ? (I - b + G - 1) / G : 0;  // gate rows b + k G, k < nA
    const int d0 = int((long long)b * H / G), d1 = int((long long)(b + 1) * H / G);
    const int nD = d1 - d0;
    const int rs1 = L.rs1;
    const int units1 = (nA + rs1 - 1) / rs1;
    const int nblk = (I + CB - 1) / CB;
    const int rpc1 = (I + G - 1) / G, rpc2 = (H + G - 1) / G;
    const int stages = L.stages;
    const StreamLayout Y = stream_layout(L.stage_bytes, stages, CW, rpc1, rpc2, (rpc1 + rs1 - 1) / rs1, nblk, I);
    unsigned char* ring = smem + Y.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Y.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + Y.empty);
    uint64_t* gdone = reinterpret_cast<uint64_t*>(smem + Y.gdone);
    uint64_t* hready = reinterpret_cast<uint64_t*>(smem + Y.hready);
    __half* hsm = reinterpret_cast<__half*>(smem + Y.hsm);
    float* sbias = reinterpret_cast<float*>(smem + Y.bias);
    float* part1 = reinterpret_cast<float*>(smem + Y.part1);
    float* part2 = reinterpret_cast<float*>(smem + Y.part2);
    uint32_t* blk = L.sync + kStreamCountBase;
    uint32_t* ctas_done = L.sync + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_failed = 0;
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), CW);
        }
        for (int j = 0; j < units1; ++j) mbar_init(smem_u32(gdone + j), CW);
        for (int c = 0; c < nblk; ++c) mbar_init(smem_u32(hready + c), 1);
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
        for (int k = 0; k < units1 + nblk; ++k) {
            if (k >= stages && !mbar_wait(smem_u32(empty + s), ph ^ 1u)) break;
            const uint32_t fb = smem_u32(full + s);
            unsigned char* dst = ring + size_t(s) * L.stage_bytes;
            if (k < units1) {  // gate rows b + (k rs1 + i) G, i < ru: Wg at [i], Wu at [rs1 + i]
                const int ru = min(rs1, nA - k * rs1);
                const uint32_t bytes = uint32_t(H) * 2u;
                mbar_arrive_expect_tx(fb, 2u * uint32_t(ru) * bytes);
                for (int i = 0; i < ru; ++i) {
                    const size_t goff = size_t(b + (k * rs1 + i) * G) * H;
                    bulk_copy_g2s(smem_u32(dst + size_t(i) * bytes), L.wg + goff, bytes, fb, pol);
                    bulk_copy_g2s(smem_u32(dst + size_t(rs1 + i) * bytes), L.wu + goff, bytes, fb, pol);
                }
            } else {  // columns [c CB, c CB + seg) of rows d0 .. d1 - 1 of Wd, row r at [r CB]
                const int c0 = (k - units1) * CB;
                const uint32_t seg = uint32_t(min(CB, I - c0)) * 2u;
                mbar_arrive_expect_tx(fb, uint32_t(nD) * seg);
                for (int r = 0; r < nD; ++r)
                    bulk_copy_g2s(smem_u32(dst + size_t(r) * CB * 2), L.wd + size_t(d0 + r) * I + c0, seg, fb, pol);
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

    if (warp == CW + 1) {
        // ------------------------------------------------------- signal warp
        // each gate stage's h rows (lane i: row i of the stage), written now and counted one
        // stage later: fence (the stores have long landed), then a relaxed add
        int pend = -1;
        for (int j = 0; j < units1; ++j) {
            if (!mbar_wait(smem_u32(gdone + j), 0u)) break;
            if (pend >= 0) {
                __threadfence();
                atomicAdd(blk + pend / CB, 1u);
                pend = -1;
            }
            const int ru = min(rs1, nA - j * rs1);
            if (lane < ru) {
                const int kk = j * rs1 + lane, row = b + kk * G;
                float ga = sbias[2 * kk], ub = sbias[2 * kk + 1];
                for (int w = 0; w < CW; ++w) {
                    ga += part1[(size_t(kk) * CW + w) * 2];
                    ub += part1[(size_t(kk) * CW + w) * 2 + 1];
                }
                L.h[row] = __float2half_rn(silu(ga) * ub);
                pend = row;
            }
        }
        if (pend >= 0) {
            __threadfence();
            atomicAdd(blk + pend / CB, 1u);
        }
        return;
    }

    if (warp == CW + 2) {
        // ------------------------------------------------------- loader warp
        // The block words of this call start at zero only once the kernel before has ended
        // (the last CTA of the previous call resets them): wait for it first.
        griddep_wait();
        for (int c = 0; c < nblk; ++c) {
            const int c0 = c * CB;
            const int seg = min(CB, I - c0);
            if (!__all_sync(0xffffffffu, wait_at_least(blk + c, uint32_t(seg)))) break;
            for (int q = lane; q < seg / 8; q += 32)
                reinterpret_cast<uint4*>(hsm + c0)[q] = __ldcg(reinterpret_cast<const uint4*>(L.h + c0) + q);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(hready + c));  // release: the block's copies first
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int t = threadIdx.x;
    for (int k = t; k < nA; k += CT) {  // biases do not depend on the previous kernel
        const int row = b + k * G;
        sbias[2 * k] = L.bg ? __half2float(L.bg[row]) : 0.f;
        sbias[2 * k + 1] = L.bu ? __half2float(L.bu[row]) : 0.f;
    }
    griddep_wait();  // x may be the previous kernel's output
    const uint32_t xe = TP ? *reinterpret_cast<volatile const uint32_t*>(tp.ctr) + 1u : 0u;  // this call's epoch
    named_barrier_sync(1, CT);  // sbias complete before the signal warp reads it (gdone orders the rest)
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;

    // ---- phase 1: gate rows b + k G; each warp reports a finished stage to the signal warp
    {
        float xr[kLayerMaxJ][8];
        load_slice<CT>(L.x, H, t, false, xr);
        const int nv = H / 8;
        auto gate = [&](auto rg, auto jv) {
            constexpr int RG = decltype(rg)::value, J = decltype(jv)::value;
            for (int k = 0; k < units1; ++k) {
                if (!mbar_wait(smem_u32(full + s), ph)) { ok = false; break; }
                const int ru = min(rs1, nA - k * rs1);
                const __half* sw = reinterpret_cast<const __half*>(ring + size_t(s) * L.stage_bytes);
                stage_rows<CW, kLayerMaxJ, 2, RG, J>(sw, ru, rs1, H, nv, xr, part1, k * rs1);
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(empty + s));
                    mbar_arrive(smem_u32(gdone + k));  // release: this warp's partials of the stage
                }
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
        };
        using I1 = std::integral_constant<int, 1>;
        using I2 = std::integral_constant<int, 2>;
        using I4 = std::integral_constant<int, 4>;
        using IJ = std::integral_constant<int, kLayerMaxJ>;
        const int jn = (nv + CT - 1) / CT;
        if (jn <= 1) gate(I4{}, I1{});
        else if (jn <= 2) gate(I2{}, I2{});
        else gate(I1{}, IJ{});
    }

    // ---- phase 2: rows [d0, d1) of Wd, block by block as h fills
    const int rslot = t / VPB, v = t % VPB;
    float acc[MAXR];
#pragma unroll
    for (int i = 0; i < MAXR; ++i) acc[i] = 0.f;
    for (int c = 0; ok && c < nblk; ++c) {
        if (!mbar_wait(smem_u32(full + s), ph) || !mbar_wait(smem_u32(hready + c), 0u)) {
            ok = false;
            break;
        }
        const int seg = min(CB, I - c * CB);
        if (v * 8 < seg) {
            const uint4 hv = *reinterpret_cast<const uint4*>(hsm + size_t(c) * CB + size_t(v) * 8);
            const uint32_t h4[4] = {hv.x, hv.y, hv.z, hv.w};
            float hf[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = half2_bits_to_float2(h4[q]);
                hf[2 * q] = f.x;
                hf[2 * q + 1] = f.y;
            }
            const __half* sw = reinterpret_cast<const __half*>(ring + size_t(s) * L.stage_bytes);
#pragma unroll
            for (int i = 0; i < MAXR; ++i) {
                const int r = rslot + RSPLIT * i;
                if (r < nD) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(sw + size_t(r) * CB + size_t(v) * 8);
                    const uint32_t u4[4] = {wv.x, wv.y, wv.z, wv.w};
                    float a = acc[i];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 f = half2_bits_to_float2(u4[q]);
                        a = fmaf(f.x, hf[2 * q], a);
                        a = fmaf(f.y, hf[2 * q + 1], a);
                    }
                    acc[i] = a;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(empty + s));
        if (++s == stages) { s = 0; ph ^= 1u; }
    }
    if (!ok) s_failed = 1;
    // each row over its slot's VPB threads: warp sums, then the slot's warps in order
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
        const float a = warp_sum(acc[i]);
        const int r = rslot + RSPLIT * i;
        if (lane == 0 && r < nD) part2[size_t(r) * CW + (v >> 5)] = a;
    }
    named_barrier_sync(1, CT);
    if (!s_failed) {
        auto row = [&](int i) {
            float a = 0.f;
            for (int j = 0; j < VPB / 32; ++j) a += part2[size_t(i) * CW + j];
            return a;
        };
        if constexpr (!TP) {
            for (int i = t; i < nD; i += CT) {
                float a = row(i);
                if (L.bd) a += __half2float(L.bd[d0 + i]);
                a += __half2float(L.x[d0 + i]);
                L.y[d0 + i] = a;
            }
        } else {
            tp_exchange_rows<CT>(tp, xe, H, d0, nD, L.y, row);
        }
    }
    // The last CTA to get here resets the block words (every CTA's loader warp has passed
    // its waits: the consumers took every block it copied) and, tensor parallel, advances
    // the exchange epoch every CTA read at its start.
    named_barrier_sync(1, CT);
    if (t == 0) {
        __threadfence();
        if (atomicAdd(ctas_done, 1u) == uint32_t(G - 1)) {
            for (int c = 0; c < nblk; ++c) blk[c] = 0u;
            *ctas_done = 0u;
            if (TP) *reinterpret_cast<volatile uint32_t*>(tp.ctr) = xe;
            __threadfence();
        }
    }
}

}  // namespace swb
