// Batch-one projection kernels for sm_100a.
//
// One kernel body computes dot(W[row], x) for every row of a row-major fp16
// matrix with fp32 accumulation, optionally a second matrix U against the same
// x (the gated SwiGLU stage), and writes one of three epilogues:
//   MODE_GATE: h = fp16(SiLU(a + bg) * (b + bu)), optionally with the eager
//              fp16 rounding points (kernels.cuh:102-106 of the reference);
//   MODE_F32 : y = a (+ bias) (+ residual), fp32;
//   MODE_F16 : the same rounded to fp16.
// These replace decode::project (include/kernels.cuh:24-114 of shubhxho/cuda-kernel).
//
// Families (one registry, csrc/registry.h):
//   ldg_kernel   -- rows spread over CTAs, 128-bit (or 32-bit) streaming loads
//                   with UNROLL loads per matrix in flight per thread, x staged
//                   once per CTA in shared memory as fp32;
//   bulk_kernel  -- persistent: each CTA owns a balanced contiguous row range and
//                   a producer thread streams it with cp.async.bulk into a ring
//                   of shared-memory stages guarded by mbarriers; consumer warps
//                   read each stage once;
//   rbulk_kernel -- as bulk_kernel, but a stage holds whole rows and each
//                   consumer thread keeps its slice of x in registers;
//                   rbulk_allreduce_kernel adds the tensor-parallel exchange;
//   sbulk_kernel -- rbulk's stages with hardware work stealing (cluster launch
//                   control) over row blocks.
// Row partial sums are combined in a fixed order, so every configuration is
// deterministic. Every wait is bounded (device.cuh).
#pragma once

#include <type_traits>

#include "device.cuh"

namespace swb {

enum Mode : int { MODE_GATE = 0, MODE_F32 = 1, MODE_F16 = 2 };

struct Params {
    const __half* w;
    const __half* u;
    const __half* x;
    const __half* bias;
    const __half* ubias;
    const __half* residual;
    float* y;   // MODE_F32 output
    __half* h;  // MODE_GATE / MODE_F16 output
    int rows;
    int cols;
    int model_round;
    int x_staged;  // ldg_kernel: x copied to shared memory as fp32
    int stages;    // bulk_kernel / rbulk_kernel: ring depth
    int row_stage; // rbulk_kernel / sbulk_kernel: whole rows per ring stage
    int rows_per_block;  // sbulk_kernel: rows per CTA index (unit of work stealing)
    int blocks;          // sbulk_kernel: number of row blocks (= grid size)
    int block_stride;    // sbulk_kernel: A in row_block = (cta * A) mod blocks, gcd(A, blocks) = 1
    int inflight;        // bulk_kernel / rbulk_kernel: copies in flight once the ring is full (0 = ring depth)
    float* y_host;       // MODE_F32: y also stored here (mapped page-locked host memory), or null
    // Tensor-parallel exchange call epoch (null otherwise): the gate kernel of a
    // call advances it (advance_call_epoch); the fused down kernel reads it after
    // griddepcontrol.wait, so both kernels of the call agree on it.
    uint32_t* epoch;
};

// In every kernel that can run as the gate of a tensor-parallel call, after its
// griddepcontrol.wait: one fire-and-forget add (no thread waits for it), made by
// thread 0 of the one CTA that `owner` names -- the CTA that owns row 0 of the
// output. For the families with a fixed row -> CTA map that is CTA 0; under work
// stealing (sbulk_kernel) CTA 0 itself may be cancelled before it starts, so
// there it is whichever CTA streams the stage holding row 0. The previous call's
// down kernel, which read the epoch, has completed by then (even when the gate
// was launched programmatically and started early); this call's down kernel
// reads it only after its own griddepcontrol.wait, when this grid's memory
// operations are complete. Epochs start at 1 in a zeroed exchange, so a slot's
// epoch field is 0 only until its first write; every call writes each slot a
// reader of its parity waits on, so when the counter wraps back to 0 no such
// slot still holds that value.
__device__ __forceinline__ void advance_call_epoch(const Params& p, bool owner) {
    if (p.epoch && owner && threadIdx.x == 0) atomicAdd(p.epoch, 1u);
}

// The producer's wait before issuing copy k into a ring of `stages` slots. The
// first `stages` copies go out at once (with programmatic launch they land while
// the previous kernel still runs); after that copy k waits until copy
// k - depth has been consumed, so at most `depth` copies stay in flight. depth =
// stages is the plain ring (wait for the slot's previous copy). Copies are
// consumed in order, so copy k - depth consumed implies slot k % stages free, and
// slot (k - depth) % stages has not started its next round: its parity is exact.
__device__ __forceinline__ bool ring_slot_ready(const uint64_t* empty, int k, int stages, int depth) {
    if (k < stages) return true;
    const int j = k - depth;
    return mbar_wait(smem_u32(empty + (j % stages)), uint32_t((j / stages) & 1));
}
__device__ __forceinline__ int ring_depth(const Params& p) {
    return p.inflight > 0 && p.inflight < p.stages ? p.inflight : p.stages;
}

template <int MODE>
__device__ __forceinline__ void write_row(const Params& p, int row, float a, float b) {
    if constexpr (MODE == MODE_GATE) {
        if (p.bias) a += __half2float(p.bias[row]);
        if (p.ubias) b += __half2float(p.ubias[row]);
        if (p.model_round) {
            a = round_half(a);
            b = round_half(b);
            const float s = round_half(silu(a));
            p.h[row] = __float2half_rn(s * b);
        } else {
            p.h[row] = __float2half_rn(silu(a) * b);
        }
    } else {
        if (p.bias) a += __half2float(p.bias[row]);
        if (p.residual) a += __half2float(p.residual[row]);
        if constexpr (MODE == MODE_F16) {
            p.h[row] = __float2half_rn(a);
        } else {
            p.y[row] = a;
            if (p.y_host) p.y_host[row] = a;  // over PCIe; consecutive threads write consecutive rows
        }
    }
}

// acc[k] += w(half2 k of the 8-half vector) . x[2k..2k+1]
__device__ __forceinline__ void dot8(const uint4& wv, const float* xf, float* acc) {
    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 wf = half2_bits_to_float2(words[k]);
        acc[k] = fmaf(wf.x, xf[2 * k], acc[k]);
        acc[k] = fmaf(wf.y, xf[2 * k + 1], acc[k]);
    }
}

__device__ __forceinline__ float fold4(const float* acc) { return (acc[0] + acc[1]) + (acc[2] + acc[3]); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

// x values for columns [c, c + PACK): from the fp32 shared copy when staged
// (vector reads when 16/8-byte aligned), else from global fp16.
template <int PACK>
__device__ __forceinline__ void load_x(const Params& p, const float* xs, int c, bool xs_vec, float* xf) {
    if (p.x_staged) {
        if (xs_vec) {
            if constexpr (PACK == 8) {
                const float4 a = *reinterpret_cast<const float4*>(xs + c);
                const float4 b = *reinterpret_cast<const float4*>(xs + c + 4);
                xf[0] = a.x; xf[1] = a.y; xf[2] = a.z; xf[3] = a.w;
                xf[4] = b.x; xf[5] = b.y; xf[6] = b.z; xf[7] = b.w;
            } else {
                const float2 a = *reinterpret_cast<const float2*>(xs + c);
                xf[0] = a.x; xf[1] = a.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < PACK; ++i) xf[i] = xs[c + i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < PACK; ++i) xf[i] = __half2float(p.x[c + i]);
    }
}

__device__ __forceinline__ float load_x1(const Params& p, const float* xs, int c) {
    return p.x_staged ? xs[c] : __half2float(p.x[c]);
}

// Copies x[0, cols) into shared memory as fp32 using threads [tid, nthreads).
// 16-byte loads when x is 16-byte aligned, four loads in flight per thread, so
// a 14336-element x costs one or two L2 round trips rather than dozens.
__device__ __forceinline__ void stage_x(const __half* __restrict__ x, float* xs, int cols, int tid, int nthreads) {
    constexpr int U = 4;
    int tail = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int nv = cols / 8;
        const uint4* xv = reinterpret_cast<const uint4*>(x);
        for (int v = tid; v < nv; v += U * nthreads) {
            uint4 a[U];
#pragma unroll
            for (int i = 0; i < U; ++i)
                if (v + i * nthreads < nv) a[i] = xv[v + i * nthreads];
#pragma unroll
            for (int i = 0; i < U; ++i) {
                const int vi = v + i * nthreads;
                if (vi < nv) {
                    const uint32_t w[4] = {a[i].x, a[i].y, a[i].z, a[i].w};
                    float f[8];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 p2 = half2_bits_to_float2(w[k]);
                        f[2 * k] = p2.x;
                        f[2 * k + 1] = p2.y;
                    }
                    float4* dst = reinterpret_cast<float4*>(xs + vi * 8);
                    dst[0] = make_float4(f[0], f[1], f[2], f[3]);
                    dst[1] = make_float4(f[4], f[5], f[6], f[7]);
                }
            }
        }
        tail = nv * 8;
    }
    for (int c = tail + tid; c < cols; c += U * nthreads) {
        float f[U];
#pragma unroll
        for (int i = 0; i < U; ++i)
            if (c + i * nthreads < cols) f[i] = __half2float(x[c + i * nthreads]);
#pragma unroll
        for (int i = 0; i < U; ++i)
            if (c + i * nthreads < cols) xs[c + i * nthreads] = f[i];
    }
}

// ======================================================================= LDG

template <int WPR, int ROWS, int PACK, int UNROLL, int MODE>
__global__ void __launch_bounds__(32 * WPR * ROWS) ldg_kernel(const Params p) {
    static_assert(WPR > 0 && (WPR & (WPR - 1)) == 0 && ROWS > 0 && 32 * WPR * ROWS <= 1024, "geometry");
    static_assert(PACK == 2 || PACK == 8, "pack");
    constexpr bool GATED = MODE == MODE_GATE;
    constexpr int NM = GATED ? 2 : 1;
    constexpr int T = 32 * WPR;      // threads sharing one row
    constexpr int VB = 2 * PACK;     // bytes per vector load
    using Vec = typename std::conditional<PACK == 8, uint4, uint32_t>::type;

    extern __shared__ __align__(16) float xs[];
    __shared__ float red[NM][ROWS * WPR];

    const int cols = p.cols;
    griddep_launch_dependents();
    // x may be the previous kernel's output (h of the gate stage).
    griddep_wait();
    advance_call_epoch(p, blockIdx.x == 0);
    if (p.x_staged) {
        stage_x(p.x, xs, cols, threadIdx.x, blockDim.x);
        __syncthreads();
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int group = warp / WPR, sub = warp % WPR;
    const int t = sub * 32 + lane;
    const int row = blockIdx.x * ROWS + group;

    float acc[NM][4];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[m][k] = 0.f;

    if (row < p.rows) {
        const __half* wr = p.w + size_t(row) * cols;
        const __half* ur = GATED ? p.u + size_t(row) * cols : nullptr;
        const uintptr_t wa = reinterpret_cast<uintptr_t>(wr);
        bool vec = true;
        if constexpr (GATED) vec = ((reinterpret_cast<uintptr_t>(ur) - wa) % VB) == 0;
        // Scalar head up to the first VB-aligned weight, vector body, scalar tail.
        int peel = vec ? int(((VB - wa % VB) % VB) / 2) : cols;
        if (peel > cols) peel = cols;
        const int nvec = (cols - peel) / PACK;
        const int tail0 = peel + nvec * PACK;
        const bool xs_vec = (peel % (PACK == 8 ? 4 : 2)) == 0;

        for (int c = t; c < peel; c += T) {
            const float xv = load_x1(p, xs, c);
            acc[0][0] = fmaf(__half2float(wr[c]), xv, acc[0][0]);
            if constexpr (GATED) acc[1][0] = fmaf(__half2float(ur[c]), xv, acc[1][0]);
        }
        const __half* wv0 = wr + peel;
        const __half* uv0 = GATED ? ur + peel : nullptr;
        int v = t;
        for (; v + (UNROLL - 1) * T < nvec; v += UNROLL * T) {
            Vec wv[UNROLL], uv[UNROLL];
#pragma unroll
            for (int i = 0; i < UNROLL; ++i) {
                const size_t off = size_t(v + i * T) * PACK;
                if constexpr (PACK == 8) {
                    wv[i] = ldg_stream_v4(wv0 + off);
                    if constexpr (GATED) uv[i] = ldg_stream_v4(uv0 + off);
                } else {
                    wv[i] = ldg_stream_b32(wv0 + off);
                    if constexpr (GATED) uv[i] = ldg_stream_b32(uv0 + off);
                }
            }
#pragma unroll
            for (int i = 0; i < UNROLL; ++i) {
                float xf[PACK];
                load_x<PACK>(p, xs, peel + (v + i * T) * PACK, xs_vec, xf);
                if constexpr (PACK == 8) {
                    dot8(wv[i], xf, acc[0]);
                    if constexpr (GATED) dot8(uv[i], xf, acc[1]);
                } else {
                    const int k = i & 3;
                    const float2 wf = half2_bits_to_float2(wv[i]);
                    acc[0][k] = fmaf(wf.y, xf[1], fmaf(wf.x, xf[0], acc[0][k]));
                    if constexpr (GATED) {
                        const float2 uf = half2_bits_to_float2(uv[i]);
                        acc[1][k] = fmaf(uf.y, xf[1], fmaf(uf.x, xf[0], acc[1][k]));
                    }
                }
            }
        }
        for (; v < nvec; v += T) {
            const size_t off = size_t(v) * PACK;
            float xf[PACK];
            load_x<PACK>(p, xs, peel + v * PACK, xs_vec, xf);
            if constexpr (PACK == 8) {
                dot8(ldg_stream_v4(wv0 + off), xf, acc[0]);
                if constexpr (GATED) dot8(ldg_stream_v4(uv0 + off), xf, acc[1]);
            } else {
                const float2 wf = half2_bits_to_float2(ldg_stream_b32(wv0 + off));
                acc[0][0] = fmaf(wf.y, xf[1], fmaf(wf.x, xf[0], acc[0][0]));
                if constexpr (GATED) {
                    const float2 uf = half2_bits_to_float2(ldg_stream_b32(uv0 + off));
                    acc[1][0] = fmaf(uf.y, xf[1], fmaf(uf.x, xf[0], acc[1][0]));
                }
            }
        }
        for (int c = tail0 + t; c < cols; c += T) {
            const float xv = load_x1(p, xs, c);
            acc[0][1] = fmaf(__half2float(wr[c]), xv, acc[0][1]);
            if constexpr (GATED) acc[1][1] = fmaf(__half2float(ur[c]), xv, acc[1][1]);
        }
    }

    float a = warp_sum(fold4(acc[0]));
    float b = 0.f;
    if constexpr (GATED) b = warp_sum(fold4(acc[1]));
    if constexpr (WPR > 1) {
        if (lane == 0) {
            red[0][warp] = a;
            if constexpr (GATED) red[NM - 1][warp] = b;
        }
        __syncthreads();
        if (sub == 0 && lane == 0) {
            a = 0.f;
            b = 0.f;
#pragma unroll
            for (int j = 0; j < WPR; ++j) {
                a += red[0][group * WPR + j];
                if constexpr (GATED) b += red[NM - 1][group * WPR + j];
            }
        }
    }
    if (row < p.rows && sub == 0 && lane == 0) write_row<MODE>(p, row, a, b);
}

// ====================================================================== BULK

// Shared-memory layout of bulk_kernel, shared by host sizing and device code.
struct BulkLayout {
    size_t ring, full, empty, xs, part, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline BulkLayout bulk_layout(int nm, int chunk, int stages, int cols, int cw,
                                                  int rows_per_cta) {
    BulkLayout L;
    L.ring = 0;
    size_t off = size_t(stages) * nm * chunk * 2;
    L.full = align_up(off, 16);
    L.empty = L.full + size_t(stages) * 8;
    L.xs = align_up(L.empty + size_t(stages) * 8, 16);
    L.part = align_up(L.xs + size_t(cols) * 4, 16);
    L.total = align_up(L.part + size_t(rows_per_cta) * cw * nm * 4, 16);
    return L;
}

template <int CW, int CHUNK, int MODE>
__global__ void __launch_bounds__((CW + 1) * 32, 1) bulk_kernel(const Params p) {
    static_assert(CHUNK % 8 == 0 && CHUNK > 0, "chunk must be whole 16-byte vectors");
    constexpr bool GATED = MODE == MODE_GATE;
    constexpr int NM = GATED ? 2 : 1;
    constexpr int CT = CW * 32;  // consumer threads

    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_failed;

    const int G = gridDim.x;
    const int r0 = int((long long)blockIdx.x * p.rows / G);
    const int r1 = int((long long)(blockIdx.x + 1) * p.rows / G);
    const int nrows = r1 - r0;
    if (nrows <= 0) return;  // whole CTA leaves together
    const int cols = p.cols;
    const int stages = p.stages;
    const int nch = (cols + CHUNK - 1) / CHUNK;
    const int units = nrows * nch;
    const int rows_per_cta = (p.rows + G - 1) / G;

    const BulkLayout L = bulk_layout(NM, CHUNK, stages, cols, CW, rows_per_cta);
    __half* ring = reinterpret_cast<__half*>(smem + L.ring);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
    float* xs = reinterpret_cast<float*>(smem + L.xs);
    float* part = reinterpret_cast<float*>(smem + L.part);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        SWB_TIMELINE(0);
        s_failed = 0;
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), CW);
        }
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch_dependents();

    // The producer starts streaming weights at once (it never reads x); the
    // consumers stage x meanwhile and meet at a named barrier before reading it.
    if (warp == CW) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first_policy();
        const int depth = ring_depth(p);
        int s = 0, row = r0, ch = 0, issued = 0;
        for (int k = 0; k < units; ++k) {
            if (!ring_slot_ready(empty, k, stages, depth)) break;
            const int c0 = ch * CHUNK;
            const int len = min(CHUNK, cols - c0);
            const uint32_t bytes = uint32_t(len) * 2u;
            const uint32_t fb = smem_u32(full + s);
            mbar_arrive_expect_tx(fb, bytes * NM);
            const size_t goff = size_t(row) * cols + c0;
            bulk_copy_g2s(smem_u32(ring + size_t(s) * NM * CHUNK), p.w + goff, bytes, fb, pol);
            if constexpr (GATED) bulk_copy_g2s(smem_u32(ring + (size_t(s) * NM + 1) * CHUNK), p.u + goff, bytes, fb, pol);
            ++issued;
            if (++ch == nch) { ch = 0; ++row; }
            if (++s == stages) s = 0;
        }
        SWB_TIMELINE(4);
        // Never leave with copies in flight: wait (bounded) for the last fills.
        const int drain = issued < stages ? issued : stages;
        for (int j = 1; j <= drain; ++j) {
            const int k = issued - j;
            if (!mbar_wait(smem_u32(full + (k % stages)), uint32_t((k / stages) & 1))) break;
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int t = threadIdx.x;
    griddep_wait();  // x may be the previous kernel's output (h of the gate stage)
    advance_call_epoch(p, blockIdx.x == 0);
    stage_x(p.x, xs, cols, t, CT);
    named_barrier_sync(1, CT);
    float acc[NM][4];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[m][k] = 0.f;

    int s = 0, row = r0, ch = 0;
    uint32_t ph = 0;
    for (int k = 0; k < units; ++k) {
        if (!mbar_wait(smem_u32(full + s), ph)) {
            s_failed = 1;
            break;
        }
        if (k == 0 && t == 0) SWB_TIMELINE(1);
        const int c0 = ch * CHUNK;
        const int nv = min(CHUNK, cols - c0) / 8;
        const __half* sw = ring + size_t(s) * NM * CHUNK;
        for (int v = t; v < nv; v += CT) {
            const uint4 wv = *reinterpret_cast<const uint4*>(sw + v * 8);
            const float4 xa = *reinterpret_cast<const float4*>(xs + c0 + v * 8);
            const float4 xb = *reinterpret_cast<const float4*>(xs + c0 + v * 8 + 4);
            const float xf[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            dot8(wv, xf, acc[0]);
            if constexpr (GATED) {
                const uint4 uv = *reinterpret_cast<const uint4*>(sw + CHUNK + v * 8);
                dot8(uv, xf, acc[1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(empty + s));
        if (++ch == nch) {
            const float a = warp_sum(fold4(acc[0]));
            float b = 0.f;
            if constexpr (GATED) b = warp_sum(fold4(acc[1]));
            if (lane == 0) {
                part[(size_t(row - r0) * CW + warp) * NM] = a;
                if constexpr (GATED) part[(size_t(row - r0) * CW + warp) * NM + 1] = b;
            }
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[m][q] = 0.f;
            ch = 0;
            ++row;
        }
        if (++s == stages) { s = 0; ph ^= 1u; }
    }
    if (t == 0) SWB_TIMELINE(2);
    named_barrier_sync(1, CT);
    if (s_failed) return;
    for (int i = t; i < nrows; i += CT) {
        float a = 0.f, b = 0.f;
        for (int j = 0; j < CW; ++j) {
            a += part[(size_t(i) * CW + j) * NM];
            if constexpr (GATED) b += part[(size_t(i) * CW + j) * NM + 1];
        }
        write_row<MODE>(p, r0 + i, a, b);
    }
    if (t == 0) SWB_TIMELINE(3);
}

// ===================================================================== RBULK

// Shared-memory layout of rbulk_kernel, shared by host sizing and device code.
__host__ __device__ inline BulkLayout rbulk_layout(int nm, int row_stage, int cols, int stages, int cw,
                                                   int rows_per_cta) {
    BulkLayout L;
    L.ring = 0;
    const size_t off = size_t(stages) * row_stage * nm * size_t(cols) * 2;
    L.full = align_up(off, 16);
    L.empty = L.full + size_t(stages) * 8;
    L.xs = align_up(L.empty + size_t(stages) * 8, 16);  // no x copy: x lives in registers
    L.part = L.xs;
    L.total = align_up(L.part + size_t(rows_per_cta) * cw * nm * 4, 16);
    return L;
}

// Sums K values (K a power of two, at most 32) over the 32 lanes of a warp.
// Each of the first log2(K) xor steps halves what a lane carries: the lane
// keeps one half of its values, sends the other half to its partner and adds
// what comes back; a plain butterfly over the remaining lane bits finishes. K
// values cost K/2 + K/4 + ... + 1 + (5 - log2 K) shuffles (9 for K = 8) instead
// of 5K, which matters when many warps of an SM reduce short rows at once.
// Lane L returns the total of value (L >> (5 - log2 K)); the order of the adds
// is fixed, so the result is deterministic.
template <int K>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[K], int lane) {
    static_assert(K >= 1 && K <= 32 && (K & (K - 1)) == 0, "K must be a power of two up to 32");
#pragma unroll
    for (int k = K, d = 16; k > 1; k >>= 1, d >>= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < k / 2; ++i) {
            const float send = upper ? v[i] : v[i + k / 2];
            const float keep = upper ? v[i + k / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
    }
    constexpr int LK = K >= 32 ? 5 : K >= 16 ? 4 : K >= 8 ? 3 : K >= 4 ? 2 : K >= 2 ? 1 : 0;
    float t = v[0];
#pragma unroll
    for (int d = 16 >> LK; d; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
    return t;
}

// Dot products of the `ru` rows of one ring stage with the consumer's register
// slice xr (vectors t + j*CT, j < J), RG rows at a time: the RG * NM row sums of
// a group are reduced together (warp_reduce_scatter), so rows that give each
// thread only a vector or two are bound neither by one dependent shuffle chain
// per row nor by the SM's shuffle throughput. The lane holding a row's sum
// stores the warp partial of row prow0 + r into part[row][warp][matrix].
template <int CW, int MAXJ, int NM, int RG, int J>
__device__ __forceinline__ void stage_rows(const __half* sw, int ru, int rs, int cols, int nv, const float (&xr)[MAXJ][8],
                                           float* part, int prow0) {
    static_assert(J <= MAXJ, "vectors per thread");
    constexpr int CT = CW * 32;
    constexpr int K = RG * NM;
    constexpr int LK = K >= 32 ? 5 : K >= 16 ? 4 : K >= 8 ? 3 : K >= 4 ? 2 : K >= 2 ? 1 : 0;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    for (int r = 0; r < ru; r += RG) {
        float acc[RG][NM][4];
#pragma unroll
        for (int g = 0; g < RG; ++g)
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[g][m][q] = 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int v = t + j * CT;
            if (v < nv) {
#pragma unroll
                for (int g = 0; g < RG; ++g) {
                    if (r + g < ru) {
                        const __half* wv = sw + size_t(r + g) * cols + size_t(v) * 8;
                        dot8(*reinterpret_cast<const uint4*>(wv), xr[j], acc[g][0]);
                        if constexpr (NM == 2)
                            dot8(*reinterpret_cast<const uint4*>(wv + size_t(rs) * cols), xr[j], acc[g][1]);
                    }
                }
            }
        }
        float red[K];
#pragma unroll
        for (int g = 0; g < RG; ++g)
#pragma unroll
            for (int m = 0; m < NM; ++m) red[g * NM + m] = fold4(acc[g][m]);
        const float total = warp_reduce_scatter<K>(red, lane);
        if ((lane & ((32 >> LK) - 1)) == 0) {
            const int idx = lane >> (5 - LK);
            const int g = idx / NM, m = idx % NM;
            if (r + g < ru) part[(size_t(prow0 + r + g) * CW + warp) * NM + m] = total;
        }
    }
}

template <int CW, int MAXJ, int MODE>
__device__ __forceinline__ bool rbulk_stream(const Params& p, unsigned char* smem, int& r0_out, int& nrows_out,
                                             float*& part_out, uint32_t* epoch_out = nullptr) {
    constexpr bool GATED = MODE == MODE_GATE;
    constexpr int NM = GATED ? 2 : 1;
    constexpr int CT = CW * 32;
    __shared__ int s_failed;

    const int G = gridDim.x;
    const int r0 = int((long long)blockIdx.x * p.rows / G);
    const int r1 = int((long long)(blockIdx.x + 1) * p.rows / G);
    const int nrows = r1 - r0;
    if (nrows <= 0) return false;  // whole CTA leaves together
    const int cols = p.cols;
    const int nv = cols / 8;
    const int rs = p.row_stage;
    const int stages = p.stages;
    const int units = (nrows + rs - 1) / rs;
    const int rows_per_cta = (p.rows + G - 1) / G;
    const size_t stage_halves = size_t(rs) * NM * cols;

    const BulkLayout L = rbulk_layout(NM, rs, cols, stages, CW, rows_per_cta);
    __half* ring = reinterpret_cast<__half*>(smem + L.ring);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
    float* part = reinterpret_cast<float*>(smem + L.part);
    r0_out = r0;
    nrows_out = nrows;
    part_out = part;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        SWB_TIMELINE(0);
        s_failed = 0;
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
        if (lane != 0) return false;
        const uint64_t pol = l2_evict_first_policy();
        const int depth = ring_depth(p);
        int s = 0, issued = 0;
        for (int k = 0; k < units; ++k) {
            if (!ring_slot_ready(empty, k, stages, depth)) break;
            const int row = r0 + k * rs;
            const int ru = min(rs, r1 - row);
            const uint32_t bytes = uint32_t(ru) * uint32_t(cols) * 2u;
            const uint32_t fb = smem_u32(full + s);
            mbar_arrive_expect_tx(fb, bytes * NM);
            const size_t goff = size_t(row) * cols;
            __half* dst = ring + size_t(s) * stage_halves;
            bulk_copy_g2s(smem_u32(dst), p.w + goff, bytes, fb, pol);
            if constexpr (GATED) bulk_copy_g2s(smem_u32(dst + size_t(rs) * cols), p.u + goff, bytes, fb, pol);
            ++issued;
            if (++s == stages) s = 0;
        }
        SWB_TIMELINE(4);
        const int drain = issued < stages ? issued : stages;
        for (int j = 1; j <= drain; ++j) {
            const int k = issued - j;
            if (!mbar_wait(smem_u32(full + (k % stages)), uint32_t((k / stages) & 1))) break;
        }
        return false;
    }

    // ----------------------------------------------------------- consumers
    const int t = threadIdx.x;
    griddep_wait();  // x may be the previous kernel's output (h of the gate stage)
    // the fused tensor-parallel down kernel reads the call epoch its gate advanced;
    // as the gate of a tensor-parallel call this kernel advances it
    if (epoch_out) {
        if (t == 0) *epoch_out = *reinterpret_cast<volatile const uint32_t*>(p.epoch);
    } else {
        advance_call_epoch(p, blockIdx.x == 0);
    }
    float xr[MAXJ][8];
    const bool x16 = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
        const int v = t + j * CT;
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[j][e] = 0.f;
        if (v < nv) {
            if (x16) {
                const uint4 q = *reinterpret_cast<const uint4*>(p.x + size_t(v) * 8);
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = half2_bits_to_float2(w4[k]);
                    xr[j][2 * k] = f.x;
                    xr[j][2 * k + 1] = f.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) xr[j][e] = __half2float(p.x[size_t(v) * 8 + e]);
            }
        }
    }

    // Rows per reduction group by the vectors each thread holds (jn): short rows
    // reduce 8 / NM at once. The choice is made once, outside the stage loop, so
    // each loop keeps only the part of xr it reads in registers.
    auto consume = [&](auto rg, auto jv) {
        constexpr int RG = decltype(rg)::value, J = decltype(jv)::value;
        int s = 0;
        uint32_t ph = 0;
        for (int k = 0; k < units; ++k) {
            if (!mbar_wait(smem_u32(full + s), ph)) {
                s_failed = 1;
                break;
            }
            if (k == 0 && t == 0) SWB_TIMELINE(1);
            const int row0 = r0 + k * rs;
            const int ru = min(rs, r1 - row0);
            const __half* sw = ring + size_t(s) * stage_halves;
            stage_rows<CW, MAXJ, NM, RG, J>(sw, ru, rs, cols, nv, xr, part, row0 - r0);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(empty + s));
            if (++s == stages) { s = 0; ph ^= 1u; }
        }
        if (t == 0) SWB_TIMELINE(2);
    };
    const int jn = (nv + CT - 1) / CT;
    if (jn <= 1)
        consume(std::integral_constant<int, 8 / NM>{}, std::integral_constant<int, 1>{});
    else if (jn <= 2)
        consume(std::integral_constant<int, 4 / NM>{}, std::integral_constant<int, (MAXJ < 2 ? MAXJ : 2)>{});
    else
        consume(std::integral_constant<int, 1>{}, std::integral_constant<int, MAXJ>{});
    named_barrier_sync(1, CT);
    return s_failed == 0;
}

// Sum of warp partials of local row i, in warp order (deterministic).
template <int CW, int NM>
__device__ __forceinline__ float row_sum(const float* part, int i, int m) {
    float a = 0.f;
    for (int j = 0; j < CW; ++j) a += part[(size_t(i) * CW + j) * NM + m];
    return a;
}

template <int CW, int MAXJ, int CPS, int MODE>
__global__ void __launch_bounds__((CW + 1) * 32, CPS) rbulk_kernel(const Params p) {
    constexpr int NM = MODE == MODE_GATE ? 2 : 1;
    constexpr int CT = CW * 32;
    extern __shared__ __align__(128) unsigned char smem[];
    int r0, nrows;
    float* part;
    if (!rbulk_stream<CW, MAXJ, MODE>(p, smem, r0, nrows, part)) return;
    for (int i = threadIdx.x; i < nrows; i += CT)
        write_row<MODE>(p, r0 + i, row_sum<CW, NM>(part, i, 0), NM == 2 ? row_sum<CW, NM>(part, i, NM - 1) : 0.f);
    if (threadIdx.x == 0) SWB_TIMELINE(3);
}

// ============================================ RBULK + one-shot all-reduce

// Tensor-parallel exchange of one layer call. Rank q's exchange buffer holds
// recv[2][world][rows] slots (parity-double-buffered partials from every rank;
// a slot is one 64-bit word {fp32 value, call epoch}, see st_slot_sys) and this
// rank's call epoch ctr[0]. Each call advances the epoch exactly once: the gate
// kernel does it (Params::epoch) before the fused down kernel reads it, or the
// fused layer kernel's CTA 0 stores the epoch every CTA read before the grid
// barrier. One epoch per call, the same for every CTA whatever the grid: with a
// per-CTA counter, consecutive calls that map rows to CTAs differently could let
// a peer's CTA b write this call's rows into the parity buffer that another CTA
// here still reads for the previous call. After a device error the exchange must
// be recreated (the epochs of the ranks may no longer agree).
constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxCtas = 1024;

struct TpParams {
    unsigned long long* recv[kTpMaxRanks];
    uint32_t* ctr;
    const __half* bias;      // added once after the sum (may be null)
    const __half* residual;  // added once after the sum (may be null)
    float* y_host;           // fp32 y also stored here (mapped page-locked host memory), or null
    int rank;
    int world;
};

// Rows [r0, r0 + n) of y: this rank's partial `own(i)` goes to slot
// [parity][my rank][row] of every other rank; then each row sums every rank's
// partial in rank order -- the same order on every rank, so y is bit-identical
// everywhere -- plus bias and residual. A rank can run at most one call ahead of
// a peer (each call waits for that peer's slots), so the parity double buffer
// keeps a slot from being rewritten before it is read.
__device__ __forceinline__ void store_out(float* y, int i, float v) { y[i] = v; }
__device__ __forceinline__ void store_out(__half* y, int i, float v) { y[i] = __float2half_rn(v); }

template <int CT, class Out, class Own>
__device__ __forceinline__ void tp_exchange_rows(const TpParams& tp, uint32_t epoch, int rows, int r0, int n, Out* y,
                                                 Own own) {
    // rank loops run to the compile-time bound, so recv[] is indexed by constants
    // and stays in the kernel's parameter space
    const int t = threadIdx.x;
    const size_t par = epoch & 1u;
    for (int i = t; i < n; i += CT) {
        const float a = own(i);
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
            if (q < tp.world && q != tp.rank)
                st_slot_sys(tp.recv[q] + (par * tp.world + tp.rank) * rows + r0 + i, a, epoch);
    }
    const unsigned long long* mine = tp.recv[0] + par * tp.world * rows;
#pragma unroll
    for (int q = 1; q < kTpMaxRanks; ++q)
        if (q == tp.rank) mine = tp.recv[q] + par * tp.world * rows;
    bool ok = true;
    for (int i = t; i < n; i += CT) {
        // every peer's word of this row first, the loads all in flight together; only the
        // words that do not carry this epoch yet are then polled (bounded), one peer at a time
        unsigned long long w[kTpMaxRanks];
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
            w[q] = (q < tp.world && q != tp.rank) ? ld_slot_sys(mine + size_t(q) * rows + r0 + i) : 0ull;
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q) {
            if (q >= tp.world) break;
            float v = 0.f;
            if (q == tp.rank) v = own(i);
            else if (uint32_t(w[q] >> 32) == epoch) v = __uint_as_float(uint32_t(w[q]));
            else if (ok) ok = wait_slot(mine + size_t(q) * rows + r0 + i, epoch, v);
            acc += v;  // rank order, whichever word came first: y is the same on every rank
        }
        if (!ok) break;  // a peer did not deliver: the error word is set, y is not written
        float add = 0.f;
        if (tp.bias) add += __half2float(tp.bias[r0 + i]);
        if (tp.residual) add += __half2float(tp.residual[r0 + i]);
        store_out(y, r0 + i, acc + add);
        if constexpr (std::is_same_v<Out, float>)
            if (tp.y_host) tp.y_host[r0 + i] = acc + add;  // over PCIe, consecutive rows per warp
    }
}

// The down projection of a tensor-parallel rank with the all-reduce fused into
// its epilogue (tp_exchange_rows). Every rank runs the same grid and row
// partition, so CTA b owns rows [r0, r1) of y on every rank. The epoch lives in
// device memory (advanced by the gate kernel), so graph replays need no reset.
// HALF_OUT writes the reduced rows rounded once to fp16 into p.h (the model
// path: fp16 y, no bias, no residual); otherwise fp32 into p.y.
template <int CW, int MAXJ, int CPS, bool HALF_OUT>
__global__ void __launch_bounds__((CW + 1) * 32, CPS) rbulk_allreduce_kernel(const Params p, const TpParams tp) {
    constexpr int CT = CW * 32;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint32_t s_epoch;
    int r0, nrows;
    float* part;
    if (!rbulk_stream<CW, MAXJ, MODE_F32>(p, smem, r0, nrows, part, &s_epoch)) return;
    named_barrier_sync(1, CT);
    auto own = [&](int i) { return row_sum<CW, 1>(part, i, 0); };
    if constexpr (HALF_OUT)
        tp_exchange_rows<CT>(tp, s_epoch, p.rows, r0, nrows, p.h, own);
    else
        tp_exchange_rows<CT>(tp, s_epoch, p.rows, r0, nrows, p.y, own);
}

// ===================================================================== SBULK

// Shared-memory layout of sbulk_kernel (host sizing and device code).
struct StealLayout {
    size_t ring, full, empty, meta, cnt, part, total;
};

__host__ __device__ inline StealLayout sbulk_layout(int nm, int row_stage, int cols, int stages, int cw) {
    StealLayout L;
    L.ring = 0;
    L.full = align_up(size_t(stages) * row_stage * nm * size_t(cols) * 2, 16);
    L.empty = L.full + size_t(stages) * 8;
    L.meta = L.empty + size_t(stages) * 8;              // int2 {first row, rows} per stage
    L.cnt = L.meta + size_t(stages) * 8;                // consumer warps done per stage
    L.part = align_up(L.cnt + size_t(stages) * 4, 16);  // [stage][row][warp][matrix] partial sums
    L.total = align_up(L.part + size_t(stages) * row_stage * cw * nm * 4, 16);
    return L;
}

// Row-stage streaming with hardware work stealing. The grid has one CTA per
// block of `rows_per_block` rows; the CTAs that fit run, and each one's producer,
// while streaming its current block, asks cluster launch control for a CTA that
// has not started and takes over that CTA's block. Faster SMs therefore take more
// blocks and the CTAs finish together. A ring stage holds up to `row_stage`
// whole rows; the producer tags each stage with its rows (or -1 to stop). As in
// rbulk_kernel, consumer thread t owns vectors t + j*CT of every row, x stays in
// registers. The last consumer warp to finish a stage sums the stage's row
// partials over the warps in a fixed order and writes those rows, so outputs are
// deterministic whatever the stealing order.
template <int CW, int MAXJ, int CPS, int MODE>
__global__ void __launch_bounds__((CW + 1) * 32, CPS) sbulk_kernel(const Params p) {
    constexpr bool GATED = MODE == MODE_GATE;
    constexpr int NM = GATED ? 2 : 1;
    constexpr int CT = CW * 32;

    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) uint4 clc_resp[2];
    __shared__ uint64_t clc_bar[2];
    __shared__ int s_failed;

    const int cols = p.cols;
    const int nv = cols / 8;
    const int rs = p.row_stage;
    const int rpb = p.rows_per_block;
    const int stages = p.stages;
    const size_t stage_halves = size_t(rs) * NM * cols;

    const StealLayout L = sbulk_layout(NM, rs, cols, stages, CW);
    __half* ring = reinterpret_cast<__half*>(smem + L.ring);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
    int2* meta = reinterpret_cast<int2*>(smem + L.meta);
    int* cnt = reinterpret_cast<int*>(smem + L.cnt);
    float* part = reinterpret_cast<float*>(smem + L.part);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        SWB_TIMELINE(0);
        s_failed = 0;
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), CW);
            cnt[s] = 0;
        }
        mbar_init(smem_u32(&clc_bar[0]), 1);
        mbar_init(smem_u32(&clc_bar[1]), 1);
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
        // Two steal requests stay in flight (slots 0 and 1, answered in the order
        // issued), so an answer is ready when a block ends. After an answer says
        // nothing was left, no new request is issued; an older outstanding one is
        // still collected and, if it did cancel a CTA, that CTA's block is done here.
        uint32_t clc_ph = 0u;  // bit k: parity of slot k's next answer
        int q_head = 0, q_len = 0;
        bool steal_failed = false;
        auto request = [&](int slot) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(smem_u32(&clc_bar[slot]), 16);
            clc_try_cancel(smem_u32(&clc_resp[slot]), smem_u32(&clc_bar[slot]));
        };
        request(0);
        request(1);
        q_len = 2;
        int block = blockIdx.x;
        bool ok = true;
        while (block >= 0 && ok) {
            // CTA index -> row block through a bijection that spreads consecutive
            // indices A blocks apart, so the CTAs in flight stream from all over the
            // matrix rather than one narrow window of it.
            const int rb = int((long long)block * p.block_stride % p.blocks);
            const int b0 = rb * rpb;
            const int b1 = min(b0 + rpb, p.rows);
            for (int row = b0; row < b1; row += rs) {
                if (issued >= stages && !mbar_wait(smem_u32(empty + s), ph ^ 1u)) { ok = false; break; }
                const int ru = min(rs, b1 - row);
                const uint32_t bytes = uint32_t(ru) * uint32_t(cols) * 2u;
                meta[s] = make_int2(row, ru);
                const uint32_t fb = smem_u32(full + s);
                mbar_arrive_expect_tx(fb, bytes * NM);
                const size_t goff = size_t(row) * cols;
                __half* dst = ring + size_t(s) * stage_halves;
                bulk_copy_g2s(smem_u32(dst), p.w + goff, bytes, fb, pol);
                if constexpr (GATED) bulk_copy_g2s(smem_u32(dst + size_t(rs) * cols), p.u + goff, bytes, fb, pol);
                ++issued;
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
            // Next block: the oldest outstanding answer that cancelled a CTA.
            block = -1;
            while (q_len > 0) {
                const int slot = q_head;
                if (!mbar_wait(smem_u32(&clc_bar[slot]), (clc_ph >> slot) & 1u)) {
                    ok = false;  // give this slot up; still try to collect the other one
                    q_head ^= 1;
                    --q_len;
                    continue;
                }
                clc_ph ^= 1u << slot;
                fence_proxy_async_smem();
                const int nb = clc_decode(clc_resp[slot]);
                q_head ^= 1;
                --q_len;
                if (nb < 0) { steal_failed = true; continue; }
                if (!steal_failed && ok) { request(slot); ++q_len; }
                block = nb;
                break;
            }
        }
        SWB_TIMELINE(4);
        // Collect any request still outstanding (its answer is written asynchronously).
        while (q_len > 0) {
            const int slot = q_head;
            if (mbar_wait(smem_u32(&clc_bar[slot]), (clc_ph >> slot) & 1u)) clc_ph ^= 1u << slot;
            else ok = false;
            q_head ^= 1;
            --q_len;
        }
        // Normal end: tag the next stage -1 and complete it without data; the
        // consumers take every filled stage, in order, before they reach it, so
        // no copy is in flight when the CTA exits.
        if (ok && (issued < stages || mbar_wait(smem_u32(empty + s), ph ^ 1u))) {
            meta[s] = make_int2(-1, 0);
            mbar_arrive(smem_u32(full + s));
            return;
        }
        // A wait gave up: never leave with copies in flight -- wait (bounded) for
        // the last fills. (Only here: after the -1 tag above their phases would
        // no longer be the most recent ones.)
        const int drain = issued < stages ? issued : stages;
        for (int j = 1; j <= drain; ++j) {
            const int k = issued - j;
            if (!mbar_wait(smem_u32(full + (k % stages)), uint32_t((k / stages) & 1))) break;
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int t = threadIdx.x;
    griddep_wait();  // x may be the previous kernel's output (h of the gate stage)
    float xr[MAXJ][8];
    const bool x16 = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
        const int v = t + j * CT;
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[j][e] = 0.f;
        if (v < nv) {
            if (x16) {
                const uint4 q = *reinterpret_cast<const uint4*>(p.x + size_t(v) * 8);
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = half2_bits_to_float2(w4[k]);
                    xr[j][2 * k] = f.x;
                    xr[j][2 * k + 1] = f.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) xr[j][e] = __half2float(p.x[size_t(v) * 8 + e]);
            }
        }
    }

    int s = 0;
    uint32_t ph = 0;
    bool first = true;
    while (true) {
        if (!mbar_wait(smem_u32(full + s), ph)) {
            s_failed = 1;
            break;
        }
        const int2 m = meta[s];
        if (m.x < 0) break;
        if (first && t == 0) SWB_TIMELINE(1);
        first = false;
        // row 0 is in exactly one stage of one CTA, whichever CTA took its block
        advance_call_epoch(p, m.x == 0);
        const __half* sw = ring + size_t(s) * stage_halves;
        float* ps = part + size_t(s) * rs * CW * NM;
        for (int r = 0; r < m.y; ++r) {
            float acc[NM][4];
#pragma unroll
            for (int mm = 0; mm < NM; ++mm)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[mm][q] = 0.f;
            const __half* wrow = sw + size_t(r) * cols;
#pragma unroll
            for (int j = 0; j < MAXJ; ++j) {
                const int v = t + j * CT;
                if (v < nv) {
                    dot8(*reinterpret_cast<const uint4*>(wrow + size_t(v) * 8), xr[j], acc[0]);
                    if constexpr (GATED)
                        dot8(*reinterpret_cast<const uint4*>(wrow + size_t(rs) * cols + size_t(v) * 8), xr[j],
                             acc[1]);
                }
            }
            const float a = warp_sum(fold4(acc[0]));
            float b = 0.f;
            if constexpr (GATED) b = warp_sum(fold4(acc[1]));
            if (lane == 0) {
                ps[(size_t(r) * CW + warp) * NM] = a;
                if constexpr (GATED) ps[(size_t(r) * CW + warp) * NM + 1] = b;
            }
        }
        // The last warp to finish this stage combines the warps' partials and writes the rows.
        int done = 0;
        if (lane == 0) {
            __threadfence_block();
            done = atomicAdd(cnt + s, 1);
        }
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done == CW - 1) {
            __threadfence_block();
            for (int r = lane; r < m.y; r += 32) {
                float a = 0.f, b = 0.f;
                for (int j = 0; j < CW; ++j) {
                    a += ps[(size_t(r) * CW + j) * NM];
                    if constexpr (GATED) b += ps[(size_t(r) * CW + j) * NM + 1];
                }
                write_row<MODE>(p, m.x + r, a, b);
            }
            if (lane == 0) cnt[s] = 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(empty + s));
        if (++s == stages) { s = 0; ph ^= 1u; }
    }
    if (t == 0) SWB_TIMELINE(2);
    (void)s_failed;
}

// ============================================================== pointwise

// kernels.cuh:134-141 of the reference: the cuBLAS path's gate epilogue.
__global__ void gate_epilogue_kernel(const float* a, const float* b, const __half* bg, const __half* bu,
                                     __half* h, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float g = a[i] + __half2float(bg[i]);
        const float v = b[i] + __half2float(bu[i]);
        h[i] = __float2half_rn(silu(g) * v);
    }
}

// kernels.cuh:142-145 of the reference: y += bias + x.
__global__ void residual_epilogue_kernel(float* y, const __half* bias, const __half* x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] += __half2float(bias[i]) + __half2float(x[i]);
}

// ===================================================== host-buffer transfers

// One step of a layer call from page-locked host x to page-locked host y
// (swb_ffn_host_ex): x in, or y out, over PCIe. The transfers are kernels, not
// copy operations, so consecutive calls stay one chain of programmatic launches:
// the next call's gate streams its weights while this call's y and the next x
// cross the bus. `src` / `dst` may be the device address of page-locked host
// memory (unified addressing). The loads are plain (not the read-only path): the
// host rewrites its buffer between calls. 16-byte pieces when both ends are
// 16-byte aligned, bytes otherwise.
__global__ void transfer_kernel(const unsigned char* src, unsigned char* dst, size_t bytes) {
    griddep_launch_dependents();
    griddep_wait();  // the previous kernel of the chain has finished with dst (or written src)
    const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n = size_t(gridDim.x) * blockDim.x;
    size_t done = 0;
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const size_t pieces = bytes / 16;
        for (size_t i = t; i < pieces; i += n) reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
        done = pieces * 16;
    }
    for (size_t i = done + t; i < bytes; i += n) dst[i] = src[i];
}

}  // namespace swb
