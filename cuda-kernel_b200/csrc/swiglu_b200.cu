// C ABI of the B200 SwiGLU decode layer (declarations: include/swiglu_b200.h).
//
// Argument guards mirror decode::launch (include/kernels.cuh:115-133) and the
// torch binding (src/torch_extension.cu:7-40) of shubhxho/cuda-kernel, in the
// same order and with the same messages, and run before any CUDA call.
// Dispatch is generated from the registry list (registry.h), as
// include/kernels.cuh:124-131 generates it from DECODE_CONFIGS.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <new>
#include <numeric>
#include <string>

#include "kernels.cuh"
#include "layer.cuh"
#include "registry.h"
#include "swiglu_b200.h"

namespace swb {
namespace {

thread_local std::string g_last_error;

int fail(int status, const char* detail = nullptr) {
    g_last_error = swb_status_string(status);
    if (detail && *detail) {
        g_last_error += ": ";
        g_last_error += detail;
    }
    return status;
}

int check_launch() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    return SWB_OK;
}

constexpr swb_config_t kConfigs[] = {
#define SWB_META(ID, FAM, W, R, PK, U, CH, ST) {ID, FAM, W, R, PK, U, CH, ST},
    SWB_CONFIGS(SWB_META)
#undef SWB_META
};
constexpr int kConfigCount = int(sizeof(kConfigs) / sizeof(kConfigs[0]));

const swb_config_t* find_config(int64_t id) {
    for (const auto& c : kConfigs)
        if (c.id == id) return &c;
    return nullptr;
}

// Geometry invariants checked at compile time for every registry entry.
#define SWB_CHECK(ID, FAM, W, R, PK, U, CH, ST)                                                     \
    static_assert(ID > 0 && ID < 1000, "ids 0 and >= 1000 stay invalid");                          \
    static_assert(FAM != SWB_FAM_LDG || (32 * W * R <= 1024 && (W & (W - 1)) == 0), "LDG block");   \
    static_assert(FAM != SWB_FAM_LDG || PK == 2 || PK == 8, "LDG pack");                            \
    static_assert(FAM != SWB_FAM_LDG || U == 1 || U == 2 || U == 4 || U == 8, "LDG unroll");        \
    static_assert(FAM != SWB_FAM_BULK || (CH % 8 == 0 && CH > 0 && ST >= 2 && (W + 1) * 32 <= 1024), \
                  "BULK geometry");                                                                \
    static_assert((FAM != SWB_FAM_RBULK && FAM != SWB_FAM_SBULK) ||                                \
                      (U >= 1 && U <= 8 && CH >= 16 && ST >= 2 && (W + 1) * 32 <= 1024),             \
                  "RBULK/SBULK geometry");
SWB_CONFIGS(SWB_CHECK)
#undef SWB_CHECK

// Shared-memory capacities of sm_100: 228 KB per SM, 227 KB opt-in per CTA,
// 1 KB reserved per resident CTA.
constexpr size_t kSmemPerSm = 233472;
constexpr size_t kSmemPerCtaMax = 232448;
// x is staged in shared memory by the LDG family while its fp32 copy fits this.
constexpr size_t kXStageLimit = 96 * 1024;

int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (dev < 64) {
        const int c = cache[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (dev < 64) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

// Raises a kernel's dynamic shared-memory limit once per device.
template <typename Kernel>
int ensure_smem(Kernel kernel, std::atomic<uint64_t>& done_mask, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch();
    const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
    if (bit && (done_mask.load(std::memory_order_acquire) & bit)) return SWB_OK;
    // Static shared memory counts against the same 227 KB per-CTA limit.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (bytes + fa.sharedSizeBytes > kSmemPerCtaMax) return fail(SWB_E_CUDA, "shared memory request too large");
    // the permitted maximum, once per kernel and device, whatever this request needs
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(kSmemPerCtaMax - fa.sharedSizeBytes));
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    // Every kernel asks for the largest shared-memory carveout, so all of them
    // run in one SM configuration: CTAs of the next kernel (the down projection,
    // launched programmatically) can join an SM beside the gate's CTAs and start
    // streaming their weights, instead of waiting for the SM to drain and be
    // reconfigured for a different L1 / shared split.
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared));
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (bit) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return SWB_OK;
}

// Launches `kernel`; with `pdl` the launch may begin before the previous kernel
// in the stream finishes (programmatic dependent launch). Used for the down
// projection right after this library's own gate kernel (the down kernel reads
// nothing the gate writes until its griddepcontrol.wait), and for the gate under
// SWB_PREFETCH_WEIGHTS (only its weight stream starts early; x, h and the
// exchange epoch wait for griddepcontrol.wait).
template <typename Kernel>
void launch_kernel(Kernel kernel, unsigned grid, unsigned block, size_t smem, cudaStream_t stream, bool pdl,
                   const Params& p) {
    if (!pdl) {
        kernel<<<grid, block, smem, stream>>>(p);
        return;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int W, int R, int PK, int U, int MODE>
int launch_ldg(Params p, cudaStream_t stream, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    p.x_staged = size_t(p.cols) * 4 <= kXStageLimit;
    const size_t smem = p.x_staged ? align_up(size_t(p.cols) * 4, 16) : 0;
    auto kernel = ldg_kernel<W, R, PK, U, MODE>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    const unsigned grid = unsigned((p.rows + R - 1) / R);
    launch_kernel(kernel, grid, 32 * W * R, smem, stream, pdl, p);
    return check_launch();
}

template <int CW, int CPS, int CH, int ST, int MODE>
int launch_bulk(Params p, cudaStream_t stream, bool pdl);

template <int MODE>
int run_fallback(Params p, cudaStream_t stream, bool pdl);

template <int MODE>
int dispatch_fallback(int64_t id, Params p, cudaStream_t stream, bool pdl);

template <int FAM, int W, int R, int PK, int U, int CH, int ST>
struct Launcher;

template <int W, int R, int PK, int U, int CH, int ST>
struct Launcher<SWB_FAM_LDG, W, R, PK, U, CH, ST> {
    template <int MODE>
    static int run(Params p, cudaStream_t s, bool pdl) {
        return launch_ldg<W, R, PK, U, MODE>(p, s, pdl);
    }
};

template <int W, int R, int PK, int U, int CH, int ST>
struct Launcher<SWB_FAM_BULK, W, R, PK, U, CH, ST> {
    template <int MODE>
    static int run(Params p, cudaStream_t s, bool pdl) {
        return launch_bulk<W, R, CH, ST, MODE>(p, s, pdl);
    }
};

// Copies a BULK / RBULK producer keeps in flight once its ring is full: enough
// for about SWB_INFLIGHT_TARGET bytes per SM (at least two, at most the ring).
// The first ring-full still goes out at once. 0 keeps the whole ring in flight.
#ifndef SWB_INFLIGHT_TARGET
#define SWB_INFLIGHT_TARGET 0
#endif
int inflight_cap(size_t stage_bytes, int cps, int stages) {
    if (SWB_INFLIGHT_TARGET <= 0 || stage_bytes == 0) return 0;
    const int d = int(size_t(SWB_INFLIGHT_TARGET) / (size_t(cps) * stage_bytes));
    return std::min(stages, std::max(2, d));
}

template <int CW, int CPS, int CH, int ST, int MODE>
int launch_bulk(Params p, cudaStream_t stream, bool pdl) {
    constexpr int NM = MODE == MODE_GATE ? 2 : 1;
    static std::atomic<uint64_t> smem_set{0};
    const bool aligned = (p.cols % 8) == 0 && (reinterpret_cast<uintptr_t>(p.w) % 16) == 0 &&
                         (NM == 1 || (reinterpret_cast<uintptr_t>(p.u) % 16) == 0);
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int G = std::min(sms * CPS, p.rows);
    const int rows_per_cta = (p.rows + G - 1) / G;
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 64;
    int stages = ST;
    while (stages >= 2 && bulk_layout(NM, CH, stages, p.cols, CW, rows_per_cta).total > budget) --stages;
    if (!aligned || stages < 2) return run_fallback<MODE>(p, stream, pdl);
    p.stages = stages;
    p.inflight = inflight_cap(size_t(NM) * CH * 2, CPS, stages);
    p.x_staged = 1;
    const size_t smem = bulk_layout(NM, CH, stages, p.cols, CW, rows_per_cta).total;
    auto kernel = bulk_kernel<CW, CH, MODE>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    launch_kernel(kernel, unsigned(G), (CW + 1) * 32, smem, stream, pdl, p);
    return check_launch();
}

template <int CW, int CPS, int MAXJ, int STAGE_BYTES, int ST, int MODE>
int launch_rbulk(Params p, cudaStream_t stream, bool pdl) {
    constexpr int NM = MODE == MODE_GATE ? 2 : 1;
    static std::atomic<uint64_t> smem_set{0};
    const int nv = p.cols / 8;
    const bool ok = (p.cols % 8) == 0 && (reinterpret_cast<uintptr_t>(p.w) % 16) == 0 &&
                    (NM == 1 || (reinterpret_cast<uintptr_t>(p.u) % 16) == 0) && nv <= MAXJ * CW * 32;
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int G = std::min(sms * CPS, p.rows);
    const int rows_per_cta = (p.rows + G - 1) / G;
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 64;
    const size_t row_bytes = size_t(NM) * p.cols * 2;
    int rs = int(std::max<size_t>(1, STAGE_BYTES / std::max<size_t>(row_bytes, 1)));
    rs = std::min(rs, rows_per_cta);
    int stages = 0;
    for (; rs >= 1; rs = rs > 1 ? rs / 2 : 0) {  // shrink the stage until at least two fit
        stages = ST;
        while (stages >= 2 && rbulk_layout(NM, rs, p.cols, stages, CW, rows_per_cta).total > budget) --stages;
        if (stages >= 2 || rs == 1) break;
    }
    if (!ok || rs < 1 || stages < 2) return dispatch_fallback<MODE>(SWB_RBULK_FALLBACK_ID, p, stream, pdl);
    // no deeper than the CTA's stages of work: a short shard then leaves shared
    // memory for the next kernel's CTAs to become resident early
    stages = std::min(stages, std::max(2, (rows_per_cta + rs - 1) / rs));
    p.stages = stages;
    p.inflight = inflight_cap(size_t(rs) * row_bytes, CPS, stages);
    p.row_stage = rs;
    const size_t smem = rbulk_layout(NM, rs, p.cols, stages, CW, rows_per_cta).total;
    auto kernel = rbulk_kernel<CW, MAXJ, CPS, MODE>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    launch_kernel(kernel, unsigned(G), (CW + 1) * 32, smem, stream, pdl, p);
    return check_launch();
}

// The fused tensor-parallel down projection (rbulk_allreduce_kernel). Every rank
// must launch the same grid: the plan depends only on the shape, the geometry
// and the SM count, which match across ranks of one machine.
template <int CW, int CPS, int MAXJ, int STAGE_BYTES, int ST, bool HALF>
int launch_rbulk_ar(Params p, const TpParams& tp, cudaStream_t stream, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    const int nv = p.cols / 8;
    if ((p.cols % 8) != 0 || (reinterpret_cast<uintptr_t>(p.w) % 16) != 0 || nv > MAXJ * CW * 32)
        return fail(SWB_E_UNSUPPORTED, "fused tensor-parallel path needs cols % 8 == 0, 16-byte rows and "
                                       "cols <= 8 * 32 * warps * unroll of the geometry");
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int G = std::min(sms * CPS, p.rows);
    if (G > kTpMaxCtas) return fail(SWB_E_UNSUPPORTED, "grid larger than the exchange supports");
    const int rows_per_cta = (p.rows + G - 1) / G;
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 128;
    const size_t row_bytes = size_t(p.cols) * 2;
    int rs = int(std::max<size_t>(1, STAGE_BYTES / std::max<size_t>(row_bytes, 1)));
    rs = std::min(rs, rows_per_cta);
    int stages = 0;
    for (; rs >= 1; rs = rs > 1 ? rs / 2 : 0) {
        stages = ST;
        while (stages >= 2 && rbulk_layout(1, rs, p.cols, stages, CW, rows_per_cta).total > budget) --stages;
        if (stages >= 2 || rs == 1) break;
    }
    if (rs < 1 || stages < 2) return fail(SWB_E_UNSUPPORTED, "shape does not fit the geometry's shared memory");
    stages = std::min(stages, std::max(2, (rows_per_cta + rs - 1) / rs));  // as launch_rbulk
    p.stages = stages;
    p.inflight = inflight_cap(size_t(rs) * row_bytes, CPS, stages);
    p.row_stage = rs;
    const size_t smem = rbulk_layout(1, rs, p.cols, stages, CW, rows_per_cta).total;
    auto kernel = rbulk_allreduce_kernel<CW, MAXJ, CPS, HALF>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    if (!pdl) {
        kernel<<<unsigned(G), (CW + 1) * 32, smem, stream>>>(p, tp);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(G));
        cfg.blockDim = dim3((CW + 1) * 32);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, kernel, p, tp);
    }
    return check_launch();
}

template <int W, int R, int PK, int U, int CH, int ST>
struct Launcher<SWB_FAM_RBULK, W, R, PK, U, CH, ST> {
    template <int MODE>
    static int run(Params p, cudaStream_t s, bool pdl) {
        return launch_rbulk<W, R, U, CH, ST, MODE>(p, s, pdl);
    }
    static int run_allreduce(const Params& p, const TpParams& tp, cudaStream_t s, bool pdl, bool half) {
        return half ? launch_rbulk_ar<W, R, U, CH, ST, true>(p, tp, s, pdl)
                    : launch_rbulk_ar<W, R, U, CH, ST, false>(p, tp, s, pdl);
    }
};

template <int CW, int CPS, int MAXJ, int STAGE_BYTES, int ST, int MODE>
int launch_sbulk(Params p, cudaStream_t stream, bool pdl) {
    constexpr int NM = MODE == MODE_GATE ? 2 : 1;
    static std::atomic<uint64_t> smem_set{0};
    const int nv = p.cols / 8;
    const bool ok = (p.cols % 8) == 0 && (reinterpret_cast<uintptr_t>(p.w) % 16) == 0 &&
                    (NM == 1 || (reinterpret_cast<uintptr_t>(p.u) % 16) == 0) && nv <= MAXJ * CW * 32;
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int resident = sms * CPS;
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 128;
    const size_t row_bytes = size_t(NM) * p.cols * 2;
    int rs = int(std::max<size_t>(1, STAGE_BYTES / std::max<size_t>(row_bytes, 1)));
    int stages = 0;
    for (; rs >= 1; rs = rs > 1 ? rs / 2 : 0) {  // shrink the stage until at least two fit
        stages = ST;
        while (stages >= 2 && sbulk_layout(NM, rs, p.cols, stages, CW).total > budget) --stages;
        if (stages >= 2 || rs == 1) break;
    }
    if (!ok || rs < 1 || stages < 2) return dispatch_fallback<MODE>(SWB_RBULK_FALLBACK_ID, p, stream, pdl);
    // About 16 blocks per resident CTA: the imbalance left at the end is under one block.
    const int per = (p.rows + resident * 16 - 1) / (resident * 16);
    const int rpb = std::max(rs, (per + rs - 1) / rs * rs);
    const int blocks = (p.rows + rpb - 1) / rpb;
    // Smallest stride >= blocks / resident that is coprime with blocks.
    int stride = std::max(1, blocks / resident);
    while (std::gcd(stride, blocks) != 1) ++stride;
    p.stages = stages;
    p.row_stage = rs;
    p.rows_per_block = rpb;
    p.blocks = blocks;
    p.block_stride = stride;
    const size_t smem = sbulk_layout(NM, rs, p.cols, stages, CW).total;
    auto kernel = sbulk_kernel<CW, MAXJ, CPS, MODE>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    launch_kernel(kernel, unsigned(blocks), (CW + 1) * 32, smem, stream, pdl, p);
    return check_launch();
}

template <int W, int R, int PK, int U, int CH, int ST>
struct Launcher<SWB_FAM_SBULK, W, R, PK, U, CH, ST> {
    template <int MODE>
    static int run(Params p, cudaStream_t s, bool pdl) {
        return launch_sbulk<W, R, U, CH, ST, MODE>(p, s, pdl);
    }
};

template <int FAM>
struct AllreduceDispatch {
    template <int W, int R, int PK, int U, int CH, int ST>
    static int run(const Params&, const TpParams&, cudaStream_t, bool, bool) {
        return fail(SWB_E_CONFIG_INVALID, "the fused tensor-parallel path needs an RBULK geometry");
    }
};

template <>
struct AllreduceDispatch<SWB_FAM_RBULK> {
    template <int W, int R, int PK, int U, int CH, int ST>
    static int run(const Params& p, const TpParams& tp, cudaStream_t s, bool pdl, bool half) {
        return Launcher<SWB_FAM_RBULK, W, R, PK, U, CH, ST>::run_allreduce(p, tp, s, pdl, half);
    }
};

int dispatch_allreduce_one(int64_t id, const Params& p, const TpParams& tp, cudaStream_t s, bool pdl, bool half);

// RBULK geometries tried, in order, when the requested one cannot hold a row of
// the shape (the fused epilogue exists only in the RBULK kernel).
constexpr int kAllreduceFallbacks[] = {87, 85, 82};

// half: fp16 rows into p.h (the model path) instead of fp32 into p.y.
int dispatch_allreduce(int64_t id, const Params& p, const TpParams& tp, cudaStream_t s, bool pdl, bool half = false) {
    int rc = dispatch_allreduce_one(id, p, tp, s, pdl, half);
    if (rc != SWB_E_UNSUPPORTED) return rc;
    for (int alt : kAllreduceFallbacks) {
        if (alt == id) continue;
        rc = dispatch_allreduce_one(alt, p, tp, s, pdl, half);
        if (rc != SWB_E_UNSUPPORTED) return rc;
    }
    return rc;
}

int dispatch_allreduce_one(int64_t id, const Params& p, const TpParams& tp, cudaStream_t s, bool pdl, bool half) {
    switch (id) {
#define SWB_AR_CASE(ID, FAM, W, R, PK, U, CH, ST) \
    case ID:                                      \
        return AllreduceDispatch<FAM>::template run<W, R, PK, U, CH, ST>(p, tp, s, pdl, half);
        SWB_CONFIGS(SWB_AR_CASE)
#undef SWB_AR_CASE
        default:
            return fail(SWB_E_CONFIG);
    }
}

template <int MODE>
int dispatch(int64_t id, const Params& p, cudaStream_t s, bool pdl = false) {
    switch (id) {
#define SWB_CASE(ID, FAM, W, R, PK, U, CH, ST) \
    case ID:                                   \
        return Launcher<FAM, W, R, PK, U, CH, ST>::template run<MODE>(p, s, pdl);
        SWB_CONFIGS(SWB_CASE)
#undef SWB_CASE
        default:
            return fail(SWB_E_CONFIG);
    }
}

template <int MODE>
int run_fallback(Params p, cudaStream_t stream, bool pdl) {
    return dispatch<MODE>(SWB_BULK_FALLBACK_ID, p, stream, pdl);
}

template <int MODE>
int dispatch_fallback(int64_t id, Params p, cudaStream_t stream, bool pdl) {
    return dispatch<MODE>(id, p, stream, pdl);
}

// ---------------------------------------------------------------- layer
template <int CW, int CPS, int TARGET, int ST, bool TP>
int launch_layer(LayerParams L, const TpParams& tp, cudaStream_t stream) {
    static std::atomic<uint64_t> smem_set{0};
    constexpr int CT = CW * 32;
    const bool ok = L.hidden % 8 == 0 && L.inter % 8 == 0 && (reinterpret_cast<uintptr_t>(L.wg) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(L.wu) % 16) == 0 && (reinterpret_cast<uintptr_t>(L.wd) % 16) == 0 &&
                    L.hidden / 8 <= kLayerMaxJ * CT && L.inter / 8 <= kLayerMaxJ * CT;
    if (!ok) return fail(SWB_E_UNSUPPORTED, "layer geometry cannot hold a row of this shape");
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int G = std::min({sms * CPS, L.inter, L.hidden});
    if (G > kLayerMaxCtas || G > kTpMaxCtas) return fail(SWB_E_UNSUPPORTED, "grid larger than the barrier table");
    const size_t row1 = size_t(4) * L.hidden, row2 = size_t(2) * L.inter;
    const size_t stage = align_up(std::max<size_t>({size_t(TARGET), row1, row2}), 16);
    const int rpc1 = (L.inter + G - 1) / G, rpc2 = (L.hidden + G - 1) / G;
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 128;
    int stages = ST;
    while (stages >= 2 && layer_layout(int(stage), stages, CW, rpc1, rpc2).total > budget) --stages;
    if (stages < 2) return fail(SWB_E_UNSUPPORTED, "layer does not fit the geometry's shared memory");
    L.stage_bytes = int(stage);
    L.stages = stages;
    L.rs1 = std::max(1, std::min(int(stage / row1), rpc1));
    L.rs2 = std::max(1, std::min(int(stage / row2), rpc2));
    const size_t smem = layer_layout(L.stage_bytes, stages, CW, rpc1, rpc2).total;
    auto kernel = layer_kernel<CW, CPS, TP>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    // The grid barrier needs every CTA resident at once: a cooperative launch
    // makes the runtime check that instead of leaving it to chance.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(G));
    cfg.blockDim = dim3((CW + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, L, tp);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SWB_E_CUDA, cudaGetErrorString(e));
    }
    return check_launch();
}

// The streaming whole-layer kernel (stream_layer_kernel); `pdl`: launched programmatically
// after the kernel before it (SWB_PREFETCH_WEIGHTS), else cooperatively. Either way the grid
// is no larger than the CTAs that fit on the GPU at once.
template <int CW, int CPS, int RSPLIT, int MAXR, int TARGET, int ST, bool TP>
int launch_stream_layer(LayerParams L, const TpParams& tp, cudaStream_t stream, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    constexpr int CT = CW * 32;
    constexpr int CB = 8 * CT / RSPLIT;
    const int H = L.hidden, I = L.inter;
    const bool ok = H % 8 == 0 && I % 8 == 0 && (reinterpret_cast<uintptr_t>(L.wg) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(L.wu) % 16) == 0 && (reinterpret_cast<uintptr_t>(L.wd) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(L.h) % 16) == 0 && H / 8 <= kLayerMaxJ * CT;
    if (!ok) return fail(SWB_E_UNSUPPORTED, "streaming layer needs 16-byte rows, h and weights, and a slice of x "
                                            "that fits the geometry");
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const int G = std::min({sms * CPS, I, H});
    if (G > kTpMaxCtas) return fail(SWB_E_UNSUPPORTED, "grid larger than the exchange supports");
    const int rpc1 = (I + G - 1) / G, rpc2 = (H + G - 1) / G;
    if ((rpc2 + RSPLIT - 1) / RSPLIT > MAXR) return fail(SWB_E_UNSUPPORTED, "more y rows per CTA than the geometry holds");
    if ((I + CB - 1) / CB > kStreamMaxBlocks) return fail(SWB_E_UNSUPPORTED, "more h blocks than the workspace holds");
    if (I > kStreamMaxInter) return fail(SWB_E_UNSUPPORTED, "h larger than the streaming layer's shared copy");
    // gate rows per stage: the target bytes, and few enough that a stage's rows (G apart) touch
    // at most two blocks of h
    int rs1 = std::max(1, TARGET / (4 * H));
    rs1 = std::max(1, std::min({rs1, 1 + (CB - 1) / G, rpc1}));
    const int stage = int(align_up(std::max<size_t>(size_t(rs1) * 4 * H, size_t(rpc2) * CB * 2), 16));
    const size_t budget = std::min(kSmemPerCtaMax, kSmemPerSm / CPS - 1024) - 128;
    const int units1 = (rpc1 + rs1 - 1) / rs1, nblk = (I + CB - 1) / CB;
    int stages = ST;
    while (stages >= 2 && stream_layout(stage, stages, CW, rpc1, rpc2, units1, nblk, I).total > budget) --stages;
    if (stages < 2) return fail(SWB_E_UNSUPPORTED, "streaming layer does not fit the geometry's shared memory");
    L.rs1 = rs1;
    L.stages = stages;
    L.stage_bytes = stage;
    const size_t smem = stream_layout(stage, stages, CW, rpc1, rpc2, units1, nblk, I).total;
    auto kernel = stream_layer_kernel<CW, CPS, RSPLIT, MAXR, TP>;
    if (int rc = ensure_smem(kernel, smem_set, smem)) return rc;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, (CW + 3) * 32, smem);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (per_sm * sms < G) return fail(SWB_E_UNSUPPORTED, "the streaming layer's CTAs do not fit at once");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(G));
    cfg.blockDim = dim3((CW + 3) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    } else {
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, L, tp);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SWB_E_CUDA, cudaGetErrorString(e));
    }
    return check_launch();
}

constexpr int kLayerIds[] = {
#define SWB_LAYER_ID(ID, CW, CPS, TGT, ST) ID,
    SWB_LAYER_CONFIGS(SWB_LAYER_ID)
#undef SWB_LAYER_ID
#define SWB_STREAM_ID(ID, CW, CPS, RS, MR, TGT, ST) ID,
    SWB_STREAM_LAYER_CONFIGS(SWB_STREAM_ID)
#undef SWB_STREAM_ID
};
static_assert(SWB_LAYER_WORKSPACE_BYTES == 4 * kLayerWorkspaceWords, "layer workspace words");

bool is_layer_config(int64_t id) {
    for (int v : kLayerIds)
        if (v == id) return true;
    return false;
}

// pdl: SWB_PREFETCH_WEIGHTS, honoured by the streaming kernels (the barrier kernels are
// always launched cooperatively).
template <bool TP>
int dispatch_layer_one(int64_t id, const LayerParams& L, const TpParams& tp, cudaStream_t s, bool pdl) {
    switch (id) {
#define SWB_LAYER_CASE(ID, CW, CPS, TGT, ST) \
    case ID:                                 \
        return launch_layer<CW, CPS, TGT, ST, TP>(L, tp, s);
        SWB_LAYER_CONFIGS(SWB_LAYER_CASE)
#undef SWB_LAYER_CASE
#define SWB_STREAM_CASE(ID, CW, CPS, RS, MR, TGT, ST) \
    case ID:                                          \
        return launch_stream_layer<CW, CPS, RS, MR, TGT, ST, TP>(L, tp, s, pdl);
        SWB_STREAM_LAYER_CONFIGS(SWB_STREAM_CASE)
#undef SWB_STREAM_CASE
        default:
            return fail(SWB_E_CONFIG);
    }
}

template <bool TP>
int dispatch_layer(int64_t id, const LayerParams& L, const TpParams& tp, cudaStream_t s, bool pdl = false) {
    int rc = dispatch_layer_one<TP>(id, L, tp, s, pdl);
    for (int i = 0; i < 2 && rc == SWB_E_UNSUPPORTED; ++i)
        if (kLayerIds[i] != id) rc = dispatch_layer_one<TP>(kLayerIds[i], L, tp, s, pdl);
    return rc;
}

bool overlaps(const void* a, size_t abytes, const void* b, size_t bbytes) {
    const uintptr_t ap = reinterpret_cast<uintptr_t>(a), bp = reinterpret_cast<uintptr_t>(b);
    return ap < bp + bbytes && bp < ap + abytes;
}

Params make_params() {
    Params p;
    std::memset(&p, 0, sizeof p);
    return p;
}

// The device address of page-locked host memory this device maps (every
// cudaHostAlloc / cudaHostRegister buffer under unified addressing), or null for
// anything else -- pageable or device memory is rejected before any launch.
const void* mapped_host(const void* p) {
    cudaPointerAttributes a;
    std::memset(&a, 0, sizeof a);
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// transfer_kernel over `bytes`: 256 threads per CTA, one 16-byte piece per thread,
// at most one CTA per SM. pdl: launched programmatically after the previous kernel.
int launch_transfer(const void* src, void* dst, size_t bytes, cudaStream_t stream, bool pdl) {
    const int sms = sm_count();
    if (sms <= 0) return check_launch();
    const size_t pieces = (bytes + 15) / 16;
    const unsigned block = 256;
    const unsigned grid = unsigned(std::max<size_t>(1, std::min<size_t>(size_t(sms), (pieces + block - 1) / block)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, transfer_kernel, static_cast<const unsigned char*>(src), static_cast<unsigned char*>(dst),
                       bytes);
    return check_launch();
}

}  // namespace
}  // namespace swb

using namespace swb;

extern "C" {

const char* swb_status_string(int status) {
    switch (status) {
        case SWB_OK: return "ok";
        case SWB_E_INPUT: return "invalid projection input";
        case SWB_E_GATE_BUFFERS: return "invalid gate buffers";
        case SWB_E_HALF_OUTPUT: return "missing half output";
        case SWB_E_FLOAT_OUTPUT: return "missing float output";
        case SWB_E_RESIDUAL: return "missing residual";
        case SWB_E_CONFIG: return "unknown kernel configuration";
        case SWB_E_SHAPE: return "invalid shape";
        case SWB_E_CONFIG_RANGE: return "configuration out of range";
        case SWB_E_CONFIG_INVALID: return "invalid configuration";
        case SWB_E_OVERLAP_INPUT: return "workspace overlaps input storage";
        case SWB_E_OVERLAP_OUTPUT: return "scratch and output overlap";
        case SWB_E_CUDA: return "CUDA error";
        case SWB_E_DEVICE: return "device-side error";
        case SWB_E_UNSUPPORTED: return "unsupported device";
        case SWB_E_WORKSPACE: return "intermediate size exceeds the built-in workspace";
        default: return "unknown status";
    }
}

const char* swb_last_error(void) { return g_last_error.c_str(); }

int swb_version(void) { return 1; }

int swb_cuda_versions(int* driver, int* runtime) {
    int d = 0, r = 0;
    cudaError_t e = cudaDriverGetVersion(&d);
    if (e == cudaSuccess) e = cudaRuntimeGetVersion(&r);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (driver) *driver = d;
    if (runtime) *runtime = r;
    return SWB_OK;
}

int swb_config_count(void) { return kConfigCount; }

int swb_config_ids(int* out, int cap) {
    if (out)
        for (int i = 0; i < kConfigCount && i < cap; ++i) out[i] = kConfigs[i].id;
    return kConfigCount;
}

int swb_valid_config(int64_t id) { return find_config(id) != nullptr; }

int swb_config_info(int64_t id, swb_config_t* out) {
    const swb_config_t* c = find_config(id);
    if (!c) return fail(SWB_E_CONFIG);
    if (out) *out = *c;
    return SWB_OK;
}

}  // extern "C"

namespace {
// swb_gate; `epoch` (tensor parallel) is the exchange's call epoch, which the
// kernel advances for the fused down kernel that follows.
int gate_impl(int config, const void* wg, const void* wu, const void* x, const void* bg, const void* bu, void* h,
              int rows, int cols, int model_round, void* stream, uint32_t* epoch, bool pdl = false) {
    if (rows <= 0 || cols <= 0 || !wg || !x) return fail(SWB_E_INPUT);
    if (!wu || !h) return fail(SWB_E_GATE_BUFFERS);
    if (!find_config(config)) return fail(SWB_E_CONFIG);
    Params p = make_params();
    p.epoch = epoch;
    p.w = static_cast<const __half*>(wg);
    p.u = static_cast<const __half*>(wu);
    p.x = static_cast<const __half*>(x);
    p.bias = static_cast<const __half*>(bg);
    p.ubias = static_cast<const __half*>(bu);
    p.h = static_cast<__half*>(h);
    p.rows = rows;
    p.cols = cols;
    p.model_round = model_round ? 1 : 0;
    return dispatch<MODE_GATE>(config, p, static_cast<cudaStream_t>(stream), pdl);
}
}  // namespace

extern "C" {

int swb_gate(int config, const void* wg, const void* wu, const void* x, const void* bg, const void* bu, void* h,
             int rows, int cols, int model_round, void* stream) {
    return gate_impl(config, wg, wu, x, bg, bu, h, rows, cols, model_round, stream, nullptr);
}

namespace {
// swb_project with an optional programmatic dependent launch (see launch_kernel).
int project_impl(int config, const void* w, const void* x, const void* bias, const void* residual, void* out,
                 int rows, int cols, unsigned flags, void* stream, bool pdl, float* y_host = nullptr) {
    if (rows <= 0 || cols <= 0 || !w || !x) return fail(SWB_E_INPUT);
    const bool half_out = (flags & SWB_HALF_OUT) != 0;
    if (!out) return fail(half_out ? SWB_E_HALF_OUTPUT : SWB_E_FLOAT_OUTPUT);
    if ((flags & SWB_RESIDUAL) && !residual) return fail(SWB_E_RESIDUAL);
    if (!find_config(config)) return fail(SWB_E_CONFIG);
    Params p = make_params();
    p.w = static_cast<const __half*>(w);
    p.x = static_cast<const __half*>(x);
    p.bias = static_cast<const __half*>(bias);
    p.residual = (flags & SWB_RESIDUAL) ? static_cast<const __half*>(residual) : nullptr;
    p.rows = rows;
    p.cols = cols;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (half_out) {
        p.h = static_cast<__half*>(out);
        return dispatch<MODE_F16>(config, p, s, pdl);
    }
    p.y = static_cast<float*>(out);
    p.y_host = y_host;
    return dispatch<MODE_F32>(config, p, s, pdl);
}
}  // namespace

int swb_project(int config, const void* w, const void* x, const void* bias, const void* residual, void* out,
                int rows, int cols, unsigned flags, void* stream) {
    return project_impl(config, w, x, bias, residual, out, rows, cols, flags, stream, false);
}

int swb_ffn(int gate_config, int down_config, const void* wg, const void* wu, const void* wd, const void* x,
            const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden, int inter,
            void* stream) {
    return swb_ffn_ex(gate_config, down_config, wg, wu, wd, x, bg, bu, bd, h, y, hidden, inter, 0u, stream);
}

int swb_ffn_ex(int gate_config, int down_config, const void* wg, const void* wu, const void* wd, const void* x,
               const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden, int inter,
               unsigned flags, void* stream) {
    if (flags & ~SWB_PREFETCH_WEIGHTS) return fail(SWB_E_INPUT, "unknown launch flags");
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG);
    if (!wd) return fail(SWB_E_INPUT);
    if (!y) return fail(SWB_E_FLOAT_OUTPUT);
    if (int rc = gate_impl(gate_config, wg, wu, x, bg, bu, h, inter, hidden, 0, stream, nullptr,
                           (flags & SWB_PREFETCH_WEIGHTS) != 0))
        return rc;
    return project_impl(down_config, wd, h, bd, x, y, hidden, inter, SWB_RESIDUAL, stream, true);
}

int swb_ffn_host_ex(int gate_config, int down_config, const void* wg, const void* wu, const void* wd,
                    const void* x_host, const void* bg, const void* bu, const void* bd, void* x, void* h, float* y,
                    float* y_host, int hidden, int inter, unsigned flags, void* stream) {
    if (flags & ~SWB_PREFETCH_WEIGHTS) return fail(SWB_E_INPUT, "unknown launch flags");
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG);
    if (hidden <= 0 || inter <= 0 || !wg || !wd || !x_host || !x) return fail(SWB_E_INPUT);
    if (!wu || !h) return fail(SWB_E_GATE_BUFFERS);
    if (!y || !y_host) return fail(SWB_E_FLOAT_OUTPUT);
    const size_t xb = size_t(hidden) * 2, hb = size_t(inter) * 2, yb = size_t(hidden) * 4;
    if (overlaps(x, xb, h, hb) || overlaps(x, xb, y, yb) || overlaps(h, hb, y, yb)) return fail(SWB_E_OVERLAP_OUTPUT);
    const void* xs = mapped_host(x_host);
    void* yd = const_cast<void*>(mapped_host(y_host));
    if (!xs || !yd)
        return fail(SWB_E_INPUT, "x_host and y_host must be page-locked host memory mapped for this device "
                                 "(cudaHostAlloc or cudaHostRegister)");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // x in; without SWB_PREFETCH_WEIGHTS after everything before the call has finished
    if (int rc = launch_transfer(xs, x, xb, s, (flags & SWB_PREFETCH_WEIGHTS) != 0)) return rc;
    // the gate may stream its weights while x crosses the bus (the transfer writes no weight)
    if (int rc = gate_impl(gate_config, wg, wu, x, bg, bu, h, inter, hidden, 0, stream, nullptr, true)) return rc;
    // y out: the BULK, RBULK and SBULK down kernels store it to the host buffer in their epilogue as
    // well (consecutive threads write consecutive rows); after an LDG down kernel, whose rows are
    // written one thread each, a transfer kernel copies it
    const swb_config_t* dc = find_config(down_config);
    const bool fold = dc->family != SWB_FAM_LDG;
    if (int rc = project_impl(down_config, wd, h, bd, x, y, hidden, inter, SWB_RESIDUAL, stream, true,
                              fold ? static_cast<float*>(yd) : nullptr))
        return rc;
    return fold ? SWB_OK : launch_transfer(y, yd, yb, s, true);
}

int swb_ffn_tp(int gate_config, int down_config, const void* wg_shard, const void* wu_shard, const void* wd_shard,
               const void* x, const void* bg_shard, const void* bu_shard, void* h_shard, float* y_partial, int hidden,
               int shard, void* stream) {
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG);
    if (!wd_shard) return fail(SWB_E_INPUT);
    if (!y_partial) return fail(SWB_E_FLOAT_OUTPUT);
    if (int rc = swb_gate(gate_config, wg_shard, wu_shard, x, bg_shard, bu_shard, h_shard, shard, hidden, 0, stream))
        return rc;
    return project_impl(down_config, wd_shard, h_shard, nullptr, nullptr, y_partial, hidden, shard, 0, stream, true);
}

int swb_swiglu_out(const void* x, const void* gate, const void* up, const void* down, void* h, void* y,
                   int64_t hidden, int64_t intermediate, int64_t gate_config, int64_t down_config, void* stream) {
    if (!(hidden > 0 && intermediate > 0 && hidden <= 100000 && intermediate <= 100000)) return fail(SWB_E_SHAPE);
    if (!(gate_config >= 0 && gate_config <= 1000 && down_config >= 0 && down_config <= 1000))
        return fail(SWB_E_CONFIG_RANGE);
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG_INVALID);
    if (!x || !gate || !down) return fail(SWB_E_INPUT);
    if (!up || !h) return fail(SWB_E_GATE_BUFFERS);
    if (!y) return fail(SWB_E_HALF_OUTPUT);
    const size_t hb = size_t(hidden) * 2, ib = size_t(intermediate) * 2, wb = size_t(hidden) * size_t(intermediate) * 2;
    const void* inputs[4] = {x, gate, up, down};
    const size_t sizes[4] = {hb, wb, wb, wb};
    for (int i = 0; i < 4; ++i)
        if (overlaps(h, ib, inputs[i], sizes[i]) || overlaps(y, hb, inputs[i], sizes[i]))
            return fail(SWB_E_OVERLAP_INPUT);
    if (overlaps(h, ib, y, hb)) return fail(SWB_E_OVERLAP_OUTPUT);
    if (int rc = swb_gate(int(gate_config), gate, up, x, nullptr, nullptr, h, int(intermediate), int(hidden), 1, stream))
        return rc;
    return project_impl(int(down_config), down, h, nullptr, nullptr, y, int(hidden), int(intermediate), SWB_HALF_OUT,
                        stream, true);
}

int swb_gate_epilogue(const float* a, const float* b, const void* bg, const void* bu, void* h, int n, void* stream) {
    if (n <= 0 || !a || !b || !bg || !bu || !h) return fail(SWB_E_INPUT);
    gate_epilogue_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        a, b, static_cast<const __half*>(bg), static_cast<const __half*>(bu), static_cast<__half*>(h), n);
    return check_launch();
}

int swb_residual_epilogue(float* y, const void* bias, const void* x, int n, void* stream) {
    if (n <= 0 || !y || !bias || !x) return fail(SWB_E_INPUT);
    residual_epilogue_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        y, static_cast<const __half*>(bias), static_cast<const __half*>(x), n);
    return check_launch();
}

int swb_device_error(int clear, int* out) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof v);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero);
        if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    }
    if (out) *out = v;
    return SWB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// swb_ffn_noalloc: the layer for callers that cannot allocate device memory.
// h lives in this fixed array (one copy per device that loads the library).
// Host code must not hand `g_noalloc_h` to a kernel directly -- on the host the
// name is only a stand-in; its device address is looked up per device below.
namespace {

static __device__ __align__(256) __half g_noalloc_h[SWB_NOALLOC_MAX_INTER];

std::atomic<void*> g_noalloc_ptr[64];

// Device address of g_noalloc_h on the current device, looked up once per device
// and kept for the life of the process (a device reset, which may reload the module
// elsewhere, needs a fresh process).
int noalloc_workspace(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(SWB_E_UNSUPPORTED, "device index beyond 63");
    void* p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        e = cudaGetSymbolAddress(&p, g_noalloc_h);
        if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
        if (!p) return fail(SWB_E_CUDA, "no device address for the built-in workspace");
        g_noalloc_ptr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return SWB_OK;
}

}  // namespace

extern "C" int swb_ffn_noalloc(int gate_config, int down_config, const void* wg, const void* wu, const void* wd,
                               const void* x, const void* bg, const void* bu, const void* bd, float* y, int hidden,
                               int inter, void* stream) {
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG);
    if (hidden <= 0 || inter <= 0 || !wg || !x || !wd) return fail(SWB_E_INPUT);
    if (!wu) return fail(SWB_E_GATE_BUFFERS);
    if (!y) return fail(SWB_E_FLOAT_OUTPUT);
    if (inter > SWB_NOALLOC_MAX_INTER)
        return fail(SWB_E_WORKSPACE, "swb_ffn_noalloc holds at most 65536 intermediate values");
    void* h = nullptr;
    if (int rc = noalloc_workspace(&h)) return rc;
    return swb_ffn(gate_config, down_config, wg, wu, wd, x, bg, bu, bd, h, y, hidden, inter, stream);
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange: one per rank, allocated once at set-up.
// A rank's exchange buffer (one cudaMalloc, mapped by every peer through CUDA IPC):
//   [recv slots: 2 parities x world x rows x 8 B][call counter: 256 B][layer grid-barrier slots]
struct swb_tp {
    int rank, world, rows, device;
    void* local;
    size_t bytes, recv_bytes;
    void* peer[kTpMaxRanks];
    bool connected;
};

namespace {
constexpr size_t kTpCounterBytes = 256;
size_t tp_recv_bytes(int world, int rows) { return align_up(size_t(2) * world * rows * 8, 256); }

TpParams tp_params(const swb_tp* tp, const void* bd, const void* x) {
    TpParams t;
    std::memset(&t, 0, sizeof t);
    for (int q = 0; q < tp->world; ++q) t.recv[q] = static_cast<unsigned long long*>(tp->peer[q]);
    t.ctr = reinterpret_cast<uint32_t*>(static_cast<char*>(tp->local) + tp->recv_bytes);
    t.bias = static_cast<const __half*>(bd);
    t.residual = static_cast<const __half*>(x);
    t.rank = tp->rank;
    t.world = tp->world;
    return t;
}
}  // namespace

extern "C" {

int swb_tp_create(int rank, int world, int rows, swb_tp_t** out) {
    if (!out || world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world || rows <= 0)
        return fail(SWB_E_INPUT, "rank, world (1..8) or rows out of range");
    swb_tp* tp = new (std::nothrow) swb_tp();
    if (!tp) return fail(SWB_E_INPUT, "out of host memory");
    tp->rank = rank;
    tp->world = world;
    tp->rows = rows;
    tp->recv_bytes = tp_recv_bytes(world, rows);
    tp->bytes = tp->recv_bytes + kTpCounterBytes + SWB_LAYER_WORKSPACE_BYTES;
    cudaError_t e = cudaGetDevice(&tp->device);
    if (e == cudaSuccess) e = cudaMalloc(&tp->local, tp->bytes);  // set-up time, once per rank
    if (e == cudaSuccess) e = cudaMemset(tp->local, 0, tp->bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (tp->local) cudaFree(tp->local);
        delete tp;
        return fail(SWB_E_CUDA, cudaGetErrorString(e));
    }
    for (int q = 0; q < kTpMaxRanks; ++q) tp->peer[q] = nullptr;
    tp->peer[rank] = tp->local;
    tp->connected = world == 1;
    *out = tp;
    return SWB_OK;
}

int swb_tp_ipc_handle(const swb_tp_t* tp, void* out) {
    if (!tp || !out) return fail(SWB_E_INPUT, "null exchange or output");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, tp->local);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    static_assert(sizeof(h) == SWB_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(out, &h, sizeof h);
    return SWB_OK;
}

int swb_tp_connect(swb_tp_t* tp, const void* handles) {
    if (!tp || !handles) return fail(SWB_E_INPUT, "null exchange or handles");
    if (tp->connected) return SWB_OK;
    for (int q = 0; q < tp->world; ++q) {
        if (q == tp->rank || tp->peer[q]) continue;  // a retry after a partial failure keeps what it opened
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + size_t(q) * SWB_TP_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
        tp->peer[q] = p;
    }
    tp->connected = true;
    return SWB_OK;
}

int swb_tp_epoch(const swb_tp_t* tp, uint32_t* out) {
    if (!tp || !out) return fail(SWB_E_INPUT, "null exchange or output");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != tp->device)
        return fail(SWB_E_INPUT, "the current device is not the exchange's device");
    uint32_t v = 0;
    const void* ctr = static_cast<const char*>(tp->local) + tp->recv_bytes;
    cudaError_t e = cudaDeviceSynchronize();  // calls on any stream have counted
    if (e == cudaSuccess) e = cudaMemcpy(&v, ctr, sizeof v, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(SWB_E_CUDA, cudaGetErrorString(e));
    *out = v;
    return SWB_OK;
}

int swb_tp_destroy(swb_tp_t* tp) {
    if (!tp) return SWB_OK;
    for (int q = 0; q < tp->world; ++q)
        if (q != tp->rank && tp->peer[q]) cudaIpcCloseMemHandle(tp->peer[q]);
    if (tp->local) cudaFree(tp->local);
    delete tp;
    return SWB_OK;
}

int swb_ffn_tp_fused(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard, const void* wu_shard,
                     const void* wd_shard, const void* x, const void* bg_shard, const void* bu_shard, const void* bd,
                     void* h_shard, float* y, int hidden, int shard, void* stream) {
    return swb_ffn_tp_fused_ex(tp, gate_config, down_config, wg_shard, wu_shard, wd_shard, x, bg_shard, bu_shard, bd,
                               h_shard, y, hidden, shard, 0u, stream);
}

namespace swb {
namespace {
// The rank's layer with the fused exchange, after the entry points' guards: a
// whole-layer id (gate_config 200+) as one persistent kernel, else the gate (which
// advances the call epoch) and the fused down + exchange kernel. pdl: the gate, or
// a streaming whole-layer kernel, is launched programmatically.
int tp_fused_launch(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard, const void* wu_shard,
                    const void* wd_shard, const void* x, const void* bg_shard, const void* bu_shard, const void* bd,
                    void* h_shard, float* y, int hidden, int shard, bool pdl, cudaStream_t stream,
                    float* y_host = nullptr) {
    TpParams t = tp_params(tp, bd, x);
    t.y_host = y_host;  // the reduced y also stored to mapped host memory (swb_ffn_tp_host_ex)
    if (is_layer_config(gate_config)) {  // one persistent kernel: gate, grid barrier, down + exchange
        if (!wg_shard || !wu_shard || !h_shard) return fail(SWB_E_GATE_BUFFERS);
        LayerParams L;
        std::memset(&L, 0, sizeof L);
        L.wg = static_cast<const __half*>(wg_shard);
        L.wu = static_cast<const __half*>(wu_shard);
        L.wd = static_cast<const __half*>(wd_shard);
        L.x = static_cast<const __half*>(x);
        L.bg = static_cast<const __half*>(bg_shard);
        L.bu = static_cast<const __half*>(bu_shard);
        L.h = static_cast<__half*>(h_shard);
        L.y = y;
        L.hidden = hidden;
        L.inter = shard;
        L.sync = reinterpret_cast<uint32_t*>(static_cast<char*>(tp->local) + tp->recv_bytes + kTpCounterBytes);
        return dispatch_layer<true>(gate_config, L, t, stream, pdl);
    }
    // the gate kernel advances the call epoch; the down kernel reads it after griddepcontrol.wait
    if (int rc = gate_impl(gate_config, wg_shard, wu_shard, x, bg_shard, bu_shard, h_shard, shard, hidden, 0, stream,
                           t.ctr, pdl))
        return rc;
    Params p = make_params();
    p.w = static_cast<const __half*>(wd_shard);
    p.x = static_cast<const __half*>(h_shard);
    p.y = y;
    p.rows = hidden;
    p.cols = shard;
    p.epoch = t.ctr;
    return dispatch_allreduce(down_config, p, t, stream, true);
}

// Guards shared by the fused tensor-parallel entry points.
int tp_fused_guards(const swb_tp_t* tp, int gate_config, int down_config, const void* wd_shard, const void* x,
                    const float* y, int hidden, unsigned flags) {
    if (flags & ~SWB_PREFETCH_WEIGHTS) return fail(SWB_E_INPUT, "unknown launch flags");
    if (!tp || !tp->connected) return fail(SWB_E_INPUT, "exchange missing or not connected");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != tp->device)
        return fail(SWB_E_INPUT, "the current device is not the exchange's device");
    if (hidden != tp->rows) return fail(SWB_E_SHAPE, "hidden differs from the exchange's rows");
    if (!is_layer_config(gate_config) && (!find_config(gate_config) || !find_config(down_config)))
        return fail(SWB_E_CONFIG);
    if (!wd_shard || !x) return fail(SWB_E_INPUT);
    if (!y) return fail(SWB_E_FLOAT_OUTPUT);
    return SWB_OK;
}
}  // namespace
}  // namespace swb

int swb_ffn_tp_fused_ex(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard, const void* wu_shard,
                        const void* wd_shard, const void* x, const void* bg_shard, const void* bu_shard,
                        const void* bd, void* h_shard, float* y, int hidden, int shard, unsigned flags,
                        void* stream) {
    if (int rc = tp_fused_guards(tp, gate_config, down_config, wd_shard, x, y, hidden, flags)) return rc;
    return tp_fused_launch(tp, gate_config, down_config, wg_shard, wu_shard, wd_shard, x, bg_shard, bu_shard, bd,
                           h_shard, y, hidden, shard, (flags & SWB_PREFETCH_WEIGHTS) != 0,
                           static_cast<cudaStream_t>(stream));
}

int swb_ffn_tp_host_ex(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard, const void* wu_shard,
                       const void* wd_shard, const void* x_host, const void* bg_shard, const void* bu_shard,
                       const void* bd, void* x, void* h_shard, float* y, float* y_host, int hidden, int shard,
                       unsigned flags, void* stream) {
    if (int rc = tp_fused_guards(tp, gate_config, down_config, wd_shard, x, y, hidden, flags)) return rc;
    if (!x_host || shard <= 0) return fail(SWB_E_INPUT);
    if (!h_shard) return fail(SWB_E_GATE_BUFFERS);
    if (!y_host) return fail(SWB_E_FLOAT_OUTPUT);
    const size_t xb = size_t(hidden) * 2, hb = size_t(shard) * 2, yb = size_t(hidden) * 4;
    if (overlaps(x, xb, h_shard, hb) || overlaps(x, xb, y, yb) || overlaps(h_shard, hb, y, yb))
        return fail(SWB_E_OVERLAP_OUTPUT);
    const void* xs = mapped_host(x_host);
    void* yd = const_cast<void*>(mapped_host(y_host));
    if (!xs || !yd)
        return fail(SWB_E_INPUT, "x_host and y_host must be page-locked host memory mapped for this device "
                                 "(cudaHostAlloc or cudaHostRegister)");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = launch_transfer(xs, x, xb, s, (flags & SWB_PREFETCH_WEIGHTS) != 0)) return rc;  // x in
    // y out: the exchange's epilogue stores the reduced rows to y_host as well (every rank the same y)
    return tp_fused_launch(tp, gate_config, down_config, wg_shard, wu_shard, wd_shard, x, bg_shard, bu_shard, bd,
                           h_shard, y, hidden, shard, true, s, static_cast<float*>(yd));
}

int swb_swiglu_tp_out(swb_tp_t* tp, const void* x, const void* gate_shard, const void* up_shard,
                      const void* down_shard, void* h_shard, void* y, int64_t hidden, int64_t shard,
                      int64_t gate_config, int64_t down_config, unsigned flags, void* stream) {
    if (flags & ~SWB_PREFETCH_WEIGHTS) return fail(SWB_E_INPUT, "unknown launch flags");
    if (!tp || !tp->connected) return fail(SWB_E_INPUT, "exchange missing or not connected");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != tp->device)
        return fail(SWB_E_INPUT, "the current device is not the exchange's device");
    // the binding's guards, in its order (src/torch_extension.cu:17-30), on the rank's shard
    if (!(hidden > 0 && shard > 0 && hidden <= 100000 && shard <= 100000)) return fail(SWB_E_SHAPE);
    if (hidden != tp->rows) return fail(SWB_E_SHAPE, "hidden differs from the exchange's rows");
    if (!(gate_config >= 0 && gate_config <= 1000 && down_config >= 0 && down_config <= 1000))
        return fail(SWB_E_CONFIG_RANGE);
    if (!find_config(gate_config) || !find_config(down_config)) return fail(SWB_E_CONFIG_INVALID);
    if (!x || !gate_shard || !down_shard) return fail(SWB_E_INPUT);
    if (!up_shard || !h_shard) return fail(SWB_E_GATE_BUFFERS);
    if (!y) return fail(SWB_E_HALF_OUTPUT);
    const size_t hb = size_t(hidden) * 2, sb = size_t(shard) * 2, wb = size_t(hidden) * size_t(shard) * 2;
    const void* inputs[4] = {x, gate_shard, up_shard, down_shard};
    const size_t sizes[4] = {hb, wb, wb, wb};
    for (int i = 0; i < 4; ++i)
        if (overlaps(h_shard, sb, inputs[i], sizes[i]) || overlaps(y, hb, inputs[i], sizes[i]))
            return fail(SWB_E_OVERLAP_INPUT);
    if (overlaps(h_shard, sb, y, hb)) return fail(SWB_E_OVERLAP_OUTPUT);
    const TpParams t = tp_params(tp, nullptr, nullptr);  // no bias, no residual: the model adds its own
    if (int rc = gate_impl(int(gate_config), gate_shard, up_shard, x, nullptr, nullptr, h_shard, int(shard),
                           int(hidden), 1, stream, t.ctr, (flags & SWB_PREFETCH_WEIGHTS) != 0))
        return rc;
    Params p = make_params();
    p.w = static_cast<const __half*>(down_shard);
    p.x = static_cast<const __half*>(h_shard);
    p.h = static_cast<__half*>(y);
    p.rows = int(hidden);
    p.cols = int(shard);
    p.epoch = t.ctr;
    return dispatch_allreduce(down_config, p, t, static_cast<cudaStream_t>(stream), true, true);
}

}  // extern "C"

extern "C" {

int swb_layer_config_count(void) { return int(sizeof(kLayerIds) / sizeof(kLayerIds[0])); }

int swb_layer_config_ids(int* out, int cap) {
    const int n = swb_layer_config_count();
    if (out)
        for (int i = 0; i < n && i < cap; ++i) out[i] = kLayerIds[i];
    return n;
}

int swb_ffn_fused(int layer_config, const void* wg, const void* wu, const void* wd, const void* x, const void* bg,
                  const void* bu, const void* bd, void* h, float* y, int hidden, int inter, void* workspace,
                  void* stream) {
    return swb_ffn_fused_ex(layer_config, wg, wu, wd, x, bg, bu, bd, h, y, hidden, inter, workspace, 0u, stream);
}

int swb_ffn_fused_ex(int layer_config, const void* wg, const void* wu, const void* wd, const void* x,
                     const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden, int inter,
                     void* workspace, unsigned flags, void* stream) {
    if (flags & ~SWB_PREFETCH_WEIGHTS) return fail(SWB_E_INPUT, "unknown launch flags");
    if (!is_layer_config(layer_config)) return fail(SWB_E_CONFIG);
    if (hidden <= 0 || inter <= 0 || !wg || !x || !wd) return fail(SWB_E_INPUT);
    if (!wu || !h) return fail(SWB_E_GATE_BUFFERS);
    if (!y) return fail(SWB_E_FLOAT_OUTPUT);
    if (!workspace) return fail(SWB_E_WORKSPACE, "swb_ffn_fused needs its SWB_LAYER_WORKSPACE_BYTES workspace");
    if (reinterpret_cast<uintptr_t>(workspace) % 16) return fail(SWB_E_WORKSPACE, "workspace must be 16-byte aligned");
    LayerParams L;
    std::memset(&L, 0, sizeof L);
    L.wg = static_cast<const __half*>(wg);
    L.wu = static_cast<const __half*>(wu);
    L.wd = static_cast<const __half*>(wd);
    L.x = static_cast<const __half*>(x);
    L.bg = static_cast<const __half*>(bg);
    L.bu = static_cast<const __half*>(bu);
    L.bd = static_cast<const __half*>(bd);
    L.h = static_cast<__half*>(h);
    L.y = y;
    L.sync = static_cast<uint32_t*>(workspace);
    L.hidden = hidden;
    L.inter = inter;
    TpParams t;
    std::memset(&t, 0, sizeof t);
    return dispatch_layer<false>(layer_config, L, t, static_cast<cudaStream_t>(stream),
                                 (flags & SWB_PREFETCH_WEIGHTS) != 0);
}

}  // extern "C"
