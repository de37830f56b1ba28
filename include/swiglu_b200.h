/*
 * swiglu_b200 -- C ABI of the B200 (sm_100a) batch-one SwiGLU decode layer.
 *
 *   gate = Wg x + bg,  up = Wu x + bu,  h = SiLU(gate) * up,  y = Wd h + bd + x
 *
 * fp16 weights/inputs, fp32 accumulation, fp16 h, fp32 (or fp16) y. Every layer
 * and projection entry point takes plain device pointers and sizes, launches
 * asynchronously on the given stream (a cudaStream_t, NULL = legacy default
 * stream) on the CURRENT device, allocates nothing, and returns 0 or a SWB_E_*
 * status; the only allocation is the tensor-parallel exchange buffer, once, in
 * swb_tp_create. Argument checks run before any CUDA call, so invalid calls fail
 * without touching a GPU.
 *
 * Each declaration names the interface of shubhxho/cuda-kernel it replaces.
 * Library: cuda-kernel_b200/lib/libswiglu_b200.so (cudart linked statically).
 */
#ifndef SWIGLU_B200_H
#define SWIGLU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef SWB_API
#define SWB_API __attribute__((visibility("default")))
#endif

/* ---- status codes; swb_status_string() gives the reference's message ---- */
#define SWB_OK 0
#define SWB_E_INPUT 1          /* "invalid projection input"      include/kernels.cuh:119 */
#define SWB_E_GATE_BUFFERS 2   /* "invalid gate buffers"          include/kernels.cuh:120 */
#define SWB_E_HALF_OUTPUT 3    /* "missing half output"           include/kernels.cuh:121 */
#define SWB_E_FLOAT_OUTPUT 4   /* "missing float output"          include/kernels.cuh:122 */
#define SWB_E_RESIDUAL 5       /* "missing residual"              include/kernels.cuh:123 */
#define SWB_E_CONFIG 6         /* "unknown kernel configuration"  include/kernels.cuh:130, config.hpp:19 */
#define SWB_E_SHAPE 7          /* "invalid shape"                 src/torch_extension.cu:17 */
#define SWB_E_CONFIG_RANGE 8   /* "configuration out of range"    src/torch_extension.cu:21 */
#define SWB_E_CONFIG_INVALID 9 /* "invalid configuration"         src/torch_extension.cu:22 */
#define SWB_E_OVERLAP_INPUT 10 /* "workspace overlaps input storage" src/torch_extension.cu:27-29 */
#define SWB_E_OVERLAP_OUTPUT 11 /* "scratch and output overlap"   src/torch_extension.cu:30 */
#define SWB_E_CUDA 12          /* CUDA runtime error; detail in swb_last_error() */
#define SWB_E_DEVICE 13        /* a kernel gave up a bounded wait (device error word set) */
#define SWB_E_UNSUPPORTED 14   /* no usable sm_100 device / feature */
#define SWB_E_WORKSPACE 15     /* size beyond the built-in workspace of swb_ffn_noalloc; a missing
                                  or misaligned swb_ffn_fused workspace */

/* project() flags (template flags of decode::launch, include/kernels.cuh:115) */
#define SWB_RESIDUAL 1u /* add residual[row] after bias (RESIDUAL) */
#define SWB_HALF_OUT 2u /* write fp16 into out instead of fp32 (HALF_OUT) */

/* kernel families in the registry */
#define SWB_FAMILY_LDG 0  /* register-streaming 128/32-bit loads, x staged in shared memory */
#define SWB_FAMILY_BULK 1 /* persistent: cp.async.bulk ring + mbarriers, one producer warp */
#define SWB_FAMILY_RBULK 2 /* persistent: whole-row ring stages, x held in registers */
#define SWB_FAMILY_SBULK 3 /* RBULK with hardware work stealing (cluster launch control) */

/* Host metadata of one launch geometry (include/config.hpp:5 struct Config). */
typedef struct swb_config {
    int id;
    int family;  /* SWB_FAMILY_* */
    int warps;   /* LDG: warps per output row. BULK: consumer warps per CTA */
    int rows;    /* LDG: rows per CTA. BULK: CTAs per SM */
    int pack;    /* halves per vector load (2 = 32-bit, 8 = 128-bit) */
    int unroll;  /* LDG: vector loads in flight per matrix per thread. RBULK: vectors of a row per thread */
    int chunk;   /* BULK: halves per matrix per stage. RBULK: target bytes per stage. 0 for LDG */
    int stages;  /* BULK, RBULK: maximum ring depth (0 for LDG) */
} swb_config_t;

SWB_API const char* swb_status_string(int status);
/* Detail of the last failing call on the calling host thread ("" if none). */
SWB_API const char* swb_last_error(void);
SWB_API int swb_version(void);
/* CUDA driver and runtime versions seen by this library (evidence metadata,
 * src/benchmark.cu:327-328); the runtime is the one linked into the library. */
SWB_API int swb_cuda_versions(int* driver, int* runtime);

/* ---- registry: replaces include/config.hpp:7-20 and torch_extension.cu:52 config_ids() ---- */
SWB_API int swb_config_count(void);
/* Writes up to cap ids in registry order; returns the total count. */
SWB_API int swb_config_ids(int* out, int cap);
/* config.hpp:13-16 valid_config(id); takes int64 so callers need not narrow first. */
SWB_API int swb_valid_config(int64_t id);
/* config.hpp:17-20 config(id); SWB_E_CONFIG for unknown ids. */
SWB_API int swb_config_info(int64_t id, swb_config_t* out);

/* ---- kernels: replace decode::launch<GATED,RESIDUAL,HALF_OUT,MODEL_ROUND>, kernels.cuh:115-133 ---- */

/* launch<true,false,false,MODEL_ROUND>: h[i] = fp16(SiLU(Wg[i].x + bg[i]) * (Wu[i].x + bu[i])).
 * Wg, Wu: [rows, cols] row-major fp16; x: [cols]; bg, bu: [rows] or NULL; h: [rows] fp16.
 * model_round != 0 rounds to fp16 after each dot, after SiLU and after the product
 * (kernels.cuh:102-106), matching eager fp16 Linear -> SiLU -> multiply. */
SWB_API int swb_gate(int config, const void* wg, const void* wu, const void* x, const void* bg, const void* bu,
             void* h, int rows, int cols, int model_round, void* stream);

/* launch<false,RESIDUAL,HALF_OUT>: out[r] = W[r].x (+ bias[r]) (+ residual[r]).
 * W: [rows, cols]; x: [cols]; bias: [rows] or NULL; residual: [rows] (required with SWB_RESIDUAL).
 * out: float[rows], or fp16[rows] with SWB_HALF_OUT. */
SWB_API int swb_project(int config, const void* w, const void* x, const void* bias, const void* residual, void* out,
                int rows, int cols, unsigned flags, void* stream);

/* Workload::custom(ffn=true), src/benchmark.cu:161-165: the whole layer with biases
 * and residual. h: [inter] fp16 workspace (overwritten); y: [hidden] fp32. */
SWB_API int swb_ffn(int gate_config, int down_config, const void* wg, const void* wu, const void* wd, const void* x,
            const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden, int inter,
            void* stream);

/* swb_ffn without a workspace argument. No counterpart in the reference.
 * Some callers cannot allocate device memory at all: code that only receives
 * raw pointers through a foreign-function boundary with no allocator bound,
 * serving runtimes that hand every byte of device memory to their own pool
 * up front, and latency-critical loops that must never hit an allocation
 * (which may synchronise the device). For them, h lives in a fixed array inside
 * this library (SWB_NOALLOC_MAX_INTER halves = 128 KiB, held by every GPU that
 * loads the library until the process exits); the caller still passes inputs
 * and y. Nothing is allocated: no cudaMalloc/cudaFree and no library routine
 * that allocates. inter > SWB_NOALLOC_MAX_INTER returns SWB_E_WORKSPACE.
 * The first call on a device looks up that device's copy of the array
 * (cudaGetSymbolAddress) and keeps its address for the life of the process --
 * make that first call before any stream capture on that device. A reset of the
 * device (cudaDeviceReset) may move the array: use a fresh process after one.
 * Every call shares the one array: h is fully rewritten by each call, so nothing
 * needs clearing, but calls that may overlap on the GPU (other streams, other
 * threads) race on it and must be serialised by the caller. */
#define SWB_NOALLOC_MAX_INTER 65536
SWB_API int swb_ffn_noalloc(int gate_config, int down_config, const void* wg, const void* wu, const void* wd,
                            const void* x, const void* bg, const void* bu, const void* bd, float* y, int hidden,
                            int inter, void* stream);

/* The whole layer in ONE persistent kernel (no counterpart in the reference), with
 * the weight stream running straight from Wg/Wu into Wd. Layer ids 200-219: gate
 * rows, a grid barrier, then down rows. Layer ids 220+ (streaming): no barrier --
 * the gate's rows are spread over the CTAs so h fills in order, each finished
 * stage's h rows are counted per block of h, and each CTA streams its rows of Wd
 * block by block as soon as a block is complete. Same arguments and outputs as
 * swb_ffn plus `workspace`: SWB_LAYER_WORKSPACE_BYTES of 16-byte aligned device
 * memory, zeroed once when allocated, then reused by every call on one stream
 * (calls sharing a workspace must not overlap; each call leaves it as it found it).
 * layer_config is a layer id (swb_layer_config_ids); a geometry that cannot hold
 * the shape falls back to 200, then 203. Needs hidden and inter multiples of 8 and
 * 16-byte aligned weights (and h, for 220+) (else SWB_E_UNSUPPORTED: use swb_ffn).
 * The launch is cooperative, every CTA resident at once; a streaming id under
 * SWB_PREFETCH_WEIGHTS (swb_ffn_fused_ex) is launched programmatically instead.
 * After a device error (swb_device_error) zero the workspace again. */
#define SWB_LAYER_WORKSPACE_BYTES 8192
SWB_API int swb_layer_config_count(void);
SWB_API int swb_layer_config_ids(int* out, int cap);
SWB_API int swb_ffn_fused(int layer_config, const void* wg, const void* wu, const void* wd, const void* x,
                          const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden, int inter,
                          void* workspace, void* stream);

/* Tensor-parallel rank of the layer (no counterpart in the reference, which is
 * single-GPU; it splits benchmark.cu:161-165 n ways). wg_shard, wu_shard: rows
 * [r*inter/n, (r+1)*inter/n) of Wg, Wu -> [shard, hidden]; wd_shard: the matching
 * columns of Wd stored contiguously -> [hidden, shard]; bg_shard, bu_shard: [shard]
 * or NULL; h_shard: [shard] fp16 workspace; y_partial: [hidden] fp32 = Wd_r h_r, no
 * bias or residual. The caller all-reduces y_partial over the ranks (sum) and then
 * applies swb_residual_epilogue(y, bd, x) once. */
SWB_API int swb_ffn_tp(int gate_config, int down_config, const void* wg_shard, const void* wu_shard,
                       const void* wd_shard, const void* x, const void* bg_shard, const void* bu_shard,
                       void* h_shard, float* y_partial, int hidden, int shard, void* stream);

/* Fused tensor parallel (no counterpart in the reference). The down projection of
 * each rank sums the ranks' partial y itself: its CTAs store their partial rows
 * straight into every peer's exchange buffer over NVLink, each value together
 * with the call's epoch in one 64-bit word (no fence, no separate flag), wait
 * (bounded: SWB_DEVERR_PEER_TIMEOUT, then no output) until every rank's words of
 * their rows carry the epoch, and add the partials in rank order plus bias and
 * residual -- no NCCL call and no separate epilogue kernel. Set-up, once per
 * rank: swb_tp_create (allocates this rank's exchange buffer), share
 * swb_tp_ipc_handle with every rank (any transport), swb_tp_connect with all
 * handles in rank order. Every rank must then make the same sequence of
 * swb_ffn_tp_fused calls with the same shapes and geometries (one exchange per
 * stream of calls; calls on one exchange must not overlap). After a device error
 * (swb_device_error) destroy and recreate the exchange on every rank. */
#define SWB_DEVERR_PEER_TIMEOUT 2
#define SWB_TP_MAX_RANKS 8
#define SWB_TP_HANDLE_BYTES 64
typedef struct swb_tp swb_tp_t;
SWB_API int swb_tp_create(int rank, int world, int rows, swb_tp_t** out);
SWB_API int swb_tp_ipc_handle(const swb_tp_t* tp, void* out);
SWB_API int swb_tp_connect(swb_tp_t* tp, const void* handles);
SWB_API int swb_tp_destroy(swb_tp_t* tp);
/* Calls this rank's exchange has counted so far (the call epoch; every call,
 * fused layer or two-kernel, advances it exactly once). Synchronises the
 * device. After a device error, ranks whose counts differ show which rank
 * fell behind. */
SWB_API int swb_tp_epoch(const swb_tp_t* tp, uint32_t* out);
/* One rank's whole layer: gate on its shard, then the fused down + all-reduce;
 * y: [hidden] fp32, identical on every rank. down_config must be an RBULK id;
 * when its rows cannot hold the shard's columns, RBULK 87, 85 or 82 runs instead.
 * With a layer id (swb_layer_config_ids) as gate_config the rank's whole layer,
 * exchange included, is one persistent kernel and down_config is ignored. */
SWB_API int swb_ffn_tp_fused(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard,
                             const void* wu_shard, const void* wd_shard, const void* x, const void* bg_shard,
                             const void* bu_shard, const void* bd, void* h_shard, float* y, int hidden, int shard,
                             void* stream);

/* swiglu_out (src/torch_extension.cu:7-40) for one tensor-parallel rank: the
 * binding's shape / config / alias guards on the rank's shard, the model-rounding
 * gate on gate_shard, up_shard ([shard, hidden]) into h_shard [shard], then the
 * fused down projection of down_shard ([hidden, shard]) + exchange; y [hidden] fp16
 * = fp16(sum over ranks of the fp32 partials, added in rank order), identical on
 * every rank, with no bias and no residual (the transformer layer adds its own).
 * Every rank makes the same calls with the same geometries; down_config is an
 * RBULK id (87, 85 or 82 run when its rows cannot hold the shard). flags:
 * SWB_PREFETCH_WEIGHTS or 0. */
SWB_API int swb_swiglu_tp_out(swb_tp_t* tp, const void* x, const void* gate_shard, const void* up_shard,
                              const void* down_shard, void* h_shard, void* y, int64_t hidden, int64_t shard,
                              int64_t gate_config, int64_t down_config, unsigned flags, void* stream);

/* swb_ffn and swb_ffn_tp_fused with launch flags (no counterpart in the reference).
 * SWB_PREFETCH_WEIGHTS: the gate kernel is launched programmatically as well, so
 * its stream of Wg/Wu may begin while the kernel before it in the stream is still
 * running -- in a chain of layers (one CUDA graph per decode step) the previous
 * layer's down kernel and exchange. The caller promises that no kernel issued
 * before the call writes this call's Wg or Wu; x, h and the exchange are still
 * touched only after the previous kernel has completed (griddepcontrol.wait).
 * For the streaming layer ids (220+) the whole-layer kernel is launched that way;
 * ignored for the barrier layer ids (200-219). Other bits: SWB_E_INPUT. */
#define SWB_PREFETCH_WEIGHTS 1u
SWB_API int swb_ffn_fused_ex(int layer_config, const void* wg, const void* wu, const void* wd, const void* x,
                             const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden,
                             int inter, void* workspace, unsigned flags, void* stream);
SWB_API int swb_ffn_ex(int gate_config, int down_config, const void* wg, const void* wu, const void* wd,
                       const void* x, const void* bg, const void* bu, const void* bd, void* h, float* y, int hidden,
                       int inter, unsigned flags, void* stream);
SWB_API int swb_ffn_tp_fused_ex(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard,
                                const void* wu_shard, const void* wd_shard, const void* x, const void* bg_shard,
                                const void* bu_shard, const void* bd, void* h_shard, float* y, int hidden, int shard,
                                unsigned flags, void* stream);

/* The layer from host x to host y: the reference's transfer-inclusive step,
 * src/benchmark.cu:177-206 (copy x in, layer, copy y out, steps back to back in
 * one stream), as one call. x_host [hidden] fp16 and y_host [hidden] fp32 must be
 * page-locked host memory this device maps (cudaHostAlloc / cudaHostRegister;
 * anything else: SWB_E_INPUT before any launch). x [hidden] fp16, h [inter] fp16
 * and y [hidden] fp32 are device buffers the call overwrites. x comes in through a
 * transfer kernel chained programmatically ahead of the gate, so the gate streams
 * Wg/Wu while x crosses the bus; the down kernel stores y to y_host in its
 * epilogue as well (BULK, RBULK and SBULK down geometries; after an LDG one a
 * transfer kernel copies it). With SWB_PREFETCH_WEIGHTS (same promise as above)
 * consecutive calls form one chain: the next call's gate streams its weights
 * while this call's y and the next x cross. y_host holds the result once the
 * stream has passed the call. No counterpart in the reference. */
SWB_API int swb_ffn_host_ex(int gate_config, int down_config, const void* wg, const void* wu, const void* wd,
                            const void* x_host, const void* bg, const void* bu, const void* bd, void* x, void* h,
                            float* y, float* y_host, int hidden, int inter, unsigned flags, void* stream);

/* swb_ffn_tp_fused_ex from host x to host y, one tensor-parallel rank: x_host in
 * (every rank passes the same x), the rank's gate and fused down + exchange, the
 * reduced y out to y_host (the same y on every rank), stored by the exchange's
 * epilogue as it writes y. Buffers and flags as swb_ffn_host_ex; gate_config may
 * be a whole-layer id. No counterpart in the reference. */
SWB_API int swb_ffn_tp_host_ex(swb_tp_t* tp, int gate_config, int down_config, const void* wg_shard,
                               const void* wu_shard, const void* wd_shard, const void* x_host, const void* bg_shard,
                               const void* bu_shard, const void* bd, void* x, void* h_shard, float* y,
                               float* y_host, int hidden, int shard, unsigned flags, void* stream);

/* swiglu_out, src/torch_extension.cu:7-40: the binding's shape / config / alias guards,
 * then the model-rounding gate into h [inter] and the fp16 down projection into
 * y [hidden] (no bias, no residual -- the residual stays in the transformer layer).
 * gate, up: [inter, hidden]; down: [hidden, inter]. Ids are checked against
 * [0, 1000] before narrowing, as the binding does. */
SWB_API int swb_swiglu_out(const void* x, const void* gate, const void* up, const void* down, void* h, void* y,
                   int64_t hidden, int64_t intermediate, int64_t gate_config, int64_t down_config,
                   void* stream);

/* ---- pointwise kernels of the cuBLAS path: kernels.cuh:134-145 ---- */
/* gate_epilogue: h[i] = fp16(SiLU(a[i] + bg[i]) * (b[i] + bu[i])) */
SWB_API int swb_gate_epilogue(const float* a, const float* b, const void* bg, const void* bu, void* h, int n,
                      void* stream);
/* residual_epilogue: y[i] += bias[i] + x[i]; also closes a tensor-parallel layer
 * after the all-reduce of the partial y. */
SWB_API int swb_residual_epilogue(float* y, const void* bias, const void* x, int n, void* stream);

/* Device error word of the current device: OR of SWB_DEVERR_* raised by kernels
 * whose bounded waits expired. Synchronises the device. clear != 0 resets it. */
#define SWB_DEVERR_TIMEOUT 1
SWB_API int swb_device_error(int clear, int* out);

#ifdef __cplusplus
}
#endif
#endif /* SWIGLU_B200_H */
