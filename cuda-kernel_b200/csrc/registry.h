// One list of launch geometries generates both the host metadata
// (swb_config_ids / swb_config_info) and the CUDA dispatch switch, the way
// DECODE_CONFIGS does in include/config.hpp:7-11 of shubhxho/cuda-kernel.
//
// X(id, family, warps, rows, pack, unroll, chunk, stages)
//
// LDG family (register streaming; x staged in shared memory as fp32):
//   warps  = warps per output row, rows = output rows per CTA,
//   pack   = halves per vector load (2 -> 32-bit, 8 -> 128-bit),
//   unroll = independent vector loads per matrix kept in flight per thread.
//   Ids 1..21 keep the reference's (id, warps, rows, pack) geometries so tuned
//   ids from the reference stay valid; ids 32+ are deep-unrolled B200 variants.
// BULK family (persistent, one CTA set per SM):
//   warps  = consumer warps (plus one producer warp), rows = CTAs per SM,
//   chunk  = halves per matrix per ring stage, stages = maximum ring depth
//   (the launcher trims it to the shared memory the shape leaves free).
//   A BULK id whose preconditions fail for a shape (cols % 8, 16-byte rows,
//   shared-memory fit) runs the LDG geometry of id 33 instead.
// RBULK family (persistent, whole rows per ring stage, x held in registers):
//   warps  = consumer warps (plus one producer warp), rows = CTAs per SM,
//   unroll = MAXJ, the 16-byte vectors of a row each consumer thread owns
//            (so cols <= 8 * 32 * warps * unroll),
//   chunk  = target bytes per ring stage (whole rows, at least one),
//   stages = maximum ring depth (trimmed to the shared memory available and
//            to the CTA's stages of work).
//   An RBULK id whose preconditions fail runs the BULK geometry of id 64.
// SBULK family (RBULK with hardware work stealing): same fields as RBULK; the
//   grid has one CTA per small block of rows and running CTAs take over blocks
//   whose CTAs have not started (cluster launch control), so SMs that stream
//   faster do more of the matrix. Falls back to id 64 like RBULK.
#pragma once

// A measurement build may append geometries to the list (ids 150-199) by
// defining SWB_EXTRA_CONFIGS(X) before this header; the library appends none.
#ifndef SWB_EXTRA_CONFIGS
#define SWB_EXTRA_CONFIGS(X)
#endif

#define SWB_FAM_LDG 0
#define SWB_FAM_BULK 1
#define SWB_FAM_RBULK 2
#define SWB_FAM_SBULK 3

#define SWB_CONFIGS(X)                                                                          \
    X(1, SWB_FAM_LDG, 1, 4, 2, 1, 0, 0)                                                         \
    X(2, SWB_FAM_LDG, 2, 4, 2, 1, 0, 0)                                                         \
    X(4, SWB_FAM_LDG, 4, 4, 2, 1, 0, 0)                                                         \
    X(8, SWB_FAM_LDG, 8, 4, 2, 1, 0, 0)                                                         \
    X(16, SWB_FAM_LDG, 1, 4, 8, 1, 0, 0)                                                        \
    X(17, SWB_FAM_LDG, 2, 4, 8, 1, 0, 0)                                                        \
    X(18, SWB_FAM_LDG, 4, 2, 8, 1, 0, 0)                                                        \
    X(19, SWB_FAM_LDG, 1, 8, 8, 1, 0, 0)                                                        \
    X(20, SWB_FAM_LDG, 2, 2, 8, 1, 0, 0)                                                        \
    X(21, SWB_FAM_LDG, 4, 1, 8, 1, 0, 0)                                                        \
    X(32, SWB_FAM_LDG, 1, 8, 8, 4, 0, 0)                                                        \
    X(33, SWB_FAM_LDG, 2, 4, 8, 4, 0, 0)                                                        \
    X(34, SWB_FAM_LDG, 4, 2, 8, 4, 0, 0)                                                        \
    X(35, SWB_FAM_LDG, 8, 1, 8, 4, 0, 0)                                                        \
    X(36, SWB_FAM_LDG, 1, 4, 8, 8, 0, 0)                                                        \
    X(37, SWB_FAM_LDG, 2, 2, 8, 8, 0, 0)                                                        \
    X(38, SWB_FAM_LDG, 4, 1, 8, 8, 0, 0)                                                        \
    X(64, SWB_FAM_BULK, 8, 1, 8, 1, 4096, 8)                                                    \
    X(65, SWB_FAM_BULK, 8, 1, 8, 1, 2048, 16)                                                   \
    X(66, SWB_FAM_BULK, 4, 1, 8, 1, 4096, 8)                                                    \
    X(67, SWB_FAM_BULK, 16, 1, 8, 1, 8192, 4)                                                   \
    X(68, SWB_FAM_BULK, 8, 2, 8, 1, 2048, 8)                                                    \
    X(69, SWB_FAM_BULK, 4, 2, 8, 1, 4096, 4)                                                    \
    X(78, SWB_FAM_RBULK, 2, 4, 8, 8, 16384, 3)                                                  \
    X(79, SWB_FAM_RBULK, 4, 3, 8, 4, 16384, 4)                                                  \
    X(80, SWB_FAM_RBULK, 4, 2, 8, 4, 16384, 8)                                                  \
    X(81, SWB_FAM_RBULK, 8, 1, 8, 4, 32768, 8)                                                  \
    X(82, SWB_FAM_RBULK, 16, 1, 8, 4, 32768, 8)                                                 \
    X(83, SWB_FAM_RBULK, 8, 2, 8, 4, 16384, 8)                                                  \
    X(85, SWB_FAM_RBULK, 8, 1, 8, 8, 32768, 8)                                                  \
    X(86, SWB_FAM_RBULK, 4, 2, 8, 8, 16384, 8)                                                  \
    X(87, SWB_FAM_RBULK, 8, 2, 8, 8, 16384, 6)                                                  \
    X(88, SWB_FAM_RBULK, 4, 1, 8, 4, 16384, 16)                                                 \
    X(89, SWB_FAM_RBULK, 4, 1, 8, 8, 32768, 12)                                                 \
    X(90, SWB_FAM_SBULK, 4, 2, 8, 4, 16384, 8)                                                  \
    X(91, SWB_FAM_SBULK, 8, 1, 8, 4, 32768, 8)                                                  \
    X(92, SWB_FAM_SBULK, 8, 2, 8, 8, 16384, 6)                                                  \
    X(93, SWB_FAM_SBULK, 16, 1, 8, 4, 32768, 8)                                                 \
    X(94, SWB_FAM_SBULK, 8, 2, 8, 4, 16384, 8)                                                  \
    X(95, SWB_FAM_SBULK, 4, 2, 8, 8, 16384, 8)                                                  \
    X(96, SWB_FAM_SBULK, 4, 3, 8, 4, 16384, 5)                                                  \
    X(97, SWB_FAM_SBULK, 6, 2, 8, 4, 16384, 8)                                                  \
    X(98, SWB_FAM_SBULK, 2, 4, 8, 8, 16384, 3)                                                  \
    X(99, SWB_FAM_SBULK, 8, 3, 8, 4, 16384, 4)                                                  \
    /* Shallow rings. With every SM streaming at once the memory fabric, not the SM,  */        \
    /* sets each SM's share, and some SMs get up to 1.4x less than others: a deep ring */        \
    /* (over ~128 KB in flight per SM) then leaves those SMs microseconds behind at   */        \
    /* the end of a launch. About 115-128 KB in flight per SM keeps HBM busy and the  */        \
    /* SMs even. 100/101: long rows; 102: short rows; 103: a small gate that leaves   */        \
    /* room for the down kernel's CTAs beside it.                                     */        \
    X(100, SWB_FAM_RBULK, 8, 2, 8, 8, 16384, 2)                                                 \
    X(101, SWB_FAM_RBULK, 16, 1, 8, 4, 32768, 4)                                                \
    X(102, SWB_FAM_RBULK, 4, 2, 8, 8, 16384, 2)                                                 \
    X(103, SWB_FAM_BULK, 8, 2, 8, 1, 2048, 4)                                                   \
    SWB_EXTRA_CONFIGS(X)

// Ids used when a BULK / RBULK geometry cannot run a shape.
#define SWB_BULK_FALLBACK_ID 33
#define SWB_RBULK_FALLBACK_ID 64

// Fused whole-layer kernels (layer.cuh), used by swb_ffn_fused and, with a layer
// id as the gate config, swb_ffn_tp_fused. Separate ids (200+): they run a whole
// layer, not one projection. X(id, consumer warps, CTAs per SM, target bytes per
// ring stage, maximum ring depth). The first two are the fallbacks, in order,
// when a requested geometry cannot hold a row of the shape.
#define SWB_LAYER_CONFIGS(X)    \
    X(200, 8, 1, 32768, 8)      \
    X(203, 16, 1, 32768, 8)     \
    X(201, 4, 2, 32768, 4)      \
    X(202, 8, 2, 16384, 8)      \
    X(204, 4, 2, 16384, 8)      \
    X(205, 8, 1, 16384, 12)     \
    X(206, 8, 1, 65536, 3)      \
    X(207, 16, 1, 65536, 3)     \
    X(208, 8, 1, 49152, 4)      \
    X(209, 8, 2, 49152, 2)      \
    X(210, 16, 1, 49152, 4)

// Streaming whole-layer kernels (layer.cuh stream_layer_kernel), layer ids 220+: no grid
// barrier; the down phase streams Wd block by block as the gate fills h. X(id, consumer
// warps, CTAs per SM, RSPLIT (row slots: a block is 8 * 32 * warps / RSPLIT h elements),
// MAXR (rows per thread, so rows per CTA <= RSPLIT * MAXR), target bytes per gate stage,
// maximum ring depth).
#define SWB_STREAM_LAYER_CONFIGS(X)     \
    X(220, 8, 2, 2, 8, 32768, 4)         \
    X(221, 8, 1, 2, 16, 32768, 6)        \
    X(223, 4, 2, 1, 16, 32768, 4)
