/*
 * CPU oracle for the batch-one SwiGLU decode layer.
 *
 * TEST INFRASTRUCTURE ONLY. This file and everything under oracle/ is the
 * checker: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load it. The product path (cuda-kernel_b200/) never links or calls it.
 *
 * It restates, in plain C, the host contract of shubhxho/cuda-kernel:
 *   include/contract.hpp:21      silu (two-branch, double)
 *   include/contract.hpp:23-34   matvec (row-major, double accumulation, float result)
 *   include/contract.hpp:36-53   compare (|a-e| / (atol + rtol|e|) <= 1, non-finite fails)
 *   include/contract.hpp:54-60   median
 *   include/contract.hpp:61-71   json_escape
 *   src/benchmark.cu:89-94       random_half (std::mt19937 + uniform_real_distribution<float>)
 *   src/benchmark.cu:116-121     workload generation order and scales
 *   src/benchmark.cu:131-141     FFN reference (projection, fp16 activation, residual output)
 *   include/kernels.cuh:102-106,110  model-rounding gate and half-output down (torch binding path)
 * Half-precision values travel as raw IEEE binary16 bit patterns (uint16_t).
 */
#ifndef SWIGLU_ORACLE_H
#define SWIGLU_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define ORC_OK 0
#define ORC_EINVAL -1

/* IEEE binary16 <-> binary32, round-to-nearest-even (the rounding __float2half_rn performs). */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_array(const float* in, uint16_t* out, size_t n);
void orc_f16_to_f32_array(const uint16_t* in, float* out, size_t n);

/* contract.hpp:21 */
double orc_silu(double x);

/* contract.hpp:23-34: y[r] = float(sum_c double(w[r*cols+c]) * double(x[c])) */
int orc_matvec(const float* w, const float* x, int rows, int cols, float* y);
/* Same arithmetic with fp16 weights and fp32 input (weights widened exactly). */
int orc_matvec_f16(const uint16_t* w, const float* x, int rows, int cols, float* y);

/* contract.hpp:36-53. Returns ORC_EINVAL for empty input or bad tolerances. */
int orc_compare(const float* actual, const float* expected, size_t n, double atol, double rtol,
                double* max_abs, double* max_scaled, int* passed);

/* contract.hpp:54-60. ORC_EINVAL on empty, non-finite or non-positive samples. */
int orc_median(const double* xs, size_t n, double* out);

/* contract.hpp:61-71. Writes at most cap bytes including the terminator; returns needed length. */
size_t orc_json_escape(const char* in, char* out, size_t cap);

/*
 * benchmark.cu:131-141. Inputs fp16 bits. Outputs:
 *   proj[I]  = matvec(Wg, x)               (the raw projection reference, fp32)
 *   act[I]   = fp16(float(silu(proj+bg) * (up+bu)))   (double math, then float, then fp16)
 *   y[H]     = matvec(Wd, act) + (x + bd)  (fp32)
 * Any output pointer may be NULL except y.
 */
int orc_ffn(const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, const uint16_t* x,
            const uint16_t* bg, const uint16_t* bu, const uint16_t* bd, int hidden, int inter,
            float* proj, uint16_t* act, float* y);

/*
 * Model-rounding path of the torch binding (kernels.cuh:102-106,110 via torch_extension.cu:34-38):
 *   a = fp16(dot(Wg,x)), b = fp16(dot(Wu,x)), s = fp16(silu(a)), h = fp16(s*b), y = fp16(dot(Wd,h)).
 * Dots are double-accumulated and rounded to float first; silu and the product in float.
 */
int orc_ffn_model(const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, const uint16_t* x,
                  int hidden, int inter, uint16_t* h, uint16_t* y);

/* Gate stage only (fp32 accumulate result with optional biases), for per-kernel checks. */
int orc_gate(const uint16_t* wg, const uint16_t* wu, const uint16_t* x, const uint16_t* bg,
             const uint16_t* bu, int rows, int cols, int model_round, uint16_t* h);

/* Plain projection y = W x (+bias) (+residual), fp32 out; half_out rounds to fp16 into yh. */
int orc_project(const uint16_t* w, const uint16_t* x, const uint16_t* bias, const uint16_t* residual,
                int rows, int cols, float* y, uint16_t* yh);

/* MT19937 (Matsumoto & Nishimura 1998), the engine behind std::mt19937. */
typedef struct { uint32_t mt[624]; int idx; } orc_mt19937;
void orc_mt_seed(orc_mt19937* s, uint32_t seed);
uint32_t orc_mt_next(orc_mt19937* s);

/* benchmark.cu:89-94: n fp16 values uniform in [-scale, scale) as libstdc++ draws them. */
void orc_random_half(orc_mt19937* s, size_t n, float scale, uint16_t* out);

/* benchmark.cu:116-121: the reference's seeded workload, in its draw order. */
int orc_reference_workload(uint32_t seed, int hidden, int inter, uint16_t* wg, uint16_t* wu,
                           uint16_t* wd, uint16_t* x, uint16_t* bg, uint16_t* bu, uint16_t* bd);

#ifdef __cplusplus
}
#endif
#endif
