/*
 * swiglu_b200_cublas -- the cuBLAS GemmEx + pointwise baseline of the SwiGLU
 * decode layer, measured beside the product kernels on the same B200.
 *
 * Replaces Workload::gemv / Workload::baseline of shubhxho/cuda-kernel
 * (src/benchmark.cu:143-160): three cublasGemmEx calls (fp16 in, fp32 out,
 * CUBLAS_COMPUTE_32F, algorithm DEFAULT or DEFAULT_TENSOR_OP) and the two
 * pointwise epilogues (include/kernels.cuh:134-145).
 * Library: cuda-kernel_b200/lib/libswiglu_b200_cublas.so. Status codes are the
 * SWB_* codes of swiglu_b200.h; SWBL_E_CUBLAS carries a cuBLAS failure.
 */
#ifndef SWIGLU_B200_CUBLAS_H
#define SWIGLU_B200_CUBLAS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef SWB_API
#define SWB_API __attribute__((visibility("default")))
#endif

#define SWBL_E_CUBLAS 100

/* Context (src/benchmark.cu:36-45): one cuBLAS handle bound to the current device. */
SWB_API int swbl_create(void** handle);
SWB_API int swbl_destroy(void* handle);
SWB_API const char* swbl_last_error(void);
/* cublasGetVersion of the handle (src/benchmark.cu:328). */
SWB_API int swbl_version(void* handle, int* out);

/* Workload::gemv (src/benchmark.cu:143-150): y[rows] (fp32) = W[rows, cols] x.
 * algo 0 = CUBLAS_GEMM_DEFAULT, 1 = CUBLAS_GEMM_DEFAULT_TENSOR_OP. */
SWB_API int swbl_gemv(void* handle, int algo, const void* w, const void* x, float* y, int rows, int cols, void* stream);

/* Workload::baseline(ffn=true) (src/benchmark.cu:151-160):
 *   g = Wg x; u = Wu x; h = gate_epilogue(g, u, bg, bu); y = Wd h; y += bd + x.
 * g, u: fp32 [inter] workspaces; h: fp16 [inter]; y: fp32 [hidden]. */
SWB_API int swbl_ffn(void* handle, int algo, const void* wg, const void* wu, const void* wd, const void* x, const void* bg,
             const void* bu, const void* bd, float* g, float* u, void* h, float* y, int hidden, int inter,
             void* stream);

#ifdef __cplusplus
}
#endif
#endif
