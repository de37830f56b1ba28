// cuBLAS GemmEx + pointwise baseline (declarations: include/swiglu_b200_cublas.h).
// A measured comparison point only; the product path never calls it.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <string>

#include "kernels.cuh"
#include "swiglu_b200.h"
#include "swiglu_b200_cublas.h"

namespace {

thread_local std::string g_error;

int fail(int status, const std::string& detail) {
    g_error = detail;
    return status;
}

int cuda_status(cudaError_t e) {
    return e == cudaSuccess ? SWB_OK : fail(SWB_E_CUDA, cudaGetErrorString(e));
}

int blas_status(cublasStatus_t s) {
    return s == CUBLAS_STATUS_SUCCESS ? SWB_OK : fail(SWBL_E_CUBLAS, "cuBLAS status " + std::to_string(int(s)));
}

}  // namespace

extern "C" {

const char* swbl_last_error(void) { return g_error.c_str(); }

int swbl_create(void** handle) {
    if (!handle) return fail(SWB_E_INPUT, "null handle slot");
    cublasHandle_t h = nullptr;
    if (int rc = blas_status(cublasCreate(&h))) return rc;
    if (int rc = blas_status(cublasSetMathMode(h, CUBLAS_DEFAULT_MATH))) {
        cublasDestroy(h);
        return rc;
    }
    *handle = h;
    return SWB_OK;
}

int swbl_version(void* handle, int* out) {
    if (!handle || !out) return fail(SWB_E_INPUT, "null handle or output");
    return blas_status(cublasGetVersion(static_cast<cublasHandle_t>(handle), out));
}

int swbl_destroy(void* handle) {
    if (!handle) return SWB_OK;
    return blas_status(cublasDestroy(static_cast<cublasHandle_t>(handle)));
}

int swbl_gemv(void* handle, int algo, const void* w, const void* x, float* y, int rows, int cols, void* stream) {
    if (!handle || !w || !x || !y || rows <= 0 || cols <= 0) return fail(SWB_E_INPUT, "invalid gemv input");
    cublasHandle_t h = static_cast<cublasHandle_t>(handle);
    if (int rc = blas_status(cublasSetStream(h, static_cast<cudaStream_t>(stream)))) return rc;
    const float alpha = 1.f, beta = 0.f;
    // Row-major W[rows, cols] is column-major [cols, rows]: y = op_T(W) x.
    return blas_status(cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, rows, 1, cols, &alpha, w, CUDA_R_16F, cols, x,
                                    CUDA_R_16F, cols, &beta, y, CUDA_R_32F, rows, CUBLAS_COMPUTE_32F,
                                    algo == 0 ? CUBLAS_GEMM_DEFAULT : CUBLAS_GEMM_DEFAULT_TENSOR_OP));
}

int swbl_ffn(void* handle, int algo, const void* wg, const void* wu, const void* wd, const void* x, const void* bg,
             const void* bu, const void* bd, float* g, float* u, void* h, float* y, int hidden, int inter,
             void* stream) {
    if (!bg || !bu || !bd || !g || !u || !h) return fail(SWB_E_INPUT, "invalid baseline buffers");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = swbl_gemv(handle, algo, wg, x, g, inter, hidden, stream)) return rc;
    if (int rc = swbl_gemv(handle, algo, wu, x, u, inter, hidden, stream)) return rc;
    swb::gate_epilogue_kernel<<<(inter + 255) / 256, 256, 0, s>>>(g, u, static_cast<const __half*>(bg),
                                                                  static_cast<const __half*>(bu),
                                                                  static_cast<__half*>(h), inter);
    if (int rc = cuda_status(cudaGetLastError())) return rc;
    if (int rc = swbl_gemv(handle, algo, wd, h, y, hidden, inter, stream)) return rc;
    swb::residual_epilogue_kernel<<<(hidden + 255) / 256, 256, 0, s>>>(y, static_cast<const __half*>(bd),
                                                                       static_cast<const __half*>(x), hidden);
    return cuda_status(cudaGetLastError());
}

}  // extern "C"
