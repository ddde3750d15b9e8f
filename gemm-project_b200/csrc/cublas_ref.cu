// cuBLAS comparator with the launcher's semantics (benchmark baseline only,
// never on the gemm_launcher path). Counterpart of the reference comparator
// src/lib/gemm_cublas.cuh:1-63: cublasGemmEx with FP16 A/B/C and
// CUBLAS_COMPUTE_32F, row-major C = A*B computed as column-major C^T = B^T A^T,
// reduced-precision reductions disallowed, K == 0 handled as C = beta*C.
// Differences: 8 arguments (the reference's 9th, column_major, is never passed
// by its ctypes caller), one handle per (host thread, device), explicit stream
// variant, and errors recorded instead of abort().
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "gemm_b200.h"

namespace {

constexpr int kMaxDevices = 64;

// C = half_rn(beta * C) for K == 0, C not read when beta == 0 (the reference's
// gemm_cublas_scale_c, src/lib/gemm_cublas.cuh:27-33).
__global__ void cublas_scale_c_kernel(half* C, size_t count, float beta) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < count) {
    const float prev = beta != 0.0f ? __half2float(C[i]) : 0.0f;
    C[i] = __float2half_rn(beta * prev);
  }
}

struct Handles {
  cublasHandle_t h[kMaxDevices] = {};
  ~Handles() {
    for (auto& x : h)
      if (x) cublasDestroy(x);
  }
};

cublasHandle_t handle_for_current_device() {
  static thread_local Handles handles;
  int dev = 0;
  cudaGetDevice(&dev);
  cublasHandle_t& h = handles.h[dev % kMaxDevices];
  if (!h) {
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) {
      std::fprintf(stderr, "gemm_cublas: cublasCreate failed\n");
      h = nullptr;
      return nullptr;
    }
    cublasSetMathMode(h, CUBLAS_MATH_DISALLOW_REDUCED_PRECISION_REDUCTION);
  }
  return h;
}

}  // namespace

extern "C" GEMM_API void gemm_cublas_stream(const half* A, const half* B, half* C, int M, int N, int K,
                                   float alpha, float beta, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return;
  if (K <= 0) {
    const size_t count = static_cast<size_t>(M) * N;
    cublas_scale_c_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(C, count, beta);
    return;
  }
  cublasHandle_t h = handle_for_current_device();
  if (!h) return;
  cublasSetStream(h, stream);
  const cublasStatus_t st =
      cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &alpha, B, CUDA_R_16F, N, A, CUDA_R_16F,
                   K, &beta, C, CUDA_R_16F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (st != CUBLAS_STATUS_SUCCESS) std::fprintf(stderr, "gemm_cublas: cublasGemmEx error %d\n", int(st));
}

extern "C" GEMM_API void gemm_cublas(const half* A, const half* B, half* C, int M, int N, int K,
                            float alpha, float beta) {
  gemm_cublas_stream(A, B, C, M, N, K, alpha, beta, 0);
}
