// gemm_f16.cu -- C(f16) = A(f16) * B(f16), fp32 accumulation.
// Replaces uk_gemm_h (src/codegen_hip.cpp:1777-1808).
#include <cuda_fp16.h>

#include "uk_common.cuh"

namespace uk {
int gemm_f16_simt(const __half* A, int64_t lda, const __half* B, int64_t ldb, __half* C, int64_t ldc, int M, int N,
                  int K, cudaStream_t st);
}

extern "C" int uk_cuda_gemm_f16_ld(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, uint16_t* C,
                                   int64_t ldc, int M, int N, int K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_f16: negative dims %d %d %d", M, N, K);
  if (lda < K || ldb < N || ldc < N)
    return uk::fail(UK_EINVAL, "gemm_f16: leading dimensions lda=%lld ldb=%lld ldc=%lld below K/N", (long long)lda,
                    (long long)ldb, (long long)ldc);
  if (M == 0 || N == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(C, "C")) return rc;
  if (K > 0) {
    if (int rc = uk::check_device_ptr(A, "A")) return rc;
    if (int rc = uk::check_device_ptr(B, "B")) return rc;
  }
  if ((M + 31) / 32 > 65535) return uk::fail(UK_EINVAL, "gemm_f16: M=%d exceeds the grid limit", M);
  cudaStream_t st = (cudaStream_t)stream;
  return uk::gemm_f16_simt((const __half*)A, lda, (const __half*)B, ldb, (__half*)C, ldc, M, N, K, st);
}

extern "C" int uk_cuda_gemm_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                                void* stream) {
  return uk_cuda_gemm_f16_ld(A, K, B, N, C, N, M, N, K, stream);
}
