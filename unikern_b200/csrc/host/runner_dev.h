// runner_dev.h -- device helpers of the KML runner (csrc/verify.cu): the
// reference's sawtooth initialisers as fill kernels and fp64 checker kernels
// that accumulate the worst per-element relative error into one device double.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// initialiser kinds (src/codegen_hip.cpp:604-605, :2167, :2338 of UNIKERN)
#define UKR_SAW_A 0     // ((i % 17) - 8) * 2^-4   (initA, initX)
#define UKR_SAW_B 1     // ((i % 13) - 6) * 2^-4   (initB)
#define UKR_SAW_W 2     // 1 + ((i % 7) - 3) * 2^-4 (initW, initS)
#define UKR_SAW_CONST 3 // 2^-6 everywhere (the reduce verify instance)

#define UKR_OP_REDUCE 0
#define UKR_OP_SOFTMAX 1
#define UKR_OP_RMSNORM 2
#define UKR_OP_CHANNELSCALE 3

int ukr_saw_fill(void* p, int64_t n, int kind, int f16, void* stream);
// the initialiser's values for indices [offset, offset + n)
int ukr_saw_fill_at(void* p, int64_t n, int64_t offset, int kind, int f16, void* stream);
// the device work of uk_cuda_gemm_streamed without its copies (B's pre-pass
// and every block's GEMM, on the ring's first slot): kernel-only timing
int ukr_gemm_streamed_kernels(void* dB, void* ring, size_t ring_bytes, int M, int N, int K, int kind,
                              int block_rows, void* stream);
int ukr_check_gemm(const void* A, const void* B, const void* C, int M, int N, int K, int f16, double* worst,
                   void* stream);
// f16 != 0: the operands and the result are IEEE binary16, else fp32
int ukr_check_conv(const void* X, const void* Wt, const void* Y, int H, int W, int C, int Kh, int Kw, int Oc,
                   int f16, double* worst, void* stream);
// row ops: REDUCE compares Y[r] with the row sum; the others compare Y[r][c]
int ukr_check_rows(int op, const void* X, const void* W, const void* Y, int64_t L, int64_t C, double eps, int f16,
                   double* worst, void* stream);

#ifdef __cplusplus
}
#endif
