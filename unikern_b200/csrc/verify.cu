// verify.cu -- device side of the runner's self-verification.
//
// The reference's runnable programs fill their operands with exact "sawtooth"
// values and compare the device result with a scalar CPU reference, per
// element, as rel = |got - ref| / max(|ref|, 1e-6), against the dtype's gate
// (src/codegen_hip.cpp:604-605, :1410-1416, :2167, :2338).  Here both halves
// run on the GPU: the fills are kernels, and the reference values come from
// independent, deliberately plain kernels that accumulate in fp64 (one thread
// or one warp per output, no tiling, no tensor cores), so a wrong tile, index
// or reduction order in the fast kernels cannot hide in the checker.  Each
// warp folds its lanes' worst rel and publishes it with one atomic max on the
// bit pattern of a device double (non-negative doubles order like their bits).
//
// Nothing here is on a hot path: these run once per verify instance.
#include <cuda_fp16.h>

#include "host/runner_dev.h"
#include "uk_common.cuh"

namespace {

// The reference indexes its initialisers with (int)i: sizes past 2^31 wrap to
// negative indices and C's remainder keeps the sign.  Kept identically.
__device__ __forceinline__ float saw_value(int64_t i, int kind) {
  const int idx = (int)(uint32_t)(uint64_t)i;
  switch (kind) {
    case UKR_SAW_A: return (float)((idx % 17) - 8) * 0.0625f;
    case UKR_SAW_B: return (float)((idx % 13) - 6) * 0.0625f;
    case UKR_SAW_W: return 1.0f + (float)((idx % 7) - 3) * 0.0625f;
    default: return 0.015625f;  // UKR_SAW_CONST: 2^-6
  }
}

// element i of the buffer holds the initialiser's value at index offset + i
__global__ void k_saw_f32(float* p, int64_t n, int64_t offset, int kind) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = saw_value(offset + i, kind);
}

__global__ void k_saw_f16(__half* p, int64_t n, int64_t offset, int kind) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = __float2half_rn(saw_value(offset + i, kind));
}

__device__ __forceinline__ double rel_of(double got, double ref) {
  const double den = fmax(fabs(ref), 1e-6);
  const double rel = fabs(got - ref) / den;
  return rel == rel ? rel : INFINITY;  // a NaN result fails the gate
}

// warp-wide max of `rel`, one atomic per warp (every lane must call it)
__device__ __forceinline__ void publish(double* worst, double rel) {
  for (int o = 16; o > 0; o >>= 1) rel = fmax(rel, __shfl_xor_sync(0xffffffffu, rel, o));
  if ((threadIdx.x & 31) == 0)
    atomicMax(reinterpret_cast<unsigned long long*>(worst), (unsigned long long)__double_as_longlong(rel));
}

// C[i][j] against sum_k A[i][k] * B[k][j] in fp64; one thread per output
template <typename T>
__global__ void k_check_gemm(const T* A, const T* B, const T* C, int M, int N, int K, double* worst) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  double rel = 0.0;
  if (j < N && i < M) {
    double s = 0.0;
    for (int k = 0; k < K; ++k) s += (double)(float)A[(int64_t)i * K + k] * (double)(float)B[(int64_t)k * N + j];
    rel = rel_of((double)(float)C[(int64_t)i * N + j], s);
  }
  publish(worst, rel);
}

__device__ __forceinline__ double val(const float* p, int64_t i) { return (double)p[i]; }
__device__ __forceinline__ double val(const __half* p, int64_t i) { return (double)__half2float(p[i]); }

// KML conv: X[H][W][C], Wt[Oc][Kh][Kw][C] -> Y[Oc][Ho][Wo], valid (fp32 or f16 data)
template <typename T>
__global__ void k_check_conv(const T* X, const T* Wt, const T* Y, int H, int W, int C, int Kh, int Kw, int Oc,
                             double* worst) {
  const int Ho = H - Kh + 1, Wo = W - Kw + 1;
  const int64_t n = (int64_t)Oc * Ho * Wo;
  double rel = 0.0;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int wo = (int)(t % Wo), ho = (int)((t / Wo) % Ho), oc = (int)(t / ((int64_t)Wo * Ho));
    double s = 0.0;
    for (int kh = 0; kh < Kh; ++kh)
      for (int kw = 0; kw < Kw; ++kw)
        for (int c = 0; c < C; ++c)
          s += val(X, ((int64_t)(ho + kh) * W + (wo + kw)) * C + c) * val(Wt, (((int64_t)oc * Kh + kh) * Kw + kw) * C + c);
    rel = fmax(rel, rel_of(val(Y, t), s));
  }
  publish(worst, rel);
}

// one warp per row: the row statistic in fp64, then every element checked
template <typename T>
__global__ void k_check_rows(int op, const T* X, const T* W, const T* Y, int64_t L, int64_t C, double eps,
                             double* worst) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  double rel = 0.0;  // this lane's worst over all its rows
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < L; r += warps) {
    const T* x = X + r * C;
    const T* y = Y + r * C;
    if (op == UKR_OP_REDUCE) {
      double s = 0.0;
      for (int64_t c = lane; c < C; c += 32) s += val(x, c);
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) rel = fmax(rel, rel_of(val(Y, r), s));
      continue;
    }
    double a = op == UKR_OP_SOFTMAX ? -INFINITY : 0.0;
    for (int64_t c = lane; c < C; c += 32) {
      const double v = val(x, c);
      if (op == UKR_OP_SOFTMAX) a = fmax(a, v);
      else if (op == UKR_OP_RMSNORM) a += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) {
      const double b = __shfl_xor_sync(0xffffffffu, a, o);
      a = op == UKR_OP_SOFTMAX ? fmax(a, b) : a + b;
    }
    double sum = 0.0;
    if (op == UKR_OP_SOFTMAX) {
      for (int64_t c = lane; c < C; c += 32) sum += exp(val(x, c) - a);
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    const double rms = op == UKR_OP_RMSNORM ? 1.0 / sqrt(a / (double)C + eps) : 0.0;
    for (int64_t c = lane; c < C; c += 32) {
      double ref;
      if (op == UKR_OP_SOFTMAX) ref = exp(val(x, c) - a) / sum;
      else if (op == UKR_OP_RMSNORM) ref = val(x, c) * rms * val(W, c);
      else ref = val(x, c) * val(W, c);  // channelscale
      rel = fmax(rel, rel_of(val(y, c), ref));
    }
  }
  publish(worst, rel);
}

int grid_for(int64_t n, int threads) {
  const int64_t cap = (int64_t)uk::sm_count() * 16;
  int64_t g = (n + threads - 1) / threads;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

extern "C" {

int ukr_saw_fill_at(void* p, int64_t n, int64_t offset, int kind, int f16, void* stream) {
  if (n <= 0) return UK_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (f16) k_saw_f16<<<grid_for(n, 256), 256, 0, s>>>(static_cast<__half*>(p), n, offset, kind);
  else k_saw_f32<<<grid_for(n, 256), 256, 0, s>>>(static_cast<float*>(p), n, offset, kind);
  return uk::check_launch("saw fill");
}

int ukr_saw_fill(void* p, int64_t n, int kind, int f16, void* stream) {
  return ukr_saw_fill_at(p, n, 0, kind, f16, stream);
}

int ukr_check_gemm(const void* A, const void* B, const void* C, int M, int N, int K, int f16, double* worst,
                   void* stream) {
  if (M <= 0 || N <= 0) return UK_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((N + 127) / 128, M);
  if (f16)
    k_check_gemm<__half><<<grid, 128, 0, s>>>(static_cast<const __half*>(A), static_cast<const __half*>(B),
                                              static_cast<const __half*>(C), M, N, K, worst);
  else
    k_check_gemm<float><<<grid, 128, 0, s>>>(static_cast<const float*>(A), static_cast<const float*>(B),
                                             static_cast<const float*>(C), M, N, K, worst);
  return uk::check_launch("check gemm");
}

int ukr_check_conv(const void* X, const void* Wt, const void* Y, int H, int W, int C, int Kh, int Kw, int Oc,
                   int f16, double* worst, void* stream) {
  const int64_t n = (int64_t)Oc * (H - Kh + 1) * (W - Kw + 1);
  if (n <= 0) return UK_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (f16)
    k_check_conv<__half><<<grid_for(n, 128), 128, 0, s>>>((const __half*)X, (const __half*)Wt, (const __half*)Y, H,
                                                          W, C, Kh, Kw, Oc, worst);
  else
    k_check_conv<float><<<grid_for(n, 128), 128, 0, s>>>((const float*)X, (const float*)Wt, (const float*)Y, H, W,
                                                         C, Kh, Kw, Oc, worst);
  return uk::check_launch("check conv");
}

int ukr_check_rows(int op, const void* X, const void* W, const void* Y, int64_t L, int64_t C, double eps, int f16,
                   double* worst, void* stream) {
  if (L <= 0) return UK_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (f16)
    k_check_rows<__half><<<grid_for(L * 32, 256), 256, 0, s>>>(op, (const __half*)X, (const __half*)W,
                                                               (const __half*)Y, L, C, eps, worst);
  else
    k_check_rows<float><<<grid_for(L * 32, 256), 256, 0, s>>>(op, (const float*)X, (const float*)W,
                                                              (const float*)Y, L, C, eps, worst);
  return uk::check_launch("check rows");
}

}  // extern "C"
