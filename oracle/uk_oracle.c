/*
 * uk_oracle.c -- CPU restatement of the reference KML operator set.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path (see uk_oracle.h
 * for the list of reference functions each routine follows).  Build with
 * -O2 -ffp-contract=off (no -ffast-math) so fp32 results keep the
 * reference's rounding sequence.
 */
#include "uk_oracle.h"

#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#define UK_NT(t) ((t) < 1 ? 1 : (t))
#endif

/* ---- sawtooth initialisers: src/codegen_hip.cpp:604-605, :2167, :2338 ---- */
float or_initA(int idx) { return ((idx % 17) - 8) * 0.0625f; }
float or_initB(int idx) { return ((idx % 13) - 6) * 0.0625f; }
float or_initW(int idx) { return 1.0f + ((idx % 7) - 3) * 0.0625f; }

void or_fill_initA(float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = or_initA((int)i);
}
void or_fill_initB(float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = or_initB((int)i);
}
void or_fill_initW(float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = or_initW((int)i);
}

/* ---- binary16: the compiler's _Float16 conversions are IEEE RNE ---- */
uint16_t or_f32_to_f16(float x) {
  _Float16 h = (_Float16)x;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}
float or_f16_to_f32(uint16_t u) {
  _Float16 h;
  memcpy(&h, &u, 2);
  return (float)h;
}
void or_f32_to_f16_n(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = or_f32_to_f16(src[i]);
}
void or_f16_to_f32_n(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = or_f16_to_f32(src[i]);
}

/* ---- gemm: src/codegen_hip.cpp:1124-1132 (i -> j -> k, s += A*B) ---- */
void or_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K,
                 int row0, int row1, int threads) {
  (void)M;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(UK_NT(threads))
#endif
  for (int i = row0; i < row1; ++i)
    for (int j = 0; j < N; ++j) {
      float s = 0.f;
      for (int k = 0; k < K; ++k) s += A[(size_t)i * K + k] * B[(size_t)k * N + j];
      C[(size_t)i * N + j] = s;
    }
  (void)threads;
}

void or_gemm_f64(const float* A, const float* B, double* C, int M, int N, int K,
                 int row0, int row1, int threads) {
  (void)M;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(UK_NT(threads))
#endif
  for (int i = row0; i < row1; ++i)
    for (int j = 0; j < N; ++j) {
      double s = 0.0;
      for (int k = 0; k < K; ++k)
        s += (double)A[(size_t)i * K + k] * (double)B[(size_t)k * N + j];
      C[(size_t)i * N + j] = s;
    }
  (void)threads;
}

/* src/codegen_hip.cpp:1851-1862: the reference quantises to half on the host,
 * widens back with __half2float and hands the widened values to cpu_ref.
 * Each C element is one fp32 accumulator fed the products A[i][k]*B[k][j] in
 * ascending k, exactly cpu_ref's sequence; the loops run i -> k -> j over a
 * row of accumulators (so B streams by rows, widened to fp32 once), which
 * leaves every element's operation sequence, and so its bits, unchanged. */
#define UK_GEMM_F16_ROWS(ACC_T)                                                      \
  float* Bf = (float*)malloc((size_t)K * N * sizeof(float));                         \
  if (!Bf) return;                                                                    \
  for (size_t t = 0; t < (size_t)K * N; ++t) Bf[t] = or_f16_to_f32(B[t]);            \
  UK_OMP_FOR(threads)                                                                 \
  for (int i = row0; i < row1; ++i) {                                                 \
    ACC_T* acc = C + (size_t)i * N;                                                   \
    for (int j = 0; j < N; ++j) acc[j] = 0;                                           \
    for (int k = 0; k < K; ++k) {                                                     \
      const ACC_T a = (ACC_T)or_f16_to_f32(A[(size_t)i * K + k]);                     \
      const float* b = Bf + (size_t)k * N;                                            \
      for (int j = 0; j < N; ++j) acc[j] += a * (ACC_T)b[j];                          \
    }                                                                                 \
  }                                                                                   \
  free(Bf);

#ifdef _OPENMP
#define UK_PRAGMA(x) _Pragma(#x)
#define UK_OMP_FOR(t) UK_PRAGMA(omp parallel for schedule(dynamic, 1) num_threads(UK_NT(t)))
#else
#define UK_OMP_FOR(t)
#endif

void or_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int M, int N,
                 int K, int row0, int row1, int threads) {
  (void)M;
  UK_GEMM_F16_ROWS(float)
  (void)threads;
}

void or_gemm_f16_f64(const uint16_t* A, const uint16_t* B, double* C, int M,
                     int N, int K, int row0, int row1, int threads) {
  (void)M;
  UK_GEMM_F16_ROWS(double)
  (void)threads;
}

double or_gemm_f16_dot_f64(const uint16_t* A, const uint16_t* B, int N, int K,
                           int i, int j) {
  double s = 0.0;
  for (int k = 0; k < K; ++k)
    s += (double)or_f16_to_f32(A[(size_t)i * K + k]) *
         (double)or_f16_to_f32(B[(size_t)k * N + j]);
  return s;
}

/* ---- conv: src/reference.cpp:6-22 ---- */
void or_conv_f32(const float* x, const float* wt, float* y, int H, int W, int C,
                 int Kh, int Kw, int Oc, int threads) {
  const int Ho = H - Kh + 1, Wo = W - Kw + 1;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(UK_NT(threads))
#endif
  for (int oc = 0; oc < Oc; ++oc)
    for (int ho = 0; ho < Ho; ++ho)
      for (int wo = 0; wo < Wo; ++wo) {
        float acc = 0.f;
        for (int c = 0; c < C; ++c)
          for (int kh = 0; kh < Kh; ++kh)
            for (int kw = 0; kw < Kw; ++kw) {
              const float xv = x[((size_t)(ho + kh) * W + (wo + kw)) * C + c];
              const float wv = wt[((size_t)(oc * Kh + kh) * Kw + kw) * C + c];
              acc += xv * wv;
            }
        y[((size_t)oc * Ho + ho) * Wo + wo] = acc;
      }
  (void)threads;
}

void or_conv_f64(const float* x, const float* wt, double* y, int H, int W,
                 int C, int Kh, int Kw, int Oc, int threads) {
  const int Ho = H - Kh + 1, Wo = W - Kw + 1;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(UK_NT(threads))
#endif
  for (int oc = 0; oc < Oc; ++oc)
    for (int ho = 0; ho < Ho; ++ho)
      for (int wo = 0; wo < Wo; ++wo) {
        double acc = 0.0;
        for (int c = 0; c < C; ++c)
          for (int kh = 0; kh < Kh; ++kh)
            for (int kw = 0; kw < Kw; ++kw) {
              const double xv = x[((size_t)(ho + kh) * W + (wo + kw)) * C + c];
              const double wv = wt[((size_t)(oc * Kh + kh) * Kw + kw) * C + c];
              acc += xv * wv;
            }
        y[((size_t)oc * Ho + ho) * Wo + wo] = acc;
      }
  (void)threads;
}

/* NCHW + zero padding: the same c -> kh -> kw accumulation, with the padded
 * border read as 0 (what the host-padded HWC form of the reference sees). */
#define UK_CONV_NCHW_BODY(ACC_T)                                                  \
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;                 \
  for (int n = n0; n < n1; ++n)                                                   \
    for (int oc = 0; oc < Oc; ++oc) {                                             \
      const ACC_T sc = s ? (ACC_T)s[oc] : (ACC_T)1;                               \
      for (int ho = 0; ho < Ho; ++ho)                                             \
        for (int wo = 0; wo < Wo; ++wo) {                                         \
          ACC_T acc = 0;                                                          \
          for (int c = 0; c < C; ++c)                                             \
            for (int kh = 0; kh < Kh; ++kh) {                                     \
              const int hi = ho + kh - pad;                                       \
              if (hi < 0 || hi >= H) continue;                                    \
              for (int kw = 0; kw < Kw; ++kw) {                                   \
                const int wi = wo + kw - pad;                                     \
                if (wi < 0 || wi >= W) continue;                                  \
                const ACC_T xv = x[(((size_t)n * C + c) * H + hi) * W + wi];      \
                const ACC_T wv = w[(((size_t)oc * C + c) * Kh + kh) * Kw + kw];   \
                acc += xv * wv;                                                   \
              }                                                                   \
            }                                                                     \
          y[(((size_t)n * Oc + oc) * Ho + ho) * Wo + wo] = acc * sc;              \
        }                                                                         \
    }

void or_conv_nchw_f64(const float* x, const float* w, const float* s, double* y,
                      int N, int C, int H, int W, int Oc, int Kh, int Kw,
                      int pad, int n0, int n1, int threads) {
  (void)N;
#ifdef _OPENMP
#pragma omp parallel num_threads(UK_NT(threads))
  {
    /* split each image's output channels across threads */
    const int nt = omp_get_num_threads(), t = omp_get_thread_num();
    const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
    for (int n = n0; n < n1; ++n)
      for (int oc = t; oc < Oc; oc += nt) {
        const double sc = s ? (double)s[oc] : 1.0;
        for (int ho = 0; ho < Ho; ++ho)
          for (int wo = 0; wo < Wo; ++wo) {
            double acc = 0;
            for (int c = 0; c < C; ++c)
              for (int kh = 0; kh < Kh; ++kh) {
                const int hi = ho + kh - pad;
                if (hi < 0 || hi >= H) continue;
                for (int kw = 0; kw < Kw; ++kw) {
                  const int wi = wo + kw - pad;
                  if (wi < 0 || wi >= W) continue;
                  acc += (double)x[(((size_t)n * C + c) * H + hi) * W + wi] *
                         (double)w[(((size_t)oc * C + c) * Kh + kh) * Kw + kw];
                }
              }
            y[(((size_t)n * Oc + oc) * Ho + ho) * Wo + wo] = acc * sc;
          }
      }
  }
#else
  (void)threads;
  UK_CONV_NCHW_BODY(double)
#endif
}

void or_conv_nchw_points_f64(const float* x, const float* w, const float* s, const int* pts, int npts,
                             double* out, int C, int H, int W, int Oc, int Kh, int Kw, int pad) {
  (void)Oc;
  for (int i = 0; i < npts; ++i) {
    const int n = pts[4 * i], oc = pts[4 * i + 1], ho = pts[4 * i + 2], wo = pts[4 * i + 3];
    double acc = 0;
    for (int c = 0; c < C; ++c)
      for (int kh = 0; kh < Kh; ++kh) {
        const int hi = ho + kh - pad;
        if (hi < 0 || hi >= H) continue;
        for (int kw = 0; kw < Kw; ++kw) {
          const int wi = wo + kw - pad;
          if (wi < 0 || wi >= W) continue;
          acc += (double)x[(((size_t)n * C + c) * H + hi) * W + wi] *
                 (double)w[(((size_t)oc * C + c) * Kh + kh) * Kw + kw];
        }
      }
    out[i] = acc * (s ? (double)s[oc] : 1.0);
  }
}

void or_conv_nchw_f32(const float* x, const float* w, const float* s, float* y,
                      int N, int C, int H, int W, int Oc, int Kh, int Kw,
                      int pad, int n0, int n1, int threads) {
  (void)N;
#ifdef _OPENMP
#pragma omp parallel num_threads(UK_NT(threads))
  {
    const int nt = omp_get_num_threads(), t = omp_get_thread_num();
    const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
    for (int n = n0; n < n1; ++n)
      for (int oc = t; oc < Oc; oc += nt) {
        const float sc = s ? s[oc] : 1.0f;
        for (int ho = 0; ho < Ho; ++ho)
          for (int wo = 0; wo < Wo; ++wo) {
            float acc = 0;
            for (int c = 0; c < C; ++c)
              for (int kh = 0; kh < Kh; ++kh) {
                const int hi = ho + kh - pad;
                if (hi < 0 || hi >= H) continue;
                for (int kw = 0; kw < Kw; ++kw) {
                  const int wi = wo + kw - pad;
                  if (wi < 0 || wi >= W) continue;
                  acc += x[(((size_t)n * C + c) * H + hi) * W + wi] *
                         w[(((size_t)oc * C + c) * Kh + kh) * Kw + kw];
                }
              }
            y[(((size_t)n * Oc + oc) * Ho + ho) * Wo + wo] = acc * sc;
          }
      }
  }
#else
  (void)threads;
  UK_CONV_NCHW_BODY(float)
#endif
}

/* ---- reduce: src/reference.cpp:24-48 ---- */
float or_reduce_f32(const float* x, int64_t n) {
  float acc = 0.f;
  for (int64_t i = 0; i < n; ++i) acc += x[i];
  return acc;
}

float or_reduce_blocked_f32(const float* x, int64_t n, int width) {
  if (width <= 0) return or_reduce_f32(x, n);
  float acc = 0.f;
  for (int b = 0; b < width; ++b) {
    float part = 0.f;
    for (int64_t i = b; i < n; i += width) part += x[i];
    acc += part;
  }
  return acc;
}

double or_reduce_f64(const float* x, int64_t n) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) acc += (double)x[i];
  return acc;
}

void or_row_reduce_f32(const float* x, float* y, int64_t rows, int64_t cols,
                       int width, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t r = 0; r < rows; ++r)
    y[r] = or_reduce_blocked_f32(x + r * cols, cols, width);
  (void)threads;
}

void or_row_reduce_f64(const float* x, double* y, int64_t rows, int64_t cols,
                       int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t r = 0; r < rows; ++r) y[r] = or_reduce_f64(x + r * cols, cols);
  (void)threads;
}

/* ---- softmax: src/codegen_hip.cpp:1999-2009 ---- */
void or_softmax_f32(const float* X, float* Y, int64_t L, int64_t C, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t l = 0; l < L; ++l) {
    const float* x = X + l * C;
    float* y = Y + l * C;
    float maxv = -INFINITY;
    for (int64_t c = 0; c < C; ++c)
      if (x[c] > maxv) maxv = x[c];
    float sum = 0.0f;
    for (int64_t c = 0; c < C; ++c) sum += expf(x[c] - maxv);
    for (int64_t c = 0; c < C; ++c) y[c] = expf(x[c] - maxv) / sum;
  }
  (void)threads;
}

void or_softmax_f64(const float* X, double* Y, int64_t L, int64_t C, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t l = 0; l < L; ++l) {
    const float* x = X + l * C;
    double* y = Y + l * C;
    double maxv = -INFINITY;
    for (int64_t c = 0; c < C; ++c)
      if (x[c] > maxv) maxv = x[c];
    double sum = 0.0;
    for (int64_t c = 0; c < C; ++c) sum += exp((double)x[c] - maxv);
    for (int64_t c = 0; c < C; ++c) y[c] = exp((double)x[c] - maxv) / sum;
  }
  (void)threads;
}

/* ---- rmsnorm: src/codegen_hip.cpp:2168-2178 (eps = 1e-6f there) ---- */
void or_rmsnorm_f32(const float* X, const float* W, float* Y, int64_t L,
                    int64_t C, float eps, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t l = 0; l < L; ++l) {
    const float* x = X + l * C;
    float* y = Y + l * C;
    float sum_sq = 0.0f;
    for (int64_t c = 0; c < C; ++c) sum_sq += x[c] * x[c];
    const float rms = 1.0f / sqrtf(sum_sq / (float)C + eps);
    for (int64_t c = 0; c < C; ++c) y[c] = x[c] * rms * W[c];
  }
  (void)threads;
}

void or_rmsnorm_f64(const float* X, const float* W, double* Y, int64_t L,
                    int64_t C, double eps, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t l = 0; l < L; ++l) {
    const float* x = X + l * C;
    double* y = Y + l * C;
    double sum_sq = 0.0;
    for (int64_t c = 0; c < C; ++c) sum_sq += (double)x[c] * (double)x[c];
    const double rms = 1.0 / sqrt(sum_sq / (double)C + eps);
    for (int64_t c = 0; c < C; ++c) y[c] = (double)x[c] * rms * (double)W[c];
  }
  (void)threads;
}

/* ---- channelscale: src/codegen_hip.cpp:2339-2344 ---- */
void or_channelscale_f32(const float* X, const float* S, float* Y, int64_t L,
                         int64_t C, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(UK_NT(threads))
#endif
  for (int64_t i = 0; i < L; ++i)
    for (int64_t c = 0; c < C; ++c) Y[i * C + c] = X[i * C + c] * S[c];
  (void)threads;
}
