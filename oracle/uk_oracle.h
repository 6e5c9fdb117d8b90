/*
 * uk_oracle.h -- CPU restatement of the reference KML operator set.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * is compared against.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it; the product
 * library (unikern_b200/_lib/libunikern_cuda.so) never links or calls it.
 *
 * Every f32 routine keeps the reference's loop order and fp32 accumulator
 * so that, compiled with -ffp-contract=off and without -ffast-math, it is
 * bit-identical to the reference's CPU code.  Sources followed (paths within
 * the UNIKERN project):
 *   gemm f32 ........ src/codegen_hip.cpp:1124-1132  (embedded cpu_ref)
 *   gemm f16 ........ src/codegen_hip.cpp:1851-1862  (quantise, then cpu_ref)
 *   conv ............ src/reference.cpp:6-22         (cpu_conv)
 *   reduce .......... src/reference.cpp:24-28        (cpu_reduce)
 *   reduce blocked .. src/reference.cpp:37-48        (cpu_reduce_blocked)
 *   softmax ......... src/codegen_hip.cpp:1999-2009  (embedded cpu_softmax)
 *   rmsnorm ......... src/codegen_hip.cpp:2168-2178  (embedded cpu_rmsnorm,
 *                     eps hard-coded 1e-6 there; a parameter here)
 *   channelscale .... src/codegen_hip.cpp:2339-2344  (embedded cpu_channelscale)
 *   sawtooth inits .. src/codegen_hip.cpp:604-605, :1998, :2167, :2338
 *
 * The *_f64 twins accumulate in double and are the yardstick for random
 * inputs, where fp32 reordering makes bit equality meaningless.
 *
 * `threads` parameters parallelise over the OUTER index only (rows of C,
 * output channels, rows of a row op), so every output element is computed
 * by the same sequential loop as the single-threaded version and the
 * results are bit-identical for any thread count.
 */
#ifndef UK_ORACLE_H
#define UK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* sawtooth initialisers of the reference's verify instances */
float or_initA(int idx); /* ((idx % 17) - 8) * 0.0625f */
float or_initB(int idx); /* ((idx % 13) - 6) * 0.0625f */
float or_initW(int idx); /* 1 + ((idx % 7) - 3) * 0.0625f (initW and initS) */
void or_fill_initA(float* dst, int64_t n);
void or_fill_initB(float* dst, int64_t n);
void or_fill_initW(float* dst, int64_t n);

/* IEEE binary16 <-> binary32, round to nearest even (the __float2half rule) */
uint16_t or_f32_to_f16(float x);
float or_f16_to_f32(uint16_t h);
void or_f32_to_f16_n(const float* src, uint16_t* dst, int64_t n);
void or_f16_to_f32_n(const uint16_t* src, float* dst, int64_t n);

/* C[M][N] = A[M][K] * B[K][N], row-major, i -> j -> k, fp32 accumulator.
 * Rows [row0, row1) only (the full product is row0 = 0, row1 = M). */
void or_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K,
                 int row0, int row1, int threads);
/* same loops, double accumulator over the fp32 inputs */
void or_gemm_f64(const float* A, const float* B, double* C, int M, int N, int K,
                 int row0, int row1, int threads);
/* half inputs: quantised values are widened to fp32 first (the reference
 * converts with __half2float before calling cpu_ref), then or_gemm_f32 loops */
void or_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int M, int N,
                 int K, int row0, int row1, int threads);
void or_gemm_f16_f64(const uint16_t* A, const uint16_t* B, double* C, int M,
                     int N, int K, int row0, int row1, int threads);
/* one dot product C[i][j] in double, for sampled checks of huge GEMMs */
double or_gemm_f16_dot_f64(const uint16_t* A, const uint16_t* B, int N, int K,
                           int i, int j);

/* valid conv: x[H][W][C], wt[Oc][Kh][Kw][C], y[Oc][Ho][Wo], order c->kh->kw */
void or_conv_f32(const float* x, const float* wt, float* y, int H, int W, int C,
                 int Kh, int Kw, int Oc, int threads);
void or_conv_f64(const float* x, const float* wt, double* y, int H, int W,
                 int C, int Kh, int Kw, int Oc, int threads);
/* NCHW batch form with zero padding `pad`, stride 1, and an optional
 * per-output-channel scale s[Oc] (NULL = 1):
 *   x[N][C][H][W], w[Oc][C][Kh][Kw], y[N][Oc][Ho][Wo], Ho = H + 2 pad - Kh + 1.
 * Images [n0, n1) only.  Double accumulator (the yardstick). */
void or_conv_nchw_f64(const float* x, const float* w, const float* s, double* y,
                      int N, int C, int H, int W, int Oc, int Kh, int Kw,
                      int pad, int n0, int n1, int threads);
/* The f64 yardstick of or_conv_nchw_f64 at `npts` single output points
 * pts[4 * i .. 4 * i + 3] = (n, oc, ho, wo) -> out[i]; for sampled checks of
 * full-batch runs whose every image would take too long on the host. */
void or_conv_nchw_points_f64(const float* x, const float* w, const float* s, const int* pts, int npts,
                             double* out, int C, int H, int W, int Oc, int Kh, int Kw, int pad);
/* same, fp32 accumulator in the reference's c->kh->kw order (timing arm) */
void or_conv_nchw_f32(const float* x, const float* w, const float* s, float* y,
                      int N, int C, int H, int W, int Oc, int Kh, int Kw,
                      int pad, int n0, int n1, int threads);

/* reduce: sequential fp32 sum in index order */
float or_reduce_f32(const float* x, int64_t n);
/* reduce: `width` strided fp32 partials folded in index order */
float or_reduce_blocked_f32(const float* x, int64_t n, int width);
double or_reduce_f64(const float* x, int64_t n);
/* row form used by the [rows x cols] -> [rows] configuration: each row is
 * reduced by or_reduce_blocked_f32 (width <= 0 selects the sequential tier) */
void or_row_reduce_f32(const float* x, float* y, int64_t rows, int64_t cols,
                       int width, int threads);
void or_row_reduce_f64(const float* x, double* y, int64_t rows, int64_t cols,
                       int threads);

/* softmax rows: max, sum of expf(x - max), y = expf(x - max) / sum */
void or_softmax_f32(const float* X, float* Y, int64_t L, int64_t C, int threads);
void or_softmax_f64(const float* X, double* Y, int64_t L, int64_t C, int threads);

/* rmsnorm rows: rms = 1 / sqrt(sum(x^2) / C + eps); y = x * rms * W[c] */
void or_rmsnorm_f32(const float* X, const float* W, float* Y, int64_t L,
                    int64_t C, float eps, int threads);
void or_rmsnorm_f64(const float* X, const float* W, double* Y, int64_t L,
                    int64_t C, double eps, int threads);

/* channelscale: Y[i*C + c] = X[i*C + c] * S[c] */
void or_channelscale_f32(const float* X, const float* S, float* Y, int64_t L,
                         int64_t C, int threads);

#ifdef __cplusplus
}
#endif

#endif /* UK_ORACLE_H */
