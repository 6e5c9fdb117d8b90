// rowops.cu -- the HBM-bound KML ops on B200: channelscale, reduce (row and
// scalar forms), RMSNorm and softmax.
//
// Design (vs. the reference's one-thread-per-row kernels,
// src/codegen_hip.cpp:1985-1996, :2154-2164, :2329-2335, :818-833):
//   * every HBM byte is touched once: a row op keeps its whole row in
//     registers (one CTA per row, 128-bit loads), so X is read once and Y
//     written once;
//   * loads/stores of single-use data use the streaming cache hint;
//   * reductions are warp shuffles + a fixed-order cross-warp step, so the
//     result bits are the same on every call (deterministic);
//   * grids are sized from the SM count (148 on B200), not from a label.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cmath>
#include <mutex>

#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace {

constexpr int kOpRms = 0;
constexpr int kOpSoftmax = 1;
constexpr int kOpScale = 2;  // channelscale: y = x * s[c], no row statistic

// ---------------------------------------------------------------------------
// channelscale: Y[i*C + c] = X[i*C + c] * S[c].  threadIdx.x walks column
// vectors (S held in registers for the whole CTA lifetime), threadIdx.y and
// the grid walk rows; RU rows are in flight per thread.
// ---------------------------------------------------------------------------
template <int W, int RU>
__global__ void __launch_bounds__(256) k_channelscale(const float* __restrict__ X,
                                                      const float* __restrict__ S,
                                                      float* __restrict__ Y, int64_t L, int64_t C) {
  const int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * W;
  if (c >= C) return;
  float s[W];
  uk_ld_g<W>(s, S + c);
  const int64_t step = (int64_t)gridDim.y * blockDim.y;
  int64_t r = (int64_t)blockIdx.y * blockDim.y + threadIdx.y;
  for (; r + (RU - 1) * step < L; r += RU * step) {
    float x[RU][W];
#pragma unroll
    for (int u = 0; u < RU; ++u) uk_ld_cs<W>(x[u], X + (r + u * step) * C + c);
#pragma unroll
    for (int u = 0; u < RU; ++u) {
#pragma unroll
      for (int w = 0; w < W; ++w) x[u][w] = x[u][w] * s[w];
      uk_st_cs<W>(Y + (r + u * step) * C + c, x[u]);
    }
  }
  for (; r < L; r += step) {
    float x[W];
    uk_ld_cs<W>(x, X + r * C + c);
#pragma unroll
    for (int w = 0; w < W; ++w) x[w] = x[w] * s[w];
    uk_st_cs<W>(Y + r * C + c, x);
  }
}

// ---------------------------------------------------------------------------
// reduce
// ---------------------------------------------------------------------------
// W consecutive elements as fp32: floats (W = 1 or 4) or binary16 (W = 1 or
// 8, one 16-byte load), streaming cache hint
template <int W>
__device__ __forceinline__ void ld_span(float (&d)[W], const float* p) {
  uk_ld_cs<W>(d, p);
}
template <int W>
__device__ __forceinline__ void ld_span(float (&d)[W], const __half* p) {
  if constexpr (W == 8) {
    const uint4 t = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint32_t q[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
      d[2 * i] = f.x;
      d[2 * i + 1] = f.y;
    }
  } else {
    static_assert(W == 1, "binary16 spans are 1 or 8 wide");
    d[0] = __half2float(__ldcs(p));
  }
}
__device__ __forceinline__ void st_sum(float* y, float v) { *y = v; }
__device__ __forceinline__ void st_sum(__half* y, float v) { *y = __float2half_rn(v); }

// U loads of W elements in flight per thread, summed in fp32; U partial sums
// combined in a fixed order, so the result does not depend on timing
template <int W, int U = 4, class T = float>
__device__ __forceinline__ float sum_span(const T* __restrict__ x, int64_t nv, int tid, int nthr) {
  float acc[U];
#pragma unroll
  for (int u = 0; u < U; ++u) acc[u] = 0.f;
  int64_t v = tid;
  for (; v + (U - 1) * (int64_t)nthr < nv; v += U * (int64_t)nthr) {
    float d[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u) ld_span<W>(d[u], x + (v + u * (int64_t)nthr) * W);
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int w = 0; w < W; ++w) acc[u] += d[u][w];
  }
  for (; v < nv; v += nthr) {
    float d[W];
    ld_span<W>(d, x + v * W);
#pragma unroll
    for (int w = 0; w < W; ++w) acc[0] += d[w];
  }
#pragma unroll
  for (int h = U / 2; h > 0; h /= 2)
#pragma unroll
    for (int u = 0; u < h; ++u) acc[u] += acc[u + h];
  return acc[0];
}

// one 256-thread CTA per row
template <int W, class T = float, class O = float>
__global__ void __launch_bounds__(256) k_rowsum_cta(const T* __restrict__ X, O* __restrict__ Y, int64_t cols) {
  __shared__ float red[33];
  const T* x = X + (int64_t)blockIdx.x * cols;
  float t = sum_span<W, 4, T>(x, cols / W, threadIdx.x, 256);
  t = uk_block_sum<256>(t, red);
  if (threadIdx.x == 0) st_sum(Y + blockIdx.x, t);
}

// one warp per row (short rows), 8 rows per CTA
template <int W, class T = float, class O = float>
__global__ void __launch_bounds__(256) k_rowsum_warp(const T* __restrict__ X, O* __restrict__ Y, int64_t rows,
                                                     int64_t cols) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float t = sum_span<W, 4, T>(X + row * cols, cols / W, threadIdx.x & 31, 32);
  t = uk_warp_sum(t);
  if ((threadIdx.x & 31) == 0) st_sum(Y + row, t);
}

// split rows: CTA (s, r) sums chunk s of row r into P[r * splits + s]
template <int W, class T = float>
__global__ void __launch_bounds__(256) k_rowsum_split(const T* __restrict__ X, float* __restrict__ P, int64_t cols,
                                                      int64_t splits, int64_t chunk) {
  __shared__ float red[33];
  const int64_t r = blockIdx.y, s = blockIdx.x;
  const int64_t c0 = s * chunk;
  const int64_t c1 = c0 + chunk < cols ? c0 + chunk : cols;
  float t = 0.f;
  if (c0 < c1) t = sum_span<W, 4, T>(X + r * cols + c0, (c1 - c0) / W, threadIdx.x, 256);
  t = uk_block_sum<256>(t, red);
  if (threadIdx.x == 0) P[r * splits + s] = t;
}

// fold the partials of each row in a fixed order (one warp per row)
template <class O = float>
__global__ void __launch_bounds__(256) k_rowsum_fold(const float* __restrict__ P, O* __restrict__ Y, int64_t rows,
                                                     int64_t splits) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  float t = 0.f;
  for (int64_t i = lane; i < splits; i += 32) t += P[row * splits + i];
  t = uk_warp_sum(t);
  if (lane == 0) st_sum(Y + row, t);
}

__global__ void k_fill_zero(float* __restrict__ Y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    Y[i] = 0.f;
}

__global__ void k_fill_zero_h(__half* __restrict__ Y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    Y[i] = __float2half_rn(0.f);
}

// ---------------------------------------------------------------------------
// RMSNorm / softmax with the row in registers: one CTA per row, THREADS x VPT
// vectors of W floats cover up to THREADS * VPT * W columns.
// ---------------------------------------------------------------------------
template <int OP, int THREADS, int VPT, int W>
__global__ void __launch_bounds__(THREADS) k_rowop(const float* __restrict__ X, const float* __restrict__ G,
                                                   float* __restrict__ Y, int64_t C, float eps) {
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const float* x = X + row * C;
  float* y = Y + row * C;
  const int64_t nv = C / W;
  float v[VPT][W];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t j = threadIdx.x + (int64_t)k * THREADS;
    if (j < nv) {
      uk_ld_cs<W>(v[k], x + j * W);
    } else {
#pragma unroll
      for (int w = 0; w < W; ++w) v[k][w] = OP == kOpSoftmax ? -INFINITY : 0.f;
    }
  }
  if constexpr (OP == kOpScale) {
    (void)red;
    (void)eps;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
        float g[W];
        uk_ld_g<W>(g, G + j * W);
#pragma unroll
        for (int w = 0; w < W; ++w) v[k][w] = v[k][w] * g[w];
        uk_st_cs<W>(y + j * W, v[k]);
      }
    }
  } else if constexpr (OP == kOpRms) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int w = 0; w < W; ++w) ss += v[k][w] * v[k][w];
    ss = uk_block_sum<THREADS>(ss, red);
    // src/codegen_hip.cpp:2175: rms = 1 / sqrt(sum_sq / C + eps) (IEEE div and sqrt)
    const float rms = 1.0f / sqrtf(ss / (float)C + eps);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
        float g[W];
        uk_ld_g<W>(g, G + j * W);
#pragma unroll
        for (int w = 0; w < W; ++w) v[k][w] = v[k][w] * rms * g[w];
        uk_st_cs<W>(y + j * W, v[k]);
      }
    }
  } else {
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int w = 0; w < W; ++w) m = fmaxf(m, v[k][w]);
    m = uk_block_max<THREADS>(m, red);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float e = expf(v[k][w] - m);
        v[k][w] = e;
        s += e;
      }
    s = uk_block_sum<THREADS>(s, red);
    const float inv = 1.0f / s;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
#pragma unroll
        for (int w = 0; w < W; ++w) v[k][w] = v[k][w] * inv;
        uk_st_cs<W>(y + j * W, v[k]);
      }
    }
  }
}

// Rows too long for registers: statistics pass over global memory, then an
// output pass (the second read usually hits L2).  Softmax uses the online
// (max, sum) recurrence per thread, merged in a fixed order.
template <int OP, int W>
__global__ void __launch_bounds__(512) k_rowop_stream(const float* __restrict__ X, const float* __restrict__ G,
                                                      float* __restrict__ Y, int64_t C, float eps) {
  __shared__ float red[33];
  __shared__ float sm_m[16], sm_s[16];
  const int64_t row = blockIdx.x;
  const float* x = X + row * C;
  float* y = Y + row * C;
  const int64_t nv = C / W;
  if constexpr (OP == kOpRms) {
    float ss = 0.f;
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W];
      uk_ld_g<W>(d, x + j * W);
#pragma unroll
      for (int w = 0; w < W; ++w) ss += d[w] * d[w];
    }
    ss = uk_block_sum<512>(ss, red);
    const float rms = 1.0f / sqrtf(ss / (float)C + eps);
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W], g[W];
      uk_ld_cs<W>(d, x + j * W);
      uk_ld_g<W>(g, G + j * W);
#pragma unroll
      for (int w = 0; w < W; ++w) d[w] = d[w] * rms * g[w];
      uk_st_cs<W>(y + j * W, d);
    }
  } else {
    float m = -INFINITY, s = 0.f;
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W];
      uk_ld_g<W>(d, x + j * W);
#pragma unroll
      for (int w = 0; w < W; ++w) {
        if (d[w] > m) {
          s = s * expf(m - d[w]) + 1.f;
          m = d[w];
        } else {
          s += expf(d[w] - m);
        }
      }
    }
    // merge (m, s) pairs: warp level, then the 16 warps in index order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mm));
      m = mm;
    }
    if (lane == 0) {
      sm_m[warp] = m;
      sm_s[warp] = s;
    }
    __syncthreads();
    float M = -INFINITY;
    for (int i = 0; i < 16; ++i) M = fmaxf(M, sm_m[i]);
    float S = 0.f;
    for (int i = 0; i < 16; ++i)
      if (sm_m[i] != -INFINITY) S += sm_s[i] * expf(sm_m[i] - M);
    const float inv = 1.0f / S;
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W];
      uk_ld_cs<W>(d, x + j * W);
#pragma unroll
      for (int w = 0; w < W; ++w) d[w] = expf(d[w] - M) * inv;
      uk_st_cs<W>(y + j * W, d);
    }
  }
}

template <int OP, int THREADS, int VPT, int W>
void launch_rowop(const float* X, const float* G, float* Y, int64_t L, int64_t C, float eps, cudaStream_t st) {
  k_rowop<OP, THREADS, VPT, W><<<(unsigned)L, THREADS, 0, st>>>(X, G, Y, C, eps);
}

// (THREADS, VPT) from uk::rowop_plan; rows too long for registers stream
template <int OP, int W>
bool dispatch_rowop(const float* X, const float* G, float* Y, int64_t L, int64_t C, float eps, cudaStream_t st) {
  int t = 0, v = 0;
  if (uk::rowop_plan(C, W, &t, &v)) {
#define UK_CASE(T, V)                                     \
  if (t == (T) && v == (V)) {                             \
    launch_rowop<OP, T, V, W>(X, G, Y, L, C, eps, st);    \
    return true;                                          \
  }
    if constexpr (W == 4) {
      UK_CASE(32, 1) UK_CASE(32, 2) UK_CASE(64, 2) UK_CASE(128, 2) UK_CASE(128, 4)
      UK_CASE(256, 4) UK_CASE(256, 8) UK_CASE(512, 8) UK_CASE(512, 16)
    } else {
      UK_CASE(32, 1) UK_CASE(64, 2) UK_CASE(128, 4) UK_CASE(256, 4) UK_CASE(256, 8)
    }
#undef UK_CASE
  }
  if constexpr (OP != kOpScale) {  // the scale op only takes rows that fit in registers
    k_rowop_stream<OP, W><<<(unsigned)L, 512, 0, st>>>(X, G, Y, C, eps);
    return true;
  }
  return false;
}

using uk::ReducePlan;

ReducePlan plan_reduce(int64_t rows, int64_t cols) { return uk::plan_reduce(rows, cols, uk::sm_count()); }

// ---------------------------------------------------------------------------
// Scratch for uk_cuda_reduce_f32_noalloc: the split-row partial sums live in
// this file-scope array instead of a caller workspace.  Every GPU that loads
// the library holds it (32 KiB) until the process exits.  In host code the
// name g_reduce_scratch is only a stand-in for the symbol, never a device
// address: the launch below passes the address cudaGetSymbolAddress returned.
// ---------------------------------------------------------------------------
constexpr int64_t kReduceScratchFloats = 8192;
static __device__ __align__(256) float g_reduce_scratch[kReduceScratchFloats];

// The current context's unique id (cuCtxGetId, reached through the runtime's
// driver entry points, so the library needs no link to libcuda); false when
// the driver cannot say.
bool current_context_id(unsigned long long* id) {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = (GetCurrent)f;
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = (GetId)f;
  });
  CUcontext ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of g_reduce_scratch on the current device.  The set-up (the
// cudaGetSymbolAddress call, with the device current) runs on the first call
// on each device and again whenever that device's context changed since (a
// cudaDeviceReset, or a context torn down and made again, retires the old
// address); where the driver cannot identify the context, every call looks
// the address up again.
int reduce_scratch_address(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  static unsigned long long ctx_of[64] = {0};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return uk::fail(UK_ECUDA, "reduce_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = 0;
  const bool known = current_context_id(&id) && id != 0;
  if (addr[dev] == nullptr || !known || ctx_of[dev] != id) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_reduce_scratch);
    if (e != cudaSuccess || p == nullptr)
      return uk::fail(UK_ECUDA, "reduce_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    addr[dev] = (float*)p;
    unsigned long long now = 0;
    ctx_of[dev] = current_context_id(&now) ? now : 0;
  }
  *out = addr[dev];
  return UK_OK;
}

int check_rows(int64_t L, int64_t C, const char* op) {
  if (L < 0 || C < 0) return uk::fail(UK_EINVAL, "%s: negative size L=%lld C=%lld", op, (long long)L, (long long)C);
  if (L > 2147483647LL) return uk::fail(UK_EINVAL, "%s: L=%lld exceeds 2^31-1 rows", op, (long long)L);
  if (C > 0 && L > INT64_MAX / C) return uk::fail(UK_EINVAL, "%s: L*C overflows", op);
  return UK_OK;
}

// binary16 rows summed in fp32, one rounding into the binary16 result; the
// f32 reduce's plan (width 0) or a pinned pass-1 width
int reduce_h(const uint16_t* Xv, uint16_t* Yv, int64_t rows, int64_t cols, int64_t width, void* workspace,
             size_t workspace_bytes, cudaStream_t st) {
  if (int rc = check_rows(rows, cols, "reduce_f16")) return rc;
  if (rows == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(Yv, "Y")) return rc;
  const __half* X = (const __half*)Xv;
  __half* Y = (__half*)Yv;
  if (cols == 0) {
    k_fill_zero_h<<<(unsigned)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096), 256, 0, st>>>(Y, rows);
    return uk::check_launch("reduce_f16(zero)");
  }
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  ReducePlan p = plan_reduce(rows, cols);
  if (width > 0) {
    const int64_t chunk = (cols + width - 1) / width;
    p = {3, (cols + chunk - 1) / chunk, chunk};
  }
  const bool vec = cols % 8 == 0 && uk::aligned16(X) && (p.mode != 3 || p.chunk % 8 == 0);
  if (p.mode == 1) {
    if (vec) k_rowsum_cta<8, __half, __half><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
    else k_rowsum_cta<1, __half, __half><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
  } else if (p.mode == 2) {
    const unsigned g = (unsigned)((rows + 7) / 8);
    if (vec) k_rowsum_warp<8, __half, __half><<<g, 256, 0, st>>>(X, Y, rows, cols);
    else k_rowsum_warp<1, __half, __half><<<g, 256, 0, st>>>(X, Y, rows, cols);
  } else {
    if (rows > 65535) return uk::fail(UK_EINVAL, "reduce_f16: a split plan takes at most 65535 rows");
    if (p.splits > 2147483647LL) return uk::fail(UK_EINVAL, "reduce_f16: width too large");
    const size_t need = (size_t)(rows * p.splits) * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need)
      return uk::fail(UK_EINVAL, "reduce_f16: needs a %zu-byte workspace (uk_cuda_reduce_workspace_size%s), got %zu",
                      need, width > 0 ? "_width" : "", workspace ? workspace_bytes : (size_t)0);
    if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
    float* P = (float*)workspace;
    const dim3 g1((unsigned)p.splits, (unsigned)rows);
    if (vec) k_rowsum_split<8, __half><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    else k_rowsum_split<1, __half><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    k_rowsum_fold<__half><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(P, Y, rows, p.splits);
  }
  return uk::check_launch("reduce_f16");
}

}  // namespace

extern "C" {

int uk_cuda_channelscale_f32(const float* X, const float* S, float* Y, int64_t L, int64_t C, void* stream) {
  if (int rc = check_rows(L, C, "channelscale")) return rc;
  if (L == 0 || C == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(S, "S")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = C % 4 == 0 && uk::aligned16(X) && uk::aligned16(S) && uk::aligned16(Y);
  int th = 0, vp = 0;
  if (vec && C >= 2048 && L <= 2147483647LL && uk::rowop_plan(C, 4, &th, &vp)) {
    // long rows: one CTA per row streams it contiguously (the row ops' kernel
    // with the scale in place of the statistic)
    dispatch_rowop<kOpScale, 4>(X, S, Y, L, C, 0.f, st);
    return uk::check_launch("channelscale");
  }
  const int W = vec ? 4 : 1;
  const int64_t ncv = (C + W - 1) / W;
  int tx = (int)(ncv < 256 ? ((ncv + 31) / 32) * 32 : 256);
  const int ty = 256 / tx;
  const int64_t gx = (ncv + tx - 1) / tx;
  int64_t gy = (uk::sm_count() * 8 + gx - 1) / gx;
  const int64_t need = (L + ty - 1) / ty;
  if (gy > need) gy = need;
  if (gy > 65535) gy = 65535;
  if (gy < 1) gy = 1;
  if (gx > 2147483647LL) return uk::fail(UK_EINVAL, "channelscale: C too large");
  dim3 grid((unsigned)gx, (unsigned)gy), block(tx, ty);
  if (vec)
    k_channelscale<4, 4><<<grid, block, 0, st>>>(X, S, Y, L, C);
  else
    k_channelscale<1, 4><<<grid, block, 0, st>>>(X, S, Y, L, C);
  return uk::check_launch("channelscale");
}

size_t uk_cuda_reduce_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  const ReducePlan p = plan_reduce(rows, cols);
  return p.mode == 3 ? (size_t)(rows * p.splits) * sizeof(float) : 0;
}

int uk_cuda_reduce_f32(const float* X, float* Y, int64_t rows, int64_t cols, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (int rc = check_rows(rows, cols, "reduce")) return rc;
  if (rows == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const ReducePlan p = plan_reduce(rows, cols);
  if (p.mode == 0) {
    k_fill_zero<<<(unsigned)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096), 256, 0, st>>>(Y, rows);
    return uk::check_launch("reduce(zero)");
  }
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  const bool vec = cols % 4 == 0 && uk::aligned16(X);
  if (p.mode == 1) {
    if (vec) k_rowsum_cta<4><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
    else k_rowsum_cta<1><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
  } else if (p.mode == 2) {
    const unsigned g = (unsigned)((rows + 7) / 8);
    if (vec) k_rowsum_warp<4><<<g, 256, 0, st>>>(X, Y, rows, cols);
    else k_rowsum_warp<1><<<g, 256, 0, st>>>(X, Y, rows, cols);
  } else {
    const size_t need = (size_t)(rows * p.splits) * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need)
      return uk::fail(UK_EINVAL, "reduce: needs a %zu-byte workspace (uk_cuda_reduce_workspace_size), got %zu",
                      need, workspace ? workspace_bytes : (size_t)0);
    if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
    float* P = (float*)workspace;
    dim3 g1((unsigned)p.splits, (unsigned)rows);
    if (rows > 65535) return uk::fail(UK_EINVAL, "reduce: internal split plan with rows > 65535");
    if (vec) k_rowsum_split<4><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    else k_rowsum_split<1><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    k_rowsum_fold<float><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(P, Y, rows, p.splits);
  }
  return uk::check_launch("reduce");
}

size_t uk_cuda_reduce_workspace_size_width(int64_t rows, int64_t cols, int64_t width) {
  if (rows <= 0 || cols <= 0 || width <= 0) return 0;
  const int64_t chunk = (cols + width - 1) / width, parts = (cols + chunk - 1) / chunk;
  return (size_t)(rows * parts) * sizeof(float);
}

int uk_cuda_reduce_f32_width(const float* X, float* Y, int64_t rows, int64_t cols, int64_t width, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (int rc = check_rows(rows, cols, "reduce")) return rc;
  if (width < 1) return uk::fail(UK_EINVAL, "reduce: width must be >= 1 (got %lld)", (long long)width);
  if (rows == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (cols == 0) {
    k_fill_zero<<<(unsigned)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096), 256, 0, st>>>(Y, rows);
    return uk::check_launch("reduce(zero)");
  }
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (rows > 65535) return uk::fail(UK_EINVAL, "reduce: a pinned width takes at most 65535 rows");
  const int64_t chunk = (cols + width - 1) / width, parts = (cols + chunk - 1) / chunk;
  if (parts > 2147483647LL) return uk::fail(UK_EINVAL, "reduce: width too large");
  const size_t need = (size_t)(rows * parts) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need)
    return uk::fail(UK_EINVAL, "reduce: needs a %zu-byte workspace (uk_cuda_reduce_workspace_size_width), got %zu",
                    need, workspace ? workspace_bytes : (size_t)0);
  if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
  float* P = (float*)workspace;
  // 16-byte loads when every chunk starts on a 16-byte boundary
  const bool vec = cols % 4 == 0 && chunk % 4 == 0 && uk::aligned16(X);
  dim3 g1((unsigned)parts, (unsigned)rows);
  if (vec) k_rowsum_split<4><<<g1, 256, 0, st>>>(X, P, cols, parts, chunk);
  else k_rowsum_split<1><<<g1, 256, 0, st>>>(X, P, cols, parts, chunk);
  k_rowsum_fold<float><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(P, Y, rows, parts);
  return uk::check_launch("reduce(width)");
}

int uk_cuda_reduce_f16(const uint16_t* X, uint16_t* Y, int64_t rows, int64_t cols, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return reduce_h(X, Y, rows, cols, 0, workspace, workspace_bytes, (cudaStream_t)stream);
}

int uk_cuda_reduce_f16_width(const uint16_t* X, uint16_t* Y, int64_t rows, int64_t cols, int64_t width,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (width < 1) return uk::fail(UK_EINVAL, "reduce_f16: width must be >= 1 (got %lld)", (long long)width);
  return reduce_h(X, Y, rows, cols, width, workspace, workspace_bytes, (cudaStream_t)stream);
}

int uk_cuda_rmsnorm_f32(const float* X, const float* W, float* Y, int64_t L, int64_t C, float eps, void* stream) {
  if (int rc = check_rows(L, C, "rmsnorm")) return rc;
  if (L == 0 || C == 0) return UK_OK;
  if (!(eps >= 0.f)) return uk::fail(UK_EINVAL, "rmsnorm: eps must be >= 0");
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(W, "W")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = C % 4 == 0 && uk::aligned16(X) && uk::aligned16(W) && uk::aligned16(Y);
  if (vec) dispatch_rowop<kOpRms, 4>(X, W, Y, L, C, eps, st);
  else dispatch_rowop<kOpRms, 1>(X, W, Y, L, C, eps, st);
  return uk::check_launch("rmsnorm");
}

int uk_cuda_softmax_f32(const float* X, float* Y, int64_t L, int64_t C, void* stream) {
  if (int rc = check_rows(L, C, "softmax")) return rc;
  if (L == 0 || C == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = C % 4 == 0 && uk::aligned16(X) && uk::aligned16(Y);
  if (vec) dispatch_rowop<kOpSoftmax, 4>(X, nullptr, Y, L, C, 0.f, st);
  else dispatch_rowop<kOpSoftmax, 1>(X, nullptr, Y, L, C, 0.f, st);
  return uk::check_launch("softmax");
}

// Same result as uk_cuda_reduce_f32 (same kernels, same plan), without a
// caller workspace: see the header for who needs this and its limits.
int uk_cuda_reduce_f32_noalloc(const float* X, float* Y, int64_t rows, int64_t cols, void* stream) {
  if (int rc = check_rows(rows, cols, "reduce_noalloc")) return rc;
  if (rows == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const ReducePlan p = plan_reduce(rows, cols);
  if (p.mode == 0) {
    k_fill_zero<<<(unsigned)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096), 256, 0, st>>>(Y, rows);
    return uk::check_launch("reduce_noalloc(zero)");
  }
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  const bool vec = cols % 4 == 0 && uk::aligned16(X);
  if (p.mode == 1) {
    if (vec) k_rowsum_cta<4><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
    else k_rowsum_cta<1><<<(unsigned)rows, 256, 0, st>>>(X, Y, cols);
  } else if (p.mode == 2) {
    const unsigned g = (unsigned)((rows + 7) / 8);
    if (vec) k_rowsum_warp<4><<<g, 256, 0, st>>>(X, Y, rows, cols);
    else k_rowsum_warp<1><<<g, 256, 0, st>>>(X, Y, rows, cols);
  } else {
    const int64_t need = rows * p.splits;
    if (need > kReduceScratchFloats)
      return uk::fail(UK_EINVAL,
                      "reduce_noalloc: rows=%lld cols=%lld need %lld partial sums, the static scratch holds %lld; "
                      "use uk_cuda_reduce_f32 with a workspace",
                      (long long)rows, (long long)cols, (long long)need, (long long)kReduceScratchFloats);
    if (rows > 65535) return uk::fail(UK_EINVAL, "reduce_noalloc: internal split plan with rows > 65535");
    float* P = nullptr;
    if (int rc = reduce_scratch_address(&P)) return rc;
    // every partial the fold reads is written by the split pass of the same
    // call, so nothing in the shared array has to be cleared first
    dim3 g1((unsigned)p.splits, (unsigned)rows);
    if (vec) k_rowsum_split<4><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    else k_rowsum_split<1><<<g1, 256, 0, st>>>(X, P, cols, p.splits, p.chunk);
    k_rowsum_fold<float><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(P, Y, rows, p.splits);
  }
  return uk::check_launch("reduce_noalloc");
}

}  // extern "C"
