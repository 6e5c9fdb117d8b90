// rowops_f16.cu -- softmax, RMSNorm and channelscale with fp16 rows (IEEE
// binary16 in and out, fp32 arithmetic).  The reference refuses these dtypes
// for the row ops (its capability gap, src/codegen_hip.cpp:81-89); this widens
// the interval with the same algorithms as the fp32 kernels of rowops.cu:
//   softmax       y = f16( exp(x - max) * (1 / sum exp(x - max)) )
//   RMSNorm       y = f16( (x * (1 / sqrt(sum x^2 / C + eps))) * w )
//   channelscale  y = f16( x * s[c] )        (one fp32 multiply, one rounding)
// Softmax takes the exponential from the hardware's fast exp2 (__expf): its
// error (2 + 1.16 |x - max| ulp of fp32, under 1e-5 relative wherever the
// result is not below f16's range) is far under the f16 output rounding
// (2^-11), and it keeps the f16 kernel memory-bound instead of bound by the
// accurate expf's instruction count.
// One CTA per row with the row in registers (16-byte vectors of 8 halves);
// rows longer than 32768 columns take two passes (online max/sum for
// softmax).  Reductions are warp shuffles plus a fixed-order cross-warp step,
// so results are deterministic.  Half the bytes of the fp32 ops per element.
#include <cuda_fp16.h>

#include "uk_common.cuh"

namespace {

constexpr int kOpRms = 0, kOpSoftmax = 1, kOpScale = 2;

template <int W>
__device__ __forceinline__ void ld_h(float (&d)[W], const __half* p, bool stream) {
  if constexpr (W == 8) {
    const uint4 t = stream ? __ldcs(reinterpret_cast<const uint4*>(p)) : __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      d[2 * i] = f.x;
      d[2 * i + 1] = f.y;
    }
  } else {
    d[0] = __half2float(stream ? __ldcs(p) : __ldg(p));
  }
}

template <int W>
__device__ __forceinline__ void st_h(__half* p, const float (&d)[W]) {
  if constexpr (W == 8) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(d[2 * i], d[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    __stcs(reinterpret_cast<uint4*>(p), make_uint4(w[0], w[1], w[2], w[3]));
  } else {
    __stcs(p, __float2half_rn(d[0]));
  }
}

// 8 halves of a 16-byte vector as fp32
__device__ __forceinline__ void unpack8(float (&d)[8], const uint4& t) {
  const uint32_t q[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
    d[2 * i] = f.x;
    d[2 * i + 1] = f.y;
  }
}

// The row stays in registers as packed halves (one uint4 per 8 columns, half
// the registers of fp32 copies), so four 512-thread CTAs fit on an SM and
// twice the bytes are in flight; values are unpacked to fp32 where used.
// Softmax takes exp(x - max) twice (for the sum, then for the output) rather
// than keep fp32 copies.
// CTAs per SM asked of the register allocator: a full SM (2048 threads) for
// short rows, three quarters for four vectors per thread
template <int THREADS, int VPT, int W>
constexpr int rowop_h_min_blocks() {
  return W != 8 ? 1 : VPT <= 2 ? 2048 / THREADS : VPT <= 4 ? (1536 / THREADS > 0 ? 1536 / THREADS : 1) : 1;
}

template <int OP, int THREADS, int VPT, int W>
__global__ void __launch_bounds__(THREADS, (rowop_h_min_blocks<THREADS, VPT, W>()))
    k_rowop_h(const __half* __restrict__ X, const __half* __restrict__ G, __half* __restrict__ Y, int64_t C,
              float eps) {
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const __half* x = X + row * C;
  __half* y = Y + row * C;
  const int64_t nv = C / W;
  if constexpr (W == 8) {
    uint4 raw[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      // -inf halves (0xFC00) pad softmax rows; zeros pad the others
      raw[k] = j < nv ? __ldcs(reinterpret_cast<const uint4*>(x + j * 8))
                      : (OP == kOpSoftmax ? make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u)
                                          : make_uint4(0u, 0u, 0u, 0u));
    }
    float scale = 1.f, m = 0.f;
    if constexpr (OP == kOpRms) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float d[8];
        unpack8(d, raw[k]);
#pragma unroll
        for (int w = 0; w < 8; ++w) ss += d[w] * d[w];
      }
      ss = uk_block_sum<THREADS>(ss, red);
      scale = 1.0f / sqrtf(ss / (float)C + eps);
    } else if constexpr (OP == kOpSoftmax) {
      m = -INFINITY;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float d[8];
        unpack8(d, raw[k]);
#pragma unroll
        for (int w = 0; w < 8; ++w) m = fmaxf(m, d[w]);
      }
      m = uk_block_max<THREADS>(m, red);
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float d[8];
        unpack8(d, raw[k]);
#pragma unroll
        for (int w = 0; w < 8; ++w) sum += __expf(d[w] - m);
      }
      sum = uk_block_sum<THREADS>(sum, red);
      scale = 1.0f / sum;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
        float d[8];
        unpack8(d, raw[k]);
        if constexpr (OP == kOpSoftmax) {
#pragma unroll
          for (int w = 0; w < 8; ++w) d[w] = __expf(d[w] - m) * scale;
        } else {
          float g[8];
          ld_h<8>(g, G + j * 8, false);
#pragma unroll
          for (int w = 0; w < 8; ++w) d[w] = OP == kOpRms ? (d[w] * scale) * g[w] : d[w] * g[w];
        }
        st_h<8>(y + j * 8, d);
      }
    }
  } else {
    float v[VPT][W];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
        ld_h<W>(v[k], x + j * W, true);
      } else {
#pragma unroll
        for (int w = 0; w < W; ++w) v[k][w] = OP == kOpSoftmax ? -INFINITY : 0.f;
      }
    }
    float scale = 1.f;
    if constexpr (OP == kOpRms) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int w = 0; w < W; ++w) ss += v[k][w] * v[k][w];
      ss = uk_block_sum<THREADS>(ss, red);
      scale = 1.0f / sqrtf(ss / (float)C + eps);
    } else if constexpr (OP == kOpSoftmax) {
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int w = 0; w < W; ++w) m = fmaxf(m, v[k][w]);
      m = uk_block_max<THREADS>(m, red);
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const float e = __expf(v[k][w] - m);
          v[k][w] = e;
          sum += e;
        }
      sum = uk_block_sum<THREADS>(sum, red);
      scale = 1.0f / sum;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t j = threadIdx.x + (int64_t)k * THREADS;
      if (j < nv) {
        if constexpr (OP == kOpSoftmax) {
#pragma unroll
          for (int w = 0; w < W; ++w) v[k][w] = v[k][w] * scale;
        } else {
          float g[W];
          ld_h<W>(g, G + j * W, false);
#pragma unroll
          for (int w = 0; w < W; ++w) v[k][w] = OP == kOpRms ? (v[k][w] * scale) * g[w] : v[k][w] * g[w];
        }
        st_h<W>(y + j * W, v[k]);
      }
    }
  }
}

// rows too long for registers: a statistics pass, then the output pass
template <int OP, int W>
__global__ void __launch_bounds__(512) k_rowop_h_stream(const __half* __restrict__ X, const __half* __restrict__ G,
                                                        __half* __restrict__ Y, int64_t C, float eps) {
  __shared__ float red[33];
  __shared__ float sm_m[16], sm_s[16];
  const int64_t row = blockIdx.x;
  const __half* x = X + row * C;
  __half* y = Y + row * C;
  const int64_t nv = C / W;
  float scale = 1.f, M = 0.f;
  if constexpr (OP == kOpRms) {
    float ss = 0.f;
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W];
      ld_h<W>(d, x + j * W, false);
#pragma unroll
      for (int w = 0; w < W; ++w) ss += d[w] * d[w];
    }
    ss = uk_block_sum<512>(ss, red);
    scale = 1.0f / sqrtf(ss / (float)C + eps);
  } else if constexpr (OP == kOpSoftmax) {
    float m = -INFINITY, s = 0.f;
    for (int64_t j = threadIdx.x; j < nv; j += 512) {
      float d[W];
      ld_h<W>(d, x + j * W, false);
#pragma unroll
      for (int w = 0; w < W; ++w) {
        if (d[w] > m) {
          s = s * __expf(m - d[w]) + 1.f;
          m = d[w];
        } else {
          s += __expf(d[w] - m);
        }
      }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
    }
    if (lane == 0) {
      sm_m[warp] = m;
      sm_s[warp] = s;
    }
    __syncthreads();
    M = -INFINITY;
    for (int i = 0; i < 16; ++i) M = fmaxf(M, sm_m[i]);
    float S = 0.f;
    for (int i = 0; i < 16; ++i)
      if (sm_m[i] != -INFINITY) S += sm_s[i] * __expf(sm_m[i] - M);
    scale = 1.0f / S;
  }
  for (int64_t j = threadIdx.x; j < nv; j += 512) {
    float d[W];
    ld_h<W>(d, x + j * W, true);
    if constexpr (OP == kOpSoftmax) {
#pragma unroll
      for (int w = 0; w < W; ++w) d[w] = __expf(d[w] - M) * scale;
    } else {
      float g[W];
      ld_h<W>(g, G + j * W, false);
#pragma unroll
      for (int w = 0; w < W; ++w) d[w] = OP == kOpRms ? (d[w] * scale) * g[w] : d[w] * g[w];
    }
    st_h<W>(y + j * W, d);
  }
}

template <int OP, int W>
void dispatch(const __half* X, const __half* G, __half* Y, int64_t L, int64_t C, float eps, cudaStream_t st) {
  const int64_t nv = C / W;
#define UK_TRY(T, V)                                                                   \
  if (nv <= (int64_t)(T) * (V)) {                                                      \
    k_rowop_h<OP, T, V, W><<<(unsigned)L, T, 0, st>>>(X, G, Y, C, eps);                \
    return;                                                                            \
  }
  if constexpr (W == 8) {
    // the most threads for a row, at most 4 vectors (32 halves) each: more
    // loads in flight and shorter per-thread chains
    UK_TRY(32, 1) UK_TRY(32, 2) UK_TRY(64, 2) UK_TRY(128, 2) UK_TRY(128, 4) UK_TRY(256, 4) UK_TRY(512, 4)
    UK_TRY(512, 8)
  } else {
    UK_TRY(32, 1) UK_TRY(64, 2) UK_TRY(128, 4) UK_TRY(256, 4) UK_TRY(256, 8)
  }
#undef UK_TRY
  k_rowop_h_stream<OP, W><<<(unsigned)L, 512, 0, st>>>(X, G, Y, C, eps);
}

int run(int op, const uint16_t* X, const uint16_t* G, uint16_t* Y, int64_t L, int64_t C, float eps, void* stream,
        const char* name) {
  if (L < 0 || C < 0) return uk::fail(UK_EINVAL, "%s: negative size L=%lld C=%lld", name, (long long)L, (long long)C);
  if (L > 2147483647LL) return uk::fail(UK_EINVAL, "%s: L=%lld exceeds 2^31-1 rows", name, (long long)L);
  if (L == 0 || C == 0) return UK_OK;
  if (op == kOpRms && !(eps >= 0.f)) return uk::fail(UK_EINVAL, "%s: eps must be >= 0", name);
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (G)
    if (int rc = uk::check_device_ptr(G, op == kOpRms ? "W" : "S")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  const bool vec = C % 8 == 0 && uk::aligned16(X) && uk::aligned16(Y) && (G == nullptr || uk::aligned16(G));
  const __half *x = (const __half*)X, *g = (const __half*)G;
  __half* y = (__half*)Y;
  if (op == kOpRms) vec ? dispatch<kOpRms, 8>(x, g, y, L, C, eps, st) : dispatch<kOpRms, 1>(x, g, y, L, C, eps, st);
  else if (op == kOpSoftmax)
    vec ? dispatch<kOpSoftmax, 8>(x, g, y, L, C, eps, st) : dispatch<kOpSoftmax, 1>(x, g, y, L, C, eps, st);
  else vec ? dispatch<kOpScale, 8>(x, g, y, L, C, eps, st) : dispatch<kOpScale, 1>(x, g, y, L, C, eps, st);
  return uk::check_launch(name);
}

}  // namespace

extern "C" {

int uk_cuda_softmax_f16(const uint16_t* X, uint16_t* Y, int64_t L, int64_t C, void* stream) {
  return run(kOpSoftmax, X, nullptr, Y, L, C, 0.f, stream, "softmax_f16");
}

int uk_cuda_rmsnorm_f16(const uint16_t* X, const uint16_t* W, uint16_t* Y, int64_t L, int64_t C, float eps,
                        void* stream) {
  if (W == nullptr) return uk::fail(UK_EINVAL, "rmsnorm_f16: W is NULL");
  return run(kOpRms, X, W, Y, L, C, eps, stream, "rmsnorm_f16");
}

int uk_cuda_channelscale_f16(const uint16_t* X, const uint16_t* S, uint16_t* Y, int64_t L, int64_t C, void* stream) {
  if (S == nullptr) return uk::fail(UK_EINVAL, "channelscale_f16: S is NULL");
  return run(kOpScale, X, S, Y, L, C, 0.f, stream, "channelscale_f16");
}

}  // extern "C"
