// gemm_f32.cu -- C = A * B in fp32 on the FFMA pipes (no TF32: the f32 KML
// contract verifies at 1e-4 against an f64 yardstick, which TF32 inputs
// would not meet).  Replaces uk_gemm (src/codegen_hip.cpp:1089-1120).
//
// Register-blocked SIMT GEMM: a CTA computes a BM x BN tile, each thread a
// TM x TN micro-tile split into 4-wide groups so shared-memory reads are
// 128-bit; the next K-slab is prefetched into registers while the current
// one is multiplied, with two shared-memory buffers (one barrier per slab).
// Each output accumulates k in ascending order with FFMA.
//
// Small problems (512^3: 128 tiles of 32 x 64 on 148 SMs) would leave each SM
// one CTA of four warps walking all of K, too little work in flight to hide
// latency.  There K is split over a thread-block cluster of KS CTAs (grid z):
// each CTA accumulates its K range in ascending order, the partial tiles meet
// in distributed shared memory, and each CTA sums its slice of rows over the
// cluster in rank order -- deterministic, no workspace.
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace {

// 4 consecutive elements -> fp32 (VEC: one 16-byte float4 or 8-byte half4 load)
__device__ __forceinline__ void ld4(float (&d)[4], const float* p) {
  const float4 t = __ldg(reinterpret_cast<const float4*>(p));
  d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
}
__device__ __forceinline__ void ld4(float (&d)[4], const __half* p) {
  const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
  d[0] = a.x; d[1] = a.y; d[2] = b.x; d[3] = b.y;
}
__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ld1(const __half* p) { return __half2float(__ldg(p)); }
__device__ __forceinline__ void st1(float* p, float v) { *p = v; }
__device__ __forceinline__ void st1(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void st4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__half* p, const float* v) {
  __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t*>(&a);
  t.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = t;
}

template <int BM, int BN, int BK, int TM, int TN, bool VEC>
struct SgemmCfg {
  static constexpr int NTX = BN / TN;
  static constexpr int NTY = BM / TM;
  static constexpr int NT = NTX * NTY;
  static constexpr int A_VECS = BM * BK / 4;  // float4 slots of the A slab
  static constexpr int B_VECS = BK * BN / 4;
  static constexpr int A_PER = (A_VECS + NT - 1) / NT;
  static constexpr int B_PER = (B_VECS + NT - 1) / NT;
  static constexpr int APAD = BM + 4;
  static_assert(TM % 4 == 0 && TN % 4 == 0, "micro-tile must be 4-aligned");
  static_assert(BK % 4 == 0, "BK must be a multiple of 4");
};

// One tile's main loop: acc += A[m0 : m0 + BM, kbeg : kend) * B[kbeg : kend, n0 : n0 + BN)
// by the NT threads (tid) that share As / Bs; `sync` is their barrier (the
// whole CTA, or one warp group of a CTA that splits K over its groups).
template <int BM, int BN, int BK, int TM, int TN, bool VEC, typename T, class Sync>
__device__ __forceinline__ void sgemm_mainloop(const T* __restrict__ A, const T* __restrict__ B, int M, int N,
                                               int64_t lda, int64_t ldb, int m0, int n0, int kbeg, int kend, int tid,
                                               float (*As)[BK][SgemmCfg<BM, BN, BK, TM, TN, VEC>::APAD],
                                               float (*Bs)[BK][BN], float (&acc)[TM][TN], Sync sync) {
  using Cfg = SgemmCfg<BM, BN, BK, TM, TN, VEC>;
  constexpr int NT = Cfg::NT, NTX = Cfg::NTX, NTY = Cfg::NTY;
  const int tx = tid % NTX, ty = tid / NTX;
  float ra[Cfg::A_PER][4], rb[Cfg::B_PER][4];

  // global -> registers for the slab starting at k0 (zero outside the matrix)
  auto load_slab = [&](int k0) {
#pragma unroll
    for (int p = 0; p < Cfg::A_PER; ++p) {
      const int i = tid + p * NT;
      if (i < Cfg::A_VECS) {
        const int m = i / (BK / 4), kq = (i % (BK / 4)) * 4;
        const int gm = m0 + m, gk = k0 + kq;
        if (VEC) {
          if (gm < M && gk < kend) {
            ld4(ra[p], A + (size_t)gm * lda + gk);
          } else {
            ra[p][0] = ra[p][1] = ra[p][2] = ra[p][3] = 0.f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ra[p][j] = (gm < M && gk + j < kend) ? ld1(A + (size_t)gm * lda + gk + j) : 0.f;
        }
      }
    }
#pragma unroll
    for (int p = 0; p < Cfg::B_PER; ++p) {
      const int i = tid + p * NT;
      if (i < Cfg::B_VECS) {
        const int k = i / (BN / 4), nq = (i % (BN / 4)) * 4;
        const int gk = k0 + k, gn = n0 + nq;
        if (VEC) {
          if (gk < kend && gn < N) {
            ld4(rb[p], B + (size_t)gk * ldb + gn);
          } else {
            rb[p][0] = rb[p][1] = rb[p][2] = rb[p][3] = 0.f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            rb[p][j] = (gk < kend && gn + j < N) ? ld1(B + (size_t)gk * ldb + gn + j) : 0.f;
        }
      }
    }
  };
  auto store_slab = [&](int buf) {
#pragma unroll
    for (int p = 0; p < Cfg::A_PER; ++p) {
      const int i = tid + p * NT;
      if (i < Cfg::A_VECS) {
        const int m = i / (BK / 4), kq = (i % (BK / 4)) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) As[buf][kq + j][m] = ra[p][j];
      }
    }
#pragma unroll
    for (int p = 0; p < Cfg::B_PER; ++p) {
      const int i = tid + p * NT;
      if (i < Cfg::B_VECS) {
        const int k = i / (BN / 4), nq = (i % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][k][nq]) = make_float4(rb[p][0], rb[p][1], rb[p][2], rb[p][3]);
      }
    }
  };

#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const int nslab = (kend - kbeg + BK - 1) / BK;
  if (nslab > 0) {
    load_slab(kbeg);
    store_slab(0);
  }
  sync();
  for (int s = 0; s < nslab; ++s) {
    const int buf = s & 1;
    if (s + 1 < nslab) load_slab(kbeg + (s + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[TM], b[TN];
#pragma unroll
      for (int g = 0; g < TM / 4; ++g) {
        const float4 t = *reinterpret_cast<const float4*>(&As[buf][k][g * NTY * 4 + ty * 4]);
        a[g * 4 + 0] = t.x; a[g * 4 + 1] = t.y; a[g * 4 + 2] = t.z; a[g * 4 + 3] = t.w;
      }
#pragma unroll
      for (int g = 0; g < TN / 4; ++g) {
        const float4 t = *reinterpret_cast<const float4*>(&Bs[buf][k][g * NTX * 4 + tx * 4]);
        b[g * 4 + 0] = t.x; b[g * 4 + 1] = t.y; b[g * 4 + 2] = t.z; b[g * 4 + 3] = t.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (s + 1 < nslab) store_slab(buf ^ 1);
    sync();
  }
}

// the K range of part `part` of `parts` (each a whole number of BK slabs)
template <int BK>
__device__ __forceinline__ void k_range(int K, int part, int parts, int* kbeg, int* kend) {
  const int kc = ((K + parts - 1) / parts + BK - 1) / BK * BK;
  *kbeg = min(K, part * kc);
  *kend = min(K, *kbeg + kc);
}

template <int BM, int BN, int BK, int TM, int TN, bool VEC, typename T, int KS = 1>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    k_sgemm(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, int M, int N, int K,
            int64_t lda, int64_t ldb, int64_t ldc) {
  using Cfg = SgemmCfg<BM, BN, BK, TM, TN, VEC>;
  constexpr int NT = Cfg::NT, NTX = Cfg::NTX, NTY = Cfg::NTY;
  __shared__ __align__(16) float As[2][BK][Cfg::APAD];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % NTX, ty = tid / NTX;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  // this CTA's K range: all of K, or its share of a K-split cluster (grid z)
  int kbeg = 0, kend = K;
  if constexpr (KS > 1) k_range<BK>(K, (int)blockIdx.z, KS, &kbeg, &kend);

  float acc[TM][TN];
  sgemm_mainloop<BM, BN, BK, TM, TN, VEC, T>(A, B, M, N, lda, ldb, m0, n0, kbeg, kend, tid, As, Bs, acc,
                                              [] { __syncthreads(); });

  if constexpr (KS > 1) {
    // the partial tile into shared memory (the slab buffers are free after the
    // loop's last barrier), then this CTA's BM / KS rows summed over the
    // cluster in rank order
    static_assert(BM * BN <= 2 * BK * Cfg::APAD + 2 * BK * BN, "partial tile fits in the slab buffers");
    static_assert(BM % KS == 0 && BN % 4 == 0, "row slices of the partial tile");
    float* red = &As[0][0][0];
#pragma unroll
    for (int gi = 0; gi < TM / 4; ++gi)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int gj = 0; gj < TN / 4; ++gj) {
          const int lm = gi * NTY * 4 + ty * 4 + i, ln = gj * NTX * 4 + tx * 4;
          const float* v = &acc[gi * 4 + i][gj * 4];
          *reinterpret_cast<float4*>(red + lm * BN + ln) = make_float4(v[0], v[1], v[2], v[3]);
        }
    uk_cluster_sync();
    constexpr int ROWS = BM / KS;
    const int r0 = (int)blockIdx.z * ROWS;
    for (int idx = tid; idx < ROWS * BN / 4; idx += NT) {
      const int lm = r0 + idx / (BN / 4), ln = (idx % (BN / 4)) * 4;
      const uint32_t a = uk_smem_u32(red + lm * BN + ln);
      float4 part[KS];
#pragma unroll
      for (int r = 0; r < KS; ++r) part[r] = uk_ld_dsmem_f32x4(uk_mapa(a, (uint32_t)r));
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < KS; ++r) {
        v[0] += part[r].x;
        v[1] += part[r].y;
        v[2] += part[r].z;
        v[3] += part[r].w;
      }
      const int gm = m0 + lm, gn = n0 + ln;
      if (gm < M) {
        T* c = C + (size_t)gm * ldc + gn;
        if (VEC && gn + 3 < N) {
          st4(c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (gn + j < N) st1(c + j, v[j]);
        }
      }
    }
    uk_cluster_sync();  // no CTA leaves while a peer still reads its partial tile
    return;
  }

#pragma unroll
  for (int gi = 0; gi < TM / 4; ++gi)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gm = m0 + gi * NTY * 4 + ty * 4 + i;
      if (gm >= M) continue;
#pragma unroll
      for (int gj = 0; gj < TN / 4; ++gj) {
        const int gn = n0 + gj * NTX * 4 + tx * 4;
        T* c = C + (size_t)gm * ldc + gn;
        const float* v = &acc[gi * 4 + i][gj * 4];
        if (VEC && gn + 3 < N) {
          st4(c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (gn + j < N) st1(c + j, v[j]);
        }
      }
    }
}

// The 32 x 64 tile with K split over KG warp groups of one CTA (128 threads
// each, named barrier g + 1 for group g): each group walks its K range through
// its own slab buffers, the partial tiles meet in the CTA's shared memory, and
// every element is summed over the groups in group order -- the arithmetic of
// the KS = KG cluster split (same K ranges, same fold order: the same bits)
// without the cluster barrier and the distributed-shared-memory reads.
constexpr int KG_BM = 32, KG_BN = 64, KG_BK = 16;
using KgCfg = SgemmCfg<KG_BM, KG_BN, KG_BK, 4, 4, true>;
constexpr int KG_GROUP_FLOATS = 2 * KG_BK * KgCfg::APAD + 2 * KG_BK * KG_BN;
static_assert(KG_BM * KG_BN <= KG_GROUP_FLOATS, "a group's partial tile fits in its slab buffers");
template <int KG>
constexpr size_t kg_smem_bytes() {
  return (size_t)KG * KG_GROUP_FLOATS * sizeof(float);
}

template <int KG, bool VEC, typename T>
__global__ void __launch_bounds__(128 * KG)
    k_sgemm_kg(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, int M, int N, int K,
               int64_t lda, int64_t ldb, int64_t ldc) {
  constexpr int BM = KG_BM, BN = KG_BN, BK = KG_BK, TM = 4, TN = 4;
  using Cfg = SgemmCfg<BM, BN, BK, TM, TN, VEC>;
  constexpr int NT = Cfg::NT, NTX = Cfg::NTX, NTY = Cfg::NTY;
  static_assert(NT == 128 && KG >= 2 && KG <= 8, "groups of 128 threads, named barriers 1..8");
  extern __shared__ __align__(16) float kg_smem[];
  const int g = (int)threadIdx.x / NT, tid = (int)threadIdx.x % NT;
  const int tx = tid % NTX, ty = tid / NTX;
  float* gs = kg_smem + g * KG_GROUP_FLOATS;
  auto As = reinterpret_cast<float (*)[BK][Cfg::APAD]>(gs);
  auto Bs = reinterpret_cast<float (*)[BK][BN]>(gs + 2 * BK * Cfg::APAD);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  int kbeg, kend;
  k_range<BK>(K, g, KG, &kbeg, &kend);

  float acc[TM][TN];
  sgemm_mainloop<BM, BN, BK, TM, TN, VEC, T>(A, B, M, N, lda, ldb, m0, n0, kbeg, kend, tid, As, Bs, acc, [g] {
    asm volatile("bar.sync %0, %1;" ::"r"(g + 1), "r"(NT) : "memory");
  });

  // the group's partial tile into its own slab buffers (its last barrier has
  // passed), then every element summed over the groups in group order
  float* red = gs;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int lm = ty * 4 + i, ln = tx * 4;
    *reinterpret_cast<float4*>(red + lm * BN + ln) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
  __syncthreads();
  for (int idx = (int)threadIdx.x; idx < BM * BN / 4; idx += NT * KG) {
    const int lm = idx / (BN / 4), ln = (idx % (BN / 4)) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < KG; ++r) {
      const float4 q = *reinterpret_cast<const float4*>(kg_smem + r * KG_GROUP_FLOATS + lm * BN + ln);
      v[0] += q.x;
      v[1] += q.y;
      v[2] += q.z;
      v[3] += q.w;
    }
    const int gm = m0 + lm, gn = n0 + ln;
    if (gm < M) {
      T* c = C + (size_t)gm * ldc + gn;
      if (VEC && gn + 3 < N) {
        st4(c, v);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gn + j < N) st1(c + j, v[j]);
      }
    }
  }
}

template <int BM, int BN, int BK, int TM, int TN, typename T>
void launch(const T* A, const T* B, T* C, int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, bool vec,
            cudaStream_t st) {
  constexpr int NT = (BM / TM) * (BN / TN);
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (vec) k_sgemm<BM, BN, BK, TM, TN, true, T><<<grid, NT, 0, st>>>(A, B, C, M, N, K, lda, ldb, ldc);
  else k_sgemm<BM, BN, BK, TM, TN, false, T><<<grid, NT, 0, st>>>(A, B, C, M, N, K, lda, ldb, ldc);
}

template <typename T>
__global__ void k_zero2d(T* C, int M, int N, int64_t ldc) {
  const int64_t n = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    st1(C + (i / N) * ldc + i % N, 0.f);
}

// a BM x BN tile (TM x TN per thread) with K split over a KS-CTA cluster
// (grid z): the 32 x 64 tile with 4 x 4 per thread, and the 64 x 64 tile with
// 8 x 8 per thread (twice the FFMAs per shared-memory load, 64 threads)
#ifndef UK_SGEMM_SPLIT_BK
#define UK_SGEMM_SPLIT_BK 16
#endif
template <int BM, int BN, int TM, int TN, int KS, typename T>
void launch_split(const T* A, const T* B, T* C, int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, bool vec,
                  cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), KS);
  cfg.blockDim = dim3((BM / TM) * (BN / TN), 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = KS;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  constexpr int BK = UK_SGEMM_SPLIT_BK;
  if (vec) cudaLaunchKernelEx(&cfg, k_sgemm<BM, BN, BK, TM, TN, true, T, KS>, A, B, C, M, N, K, lda, ldb, ldc);
  else cudaLaunchKernelEx(&cfg, k_sgemm<BM, BN, BK, TM, TN, false, T, KS>, A, B, C, M, N, K, lda, ldb, ldc);
}

// the 32 x 64 tile with K split over KG warp groups of one CTA
template <int KG, typename T>
int launch_groups(const T* A, const T* B, T* C, int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, bool vec,
                  cudaStream_t st) {
  static std::once_flag once[64];
  static int rc[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    std::call_once(once[dev], [&] {
      if (cudaFuncSetAttribute(k_sgemm_kg<KG, true, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kg_smem_bytes<KG>()) != cudaSuccess ||
          cudaFuncSetAttribute(k_sgemm_kg<KG, false, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kg_smem_bytes<KG>()) != cudaSuccess)
        rc[dev] = 1;
    });
    if (rc[dev]) return uk::check_launch("gemm: k-group kernel attributes");
  }
  const dim3 grid((unsigned)((N + KG_BN - 1) / KG_BN), (unsigned)((M + KG_BM - 1) / KG_BM));
  if (vec) k_sgemm_kg<KG, true, T><<<grid, 128 * KG, kg_smem_bytes<KG>(), st>>>(A, B, C, M, N, K, lda, ldb, ldc);
  else k_sgemm_kg<KG, false, T><<<grid, 128 * KG, kg_smem_bytes<KG>(), st>>>(A, B, C, M, N, K, lda, ldb, ldc);
  return UK_OK;
}

// A pinned FFMA plan from UK_SGEMM_PLAN="bm,bn,ks[,kg]" (a measurement knob,
// like the reference's UK_CONV_TILE): one of the compiled variants 128,128,1 /
// 64,64,1 / 32,64,{1,2,4,8} (K split over a cluster of ks CTAs) / 64,64,{4,8}
// (8 x 8 per thread, K split over a cluster) /
// 32,64,1,{2,4,8} (K split over kg warp groups of one CTA).  Returns 0 with
// *c set, 1 when unset, 2 when the value names no compiled variant (the call
// is then refused).
int pinned_plan(uk::Candidate* c) {
  const char* e = getenv("UK_SGEMM_PLAN");
  if (e == nullptr || e[0] == 0) return 1;
  int bm = 0, bn = 0, ks = 0, kg = 1;
  const int got = sscanf(e, "%d,%d,%d,%d", &bm, &bn, &ks, &kg);
  if (got != 3 && got != 4) return 2;
  if (kg > 1) {
    if (!(bm == 32 && bn == 64 && ks == 1 && (kg == 2 || kg == 4 || kg == 8))) return 2;
    *c = uk::Candidate{uk::kFamSgemmGroups, uk::Tile{32, 64, 16, 2}, kg, 0.0};
    return 0;
  }
  const bool ok = kg == 1 && ((bm == 128 && bn == 128 && ks == 1) ||
                              (bm == 64 && bn == 64 && (ks == 1 || ks == 4 || ks == 8)) ||
                              (bm == 32 && bn == 64 && (ks == 1 || ks == 2 || ks == 4 || ks == 8)));
  if (!ok) return 2;
  *c = uk::Candidate{uk::kFamSgemm, uk::Tile{bm, bn, (bm == 32 || ks > 1) ? 16 : 8, 2}, ks, 0.0};
  return 0;
}

// tile and K split: the solver's argmin over the FFMA candidates
// (uk::solve_gemm; 512^3 -> 32 x 64 tiles, K split over 4-CTA clusters)
template <typename T>
int simt_gemm(const T* A, const T* B, T* C, int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, bool vec,
              cudaStream_t st) {
  uk::Candidate c = uk::solve_gemm(M, N, K, /*f16*/ false, /*allow_tc*/ false, uk::sm_count());
  const int pin = pinned_plan(&c);
  if (pin == 2)
    return uk::fail(UK_EINVAL,
                    "gemm: UK_SGEMM_PLAN=%s names no compiled FFMA plan (128,128,1 64,64,{1,4,8} "
                    "32,64,{1,2,4,8} 32,64,1,{2,4,8})",
                    getenv("UK_SGEMM_PLAN"));
  if (pin == 0 && c.ksplit > 1 && K / c.ksplit < 16)
    return uk::fail(UK_EINVAL, "gemm: UK_SGEMM_PLAN k split %d leaves less than 16 of K=%d per CTA", c.ksplit, K);
  uk::note_launch(c);
  if (c.family == uk::kFamSgemmGroups) {
    if (c.ksplit == 8) return launch_groups<8>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
    if (c.ksplit == 4) return launch_groups<4>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
    return launch_groups<2>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  }
  if (c.tile.bm == 128) {
    launch<128, 128, 8, 8, 8>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.tile.bm == 64 && c.ksplit == 8) {
    launch_split<64, 64, 8, 8, 8>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.tile.bm == 64 && c.ksplit == 4) {
    launch_split<64, 64, 8, 8, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.tile.bm == 64) {
    launch<64, 64, 8, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.ksplit == 8) {
    launch_split<32, 64, 4, 4, 8>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.ksplit == 4) {
    launch_split<32, 64, 4, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else if (c.ksplit == 2) {
    launch_split<32, 64, 4, 4, 2>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  } else {
    launch<32, 64, 16, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, st);
  }
  return UK_OK;
}

}  // namespace

namespace uk {
// CUDA-core f16 GEMM (f16 in, fp32 FFMA accumulation, f16 out): the path for
// shapes the tensor-core kernel does not take.
int gemm_f16_simt(const __half* A, int64_t lda, const __half* B, int64_t ldb, __half* C, int64_t ldc, int M, int N,
                  int K, cudaStream_t st) {
  if (K == 0) {
    k_zero2d<__half><<<1024, 256, 0, st>>>(C, M, N, ldc);
    return check_launch("gemm_f16(zero)");
  }
  const bool vec = K % 4 == 0 && N % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 && ldc % 4 == 0 &&
                   ((uintptr_t)A & 7) == 0 && ((uintptr_t)B & 7) == 0 && ((uintptr_t)C & 7) == 0;
  if (int rc = simt_gemm<__half>(A, B, C, M, N, K, lda, ldb, ldc, vec, st)) return rc;
  return check_launch("gemm_f16(simt)");
}
}  // namespace uk

extern "C" int uk_cuda_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_f32: negative dims %d %d %d", M, N, K);
  if (M == 0 || N == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(C, "C")) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 0) {
    k_zero2d<float><<<1024, 256, 0, st>>>(C, M, N, N);
    return uk::check_launch("gemm_f32(zero)");
  }
  if (int rc = uk::check_device_ptr(A, "A")) return rc;
  if (int rc = uk::check_device_ptr(B, "B")) return rc;
  if ((M + 31) / 32 > 65535) return uk::fail(UK_EINVAL, "gemm_f32: M=%d exceeds the grid limit", M);
  const bool vec = K % 4 == 0 && N % 4 == 0 && uk::aligned16(A) && uk::aligned16(B) && uk::aligned16(C);
  if (int rc = simt_gemm<float>(A, B, C, M, N, K, K, N, N, vec, st)) return rc;
  return uk::check_launch("gemm_f32");
}
