// decode.cu -- the decode-layer chain's GEMM with the RMSNorm in front of it:
//
//   Y(f16)[b][n] = sum_k f16((X[b][k] * rms_b) * gamma[k]) * W[k][n],
//   rms_b = 1 / sqrt(sum_k X[b][k]^2 / K + eps),   fp32 accumulation,
//
// for a handful of token rows b < B <= 32 (decode) against a large f16
// weight W[K][N] (Llama-3-8B: 4096 x 14336, 112 MiB).  The op is bound by
// streaming W from HBM once; everything is arranged around that.
//
// Two kernels, overlapped by programmatic dependent launch:
// * k_rms_f16: one CTA per token row forms rms_b and writes the normalised
//   row as f16 into the caller's workspace Xn[B][K] (B*K*2 bytes).  It lets
//   the GEMM launch at once, so the GEMM's first weight loads are in flight
//   while the norm runs.
// * k_skinny_gemm: tensor cores on the transposed product
//   D[n][b] = W^T[n][k] * Xn^T[k][b]: a 128-column slice of W is the UMMA A
//   operand (M = 128, MN-major, loaded straight from row-major W by TMA),
//   the normalised tokens are the B operand (N = 32, K-major, rows >= B
//   zero-filled by TMA), the accumulator is 128 TMEM lanes x 32 columns.  One
//   thread streams W and Xn through an 8-stage ring (20 KiB per 64-deep k
//   block), one thread issues the MMAs, so each SM keeps ~160 KiB of W in
//   flight.  When N gives too few 128-column tiles to fill the GPU (a
//   weight-column shard on 8 GPUs: 14 tiles), K is split over a
//   thread-block cluster and the partial tiles are summed through
//   distributed shared memory in a fixed rank order (deterministic).  Any
//   cluster size up to 16 folds correctly (ragged k-block ranges and row
//   slices); a split that puts several CTAs on one SM gets a shallower ring
//   so the bytes in flight per SM stay about the same.  Splitting the full
//   Llama-3-8B width (112 tiles) over 4-, 5- or 6-CTA clusters, so that all
//   148 SMs stream, measured slower than the unsplit 112 CTAs (44.4 / 54.7 /
//   47.1 us against 40.8 us per chain), so the split is only taken when the
//   tiles alone leave most of the GPU idle.
//   The f16 result can be stored into up to 8 copies of Y (other GPUs'
//   buffers over NVLink): the weight-column sharding of the decode layer with
//   its all-gather fused into the store.
//
// Every mbarrier wait is bounded (2 s); a timeout records a bit in this
// file's fault word (read through uk_cuda_pipeline_fault) and every CTA still
// passes every cluster barrier, so no peer is left waiting.  TMA loads are
// plain single-CTA loads of this GPU's memory, each into its own CTA.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace uk {
__device__ unsigned int g_decode_fault = 0;
}  // namespace uk

namespace {

constexpr int TM = 128;        // W columns per tile (UMMA M)
constexpr int BP = 32;         // token rows, zero-padded (UMMA N)
constexpr int BK = 64;         // K per k-block (one 128-byte swizzle row of f16)
constexpr int CL_MAX = 16;     // CTAs per cluster (K split)
constexpr int THREADS = 128;   // 4 warps = the 4 TMEM lane quadrants
constexpr int MAX_OUT = 8;
constexpr int W_BOX = BK * 64 * 2;        // 8 KiB: 64 k rows x 64 W columns
constexpr int W_BLOCK = 2 * W_BOX;        // 16 KiB per k-block
constexpr int X_BLOCK = BP * BK * 2;      // 4 KiB per k-block
constexpr int STAGE_BYTES = W_BLOCK + X_BLOCK;
constexpr int RED_BYTES = TM * BP * 4;    // 16 KiB: this CTA's fp32 partial tile
constexpr uint32_t IDESC = uk_idesc_f16_ab(TM, BP, /*A MN-major*/ 1, /*B K-major*/ 0);
constexpr uint64_t WAIT_NS = 2000000000ull;

struct YList {
  uint16_t* y[MAX_OUT];  // y[0] on this GPU; y[1..] other GPUs' copies (same layout)
  int n;
};

template <int STAGES>
struct Ctl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int acc_ok;
};

template <int STAGES>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)STAGES * STAGE_BYTES + sizeof(Ctl<STAGES>);
}
static_assert(smem_bytes<8>() <= 232448, "shared memory per block on sm_100");
// the fp32 partial tile of a K-split cluster reuses the ring (all loads have
// landed once the last MMA completed)
static_assert(RED_BYTES <= 2 * STAGE_BYTES, "partial tile fits in the shallowest ring");

template <class CtlT>
__device__ __forceinline__ void fault(CtlT* ctl, unsigned bit) {
  atomicOr(&uk::g_decode_fault, bit);
  ctl->abort = 1;
}

// ---- 1. RMSNorm into f16 ------------------------------------------------------
// One CTA of 1024 threads per token row.  Rows up to 16384 columns stay in
// registers (at most four 16-byte vectors per thread): one read of X, a
// fixed-order block sum, the scaled f16 row out.  Longer rows take two passes.
constexpr int RMS_THREADS = 1024;
constexpr int RMS_VPT = 4;

__global__ void __launch_bounds__(RMS_THREADS) k_rms_f16(const float* __restrict__ X, const float* __restrict__ gamma,
                                                         float eps, __half* __restrict__ Xn, int K) {
  uk_pdl_launch_dependents();  // the GEMM may start streaming W now
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(X + (int64_t)b * K);
  const float4* gr = reinterpret_cast<const float4*>(gamma);
  uint2* out = reinterpret_cast<uint2*>(Xn + (int64_t)b * K);
  const int n4 = K / 4;
  float ss = 0.f;
  if (n4 <= RMS_VPT * RMS_THREADS) {
    float4 v[RMS_VPT];
#pragma unroll
    for (int u = 0; u < RMS_VPT; ++u) {
      const int k4 = threadIdx.x + u * RMS_THREADS;
      v[u] = k4 < n4 ? __ldg(xr + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    }
    ss = uk_block_sum<RMS_THREADS>(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
    for (int u = 0; u < RMS_VPT; ++u) {
      const int k4 = threadIdx.x + u * RMS_THREADS;
      if (k4 < n4) {
        const float4 g = __ldg(gr + k4);
        __half2 h0 = __floats2half2_rn((v[u].x * r) * g.x, (v[u].y * r) * g.y);
        __half2 h1 = __floats2half2_rn((v[u].z * r) * g.z, (v[u].w * r) * g.w);
        out[k4] = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
      }
    }
    return;
  }
  for (int k4 = threadIdx.x; k4 < n4; k4 += RMS_THREADS) {
    const float4 v = __ldg(xr + k4);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = uk_block_sum<RMS_THREADS>(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)K + eps);
  for (int k4 = threadIdx.x; k4 < n4; k4 += RMS_THREADS) {
    const float4 v = __ldg(xr + k4), g = __ldg(gr + k4);
    __half2 h0 = __floats2half2_rn((v.x * r) * g.x, (v.y * r) * g.y);
    __half2 h1 = __floats2half2_rn((v.z * r) * g.z, (v.w * r) * g.w);
    out[k4] = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
  }
}

// ---- 2. skinny GEMM -------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(THREADS)
    k_skinny_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, YList out,
                  int64_t ldy, int B, int N, int K, int64_t col_offset, int kb_per_cta) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* red = smem;
  Ctl<STAGES>* ctl = (Ctl<STAGES>*)(smem + (size_t)STAGES * STAGE_BYTES);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = uk_cluster_ctarank();
  const uint32_t csize = gridDim.x;  // the cluster spans grid x (K split)
  const int n0 = blockIdx.y * TM;
  const int kb_total = (K + BK - 1) / BK;
  const int kb0 = (int)crank * kb_per_cta;
  const int nkb = max(0, min(kb_per_cta, kb_total - kb0));

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      uk_mbar_init(&ctl->full[s], 1);
      uk_mbar_init(&ctl->empty[s], 1);
    }
    uk_mbar_init(&ctl->mma_done, 1);
    ctl->abort = 0;
    ctl->acc_ok = 0;
    uk_fence_mbar_init();
    uk_tma_prefetch_desc(&tmW);
    uk_tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    uk_tmem_alloc(&ctl->tmem_base, 32);
    uk_tmem_relinquish();
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (tid == 0) {
    // ---- producer: W does not depend on the norm kernel, Xn does ----
    const int pre = min(STAGES, nkb);
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + (size_t)i * STAGE_BYTES;
      uk_mbar_expect_tx(&ctl->full[i], STAGE_BYTES);
      uk_tma_load_2d(st, &tmW, &ctl->full[i], n0, (kb0 + i) * BK);
      uk_tma_load_2d(st + W_BOX, &tmW, &ctl->full[i], n0 + 64, (kb0 + i) * BK);
    }
    uk_pdl_wait();  // Xn is complete and visible from here on
    for (int i = 0; i < pre; ++i)
      uk_tma_load_2d(smem + (size_t)i * STAGE_BYTES + W_BLOCK, &tmX, &ctl->full[i], (kb0 + i) * BK, 0);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!uk_mbar_wait(&ctl->empty[s], ph ^ 1u, &ctl->abort, WAIT_NS)) {
        fault(ctl, UK_FAULT_PRODUCER);
        break;
      }
      uint8_t* st = smem + (size_t)s * STAGE_BYTES;
      uk_mbar_expect_tx(&ctl->full[s], STAGE_BYTES);
      uk_tma_load_2d(st, &tmW, &ctl->full[s], n0, (kb0 + i) * BK);
      uk_tma_load_2d(st + W_BOX, &tmW, &ctl->full[s], n0 + 64, (kb0 + i) * BK);
      uk_tma_load_2d(st + W_BLOCK, &tmX, &ctl->full[s], (kb0 + i) * BK, 0);
    }
  } else if (tid == 32) {
    // ---- MMA issuer ----
    bool ok = true;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!uk_mbar_wait(&ctl->full[s], ph, &ctl->abort, WAIT_NS)) {
        fault(ctl, UK_FAULT_MMA);
        ok = false;
        break;
      }
      uk_tc_fence_after();
      const uint32_t aw = uk_smem_u32(smem + (size_t)s * STAGE_BYTES);
      const uint32_t ax = aw + W_BLOCK;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        // W: MN-major, the two 64-column chunks 8 KiB apart (LBO), 8-row K
        // groups 1 KiB apart (SBO), +16 rows (2 KiB) per 16 K
        const uint64_t ad = uk_desc_sw128(aw + k * 2048, W_BOX, 1024);
        // Xn: K-major, +32 bytes per 16 K inside the swizzle atom
        const uint64_t bd = uk_desc_sw128(ax + k * 32, 16, 1024);
        uk_umma_f16(tmem, ad, bd, IDESC, (i > 0 || k > 0) ? 1u : 0u);
      }
      uk_umma_commit(&ctl->empty[s]);  // frees the stage when these MMAs finish
    }
    if (nkb > 0) {
      // arrives once every MMA issued above has finished (also after a
      // timeout, so TMEM is never released under an MMA in flight)
      uk_umma_commit(&ctl->mma_done);
      if (!uk_mbar_wait(&ctl->mma_done, 0, nullptr, WAIT_NS)) fault(ctl, UK_FAULT_TEARDOWN);
      else ctl->acc_ok = ok ? 1 : 0;
    }
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_tc_fence_after();

  // ---- epilogue: lane m of the accumulator is W column n0 + m ----
  const int m = warp * 32 + lane;
  uint32_t v[32];
  if (ctl->acc_ok) {
    uk_tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
    uk_tmem_ld_wait();
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0u;
  }
  if (csize == 1) {
    const int n = n0 + m;
    if (n < N) {
#pragma unroll
      for (int b = 0; b < BP; ++b) {
        if (b < B) {
          const uint16_t h = __half_as_ushort(__float2half_rn(__uint_as_float(v[b])));
          const int64_t off = (int64_t)b * ldy + col_offset + n;
          for (int o = 0; o < out.n; ++o) out.y[o][off] = h;
        }
      }
    }
  } else {
    // partial tile -> shared memory (16-byte chunk c of row m at
    // m * 128 + ((c ^ (m & 7)) * 16)), then this CTA's slice of rows is summed
    // over the cluster in rank order
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(red + m * 128 + ((c ^ (m & 7)) * 16)) =
          make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    uk_cluster_sync();
    const int per = (TM + (int)csize - 1) / (int)csize;
    const int m_lo = min(TM, (int)crank * per);
    const int rows = min(TM, m_lo + per) - m_lo;
    for (int idx = tid; idx < rows * 8; idx += THREADS) {
      const int mm = m_lo + idx % rows, c = idx / rows;
      const uint32_t a = uk_smem_u32(red + mm * 128 + ((c ^ (mm & 7)) * 16));
      float4 part[CL_MAX];
#pragma unroll
      for (int r = 0; r < CL_MAX; ++r)
        if (r < (int)csize) part[r] = uk_ld_dsmem_f32x4(uk_mapa(a, (uint32_t)r));
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < CL_MAX; ++r)
        if (r < (int)csize) {
          s.x += part[r].x;
          s.y += part[r].y;
          s.z += part[r].z;
          s.w += part[r].w;
        }
      const int n = n0 + mm;
      const float sv[4] = {s.x, s.y, s.z, s.w};
      if (n < N) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int b = c * 4 + j;
          if (b < B) {
            const uint16_t h = __half_as_ushort(__float2half_rn(sv[j]));
            const int64_t off = (int64_t)b * ldy + col_offset + n;
            for (int o = 0; o < out.n; ++o) out.y[o][off] = h;
          }
        }
      }
    }
    uk_cluster_sync();  // no CTA leaves while a peer still reads its shared memory
  }
  if (out.n > 1) __threadfence_system();

  uk_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    uk_tc_fence_after();
    uk_tmem_dealloc(tmem, 32);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

int make_map_f16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                 uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return uk::fail(UK_ECUDA, "decode_rmsnorm_gemm: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return uk::fail(UK_ECUDA, "decode_rmsnorm_gemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);
  return UK_OK;
}

using SkinnyFn = void (*)(CUtensorMap, CUtensorMap, YList, int64_t, int, int, int, int64_t, int);

// ---- the K split ------------------------------------------------------------
// A plan runs `tiles` clusters of cs CTAs; CTA r of a cluster streams k-blocks
// [r * ceil(kb/cs), ...).  Policy (measured): no split while the tiles alone
// give about 100 CTAs; otherwise the smallest power-of-two cs that does, each
// CTA keeping at least one k-block, halved while the GPU cannot co-schedule
// the cluster (its own occupancy answer).  per_sm = ceil(tiles * cs / SMs)
// CTAs share the busiest SM; the ring is 8 stages for one CTA per SM and
// shallower for more (4 for two, 3 for three, 2 for four or five), with the
// dynamic shared memory padded so that no SM takes more than per_sm.
// UK_DECODE_KSPLIT=<cs> pins any cluster size up to 16 (a measurement knob;
// refused when the cluster cannot be scheduled or needs more than five CTAs
// per SM).
struct SplitPlan {
  int cs = 1, per_sm = 1, stages = 8;
  size_t smem = 0;
  SkinnyFn kernel = nullptr;
};

constexpr int kMaxPerSm = 5;
constexpr int kMinCtas = 100;

int stages_for(int per_sm) { return per_sm <= 1 ? 8 : per_sm == 2 ? 4 : per_sm == 3 ? 3 : 2; }

SkinnyFn kernel_for(int stages) {
  switch (stages) {
    case 8: return k_skinny_gemm<8>;
    case 4: return k_skinny_gemm<4>;
    case 3: return k_skinny_gemm<3>;
    default: return k_skinny_gemm<2>;
  }
}

size_t ring_smem(int stages) {
  switch (stages) {
    case 8: return smem_bytes<8>();
    case 4: return smem_bytes<4>();
    case 3: return smem_bytes<3>();
    default: return smem_bytes<2>();
  }
}

void launch_config(const SplitPlan& plan, int tiles, cudaStream_t st, cudaLaunchConfig_t* cfg,
                   cudaLaunchAttribute* attr) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)plan.cs, (unsigned)tiles, 1);
  cfg->blockDim = dim3(THREADS, 1, 1);
  cfg->dynamicSmemBytes = plan.smem;
  cfg->stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)plan.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg->attrs = attr;
  cfg->numAttrs = 2;
}

// shared memory that fits at most per_sm CTAs on one SM (at least the ring)
size_t padded_smem(int stages, int per_sm, int sm_smem, int reserved) {
  const size_t ring = ring_smem(stages);
  if (per_sm >= kMaxPerSm) return ring;
  // one CTA more than per_sm must not fit: (per_sm + 1) * (smem + reserved) > sm_smem
  const size_t cap = (size_t)sm_smem / (size_t)(per_sm + 1) - (size_t)reserved + 1024;
  return std::max(ring, std::min(cap, (size_t)232448));
}

// the plan for cluster size cs, or false when the GPU cannot co-schedule it
bool make_plan(int dev, int cs, int tiles, int nsm, int sm_smem, int reserved, SplitPlan* c) {
  c->cs = cs;
  c->per_sm = (int)(((long)tiles * cs + nsm - 1) / nsm);
  if (c->per_sm > kMaxPerSm) return false;
  c->stages = stages_for(c->per_sm);
  c->kernel = kernel_for(c->stages);
  c->smem = padded_smem(c->stages, c->per_sm, sm_smem, reserved);
  if (cs == 1) return true;
  // the answer per (device, cluster size, per_sm) is asked once: 1 yes, -1 no
  static signed char fits[64][CL_MAX + 1][kMaxPerSm + 1] = {};
  signed char* slot = (dev >= 0 && dev < 64) ? &fits[dev][cs][c->per_sm] : nullptr;
  if (slot && *slot != 0) return *slot > 0;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[2];
  launch_config(*c, tiles, nullptr, &cfg, attr);
  int active = 0;
  const bool ok = cudaOccupancyMaxActiveClusters(&active, c->kernel, &cfg) == cudaSuccess && active > 0;
  cudaGetLastError();
  if (slot) *slot = ok ? 1 : -1;
  return ok;
}

int plan_split(int dev, int tiles, int kb_total, SplitPlan* out) {
  int nsm = 0, sm_smem = 0, reserved = 0;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
    return uk::check_launch("decode_rmsnorm_gemm: device attributes");
  static std::once_flag attr_once[64];
  static int attr_rc[64] = {};
  if (dev >= 0 && dev < 64) {
    std::call_once(attr_once[dev], [&] {
      for (int stg : {8, 4, 3, 2}) {
        const SkinnyFn f = kernel_for(stg);
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024) != cudaSuccess ||
            cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
          attr_rc[dev] = 1;
      }
    });
    if (attr_rc[dev]) return uk::check_launch("decode_rmsnorm_gemm: function attributes");
  }
  if (const char* e = getenv("UK_DECODE_KSPLIT")) {
    const int pin = atoi(e);
    if (pin < 1 || pin > CL_MAX || !make_plan(dev, pin, tiles, nsm, sm_smem, reserved, out))
      return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: UK_DECODE_KSPLIT=%s cannot be scheduled (1..%d, at most %d "
                      "CTAs per SM)", e, CL_MAX, kMaxPerSm);
    return UK_OK;
  }
  int cs = 1;
  while (tiles * cs < kMinCtas && cs < CL_MAX && kb_total >= 2 * cs) cs *= 2;
  for (; cs > 1; cs /= 2)
    if (make_plan(dev, cs, tiles, nsm, sm_smem, reserved, out)) return UK_OK;
  make_plan(dev, 1, tiles, nsm, sm_smem, reserved, out);
  return UK_OK;
}

}  // namespace

namespace uk {

// fault bits of the decode kernels since the last call (clears them)
unsigned decode_fault_take() {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_fault, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned zero = 0;
  cudaMemcpyToSymbol(g_decode_fault, &zero, sizeof(zero));
  return v;
}

}  // namespace uk

extern "C" size_t uk_cuda_decode_workspace_size(int B, int K) {
  if (B < 1 || K < 1) return 0;
  return ((size_t)B * (size_t)K * 2 + 255) / 256 * 256;
}

extern "C" int uk_cuda_decode_rmsnorm_gemm_f16(const float* X, const float* gamma, float eps, const uint16_t* W,
                                               int64_t ldw, uint16_t* const* Y_list, int n_y, int64_t ldy, int B,
                                               int N_shard, int K, int64_t col_offset, void* workspace,
                                               size_t workspace_bytes, void* stream) {
  if (B < 1 || B > BP) return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: B=%d token rows (1..%d)", B, BP);
  if (K <= 0 || K % 8 != 0) return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: K=%d must be a positive multiple of 8", K);
  if (N_shard < 0 || ldw < N_shard || ldw % 8 != 0)
    return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: N_shard=%d, ldw=%lld (ldw >= N_shard, multiple of 8)", N_shard,
                    (long long)ldw);
  if (col_offset < 0 || col_offset + N_shard > ldy)
    return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: columns [%lld, %lld) outside ldy=%lld", (long long)col_offset,
                    (long long)(col_offset + N_shard), (long long)ldy);
  if (!(eps >= 0.f)) return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: eps must be >= 0");
  if (Y_list == nullptr || n_y < 1 || n_y > MAX_OUT)
    return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: 1..%d outputs, got %d", MAX_OUT, n_y);
  const size_t need = uk_cuda_decode_workspace_size(B, K);
  if (workspace == nullptr || workspace_bytes < need)
    return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: needs a %zu-byte workspace (uk_cuda_decode_workspace_size)",
                    need);
  if (N_shard == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(gamma, "gamma")) return rc;
  if (int rc = uk::check_device_ptr(W, "W")) return rc;
  if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
  if (int rc = uk::check_device_ptr(Y_list[0], "Y_list[0]")) return rc;
  if (!uk::aligned16(X) || !uk::aligned16(gamma) || !uk::aligned16(W) || !uk::aligned16(workspace))
    return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: X, gamma, W and the workspace must be 16-byte aligned");
  YList out{};
  for (int i = 0; i < n_y; ++i) {
    if (Y_list[i] == nullptr) return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: Y_list[%d] is NULL", i);
    if (i > 0) {
      cudaPointerAttributes a{};
      if (cudaPointerGetAttributes(&a, Y_list[i]) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return uk::fail(UK_ERESIDENCY, "decode_rmsnorm_gemm: Y_list[%d] is not device memory", i);
      }
    }
    out.y[i] = Y_list[i];
  }
  out.n = n_y;

  const int kb_total = (K + BK - 1) / BK;
  const int tiles = (N_shard + TM - 1) / TM;
  if (tiles > 65535) return uk::fail(UK_EINVAL, "decode_rmsnorm_gemm: N_shard too large");

  CUtensorMap tmW, tmX;
  if (int rc = make_map_f16(&tmW, W, (uint64_t)N_shard, (uint64_t)K, (uint64_t)ldw, 64, BK)) return rc;
  if (int rc = make_map_f16(&tmX, workspace, (uint64_t)K, (uint64_t)B, (uint64_t)K, BK, BP)) return rc;

  int dev = 0;
  cudaGetDevice(&dev);
  SplitPlan plan;
  if (int rc = plan_split(dev, tiles, kb_total, &plan)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  launch_config(plan, tiles, st, &cfg, attr);
  const int kb_per_cta = (kb_total + plan.cs - 1) / plan.cs;
  {
    uk::Candidate c;  // the skinny decode GEMM (tile = W columns x token rows x k-block)
    c.family = uk::kFamSkinny;
    c.tile = uk::Tile{TM, BP, BK, plan.stages};
    c.ksplit = plan.cs;
    c.us = 0.0;
    uk::note_launch(c);
  }

  k_rms_f16<<<B, RMS_THREADS, 0, st>>>(X, gamma, eps, (__half*)workspace, K);
  if (int rc = uk::check_launch("decode_rmsnorm_gemm(norm)")) return rc;

  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, plan.kernel, tmW, tmX, out, ldy, B, N_shard, K, col_offset, kb_per_cta);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "decode_rmsnorm_gemm: launch: %s", cudaGetErrorString(e));
  return uk::check_launch("decode_rmsnorm_gemm");
}
