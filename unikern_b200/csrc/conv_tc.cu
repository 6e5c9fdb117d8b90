// conv_tc.cu -- 2-D convolution (stride 1, zero padding, fused per-output-
// channel scale) as an implicit GEMM on the tcgen05 tensor cores, at fp32
// accuracy through split-tf32 operands ("3xTF32").
//
// GEMM view: rows = output pixels of one image (a 2 x 64 patch of (ho, wo)
// per tile, UMMA M = 128), columns = output channels (UMMA N = 256), inner
// dimension k = (kh, kw, c) in 32-channel steps.  The input lives in the
// workspace as NHWC, so for one filter tap (kh, kw) and 32 channels the A
// tile is a single 4-D TMA box [32 c][64 w][2 h][1 n] at (c0, wo0 + kw - pad,
// ho0 + kh - pad, n): each pixel's 32 channels are one 128-byte swizzled row
// (the K-major UMMA layout) and the zero padding is TMA's out-of-bounds fill
// (only the channel coordinate, always a multiple of 32, is innermost).  The
// weights are [Oc][kh][kw][c] in the workspace: the B tile is one 2-D box
// [32 k][256 oc].
//
// Accuracy: an fp32 value x is carried as hi = tf32(x) plus lo = tf32(x - hi)
// (the pre-pass stores both), and each k-step issues lo*hi + hi*lo + hi*hi
// into the fp32 accumulator (the lo*lo term is below fp32 resolution).  The
// result matches an fp32 FFMA convolution to a few ulps of the output scale:
// the fp32 gate (1e-4 relative to an fp64 reference) holds with margin.
//
// Structure (the f16 GEMM's): a persistent CTA per SM, 192 threads; warp 0
// issues the TMA loads into a 2-stage ring (96 KiB per stage: A hi/lo, B
// hi/lo), warp 1 owns 512 TMEM columns (two 256-column accumulators) and one
// thread issues the MMAs, warps 2-5 drain the accumulator of the previous tile
// (tcgen05.ld, scale, coalesced stores to NCHW) while the next tile's MMAs
// run.  Every mbarrier wait is bounded (2 s); a timeout sets this file's fault
// word (uk_cuda_pipeline_fault) and the CTA unwinds.  Plain single-CTA TMA
// loads of this GPU's memory only, each into its own CTA.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace uk {
__device__ unsigned int g_conv_fault = 0;
int conv2d_ffma(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh, int Kw, int Oc,
                int pad, const float* scale, int layout, cudaStream_t st);
}  // namespace uk

namespace {

constexpr int BH = 2, BW = 64, BM = BH * BW;  // output pixels per tile
constexpr int BN = 256;                        // output channels per tile
constexpr int BK = 32;                         // channels per k-step (128-byte rows)
constexpr int STAGES = 2;
constexpr int A_BYTES = BM * BK * 4;  // 16 KiB
constexpr int B_BYTES = BN * BK * 4;  // 32 KiB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = uk_idesc_tf32(BM, BN, 0, 0);
constexpr uint64_t WAIT_NS = 2000000000ull;

struct SmemCtl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + sizeof(SmemCtl);
static_assert(SMEM_BYTES <= 232448, "shared memory per block on sm_100");

constexpr int MAX_COPIES = 7;  // copies of Y beyond p.y (the fused all-gather over up to 8 GPUs)

struct ConvTc {
  void* y;            // float (fp32 conv) or __half (fp16 conv)
  const void* scale;  // same type as y
  // more copies of Y (other GPUs' buffers over NVLink, at the same offsets):
  // every output the pair kernel and the tail store goes to y and to these
  void* yc[MAX_COPIES];
  int nyc;
  int N, Ho, Wo, Oc, C, Kh, Kw, pad;
  int tiles_w, tiles_h, tiles_oc, num_tiles;
  // SM-pair kernel work items: tiles [0, num_full) whole, then each of the
  // remaining tiles (the last, partial round) as `splits` k-ranges whose fp32
  // partial tiles go to `part` and are summed by k_conv_tail
  int num_items, num_full, splits;
  float* part;
};

__device__ __forceinline__ void tile_coords(const ConvTc& p, int t, int& n, int& ho0, int& wo0, int& oc0) {
  const int oct = t % p.tiles_oc;
  t /= p.tiles_oc;
  const int wt = t % p.tiles_w;
  t /= p.tiles_w;
  const int ht = t % p.tiles_h;
  n = t / p.tiles_h;
  ho0 = ht * BH;
  wo0 = wt * BW;
  oc0 = oct * BN;
}

__device__ __forceinline__ void raise_fault(SmemCtl* ctl, unsigned bit) {
  atomicOr(&uk::g_conv_fault, bit);
  ctl->abort = 1;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_conv_tc(const __grid_constant__ CUtensorMap tmXh, const __grid_constant__ CUtensorMap tmXl,
              const __grid_constant__ CUtensorMap tmWh, const __grid_constant__ CUtensorMap tmWl, const ConvTc p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  SmemCtl* ctl = (SmemCtl*)(smem + (size_t)STAGES * STAGE_BYTES);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int csteps = p.C / BK;
  const int ksteps = p.Kh * p.Kw * csteps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      uk_mbar_init(&ctl->full[s], 1);
      uk_mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      uk_mbar_init(&ctl->tfull[b], 1);
      uk_mbar_init(&ctl->tempty[b], EPI_WARPS);
    }
    uk_mbar_init(&ctl->teardown, 1);
    ctl->abort = 0;
    uk_fence_mbar_init();
    uk_tma_prefetch_desc(&tmXh);
    uk_tma_prefetch_desc(&tmXl);
    uk_tma_prefetch_desc(&tmWh);
    uk_tma_prefetch_desc(&tmWl);
  }
  if (warp == 1) {
    uk_tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    uk_tmem_relinquish();
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort; t += gridDim.x) {
        int n, ho0, wo0, oc0;
        tile_coords(p, t, n, ho0, wo0, oc0);
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait(&ctl->empty[s], ph ^ 1u, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_PRODUCER);
            ok = false;
            break;
          }
          const int tap = ks / csteps, c0 = (ks - tap * csteps) * BK;
          const int kh = tap / p.Kw, kw = tap - kh * p.Kw;
          uint8_t* st = smem + (size_t)s * STAGE_BYTES;
          uk_mbar_expect_tx(&ctl->full[s], STAGE_BYTES);
          uk_tma_load_4d(st, &tmXh, &ctl->full[s], c0, wo0 + kw - p.pad, ho0 + kh - p.pad, n);
          uk_tma_load_4d(st + A_BYTES, &tmXl, &ctl->full[s], c0, wo0 + kw - p.pad, ho0 + kh - p.pad, n);
          const int kcol = tap * p.C + c0;
          uk_tma_load_2d(st + 2 * A_BYTES, &tmWh, &ctl->full[s], kcol, oc0);
          uk_tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tmWl, &ctl->full[s], kcol, oc0);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort; t += gridDim.x, ++tl) {
        const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
        if (!uk_mbar_wait(&ctl->tempty[buf], tph ^ 1u, abort, WAIT_NS)) {
          raise_fault(ctl, UK_FAULT_MMA);
          break;
        }
        uk_tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait(&ctl->full[s], ph, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_MMA);
            ok = false;
            break;
          }
          uk_tc_fence_after();
          const uint32_t ah = uk_smem_u32(smem + (size_t)s * STAGE_BYTES);
          const uint32_t al = ah + A_BYTES, bh = ah + 2 * A_BYTES, bl = bh + B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            // K-major, 128-byte swizzle: +32 bytes per 8 tf32 inside the atom,
            // 8-row groups 1 KiB apart
            const uint64_t dah = uk_desc_sw128(ah + kk * 32, 16, 1024);
            const uint64_t dal = uk_desc_sw128(al + kk * 32, 16, 1024);
            const uint64_t dbh = uk_desc_sw128(bh + kk * 32, 16, 1024);
            const uint64_t dbl = uk_desc_sw128(bl + kk * 32, 16, 1024);
            uk_umma_tf32(d, dal, dbh, IDESC, (ks > 0 || kk > 0) ? 1u : 0u);  // small terms first
            uk_umma_tf32(d, dah, dbl, IDESC, 1u);
            uk_umma_tf32(d, dah, dbh, IDESC, 1u);
          }
          uk_umma_commit(&ctl->empty[s]);
        }
        if (!ok) break;
        uk_umma_commit(&ctl->tfull[buf]);
      }
      uk_umma_commit(&ctl->teardown);
      if (!uk_mbar_wait(&ctl->teardown, 0, nullptr, WAIT_NS)) atomicOr(&uk::g_conv_fault, UK_FAULT_TEARDOWN);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2 .. 5) ----------------
    // lane = tile row m = pixel (m / 64, m % 64) of the 2 x 64 patch; the 32
    // lanes of a warp are 32 consecutive wo of one output row, so every
    // column (output channel) is one coalesced 128-byte store
    const int q = warp & 3;
    const int m = q * 32 + lane;
    uint32_t tl = 0;
    for (int t = blockIdx.x; t < p.num_tiles && !*abort; t += gridDim.x, ++tl) {
      int n, ho0, wo0, oc0;
      tile_coords(p, t, n, ho0, wo0, oc0);
      const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
      if (!uk_mbar_wait(&ctl->tfull[buf], tph, abort, WAIT_NS)) {
        raise_fault(ctl, UK_FAULT_EPILOGUE);
        break;
      }
      uk_tc_fence_after();
      const int ho = ho0 + m / BW, wo = wo0 + m % BW;
      const bool valid = ho < p.Ho && wo < p.Wo;
      float* ybase = (float*)p.y + (((int64_t)n * p.Oc + oc0) * p.Ho + ho) * p.Wo + wo;
      const int64_t ocs = (int64_t)p.Ho * p.Wo;
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j) {
        uint32_t v[32];
        uk_tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * BN + j * 32, v);
        uk_tmem_ld_wait();
        const int ocj = oc0 + j * 32;
        const float sc_lane =
            (p.scale != nullptr && ocj + lane < p.Oc) ? __ldg((const float*)p.scale + ocj + lane) : 1.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float sc = __shfl_sync(0xffffffffu, sc_lane, i);
          if (valid && ocj + i < p.Oc) ybase[(int64_t)(j * 32 + i) * ocs] = __uint_as_float(v[i]) * sc;
        }
      }
      uk_tc_fence_before();
      __syncwarp();
      if (lane == 0) uk_mbar_arrive(&ctl->tempty[buf]);
    }
  }

  uk_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    uk_tc_fence_after();
    uk_tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- the same convolution on SM pairs (tcgen05 cta_group::2) -------------------
// A pair of CTAs (a 2-CTA cluster) shares a 256-pixel x 256-channel tile: the
// leader holds output rows ho0, ho0+1 and the peer ho0+2, ho0+3 (a 2 x 64
// patch each, its A operand), and each holds 128 of the 256 channels of the
// weights (its half of the B operand).  The leader issues M = 256 MMAs over
// both CTAs' shared memory; each CTA's TMEM receives its 128 pixels.  Loads
// count on the leader's full barrier; the leader commits MMA completion to
// both CTAs' barriers; the epilogues arrive remotely on the leader's
// tile-empty barrier (the f16 GEMM's pair pipeline).
//
// One kernel, two operand formats (each k-step is one 128-byte row per pixel
// and per output channel):
//   PairF32  fp32 data as tf32 (hi, lo) tiles, 32 channels per k-step, three
//            kind::tf32 MMAs (lo*hi, hi*lo, hi*hi) per 8-deep slice; 64 KiB
//            per stage per SM, 3 stages; fp32 output
//   PairF16  fp16 data, 64 channels per k-step, one kind::f16 MMA per 16-deep
//            slice; 32 KiB per stage per SM, 6 stages; fp16 output (fp32
//            accumulation and scale, one rounding)
constexpr int P_BH = 4;                       // output rows per pair tile
constexpr int P_BNC = BN / 2;                 // channels of B per CTA
constexpr int P_TILE_BYTES = 128 * 128;       // 128 rows x 128 bytes (A, or this CTA's half of B)
constexpr uint16_t P_PAIR = 0x3;

struct PairF32 {
  using Out = float;
  static constexpr int BKE = 32, TILES = 2, STAGES = 3;
  static constexpr uint32_t IDESC = uk_idesc_tf32(2 * BM, BN, 0, 0);
};
struct PairF16 {
  using Out = __half;
  static constexpr int BKE = 64, TILES = 1, STAGES = 6;
  static constexpr uint32_t IDESC = uk_idesc_f16_ab(2 * BM, BN, 0, 0);
};

// fp32 accuracy over long K: the tensor cores' fp32 accumulator does not round
// to nearest, and its error grows with the number of MMAs summed into it.  The
// fp32 kernel therefore accumulates at most P_KC k-steps (1024 channels) in
// TMEM: the first chunk of a tile goes to the tile's accumulator, each later
// chunk to the other TMEM buffer, and the epilogue warps add it into the
// tile's accumulator with CUDA-core fp32 adds ("promotion") before the MMAs
// reuse that buffer.  A K of at most P_KC k-steps (1024 fp32 channels x
// taps) is one chunk and needs no promotion; the 3 x 3 x 256 convolution
// (72 k-steps) promotes twice per tile.
constexpr int P_KC = 32;

template <class Tr>
struct PairCtl {
  uint64_t full[Tr::STAGES];
  uint64_t empty[Tr::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t pfull;   // a later chunk's partial sum is in the other buffer (MMA -> epilogue)
  uint64_t pempty;  // it was added into the tile's accumulator (epilogue -> MMA)
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};

template <class Tr>
constexpr int pair_stage_bytes() {
  return 2 * Tr::TILES * P_TILE_BYTES;  // A tiles then B tiles
}
// the epilogue transposes each 32-pixel x 32-channel chunk through a per-warp
// staging tile so that it stores 16-byte vectors of consecutive pixels
template <class Tr>
constexpr int pair_stg_bytes() {
  return EPI_WARPS * 32 * 32 * (int)sizeof(typename Tr::Out);
}
template <class Tr>
constexpr size_t pair_smem_bytes() {
  return 1024 + (size_t)Tr::STAGES * pair_stage_bytes<Tr>() + pair_stg_bytes<Tr>() + sizeof(PairCtl<Tr>);
}
static_assert(pair_smem_bytes<PairF32>() <= 232448 && pair_smem_bytes<PairF16>() <= 232448,
              "shared memory per block on sm_100");

__device__ __forceinline__ void pair_tile_coords(const ConvTc& p, int t, int& n, int& ho0, int& wo0, int& oc0) {
  const int oct = t % p.tiles_oc;
  t /= p.tiles_oc;
  const int wt = t % p.tiles_w;
  t /= p.tiles_w;
  const int ht = t % p.tiles_h;  // tiles_h counts 4-row pair tiles here
  n = t / p.tiles_h;
  ho0 = ht * P_BH;
  wo0 = wt * BW;
  oc0 = oct * BN;
}

// work item -> tile t and k-steps [k0, k0 + kn); j = the split item's index
// among all split items, -1 for a whole tile
__device__ __forceinline__ void pair_item(const ConvTc& p, int item, int ksteps, int& t, int& k0, int& kn, int& j) {
  if (item < p.num_full) {
    t = item;
    k0 = 0;
    kn = ksteps;
    j = -1;
    return;
  }
  j = item - p.num_full;
  t = p.num_full + j / p.splits;
  const int sidx = j - (j / p.splits) * p.splits;
  k0 = (int)((int64_t)sidx * ksteps / p.splits);
  kn = (int)((int64_t)(sidx + 1) * ksteps / p.splits) - k0;
}

__device__ __forceinline__ float out_scale(const float* s, int i) { return __ldg(s + i); }
__device__ __forceinline__ float out_scale(const __half* s, int i) { return __half2float(__ldg(s + i)); }
__device__ __forceinline__ void out_store(float* y, float v) { *y = v; }
__device__ __forceinline__ void out_store(__half* y, float v) { *y = __float2half_rn(v); }

// tmX0/tmW0: the input / weights (fp32 hi, or fp16); tmX1/tmW1: the lo tiles
// (fp32 only).  p.y / p.scale are of the traits' output type.
template <class Tr>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_conv_pair(const __grid_constant__ CUtensorMap tmX0, const __grid_constant__ CUtensorMap tmX1,
                const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1, const ConvTc p) {
  using Out = typename Tr::Out;
  constexpr int STAGES = Tr::STAGES, STAGE_BYTES = pair_stage_bytes<Tr>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stg_base = smem + (size_t)STAGES * STAGE_BYTES;
  PairCtl<Tr>* ctl = (PairCtl<Tr>*)(stg_base + pair_stg_bytes<Tr>());
  volatile int* abort = &ctl->abort;
  Out* Y = (Out*)p.y;
  const Out* scale = (const Out*)p.scale;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = uk_cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int csteps = p.C / Tr::BKE;
  const int ksteps = p.Kh * p.Kw * csteps;
  const int kc = Tr::TILES == 2 ? P_KC : ksteps;  // k-steps per TMEM chunk

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      uk_mbar_init(&ctl->full[s], 1);
      uk_mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      uk_mbar_init(&ctl->tfull[b], 1);
      uk_mbar_init(&ctl->tempty[b], 2 * EPI_WARPS);
    }
    uk_mbar_init(&ctl->pfull, 1);
    uk_mbar_init(&ctl->pempty, 2 * EPI_WARPS);
    uk_mbar_init(&ctl->teardown, 1);
    ctl->abort = 0;
    uk_fence_mbar_init();
    uk_tma_prefetch_desc(&tmX0);
    uk_tma_prefetch_desc(&tmW0);
    if (Tr::TILES == 2) {
      uk_tma_prefetch_desc(&tmX1);
      uk_tma_prefetch_desc(&tmW1);
    }
  }
  if (warp == 1) {
    uk_tmem_alloc_cg2(&ctl->tmem_base, TMEM_COLS);
    uk_tmem_relinquish_cg2();
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_cluster_sync();
  uk_tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int item = pair; item < p.num_items && !*abort; item += npairs) {
        int t, k0, kn, j;
        pair_item(p, item, ksteps, t, k0, kn, j);
        int n, ho0, wo0, oc0;
        pair_tile_coords(p, t, n, ho0, wo0, oc0);
        const int hr = ho0 + (int)crank * BH;  // this CTA's first output row
        // the pairs running side by side would all fetch the same weight (or,
        // for the GEMM, the same B^T) tile at the same moment; each tile walks
        // its k-steps from its own offset instead, a function of the tile's
        // position in the image and channel grid only (never of the image
        // index), so a result does not depend on which pair or which GPU of a
        // batch shard computes it
        const int rot =
            j >= 0 ? 0 : (int)(((int64_t)(ho0 / P_BH) * 7 + (int64_t)(wo0 / BW) * 3 + (int64_t)(oc0 / BN) * 5) % ksteps);
        bool ok = true;
        for (int ks = 0; ks < kn; ++ks, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait_cluster(&ctl->empty[s], ph ^ 1u, abort, WAIT_NS)) {
            atomicOr(&uk::g_conv_fault, UK_FAULT_PRODUCER);
            ctl->abort = 1;
            ok = false;
            break;
          }
          const int kq = k0 + (ks + rot < kn ? ks + rot : ks + rot - kn);
          const int tap = kq / csteps, c0 = (kq - tap * csteps) * Tr::BKE;
          const int kh = tap / p.Kw, kw = tap - kh * p.Kw;
          uint8_t* st = smem + (size_t)s * STAGE_BYTES;
          const uint32_t bar = uk_mapa(uk_smem_u32(&ctl->full[s]), 0);
          if (crank == 0) uk_mbar_expect_tx(&ctl->full[s], 2 * STAGE_BYTES);
          const int kcol = tap * p.C + c0;
          uk_tma_load_4d_cg2(st, &tmX0, bar, c0, wo0 + kw - p.pad, hr + kh - p.pad, n);
          uk_tma_load_2d_cg2(st + Tr::TILES * P_TILE_BYTES, &tmW0, bar, kcol, oc0 + (int)crank * P_BNC);
          if (Tr::TILES == 2) {
            uk_tma_load_4d_cg2(st + P_TILE_BYTES, &tmX1, bar, c0, wo0 + kw - p.pad, hr + kh - p.pad, n);
            uk_tma_load_2d_cg2(st + 3 * P_TILE_BYTES, &tmW1, bar, kcol, oc0 + (int)crank * P_BNC);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (crank == 0 && lane == 0) {
      uint32_t it = 0, tl = 0, np = 0;  // np: chunks handed to the epilogue for promotion
      for (int item = pair; item < p.num_items && !*abort; item += npairs, ++tl) {
        int t, k0, kn, j;
        pair_item(p, item, ksteps, t, k0, kn, j);
        const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
        // the tile's accumulator: drained two tiles ago, and no longer read
        // by the previous tile's last promotion
        if (!uk_mbar_wait_cluster(&ctl->tempty[buf], tph ^ 1u, abort, WAIT_NS) ||
            (np > 0 && !uk_mbar_wait_cluster(&ctl->pempty, (np - 1) & 1u, abort, WAIT_NS))) {
          atomicOr(&uk::g_conv_fault, UK_FAULT_MMA);
          ctl->abort = 1;
          break;
        }
        uk_tc_fence_after();
        bool ok = true;
        for (int ks = 0; ks < kn; ++ks, ++it) {
          const int c = ks / kc, kin = ks - c * kc;
          if (c >= 1 && kin == 0) {
            // a later chunk goes to the other buffer: the previous tile's
            // accumulator until drained (chunk 1), then the previous chunk's
            // partial until promoted
            const bool w = c == 1 ? uk_mbar_wait_cluster(&ctl->tempty[buf ^ 1u], ((tl - 1u) >> 1) & 1u, abort, WAIT_NS)
                                  : uk_mbar_wait_cluster(&ctl->pempty, (np - 1) & 1u, abort, WAIT_NS);
            if (!w) {
              atomicOr(&uk::g_conv_fault, UK_FAULT_MMA);
              ctl->abort = 1;
              ok = false;
              break;
            }
            uk_tc_fence_after();
          }
          const uint32_t d = tmem + (c == 0 ? buf : (buf ^ 1u)) * BN;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait_cluster(&ctl->full[s], ph, abort, WAIT_NS)) {
            atomicOr(&uk::g_conv_fault, UK_FAULT_MMA);
            ctl->abort = 1;
            ok = false;
            break;
          }
          uk_tc_fence_after();
          const uint32_t a0 = uk_smem_u32(smem + (size_t)s * STAGE_BYTES);
          const uint32_t b0 = a0 + Tr::TILES * P_TILE_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // K-major, 128-byte swizzle: +32 bytes per MMA slice (8 tf32 or
            // 16 f16) inside the atom, 8-row groups 1 KiB apart
            const uint64_t da = uk_desc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t db = uk_desc_sw128(b0 + kk * 32, 16, 1024);
            const uint32_t acc = (kin > 0 || kk > 0) ? 1u : 0u;
            if constexpr (Tr::TILES == 2) {
              const uint64_t dal = uk_desc_sw128(a0 + P_TILE_BYTES + kk * 32, 16, 1024);
              const uint64_t dbl = uk_desc_sw128(b0 + P_TILE_BYTES + kk * 32, 16, 1024);
              uk_umma_tf32_cg2(d, dal, db, Tr::IDESC, acc);  // small terms first
              uk_umma_tf32_cg2(d, da, dbl, Tr::IDESC, 1u);
              uk_umma_tf32_cg2(d, da, db, Tr::IDESC, 1u);
            } else {
              uk_umma_f16_cg2(d, da, db, Tr::IDESC, acc);
            }
          }
          uk_umma_commit_cg2(&ctl->empty[s], P_PAIR);
          if (c >= 1 && (kin == kc - 1 || ks == kn - 1)) {
            uk_umma_commit_cg2(&ctl->pfull, P_PAIR);
            ++np;
          }
        }
        if (!ok) break;
        uk_umma_commit_cg2(&ctl->tfull[buf], P_PAIR);
      }
      uk_umma_commit_cg2(&ctl->teardown, P_PAIR);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const uint32_t tempty_leader[2] = {uk_mapa(uk_smem_u32(&ctl->tempty[0]), 0),
                                       uk_mapa(uk_smem_u32(&ctl->tempty[1]), 0)};
    const uint32_t pempty_leader = uk_mapa(uk_smem_u32(&ctl->pempty), 0);
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t tl = 0, pi = 0;  // pi: promotions done
    for (int item = pair; item < p.num_items && !*abort; item += npairs, ++tl) {
      int t, k0, kn, j;
      pair_item(p, item, ksteps, t, k0, kn, j);
      int n, ho0, wo0, oc0;
      pair_tile_coords(p, t, n, ho0, wo0, oc0);
      const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
      // promotions: each later chunk's partial sum, added in fp32 (round to
      // nearest) into the tile's accumulator
      bool ok = true;
      const int nch = (kn + kc - 1) / kc;
      for (int c = 1; c < nch; ++c, ++pi) {
        if (!uk_mbar_wait_cluster(&ctl->pfull, pi & 1u, abort, WAIT_NS)) {
          atomicOr(&uk::g_conv_fault, UK_FAULT_EPILOGUE);
          ctl->abort = 1;
          ok = false;
          break;
        }
        uk_tc_fence_after();
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          uint32_t x[32], a[32];
          uk_tmem_ld32(trow + (buf ^ 1u) * BN + j * 32, x);
          uk_tmem_ld32(trow + buf * BN + j * 32, a);
          uk_tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = __float_as_uint(__uint_as_float(a[i]) + __uint_as_float(x[i]));
          uk_tmem_st32(trow + buf * BN + j * 32, a);
        }
        uk_tmem_st_wait();
        uk_tc_fence_before();
        __syncwarp();
        if (lane == 0) uk_mbar_arrive_cluster(pempty_leader);
      }
      if (!ok) break;
      if (!uk_mbar_wait_cluster(&ctl->tfull[buf], tph, abort, WAIT_NS)) {
        atomicOr(&uk::g_conv_fault, UK_FAULT_EPILOGUE);
        ctl->abort = 1;
        break;
      }
      uk_tc_fence_after();
      // the warp's 32 pixels are one run of an output row: row ho_w,
      // columns wo_w .. wo_w + 31; lane m's accumulator row is pixel wo_w + lane
      const int ho_w = ho0 + (int)crank * BH + (q * 32) / BW, wo_w = wo0 + (q * 32) % BW;
      constexpr int VEC = 16 / (int)sizeof(Out);  // pixels per 16-byte store
      constexpr int LPR = 32 / VEC;                // lanes per channel row
      constexpr int RPR = 32 / LPR;                // channel rows per store round
      Out* stg = (Out*)(stg_base + (size_t)(warp - 2) * 32 * 32 * sizeof(Out));  // [32 ch][32 px]
      const bool vec_ok = p.Wo % VEC == 0 && ((uintptr_t)Y & 15) == 0;
      const int px = (lane % LPR) * VEC, wo = wo_w + px;
      if (j >= 0) {
        // a split item: its fp32 partial tile, [BN channels][128 pixels] per
        // CTA, for k_conv_tail to sum (no scale yet)
        float* pp = p.part + (size_t)(j * 2 + (int)crank) * BN * 128;
#pragma unroll 1
        for (int jc = 0; jc < BN / 32; ++jc) {
          uint32_t v[32];
          uk_tmem_ld32(trow + buf * BN + jc * 32, v);
          uk_tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) pp[(size_t)(jc * 32 + i) * 128 + m] = __uint_as_float(v[i]);
        }
      } else {
#pragma unroll 1
        for (int jc = 0; jc < BN / 32; ++jc) {
          uint32_t v[32];
          uk_tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * BN + jc * 32, v);
          uk_tmem_ld_wait();
          const int ocj = oc0 + jc * 32;
          const float sc_lane = (scale != nullptr && ocj + lane < p.Oc) ? out_scale(scale, ocj + lane) : 1.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float sc = __shfl_sync(0xffffffffu, sc_lane, i);
            out_store(stg + i * 32 + lane, __uint_as_float(v[i]) * sc);
          }
          __syncwarp();
#pragma unroll
          for (int r = 0; r < 32 / RPR; ++r) {
            const int oi = r * RPR + lane / LPR, oc = ocj + oi;
            if (oc < p.Oc && ho_w < p.Ho && wo < p.Wo) {
              const int64_t off = (((int64_t)n * p.Oc + oc) * p.Ho + ho_w) * p.Wo + wo;
              const Out* src = stg + oi * 32 + px;
              for (int o = 0; o <= p.nyc; ++o) {
                Out* dst = (o == 0 ? Y : (Out*)p.yc[o - 1]) + off;
                if (vec_ok && wo + VEC <= p.Wo) {
                  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
                } else {
#pragma unroll
                  for (int e = 0; e < VEC; ++e)
                    if (wo + e < p.Wo) dst[e] = src[e];
                }
              }
            }
          }
          __syncwarp();
        }
      }
      uk_tc_fence_before();
      __syncwarp();
      if (lane == 0) uk_mbar_arrive_cluster(tempty_leader[buf]);
    }
    // stores into other GPUs' copies are visible system-wide before the CTA
    // retires (the ranks are ordered after the kernel)
    if (p.nyc > 0) __threadfence_system();
  }

  if (warp == 1 && lane == 0) {
    if (!uk_mbar_wait_cluster(&ctl->teardown, 0, nullptr, WAIT_NS)) atomicOr(&uk::g_conv_fault, UK_FAULT_TEARDOWN);
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_cluster_sync();
  if (warp == 1) {
    uk_tc_fence_after();
    uk_tmem_dealloc_cg2(tmem, TMEM_COLS);
  }
}

// the split tiles of the last round: every output element of those tiles is
// the sum of its `splits` partials in split order (deterministic), scaled
// and stored; one thread per element, pixels fastest (coalesced reads of the
// partials and stores along each output row)
template <class Out>
__global__ void __launch_bounds__(256) k_conv_tail(const ConvTc p) {
  const int64_t total = (int64_t)(p.num_tiles - p.num_full) * 2 * BN * 128;
  Out* Y = (Out*)p.y;
  const Out* scale = (const Out*)p.scale;
  for (int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * 256) {
    const int m = (int)(idx % 128);
    int64_t r = idx / 128;
    const int ocl = (int)(r % BN);
    r /= BN;
    const int crank = (int)(r % 2), tt = (int)(r / 2);
    int n, ho0, wo0, oc0;
    pair_tile_coords(p, p.num_full + tt, n, ho0, wo0, oc0);
    const int ho = ho0 + crank * BH + m / BW, wo = wo0 + m % BW, oc = oc0 + ocl;
    if (ho >= p.Ho || wo >= p.Wo || oc >= p.Oc) continue;
    const float* src = p.part + ((size_t)((size_t)tt * p.splits * 2 + crank) * BN + ocl) * 128 + m;
    const size_t step = (size_t)2 * BN * 128;  // from one split's partial tile to the next
    // the loads are independent (only the adds are ordered): 8 in flight
    float v = 0.f;
    int sidx = 0;
    for (; sidx + 8 <= p.splits; sidx += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = __ldcs(src + (size_t)(sidx + u) * step);
#pragma unroll
      for (int u = 0; u < 8; ++u) v += t[u];
    }
    for (; sidx < p.splits; ++sidx) v += __ldcs(src + (size_t)sidx * step);
    const int64_t off = (((int64_t)n * p.Oc + oc) * p.Ho + ho) * p.Wo + wo;
    const float out = scale != nullptr ? v * out_scale(scale, oc) : v;
    for (int o = 0; o <= p.nyc; ++o) out_store((o == 0 ? Y : (Out*)p.yc[o - 1]) + off, out);
  }
  if (p.nyc > 0) __threadfence_system();
}

// ---- pre-pass: fp32 -> (hi, lo) tf32 pairs, NCHW -> NHWC ------------------------
__device__ __forceinline__ void split(float v, float& hi, float& lo) {
  hi = uk_tf32_rna(v);
  lo = uk_tf32_rna(v - hi);
}

// X[n][c][h][w] -> Xh/Xl[n][h][w][c] through a 32 x 32 shared-memory tile
__global__ void k_split_nchw_nhwc(const float* __restrict__ X, float* __restrict__ Xh, float* __restrict__ Xl, int C,
                                  int H, int W) {
  __shared__ float tile[32][33];
  const int tiles_w = (W + 31) / 32;
  const int64_t nh = blockIdx.x / tiles_w;
  const int w0 = (int)(blockIdx.x % tiles_w) * 32, c0 = blockIdx.y * 32;
  const int n = (int)(nh / H), h = (int)(nh % H);
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, w = w0 + threadIdx.x;
    tile[r][threadIdx.x] = (c < C && w < W) ? __ldcs(X + (((int64_t)n * C + c) * H + h) * W + w) : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int w = w0 + r, c = c0 + threadIdx.x;
    if (w < W && c < C) {
      float hi, lo;
      split(tile[threadIdx.x][r], hi, lo);
      const int64_t o = (((int64_t)n * H + h) * W + w) * C + c;
      Xh[o] = hi;
      Xl[o] = lo;
    }
  }
}

// One CTA per input row (n, h): the C x W plane of that row is staged in
// shared memory ([w][c], padded to C + 1 so the column-wise writes are
// conflict free), then written out as the contiguous NHWC row (W * C floats)
// with 16-byte stores, hi and lo.  Used when the plane fits in shared memory.
constexpr int ROW_THREADS = 512;

__global__ void __launch_bounds__(ROW_THREADS) k_split_row_nhwc(const float* __restrict__ X, float* __restrict__ Xh,
                                                                 float* __restrict__ Xl, int C, int H, int W) {
  extern __shared__ float plane[];  // [W][C + 1]
  const int64_t nh = blockIdx.x;
  const int n = (int)(nh / H), h = (int)(nh % H);
  const int cp = C + 1;
  const float* src = X + ((int64_t)n * C * H + h) * W;  // + c * H * W + w
  const int64_t cw = (int64_t)C * W;
  if (W % 4 == 0) {
    // 16-byte loads, eight per thread issued before any is consumed
    constexpr int UNR = 8;
    const int w4n = W / 4;
    const int64_t n4 = cw / 4;
    for (int64_t base = threadIdx.x; base < n4; base += (int64_t)ROW_THREADS * UNR) {
      float4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int64_t i = base + (int64_t)u * ROW_THREADS;
        if (i < n4) {
          const int c = (int)(i / w4n), w4 = (int)(i - (int64_t)c * w4n);
          v[u] = __ldcs(reinterpret_cast<const float4*>(src + (int64_t)c * H * W) + w4);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int64_t i = base + (int64_t)u * ROW_THREADS;
        if (i < n4) {
          const int c = (int)(i / w4n), w = 4 * (int)(i - (int64_t)c * w4n);
          plane[w * cp + c] = v[u].x;
          plane[(w + 1) * cp + c] = v[u].y;
          plane[(w + 2) * cp + c] = v[u].z;
          plane[(w + 3) * cp + c] = v[u].w;
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < cw; i += ROW_THREADS) {
      const int c = (int)(i / W), w = (int)(i - (int64_t)c * W);
      plane[w * cp + c] = __ldcs(src + (int64_t)c * H * W + w);
    }
  }
  __syncthreads();
  float4* dh = reinterpret_cast<float4*>(Xh + nh * cw);
  float4* dl = reinterpret_cast<float4*>(Xl + nh * cw);
  for (int64_t i = threadIdx.x; i < cw / 4; i += ROW_THREADS) {
    const int64_t e = i * 4;
    const int w = (int)(e / C), c = (int)(e - (int64_t)w * C);
    const float* p = plane + w * cp + c;
    float h0, h1, h2, h3, l0, l1, l2, l3;
    split(p[0], h0, l0);
    split(p[1], h1, l1);
    split(p[2], h2, l2);
    split(p[3], h3, l3);
    dh[i] = make_float4(h0, h1, h2, h3);
    dl[i] = make_float4(l0, l1, l2, l3);
  }
}

// X[n][c][hw] -> [n][hw][c] through a 64 (c) x 64 (hw) shared-memory tile held
// as fp32 (exact for halves): 16- (fp32) or 8-byte (f16) loads along hw by 16
// threads per row, stores of 4 consecutive channels along c.  F16: binary16
// in and out (O0); else fp32 in and tf32 (hi, lo) pairs out (O0, O1).  Needs
// HW % 4 == 0, C % 4 == 0, X aligned to its vector size.
template <bool F16>
__global__ void __launch_bounds__(256) k_tile_nhwc(const void* __restrict__ Xv, void* __restrict__ O0,
                                                   void* __restrict__ O1, int C, int64_t HW) {
  __shared__ float t[64][65];
  const int64_t hw0 = (int64_t)blockIdx.x * 64;
  const int c0 = blockIdx.y * 64;
  const int64_t n = blockIdx.z;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int c = ty + 16 * r;
    const int64_t hw = hw0 + 4 * tx;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (c0 + c < C && hw < HW) {
      const int64_t off = (n * C + c0 + c) * HW + hw;
      if constexpr (F16) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>((const __half*)Xv + off));
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
      } else {
        const float4 f = __ldcs(reinterpret_cast<const float4*>((const float*)Xv + off));
        v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) t[c][4 * tx + j] = v[j];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int hl = ty + 16 * r, c = 4 * tx;
    const int64_t hw = hw0 + hl;
    if (hw >= HW || c0 + c >= C) continue;
    const int64_t off = (n * HW + hw) * C + c0 + c;
    if constexpr (F16) {
      const __half2 a = __floats2half2_rn(t[c][hl], t[c + 1][hl]);
      const __half2 b = __floats2half2_rn(t[c + 2][hl], t[c + 3][hl]);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&a);
      u.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>((__half*)O0 + off) = u;
    } else {
      float4 h, l;
      split(t[c][hl], h.x, l.x);
      split(t[c + 1][hl], h.y, l.y);
      split(t[c + 2][hl], h.z, l.z);
      split(t[c + 3][hl], h.w, l.w);
      *reinterpret_cast<float4*>((float*)O0 + off) = h;
      *reinterpret_cast<float4*>((float*)O1 + off) = l;
    }
  }
}

// elementwise split (the KML input is already HWC)
__global__ void k_split_flat(const float* __restrict__ X, float* __restrict__ Xh, float* __restrict__ Xl, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float hi, lo;
    split(__ldcs(X + i), hi, lo);
    Xh[i] = hi;
    Xl[i] = lo;
  }
}

// weights -> [Oc][kh][kw][c] hi/lo (NCHW weights are [Oc][c][kh][kw])
__global__ void k_split_weights(const float* __restrict__ Wt, float* __restrict__ Wh, float* __restrict__ Wl, int Oc,
                                int C, int Kh, int Kw, int nchw) {
  const int64_t K = (int64_t)C * Kh * Kw, total = (int64_t)Oc * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t oc = i / K;
    const int k = (int)(i - oc * K);
    int64_t src = i;
    if (nchw) {
      const int tap = k / C, c = k - tap * C, kh = tap / Kw, kw = tap - kh * Kw;
      src = ((oc * C + c) * Kh + kh) * Kw + kw;
    }
    float hi, lo;
    split(__ldg(Wt + src), hi, lo);
    Wh[i] = hi;
    Wl[i] = lo;
  }
}

// NCHW weights [Oc][C][Kh][Kw] -> [Oc][kh][kw][c], one CTA per output channel:
// its C * taps weights staged in shared memory (as fp32, exact for halves) by
// contiguous loads, then written in the new order by contiguous stores.  F16:
// binary16 in and out (O0); else fp32 in, tf32 (hi, lo) pairs out (O0, O1).
// Needs C * taps * 4 <= kPermuteSmem.
constexpr int kPermuteSmem = 48 * 1024;
template <bool F16>
__global__ void __launch_bounds__(256) k_permute_w(const void* __restrict__ Wt, void* __restrict__ O0,
                                                   void* __restrict__ O1, int C, int taps) {
  extern __shared__ float wst[];
  const int K = C * taps;
  const int64_t base = (int64_t)blockIdx.x * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x)
    wst[i] = F16 ? __half2float(__ldg((const __half*)Wt + base + i)) : __ldg((const float*)Wt + base + i);
  __syncthreads();
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    const int tap = i / C, c = i - tap * C;
    const float v = wst[c * taps + tap];
    if constexpr (F16) {
      ((__half*)O0)[base + i] = __float2half_rn(v);  // exact: v came from a half
    } else {
      float hi, lo;
      split(v, hi, lo);
      ((float*)O0)[base + i] = hi;
      ((float*)O1)[base + i] = lo;
    }
  }
}

// B[K][N] -> Bt[N][K] as (hi, lo) pairs, 32 x 32 tiles through shared memory
// (K % 32 == 0 and N % 32 == 0: every tile is whole)
__global__ void __launch_bounds__(256) k_split_transpose(const float* __restrict__ B, float* __restrict__ Th,
                                                         float* __restrict__ Tl, int K, int N) {
  __shared__ float t[32][33];
  const int64_t n0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
#pragma unroll
  for (int i = threadIdx.y; i < 32; i += 8) t[i][threadIdx.x] = __ldcs(B + (k0 + i) * N + n0 + threadIdx.x);
  __syncthreads();
#pragma unroll
  for (int i = threadIdx.y; i < 32; i += 8) {
    float hi, lo;
    split(t[threadIdx.x][i], hi, lo);
    const int64_t o = (n0 + i) * K + k0 + threadIdx.x;
    Th[o] = hi;
    Tl[o] = lo;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  });
  return fn;
}

int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
           const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return uk::fail(UK_ECUDA, "conv2d: cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return uk::fail(UK_ECUDA, "conv2d: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return UK_OK;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// the SM-pair kernel unless UNIKERN_CONV_PAIR=0 (for comparisons)
bool use_pair_kernel() {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("UNIKERN_CONV_PAIR");
    env = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return env == 1;
}

bool tc_applies(int N, int H, int W, int C, int Kh, int Kw, int Oc, int pad, int layout) {
  (void)Oc;
  if (C < BK || C % BK != 0) return false;
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  if (Ho <= 0 || Wo <= 0 || N <= 0) return false;
  if (layout == UK_CONV_KML && (N != 1 || pad != 0)) return false;
  return true;
}

// Work items of the SM-pair kernels.  Tiles go round-robin over the pairs,
// so the last round is partial (448 conv tiles on 74 pairs: 6 full rounds and
// 4 tiles).  When there is room in the workspace, each tile of that last
// round is cut into `splits` k-ranges (at least 4 k-steps each) so that the
// idle pairs share it; k_conv_tail sums the fp32 partial tiles.
struct TailPlan {
  int pairs, num_items, num_full, splits;
  size_t bytes;
};

TailPlan tail_plan(int64_t tiles, int ksteps, size_t room) {
  TailPlan tp{};
  const int sm2 = uk::sm_count() / 2;
  const int r = (int)(tiles % sm2);  // tiles in the last round (all of them when tiles < sm2)
  int S = r > 0 ? sm2 / r : 1;
  if (S > ksteps / 4) S = ksteps / 4;
  const size_t bytes = S >= 2 ? (size_t)r * S * 2 * BN * 128 * sizeof(float) : 0;
  if (S < 2 || bytes > room) {
    tp.num_full = (int)tiles;
    tp.splits = 1;
    tp.num_items = (int)tiles;
  } else {
    tp.num_full = (int)(tiles - r);
    tp.splits = S;
    tp.num_items = tp.num_full + r * S;
    tp.bytes = bytes;
  }
  tp.pairs = tp.num_items < sm2 ? tp.num_items : sm2;
  return tp;
}

size_t tail_bytes(int64_t tiles, int ksteps) { return align256(tail_plan(tiles, ksteps, (size_t)-1).bytes); }

// pair tiles of a convolution (the SM-pair kernels' tiling)
int64_t pair_tiles(int N, int Ho, int Wo, int Oc) {
  return (int64_t)N * ((Ho + P_BH - 1) / P_BH) * ((Wo + BW - 1) / BW) * ((Oc + BN - 1) / BN);
}

// fill the work-item fields of p from the plan (launch the tail kernel after)
void apply_tail(ConvTc& p, const TailPlan& tp, float* part) {
  p.num_items = tp.num_items;
  p.num_full = tp.num_full;
  p.splits = tp.splits;
  p.part = tp.splits >= 2 ? part : nullptr;
}

// the split-tf32 kernel over prepared operands: Xh/Xl the input as NHWC
// (hi, lo) pairs, Wh/Wl the weights as [Oc][kh][kw][c] pairs
int run_tc(const float* Xh, const float* Xl, const float* Wh, const float* Wl, float* Y, const float* scale, int N,
           int H, int W, int C, int Kh, int Kw, int Oc, int pad, float* part, size_t part_room, cudaStream_t st,
           float* const* ycopies = nullptr, int nyc = 0) {
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  // tensor maps: input [N][H][W][C] as 4-D (C innermost), weights [Oc][K]
  CUtensorMap txh, txl, twh, twl;
  const cuuint64_t xdims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
  const cuuint64_t xstr[3] = {(cuuint64_t)C * 4, (cuuint64_t)W * C * 4, (cuuint64_t)H * W * C * 4};
  const cuuint32_t xbox[4] = {BK, BW, BH, 1};
  const int64_t K = (int64_t)Kh * Kw * C;
  const cuuint64_t wdims[2] = {(cuuint64_t)K, (cuuint64_t)Oc};
  const cuuint64_t wstr[1] = {(cuuint64_t)K * 4};
  const bool pair = use_pair_kernel();
  const cuuint32_t wbox[2] = {BK, (cuuint32_t)(pair ? P_BNC : BN)};
  if (int rc = encode(&txh, Xh, 4, xdims, xstr, xbox)) return rc;
  if (int rc = encode(&txl, Xl, 4, xdims, xstr, xbox)) return rc;
  if (int rc = encode(&twh, Wh, 2, wdims, wstr, wbox)) return rc;
  if (int rc = encode(&twl, Wl, 2, wdims, wstr, wbox)) return rc;

  ConvTc p{};
  p.y = Y;
  p.scale = scale;
  if (nyc < 0 || nyc > MAX_COPIES) return uk::fail(UK_EINVAL, "conv2d: %d extra copies of Y (0..%d)", nyc, MAX_COPIES);
  if (nyc > 0 && !pair) return uk::fail(UK_EINVAL, "conv2d: copies of Y need the SM-pair kernel");
  for (int i = 0; i < nyc; ++i) p.yc[i] = ycopies[i];
  p.nyc = nyc;
  p.N = N;
  p.Ho = Ho;
  p.Wo = Wo;
  p.Oc = Oc;
  p.C = C;
  p.Kh = Kh;
  p.Kw = Kw;
  p.pad = pad;
  p.tiles_w = (Wo + BW - 1) / BW;
  p.tiles_h = pair ? (Ho + P_BH - 1) / P_BH : (Ho + BH - 1) / BH;
  p.tiles_oc = (Oc + BN - 1) / BN;
  const int64_t tiles = (int64_t)N * p.tiles_h * p.tiles_w * p.tiles_oc;
  if (tiles > 2147483647LL) return uk::fail(UK_EINVAL, "conv2d: too many tiles");
  p.num_tiles = (int)tiles;
  const TailPlan tp = tail_plan(tiles, Kh * Kw * (C / BK), pair && part != nullptr ? part_room : 0);
  apply_tail(p, tp, part);

  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(k_conv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_conv_pair<PairF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)pair_smem_bytes<PairF32>()) != cudaSuccess)
      return uk::check_launch("conv2d: smem attribute");
    attr_done[dev] = true;
  }
  if (!pair) {
    const int grid = p.num_tiles < uk::sm_count() ? p.num_tiles : uk::sm_count();
    k_conv_tc<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(txh, txl, twh, twl, p);
    return uk::check_launch("conv2d(tcgen05)");
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * tp.pairs), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = pair_smem_bytes<PairF32>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_conv_pair<PairF32>, txh, txl, twh, twl, p);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "conv2d(pair): launch: %s", cudaGetErrorString(e));
  if (tp.splits >= 2) {
    const int64_t total = (int64_t)(p.num_tiles - p.num_full) * 2 * BN * 128;
    const int64_t g = std::min<int64_t>((total + 255) / 256, (int64_t)uk::sm_count() * 8);
    k_conv_tail<float><<<(unsigned)g, 256, 0, st>>>(p);
  }
  return uk::check_launch("conv2d(tcgen05 pair)");
}
}  // namespace

namespace uk {

unsigned conv_fault_take() {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_conv_fault, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned zero = 0;
  cudaMemcpyToSymbol(g_conv_fault, &zero, sizeof(zero));
  return v;
}

}  // namespace uk

extern "C" size_t uk_cuda_conv2d_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc, int pad,
                                                int layout) {
  if (!tc_applies(N, H, W, C, Kh, Kw, Oc, pad, layout)) return 0;
  const size_t xs = align256((size_t)N * H * W * C * 4), ws = align256((size_t)Oc * Kh * Kw * C * 4);
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  // + the last round's split partial tiles (SM-pair kernel)
  const size_t tail = use_pair_kernel() ? tail_bytes(pair_tiles(N, Ho, Wo, Oc), Kh * Kw * (C / BK)) : 0;
  return 2 * xs + 2 * ws + tail;
}

namespace {

// the tensor-core fp32 conv, its output stored into Y and the nyc copies
int conv2d_f32_tc(const float* X, const float* Wt, float* Y, float* const* ycopies, int nyc, int N, int H, int W,
                  int C, int Kh, int Kw, int Oc, int pad, const float* scale, int layout, void* workspace,
                  size_t workspace_bytes, void* stream) {
  const cudaStream_t st = (cudaStream_t)stream;
  if (layout != UK_CONV_KML && layout != UK_CONV_NCHW)
    return uk::fail(UK_EINVAL, "conv2d: unknown layout %d", layout);
  if (N < 0 || H <= 0 || W <= 0 || C <= 0 || Kh <= 0 || Kw <= 0 || Oc <= 0 || pad < 0)
    return uk::fail(UK_EINVAL, "conv2d: invalid dims N=%d H=%d W=%d C=%d Kh=%d Kw=%d Oc=%d pad=%d", N, H, W, C, Kh,
                    Kw, Oc, pad);
  if (!tc_applies(N, H, W, C, Kh, Kw, Oc, pad, layout)) {
    if (nyc > 0) return uk::fail(UK_EINVAL, "conv2d: copies of Y need the tensor-core path (C a multiple of 32)");
    return uk::conv2d_ffma(X, Wt, Y, N, H, W, C, Kh, Kw, Oc, pad, scale, layout, st);
  }
  // the operand pairs are required; the split partials of the last round
  // are used when the workspace has room for them (the size query includes it)
  const size_t need = 2 * align256((size_t)N * H * W * C * 4) + 2 * align256((size_t)Oc * Kh * Kw * C * 4);
  if (workspace == nullptr || workspace_bytes < need)
    return uk::fail(UK_EINVAL, "conv2d: needs a %zu-byte workspace (uk_cuda_conv2d_workspace_size), got %zu", need,
                    workspace ? workspace_bytes : (size_t)0);
  if ((int64_t)N * H * W * C > ((int64_t)1 << 40)) return uk::fail(UK_EINVAL, "conv2d: input too large");
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(Wt, "Wt")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
  if (scale)
    if (int rc = uk::check_device_ptr(scale, "scale")) return rc;
  if (!uk::aligned16(workspace)) return uk::fail(UK_EINVAL, "conv2d: the workspace must be 16-byte aligned");

  const size_t xs = align256((size_t)N * H * W * C * 4), wsz = align256((size_t)Oc * Kh * Kw * C * 4);
  float* Xh = (float*)workspace;
  float* Xl = (float*)((uint8_t*)workspace + xs);
  float* Wh = (float*)((uint8_t*)workspace + 2 * xs);
  float* Wl = (float*)((uint8_t*)workspace + 2 * xs + wsz);

  // pre-pass: operands as tf32 (hi, lo) pairs, input as NHWC
  if (N == 0) return UK_OK;
  const size_t plane_bytes = (size_t)W * (C + 1) * 4;
  const int64_t HW = (int64_t)H * W;
  if (layout == UK_CONV_NCHW && HW % 4 == 0 && uk::aligned16(X) && (HW + 63) / 64 <= 2147483647LL && N <= 65535) {
    // the tiled transpose: vector loads along hw, vector stores along c
    const dim3 g((unsigned)((HW + 63) / 64), (unsigned)((C + 63) / 64), (unsigned)N);
    k_tile_nhwc<false><<<g, 256, 0, st>>>(X, Xh, Xl, C, HW);
  } else if (layout == UK_CONV_NCHW && plane_bytes <= 100 * 1024 && (W % 4 != 0 || uk::aligned16(X))) {
    static bool plane_attr[64] = {false};
    int d = 0;
    cudaGetDevice(&d);
    if (d >= 0 && d < 64 && !plane_attr[d]) {
      if (cudaFuncSetAttribute(k_split_row_nhwc, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024) !=
          cudaSuccess)
        return uk::check_launch("conv2d: pre-pass attribute");
      plane_attr[d] = true;
    }
    if ((int64_t)N * H > 2147483647LL) return uk::fail(UK_EINVAL, "conv2d: N*H too large");
    k_split_row_nhwc<<<(unsigned)((int64_t)N * H), ROW_THREADS, plane_bytes, st>>>(X, Xh, Xl, C, H, W);
  } else if (layout == UK_CONV_NCHW) {
    const int64_t gx = (int64_t)((W + 31) / 32) * N * H;
    if (gx > 2147483647LL || C / 32 > 65535) return uk::fail(UK_EINVAL, "conv2d: input too large for the pre-pass");
    const dim3 g((unsigned)gx, (unsigned)(C / 32), 1);
    k_split_nchw_nhwc<<<g, dim3(32, 8), 0, st>>>(X, Xh, Xl, C, H, W);
  } else {
    const int64_t n = (int64_t)H * W * C;
    k_split_flat<<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)uk::sm_count() * 16), 256, 0, st>>>(X, Xh,
                                                                                                            Xl, n);
  }
  if (layout == UK_CONV_NCHW && (int64_t)C * Kh * Kw * 4 <= kPermuteSmem) {
    k_permute_w<false><<<(unsigned)Oc, 256, (size_t)C * Kh * Kw * 4, st>>>(Wt, Wh, Wl, C, Kh * Kw);
  } else {
    const int64_t n = (int64_t)Oc * Kh * Kw * C;
    k_split_weights<<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)uk::sm_count() * 8), 256, 0, st>>>(
        Wt, Wh, Wl, Oc, C, Kh, Kw, layout == UK_CONV_NCHW ? 1 : 0);
  }
  if (int rc = uk::check_launch("conv2d(split)")) return rc;

  return run_tc(Xh, Xl, Wh, Wl, Y, scale, N, H, W, C, Kh, Kw, Oc, pad, (float*)((uint8_t*)workspace + need),
                workspace_bytes - need, st, ycopies, nyc);
}

}  // namespace

extern "C" int uk_cuda_conv2d_f32_ws(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh,
                                     int Kw, int Oc, int pad, const float* scale, int layout, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  return conv2d_f32_tc(X, Wt, Y, nullptr, 0, N, H, W, C, Kh, Kw, Oc, pad, scale, layout, workspace, workspace_bytes,
                       stream);
}

extern "C" int uk_cuda_conv2d_f32_allgather(const float* X, const float* Wt, float* const* Y_list, int n_y, int N,
                                            int H, int W, int C, int Kh, int Kw, int Oc, int pad, const float* scale,
                                            void* workspace, size_t workspace_bytes, void* stream) {
  if (Y_list == nullptr || n_y < 1 || n_y > MAX_COPIES + 1)
    return uk::fail(UK_EINVAL, "conv2d_allgather: 1..%d copies of Y, got %d", MAX_COPIES + 1, n_y);
  for (int i = 1; i < n_y; ++i) {
    cudaPointerAttributes a{};
    if (Y_list[i] == nullptr || cudaPointerGetAttributes(&a, Y_list[i]) != cudaSuccess ||
        a.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return uk::fail(UK_ERESIDENCY, "conv2d_allgather: Y_list[%d] is not device memory", i);
    }
  }
  return conv2d_f32_tc(X, Wt, Y_list[0], Y_list + 1, n_y - 1, N, H, W, C, Kh, Kw, Oc, pad, scale, UK_CONV_NCHW,
                       workspace, workspace_bytes, stream);
}

// ---- the fp32 GEMM as a 1 x 1 convolution -------------------------------------------
// C[M][N] = A[M][K] * B[K][N] is the 1 x 1 convolution of one (N/64) x 64
// image of K channels, X[h][w][c] = B[c][64h + w] (B transposed), with M
// filters Wt[m][c] = A[m][c]: output channel m at pixel n = 64h + w is
// C[m][n], and the output planes Y[m][h][w] are C row-major.  So the
// split-tf32 convolution kernels above run it unchanged, at fp32 accuracy on
// the tensor cores; the pre-passes write B^T and A as tf32 (hi, lo) pairs.
namespace uk {

bool gemm_f32_tc_shape(int M, int N, int K) { return M > 0 && N >= 64 && N % 64 == 0 && K >= BK && K % BK == 0; }

size_t gemm_f32_tc_b_bytes(int N, int K) { return 2 * align256((size_t)N * K * 4); }
size_t gemm_f32_tc_a_bytes(int M, int K) { return 2 * align256((size_t)M * K * 4); }
// the last round's split partial tiles of the GEMM's convolution
size_t gemm_f32_tc_tail_bytes(int M, int N, int K) {
  return use_pair_kernel() ? tail_bytes(pair_tiles(1, N / 64, 64, M), K / BK) : 0;
}

// B (device, K x N) -> the (hi, lo) pairs of B^T in bws (gemm_f32_tc_b_bytes)
int gemm_f32_tc_prep_b(const float* B, void* bws, int N, int K, cudaStream_t st) {
  if ((int64_t)K / 32 > 65535) return uk::fail(UK_EINVAL, "gemm_f32: K=%d too large for the transpose pre-pass", K);
  float* Th = (float*)bws;
  float* Tl = (float*)((uint8_t*)bws + align256((size_t)N * K * 4));
  k_split_transpose<<<dim3((unsigned)(N / 32), (unsigned)(K / 32)), dim3(32, 8), 0, st>>>(B, Th, Tl, K, N);
  return uk::check_launch("gemm_f32(transpose split)");
}

// C = A * B over a prepared B: splits A into aws (gemm_f32_tc_a_bytes), then
// runs the convolution kernel
int gemm_f32_tc_run(const float* A, const void* bws, void* aws, float* C, int M, int N, int K, cudaStream_t st,
                    float* part, size_t part_room) {
  float* Ah = (float*)aws;
  float* Al = (float*)((uint8_t*)aws + align256((size_t)M * K * 4));
  const int64_t n = (int64_t)M * K;
  k_split_flat<<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)uk::sm_count() * 16), 256, 0, st>>>(A, Ah, Al,
                                                                                                          n);
  if (int rc = uk::check_launch("gemm_f32(split)")) return rc;
  const float* Th = (const float*)bws;
  const float* Tl = (const float*)((const uint8_t*)bws + align256((size_t)N * K * 4));
  note_launch(Candidate{kFamTf32x3, kConvPairF32Tile, 1, 0.0});
  return run_tc(Th, Tl, Ah, Al, C, nullptr, 1, N / 64, 64, K, 1, 1, M, 0, part, part_room, st);
}

}  // namespace uk

extern "C" size_t uk_cuda_gemm_f32_workspace_size(int M, int N, int K) {
  if (!uk::gemm_f32_tc_shape(M, N, K)) return 0;
  return uk::gemm_f32_tc_b_bytes(N, K) + uk::gemm_f32_tc_a_bytes(M, K) + uk::gemm_f32_tc_tail_bytes(M, N, K);
}

extern "C" int uk_cuda_gemm_f32_prefers_tc(int M, int N, int K) {
  // the solver's argmin over the FFMA and split-tf32 candidates (the latter
  // only from 2^30 multiply-adds; below, its pre-passes are never repaid)
  if (!uk::gemm_f32_tc_shape(M, N, K)) return 0;
  return uk::solve_gemm(M, N, K, false, true, uk::sm_count()).family == uk::kFamTf32x3;
}

extern "C" int uk_cuda_gemm_f32_ws(const float* A, const float* B, float* C, int M, int N, int K, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  const cudaStream_t st = (cudaStream_t)stream;
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_f32: negative dims %d %d %d", M, N, K);
  if (workspace == nullptr || workspace_bytes == 0) return uk_cuda_gemm_f32(A, B, C, M, N, K, stream);
  if (!uk::gemm_f32_tc_shape(M, N, K))
    return uk::fail(UK_EINVAL, "gemm_f32: the tensor-core path needs K %% 32 == 0 and N %% 64 == 0 (M=%d N=%d K=%d); "
                    "call without a workspace", M, N, K);
  const size_t bb = uk::gemm_f32_tc_b_bytes(N, K), need = bb + uk::gemm_f32_tc_a_bytes(M, K);  // + optional tail
  if (workspace_bytes < need)
    return uk::fail(UK_EINVAL, "gemm_f32: the tensor-core path needs a %zu-byte workspace, got %zu", need,
                    workspace_bytes);
  if (int rc = uk::check_device_ptr(A, "A")) return rc;
  if (int rc = uk::check_device_ptr(B, "B")) return rc;
  if (int rc = uk::check_device_ptr(C, "C")) return rc;
  if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
  if (!uk::aligned16(workspace)) return uk::fail(UK_EINVAL, "gemm_f32: the workspace must be 16-byte aligned");
  if (int rc = uk::gemm_f32_tc_prep_b(B, workspace, N, K, st)) return rc;
  return uk::gemm_f32_tc_run(A, workspace, (uint8_t*)workspace + bb, C, M, N, K, st,
                             (float*)((uint8_t*)workspace + need), workspace_bytes - need);
}

// ---- fp16 convolution -------------------------------------------------------------
namespace {

// X[n][c][h][w] (f16) -> Xt[n][h][w][c] (f16): one CTA per input row, the C x W
// plane staged in shared memory (as fp32, exact), contiguous 16-byte stores
__global__ void __launch_bounds__(ROW_THREADS) k_row_nhwc_h(const __half* __restrict__ X, __half* __restrict__ Xt,
                                                             int C, int H, int W) {
  extern __shared__ float plane_h[];  // [W][C + 1]
  const int64_t nh = blockIdx.x;
  const int n = (int)(nh / H), h = (int)(nh % H);
  const int cp = C + 1;
  const __half* src = X + ((int64_t)n * C * H + h) * W;
  const int64_t cw = (int64_t)C * W;
  if (W % 8 == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0) {
    // 16-byte loads of 8 w, eight per thread issued before any is consumed
    constexpr int UNR = 8;
    const int w8n = W / 8;
    const int64_t n8 = cw / 8;
    for (int64_t base = threadIdx.x; base < n8; base += (int64_t)ROW_THREADS * UNR) {
      uint4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int64_t i = base + (int64_t)u * ROW_THREADS;
        if (i < n8) {
          const int c = (int)(i / w8n), w8 = (int)(i - (int64_t)c * w8n);
          v[u] = __ldcs(reinterpret_cast<const uint4*>(src + (int64_t)c * H * W) + w8);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int64_t i = base + (int64_t)u * ROW_THREADS;
        if (i < n8) {
          const int c = (int)(i / w8n), w = 8 * (int)(i - (int64_t)c * w8n);
          const uint32_t q[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[j]));
            plane_h[(w + 2 * j) * cp + c] = f.x;
            plane_h[(w + 2 * j + 1) * cp + c] = f.y;
          }
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < cw; i += ROW_THREADS) {
      const int c = (int)(i / W), w = (int)(i - (int64_t)c * W);
      plane_h[w * cp + c] = __half2float(__ldcs(src + (int64_t)c * H * W + w));
    }
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(Xt + nh * cw);
  for (int64_t i = threadIdx.x; i < cw / 8; i += ROW_THREADS) {
    const int64_t e = i * 8;
    const int w = (int)(e / C), c = (int)(e - (int64_t)w * C);
    const float* q = plane_h + w * cp + c;
    uint32_t u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 hh = __floats2half2_rn(q[2 * j], q[2 * j + 1]);
      u[j] = *reinterpret_cast<uint32_t*>(&hh);
    }
    dst[i] = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

// weights [Oc][C][Kh][Kw] -> [Oc][kh][kw][c] (f16)
__global__ void k_permute_weights_h(const __half* __restrict__ Wt, __half* __restrict__ Wp, int Oc, int C, int Kh,
                                    int Kw) {
  const int64_t K = (int64_t)C * Kh * Kw, total = (int64_t)Oc * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t oc = i / K;
    const int k = (int)(i - oc * K);
    const int tap = k / C, c = k - tap * C, kh = tap / Kw, kw = tap - kh * Kw;
    Wp[i] = Wt[((oc * C + c) * Kh + kh) * Kw + kw];
  }
}

int encode_h(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
             const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return uk::fail(UK_ECUDA, "conv2d_f16: cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return uk::fail(UK_ECUDA, "conv2d_f16: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return UK_OK;
}

}  // namespace

extern "C" size_t uk_cuda_conv2d_f16_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc, int pad,
                                                    int layout) {
  if ((layout != UK_CONV_NCHW && layout != UK_CONV_KML) || N <= 0 || H <= 0 || W <= 0 || C <= 0 || C % 64 != 0 ||
      Kh <= 0 || Kw <= 0 || Oc <= 0 || pad < 0)
    return 0;
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  if (Ho <= 0 || Wo <= 0) return 0;
  // NCHW: the NHWC copy and the permuted weights; both layouts: the last
  // round's split partial tiles (the KML layout runs without a workspace too)
  const size_t base = layout == UK_CONV_NCHW
                          ? align256((size_t)N * H * W * C * 2) + align256((size_t)Oc * Kh * Kw * C * 2)
                          : 0;
  return base + tail_bytes(pair_tiles(N, Ho, Wo, Oc), Kh * Kw * (C / PairF16::BKE));
}

extern "C" int uk_cuda_conv2d_f16(const uint16_t* X, const uint16_t* Wt, uint16_t* Y, int N, int H, int W, int C,
                                  int Kh, int Kw, int Oc, int pad, const uint16_t* scale, int layout, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  const cudaStream_t st = (cudaStream_t)stream;
  if (layout != UK_CONV_KML && layout != UK_CONV_NCHW)
    return uk::fail(UK_EINVAL, "conv2d_f16: unknown layout %d", layout);
  if (N < 0 || H <= 0 || W <= 0 || C <= 0 || Kh <= 0 || Kw <= 0 || Oc <= 0 || pad < 0)
    return uk::fail(UK_EINVAL, "conv2d_f16: invalid dims N=%d H=%d W=%d C=%d Kh=%d Kw=%d Oc=%d pad=%d", N, H, W, C,
                    Kh, Kw, Oc, pad);
  if (C % 64 != 0)
    return uk::fail(UK_EINVAL, "conv2d_f16: C=%d must be a multiple of 64 (one 128-byte row of channels per step)", C);
  if (layout == UK_CONV_KML && (N != 1 || pad != 0))
    return uk::fail(UK_EINVAL, "conv2d_f16: the KML layout is one image with valid padding (N=1, pad=0)");
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  if (Ho <= 0 || Wo <= 0) return uk::fail(UK_EINVAL, "conv2d_f16: the filter is larger than the padded input");
  if (N == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(Wt, "Wt")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  if (scale)
    if (int rc = uk::check_device_ptr(scale, "scale")) return rc;
  const uint16_t* Xn = X;   // NHWC input
  const uint16_t* Wk = Wt;  // [Oc][kh][kw][c] weights
  float* part = (float*)workspace;  // the split partial tiles, after the NCHW layout's copies
  size_t part_room = workspace != nullptr ? workspace_bytes : 0;
  if (workspace != nullptr && !uk::aligned16(workspace))
    return uk::fail(UK_EINVAL, "conv2d_f16: the workspace must be 16-byte aligned");
  if (workspace != nullptr)
    if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
  if (layout == UK_CONV_NCHW) {
    const size_t need = align256((size_t)N * H * W * C * 2) + align256((size_t)Oc * Kh * Kw * C * 2);
    if (workspace == nullptr || workspace_bytes < need)
      return uk::fail(UK_EINVAL, "conv2d_f16: needs a %zu-byte workspace (uk_cuda_conv2d_f16_workspace_size), got %zu",
                      need, workspace ? workspace_bytes : (size_t)0);
    if (int rc = uk::check_device_ptr(workspace, "workspace")) return rc;
    if (!uk::aligned16(workspace)) return uk::fail(UK_EINVAL, "conv2d_f16: the workspace must be 16-byte aligned");
    const size_t plane = (size_t)W * (C + 1) * 4;
    uint16_t* Xt = (uint16_t*)workspace;
    uint16_t* Wp = (uint16_t*)((uint8_t*)workspace + align256((size_t)N * H * W * C * 2));
    static bool attr[64] = {false};
    int d = 0;
    cudaGetDevice(&d);
    if (d >= 0 && d < 64 && !attr[d]) {
      if (cudaFuncSetAttribute(k_row_nhwc_h, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
        return uk::check_launch("conv2d_f16: pre-pass attribute");
      attr[d] = true;
    }
    if ((int64_t)N * H > 2147483647LL) return uk::fail(UK_EINVAL, "conv2d_f16: N*H too large");
    const int64_t HW = (int64_t)H * W;
    if (HW % 4 == 0 && ((uintptr_t)X & 7) == 0 && N <= 65535) {
      const dim3 g((unsigned)((HW + 63) / 64), (unsigned)(C / 64), (unsigned)N);
      k_tile_nhwc<true><<<g, 256, 0, st>>>(X, Xt, nullptr, C, HW);
    } else {
      // the row-staged fallback holds one C x W plane in shared memory
      if (plane > 200 * 1024) return uk::fail(UK_EINVAL, "conv2d_f16: W*C too large for the layout pre-pass");
      k_row_nhwc_h<<<(unsigned)((int64_t)N * H), ROW_THREADS, plane, st>>>((const __half*)X, (__half*)Xt, C, H, W);
    }
    const int64_t nw = (int64_t)Oc * Kh * Kw * C;
    if ((int64_t)C * Kh * Kw * 4 <= kPermuteSmem)
      k_permute_w<true><<<(unsigned)Oc, 256, (size_t)C * Kh * Kw * 4, st>>>(Wt, Wp, nullptr, C, Kh * Kw);
    else
      k_permute_weights_h<<<(unsigned)std::min<int64_t>((nw + 255) / 256, (int64_t)uk::sm_count() * 8), 256, 0,
                            st>>>((const __half*)Wt, (__half*)Wp, Oc, C, Kh, Kw);
    if (int rc = uk::check_launch("conv2d_f16(pre-pass)")) return rc;
    Xn = Xt;
    Wk = Wp;
    part = (float*)((uint8_t*)workspace + need);
    part_room = workspace_bytes - need;
  } else if (!uk::aligned16(X) || !uk::aligned16(Wt)) {
    return uk::fail(UK_EINVAL, "conv2d_f16: X and Wt must be 16-byte aligned");
  }

  CUtensorMap tx, tw;
  const cuuint64_t xdims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
  const cuuint64_t xstr[3] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2, (cuuint64_t)H * W * C * 2};
  const cuuint32_t xbox[4] = {(cuuint32_t)PairF16::BKE, BW, BH, 1};
  const int64_t K = (int64_t)Kh * Kw * C;
  const cuuint64_t wdims[2] = {(cuuint64_t)K, (cuuint64_t)Oc};
  const cuuint64_t wstr[1] = {(cuuint64_t)K * 2};
  const cuuint32_t wbox[2] = {(cuuint32_t)PairF16::BKE, (cuuint32_t)P_BNC};
  if (int rc = encode_h(&tx, Xn, 4, xdims, xstr, xbox)) return rc;
  if (int rc = encode_h(&tw, Wk, 2, wdims, wstr, wbox)) return rc;

  ConvTc p{};
  p.y = Y;
  p.scale = scale;
  p.N = N;
  p.Ho = Ho;
  p.Wo = Wo;
  p.Oc = Oc;
  p.C = C;
  p.Kh = Kh;
  p.Kw = Kw;
  p.pad = pad;
  p.tiles_w = (Wo + BW - 1) / BW;
  p.tiles_h = (Ho + P_BH - 1) / P_BH;
  p.tiles_oc = (Oc + BN - 1) / BN;
  const int64_t tiles = (int64_t)N * p.tiles_h * p.tiles_w * p.tiles_oc;
  if (tiles > 2147483647LL) return uk::fail(UK_EINVAL, "conv2d_f16: too many tiles");
  p.num_tiles = (int)tiles;
  const TailPlan tp = tail_plan(tiles, Kh * Kw * (C / PairF16::BKE), workspace != nullptr ? part_room : 0);
  apply_tail(p, tp, part);

  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(k_conv_pair<PairF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)pair_smem_bytes<PairF16>()) != cudaSuccess)
      return uk::check_launch("conv2d_f16: smem attribute");
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * tp.pairs), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = pair_smem_bytes<PairF16>();
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_conv_pair<PairF16>, tx, tx, tw, tw, p);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "conv2d_f16: launch: %s", cudaGetErrorString(e));
  if (tp.splits >= 2) {
    const int64_t total = (int64_t)(p.num_tiles - p.num_full) * 2 * BN * 128;
    const int64_t g = std::min<int64_t>((total + 255) / 256, (int64_t)uk::sm_count() * 8);
    k_conv_tail<__half><<<(unsigned)g, 256, 0, st>>>(p);
  }
  return uk::check_launch("conv2d_f16(tcgen05 pair)");
}
