// gemm_f16_2sm.cu -- the f16 GEMM (f32 accumulation, f16 out) on CTA pairs:
// tcgen05.mma.cta_group::2 with a 256 x 256 tile per pair of SMs.
//
// Each CTA of a 2-CTA cluster holds its own 128 rows of the A tile and one half
// (128 columns) of the B tile; the even (leader) CTA issues M = 256 MMAs whose
// operands come from the same shared-memory offsets in both CTAs, and each
// CTA's TMEM receives its 128 rows of the accumulator.  Compared with the
// single-SM kernel (128 x 256 per SM), every SM loads half as much B per
// k-block (32 KiB per stage instead of 48), so the ring is 6 stages deep and
// the L2 -> SM operand traffic per MMA flop drops by a third.
//
// Pipeline (per CTA, 192 threads):
//   warp 0      TMA producer of this CTA's A half and B half; the loads count
//               their bytes on the LEADER's full barrier (the leader posts
//               the expected bytes of both CTAs), so one barrier tells the
//               MMA issuer that the whole 256 x 64 / 64 x 256 stage landed
//   warp 1      TMEM (cta_group::2 alloc of 512 columns = two accumulators);
//               in the leader, one thread issues the MMAs and commits their
//               completion to the empty / tile-full barriers of BOTH CTAs
//   warps 2-5   epilogue of this CTA's 128 rows (as the single-SM kernel:
//               tcgen05.ld, f16, swizzled staging, 128-byte row stores), then
//               a remote arrive on the leader's tile-empty barrier
// The all-gather of the N-sharded multi-GPU GEMM writes each tile to every
// copy of C.  A second epilogue (TMA_OUT, opt-in) stores through the TMA:
// each warp stages its 32 x 64 block in one of two 4 KiB slots with the
// 128-byte swizzle a tensor map expects, one lane issues a TMA tensor store
// of the block to every copy (peers' buffers over NVLink included) and the
// accumulator goes back to the MMA issuer as soon as the tile is staged.
// Measured on 2 and 4 GPUs it is no faster than the lane stores (0.294 vs
// 0.273 ms per launch on 4), so the lane stores stay the default.
// Every mbarrier wait is bounded (2 s); a timeout sets the fault word and the
// CTA unwinds; both CTAs pass the same cluster barriers on every path.  Each
// TMA load is a plain load of this GPU's memory into the issuing CTA's own
// shared memory: only its completion count goes to the peer's barrier.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace uk {
__device__ unsigned int g_fault_word_2sm = 0;
}  // namespace uk

namespace {

constexpr int BMC = 128;           // rows per CTA (256 per pair)
constexpr int BN = 256;            // columns per pair tile
constexpr int BNC = BN / 2;        // B columns per CTA
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_BYTES = BMC * BK * 2;        // 16 KiB
constexpr int B_BOX_BYTES = BK * 64 * 2;     // 8 KiB
constexpr int B_BYTES = BNC * BK * 2;        // 16 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;         // pair-rows (of 256) per raster group
constexpr int MAX_OUT = 8;
constexpr uint32_t IDESC = uk_idesc_f16(2 * BMC, BN, /*B MN-major*/ 1);
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr uint16_t PAIR = 0x3;     // both CTAs of the cluster
static_assert(2 * BMC == uk::kGemmF16PairTile.bm && BN == uk::kGemmF16PairTile.bn && BK == uk::kGemmF16PairTile.bk &&
                  STAGES == uk::kGemmF16PairTile.stages,
              "the plan query must report the tile this kernel is built for");

struct OutList {
  uint16_t* c[MAX_OUT];
  int n;
};

// TMA_OUT: one tensor map per copy of C ([M][N] at stride ldc, box 64 x 32,
// 128-byte swizzle)
struct OutMaps {
  CUtensorMap m[MAX_OUT];
};

struct SmemCtl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};

constexpr int STG_BYTES = 32 * 64 * 2;
template <bool TMA_OUT>
constexpr size_t smem_bytes() {
  return (size_t)STAGES * STAGE_BYTES + EPI_WARPS * (TMA_OUT ? 2 : 1) * STG_BYTES + sizeof(SmemCtl) + 1024;
}
static_assert(smem_bytes<true>() <= 232448 && smem_bytes<false>() <= 232448, "shared memory per block on sm_100");

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int r = t - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

__device__ __forceinline__ void raise_fault(SmemCtl* ctl, unsigned bit) {
  atomicOr(&uk::g_fault_word_2sm, bit);
  ctl->abort = 1;
}

template <bool TMA_OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_f16_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ OutMaps omaps, OutList out, int M, int N, int K, int64_t ldc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* staging = smem + (size_t)STAGES * STAGE_BYTES;  // 1024-byte aligned: the swizzle atom
  SmemCtl* ctl = (SmemCtl*)(staging + EPI_WARPS * (TMA_OUT ? 2 : 1) * STG_BYTES);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = uk_cluster_ctarank();  // 0 = leader, 1 = peer
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + 2 * BMC - 1) / (2 * BMC), num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      uk_mbar_init(&ctl->full[s], 1);
      uk_mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      uk_mbar_init(&ctl->tfull[b], 1);
      uk_mbar_init(&ctl->tempty[b], 2 * EPI_WARPS);  // both CTAs' epilogue warps (leader's copy is used)
    }
    uk_mbar_init(&ctl->teardown, 1);
    ctl->abort = 0;
    uk_fence_mbar_init();
    uk_tma_prefetch_desc(&tmA);
    uk_tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    uk_tmem_alloc_cg2(&ctl->tmem_base, TMEM_COLS);
    uk_tmem_relinquish_cg2();
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  uk_tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = pair; t < num_tiles && !*abort; t += npairs) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait_cluster(&ctl->empty[s], ph ^ 1u, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_PRODUCER);
            break;
          }
          uint8_t* sa = smem + (size_t)s * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          const uint32_t bar = uk_mapa(uk_smem_u32(&ctl->full[s]), 0);  // the leader's full barrier
          if (crank == 0) uk_mbar_expect_tx(&ctl->full[s], 2 * STAGE_BYTES);
          uk_tma_load_2d_cg2(sa, &tmA, bar, kb * BK, mb * 2 * BMC + (int)crank * BMC);
#pragma unroll
          for (int j = 0; j < BNC / 64; ++j)
            uk_tma_load_2d_cg2(sb + j * B_BOX_BYTES, &tmB, bar, nb * BN + (int)crank * BNC + j * 64, kb * BK);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (crank == 0 && lane == 0) {
      uint32_t it = 0, tl = 0;
      for (int t = pair; t < num_tiles && !*abort; t += npairs, ++tl) {
        const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
        if (!uk_mbar_wait_cluster(&ctl->tempty[buf], tph ^ 1u, abort, WAIT_NS)) {
          raise_fault(ctl, UK_FAULT_MMA);
          break;
        }
        uk_tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait_cluster(&ctl->full[s], ph, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_MMA);
            ok = false;
            break;
          }
          uk_tc_fence_after();
          const uint32_t sa = uk_smem_u32(smem + (size_t)s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: K-major, +32 bytes per 16 K; B: MN-major, 64-column chunks
            // 8 KiB apart (LBO), 8-row K groups 1 KiB apart (SBO), +2 KiB per 16 K
            const uint64_t ad = uk_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = uk_desc_sw128(sb + k * 2048, B_BOX_BYTES, 1024);
            uk_umma_f16_cg2(d, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          uk_umma_commit_cg2(&ctl->empty[s], PAIR);  // frees the stage in both CTAs
        }
        if (!ok) break;
        uk_umma_commit_cg2(&ctl->tfull[buf], PAIR);  // both halves of the accumulator ready
      }
      uk_umma_commit_cg2(&ctl->teardown, PAIR);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2 .. 5, both CTAs) ----------------
    const int q = warp & 3;
    uint8_t* stg = staging + (warp - 2) * (TMA_OUT ? 2 : 1) * STG_BYTES;
    const uint32_t tempty_leader[2] = {uk_mapa(uk_smem_u32(&ctl->tempty[0]), 0),
                                       uk_mapa(uk_smem_u32(&ctl->tempty[1]), 0)};
    uint32_t tl = 0;
    int slot = 0;  // TMA_OUT: the staging slot of the next block (two per warp)
    for (int t = pair; t < num_tiles && !*abort; t += npairs, ++tl) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
      if (!uk_mbar_wait_cluster(&ctl->tfull[buf], tph, abort, WAIT_NS)) {
        raise_fault(ctl, UK_FAULT_EPILOGUE);
        break;
      }
      uk_tc_fence_after();
      const int row0 = mb * 2 * BMC + (int)crank * BMC + q * 32;
      const int n0 = nb * BN;
#pragma unroll 1
      for (int h = 0; h < BN / 64; ++h) {
        uint32_t v0[32], v1[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + buf * BN + h * 64;
        uk_tmem_ld32(taddr, v0);
        uk_tmem_ld32(taddr + 32, v1);
        uk_tmem_ld_wait();
        uint8_t* blk = stg;
        if constexpr (TMA_OUT) {
          blk = stg + slot * STG_BYTES;
          // the stores issued from this slot two blocks ago have read it
          if (lane == 0) uk_bulk_wait_read<1>();
          __syncwarp();
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? &v0[(c & 3) * 8] : &v1[(c & 3) * 8];
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            __half2 h2 = __floats2half2_rn(__uint_as_float(src[2 * i]), __uint_as_float(src[2 * i + 1]));
            w[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(blk + lane * 128 + ((c ^ (lane & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if constexpr (TMA_OUT) {
          // staging writes -> async proxy, then one lane stores the block to
          // every copy (boxes wholly past M or N are skipped; partial ones
          // are clipped by the tensor map)
          uk_fence_proxy_async_smem();
          __syncwarp();
          const int bx = n0 + h * 64;
          if (lane == 0 && bx < N && row0 < M) {
            for (int o = 0; o < out.n; ++o) uk_tma_store_2d(&omaps.m[o], blk, bx, row0);
            uk_bulk_commit();
          }
          slot ^= 1;
          continue;
        }
        __syncwarp();
        const int c = lane & 7;
        const int gn = n0 + h * 64 + c * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = i * 4 + (lane >> 3);
          const uint4 val = *reinterpret_cast<const uint4*>(stg + r * 128 + ((c ^ (r & 7)) * 16));
          const int gm = row0 + r;
          if (gm < M && gn < N) {
            const size_t off = (size_t)gm * ldc + gn;
            for (int o = 0; o < out.n; ++o) *reinterpret_cast<uint4*>(out.c[o] + off) = val;
          }
        }
        __syncwarp();
      }
      uk_tc_fence_before();
      __syncwarp();
      if (lane == 0) uk_mbar_arrive_cluster(tempty_leader[buf]);
    }
    // TMA_OUT: every store this warp issued has been performed before the
    // CTA retires; stores into other GPUs' buffers are made visible
    // system-wide (the host orders the ranks after the kernel)
    if constexpr (TMA_OUT) {
      if (lane == 0) uk_bulk_wait<0>();
      __syncwarp();
    }
    if (out.n > 1) __threadfence_system();
  }

  // teardown: every MMA has completed (the leader's last commit), both CTAs'
  // epilogues are done with TMEM, then the pair releases it together
  if (warp == 1 && lane == 0) {
    if (!uk_mbar_wait_cluster(&ctl->teardown, 0, nullptr, WAIT_NS)) atomicOr(&uk::g_fault_word_2sm, UK_FAULT_TEARDOWN);
  }
  uk_tc_fence_before();
  __syncthreads();
  uk_cluster_sync();
  if (warp == 1) {
    uk_tc_fence_after();
    uk_tmem_dealloc_cg2(tmem, TMEM_COLS);
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

int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
             uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return uk::fail(UK_ECUDA, "gemm_f16: cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return uk::fail(UK_ECUDA, "gemm_f16: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return UK_OK;
}

}  // namespace

namespace uk {

unsigned fault_take_2sm() {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fault_word_2sm, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned zero = 0;
  cudaMemcpyToSymbol(g_fault_word_2sm, &zero, sizeof(zero));
  return v;
}

// The pair kernel, for shapes the single-SM kernel takes (same preconditions).
int gemm_f16_tc_2sm(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, uint16_t* const* Cs, int nc,
                    int64_t ldc, int M, int N, int K, cudaStream_t st) {
  if (nc < 1 || nc > MAX_OUT) return fail(UK_EINVAL, "gemm_f16: 1..%d outputs, got %d", MAX_OUT, nc);
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BMC)) return rc;
  if (int rc = make_map(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK)) return rc;
  // copies of C go out through the lane stores of the one-copy epilogue;
  // UNIKERN_GEMM_F16_TMA_OUT=1 selects the TMA-store epilogue instead (on 4
  // GPUs the lane stores measured 0.273 ms per launch against 0.294)
  static int tma_env = -1;
  if (tma_env < 0) {
    const char* e = getenv("UNIKERN_GEMM_F16_TMA_OUT");
    tma_env = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  const bool tma_out = nc > 1 && tma_env == 1;
  static bool attr_done[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[tma_out][dev]) {
    const cudaError_t e =
        tma_out ? cudaFuncSetAttribute(k_gemm_f16_tc2<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_bytes<true>())
                : cudaFuncSetAttribute(k_gemm_f16_tc2<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_bytes<false>());
    if (e != cudaSuccess) return fail(UK_ECUDA, "gemm_f16: smem attribute: %s", cudaGetErrorString(e));
    attr_done[tma_out][dev] = true;
  }
  OutList out{};
  for (int i = 0; i < nc; ++i) out.c[i] = Cs[i];
  out.n = nc;
  // the copies' tensor maps: [M][N] at stride ldc (each copy already offset
  // to this rank's first column), 64 x 32 boxes, 128-byte swizzle
  OutMaps omaps{};
  if (tma_out)
    for (int i = 0; i < nc; ++i)
      if (int rc = make_map(&omaps.m[i], Cs[i], (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 64, 32)) return rc;
  const int tiles = ((M + 2 * BMC - 1) / (2 * BMC)) * ((N + BN - 1) / BN);
  const int pairs = tiles < sm_count() / 2 ? tiles : sm_count() / 2;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = tma_out ? smem_bytes<true>() : smem_bytes<false>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = tma_out ? cudaLaunchKernelEx(&cfg, k_gemm_f16_tc2<true>, ta, tb, omaps, out, M, N, K, ldc)
                                : cudaLaunchKernelEx(&cfg, k_gemm_f16_tc2<false>, ta, tb, omaps, out, M, N, K, ldc);
  if (e != cudaSuccess) return fail(UK_ECUDA, "gemm_f16(2sm): launch: %s", cudaGetErrorString(e));
  return check_launch("gemm_f16(tcgen05 pair)");
}

}  // namespace uk
