// gemm_f16.cu -- C(f16) = A(f16) * B(f16) with fp32 accumulation on the
// 5th-generation tensor cores (tcgen05, accumulators in TMEM, operands staged
// by TMA).  Replaces uk_gemm_h (src/codegen_hip.cpp:1777-1808), which ran the
// product on SIMT FMA from fp32 copies in shared memory.
//
// Kernel structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: per 64-wide K block, one 128x64 box of A
//               (K-major) and four 64x64 boxes of B (row-major B is the
//               MN-major operand), 128-byte swizzle, into a 4-stage ring
//   warp 1      TMEM owner (alloc/dealloc 512 columns) and MMA issuer: one
//               thread issues tcgen05.mma M=128 N=256 K=16 (4 per K block)
//               into one of two 256-column fp32 accumulators
//   warps 2-5   epilogue, one warp per TMEM lane quadrant: tcgen05.ld
//               32 lanes x 32 columns, convert
//               to f16 (round to nearest even), stage in swizzled shared
//               memory, store 128-byte row segments; with the second
//               accumulator the epilogue of tile i overlaps the MMAs of i+1
// The epilogue can also write each tile to up to 7 more buffers (other GPUs'
// copies of C reached over NVLink): that is the all-gather of the N-sharded
// multi-GPU GEMM, fused into the store.
// Tiles are visited in groups of 16 M-blocks so the A and B panels a wave of
// 148 CTAs touches stay in L2.
//
// Every mbarrier wait is bounded (uk_mbar_wait); a timeout sets the fault word
// read by uk_cuda_pipeline_fault() and the CTA unwinds.  Every TMA load is a
// plain single-CTA load of this GPU's own memory.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace uk {
// device fault word of this translation unit (no relocatable device code, so
// each TU that runs bounded waits owns one); read by uk_cuda_pipeline_fault
__device__ unsigned int g_fault_word = 0;
int gemm_f16_simt(const __half* A, int64_t lda, const __half* B, int64_t ldb, __half* C, int64_t ldc, int M, int N,
                  int K, cudaStream_t st);
}  // namespace uk

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
static_assert(BM == uk::kGemmF16Tile.bm && BN == uk::kGemmF16Tile.bn && BK == uk::kGemmF16Tile.bk &&
                  STAGES == uk::kGemmF16Tile.stages,
              "the plan query must report the tile this kernel is built for");
constexpr int A_BYTES = BM * BK * 2;      // 16 KiB
constexpr int B_BOX_BYTES = BK * 64 * 2;  // 8 KiB: 64 K rows x 64 N columns
constexpr int B_BYTES = BK * BN * 2;      // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;  // one per TMEM lane quadrant (8 measured slower: more remote stores in flight per SM congest NVLink)
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;
constexpr int MAX_OUT = 8;
constexpr uint32_t IDESC = uk_idesc_f16(BM, BN, /*B MN-major*/ 1);
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait

struct OutList {
  uint16_t* c[MAX_OUT];  // c[0]: this GPU's C; c[1..]: peers' C (same layout)
  int n;
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

// epilogue staging: per epilogue warp one 32-row x 64-column f16 block (4 KiB)
constexpr int STG_BYTES = 32 * 64 * 2;
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + EPI_WARPS * STG_BYTES + sizeof(SmemCtl) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory per block on sm_100");

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
  atomicOr(&uk::g_fault_word, bit);
  ctl->abort = 1;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_f16_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, OutList out,
                  int M, int N, int K, int64_t ldc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* staging = smem + (size_t)STAGES * STAGE_BYTES;
  SmemCtl* ctl = (SmemCtl*)(staging + EPI_WARPS * STG_BYTES);
  volatile int* abort = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

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
    uk_tma_prefetch_desc(&tmA);
    uk_tma_prefetch_desc(&tmB);
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
      for (int t = blockIdx.x; t < num_tiles && !*abort; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait(&ctl->empty[s], ph ^ 1u, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_PRODUCER);
            break;
          }
          uint8_t* sa = smem + (size_t)s * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          uk_mbar_expect_tx(&ctl->full[s], STAGE_BYTES);
          uk_tma_load_2d(sa, &tmA, &ctl->full[s], kb * BK, mb * BM);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            uk_tma_load_2d(sb + j * B_BOX_BYTES, &tmB, &ctl->full[s], nb * BN + j * 64, kb * BK);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort; t += gridDim.x, ++tl) {
        const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
        if (!uk_mbar_wait(&ctl->tempty[buf], tph ^ 1u, abort, WAIT_NS)) {
          raise_fault(ctl, UK_FAULT_MMA);
          break;
        }
        uk_tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!uk_mbar_wait(&ctl->full[s], ph, abort, WAIT_NS)) {
            raise_fault(ctl, UK_FAULT_MMA);
            ok = false;
            break;
          }
          uk_tc_fence_after();
          const uint32_t sa = uk_smem_u32(smem + (size_t)s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: K-major, +32 bytes per 16 K inside the 128-byte swizzle atom
            const uint64_t ad = uk_desc_sw128(sa + k * 32, 16, 1024);
            // B: MN-major, 64-column chunks 8 KiB apart (LBO), 8-row K groups
            // 1 KiB apart (SBO), +16 rows (2 KiB) per 16 K
            const uint64_t bd = uk_desc_sw128(sb + k * 2048, B_BOX_BYTES, 1024);
            uk_umma_f16(d, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          uk_umma_commit(&ctl->empty[s]);  // frees the stage when these MMAs finish
        }
        if (!ok) break;
        uk_umma_commit(&ctl->tfull[buf]);  // accumulator ready for the epilogue
      }
      // all MMAs issued by this thread complete before TMEM is released
      uk_umma_commit(&ctl->teardown);
      if (!uk_mbar_wait(&ctl->teardown, 0, nullptr, WAIT_NS)) atomicOr(&uk::g_fault_word, UK_FAULT_TEARDOWN);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2 .. 2 + EPI_WARPS) ----------------
    // TMEM -> registers (each lane one row) -> f16 -> swizzled staging block
    // -> coalesced 128-byte row segments to every copy of C.  Staging chunk
    // c (16 bytes) of row r sits at r*128 + ((c ^ (r & 7)) * 16), so both the
    // row-wise writes and the column-wise reads are bank-conflict free.
    const int q = warp & 3;                       // TMEM lane quadrant this warp may access
    constexpr int COLS = BN * 4 / EPI_WARPS;      // columns of the tile this warp drains
    const int half = (warp - 2) >> 2;             // which COLS-wide part of the tile
    uint8_t* stg = staging + (warp - 2) * STG_BYTES;
    uint32_t tl = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort; t += gridDim.x, ++tl) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const uint32_t buf = tl & 1u, tph = (tl >> 1) & 1u;
      if (!uk_mbar_wait(&ctl->tfull[buf], tph, abort, WAIT_NS)) {
        raise_fault(ctl, UK_FAULT_EPILOGUE);
        break;
      }
      uk_tc_fence_after();
      const int row0 = mb * BM + q * 32;
      const int n0 = nb * BN;
#pragma unroll 1
      for (int h = half * (COLS / 64); h < (half + 1) * (COLS / 64); ++h) {
        uint32_t v0[32], v1[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + buf * BN + h * 64;
        uk_tmem_ld32(taddr, v0);
        uk_tmem_ld32(taddr + 32, v1);
        uk_tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? &v0[(c & 3) * 8] : &v1[(c & 3) * 8];
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            __half2 h2 = __floats2half2_rn(__uint_as_float(src[2 * i]), __uint_as_float(src[2 * i + 1]));
            w[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
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
      if (lane == 0) uk_mbar_arrive(&ctl->tempty[buf]);
    }
    // stores into other GPUs' buffers are made visible system-wide before
    // this CTA retires (the host orders ranks after the kernel)
    if (out.n > 1) __threadfence_system();
  }

  uk_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    uk_tc_fence_after();
    uk_tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- host side ----------------------------------------------------------------

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

// 2-D f16 tensor map: `inner` contiguous elements per row, `outer` rows,
// `ld` elements between rows; box = box_inner x box_outer, 128-byte swizzle.
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

bool tc_shape_ok(const void* A, int64_t lda, const void* B, int64_t ldb, const void* const* Cs, int nc, int64_t ldc,
                 int N, int K) {
  if (K % 8 != 0 || N % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 || ldc % 8 != 0) return false;
  if (!uk::aligned16(A) || !uk::aligned16(B)) return false;
  for (int i = 0; i < nc; ++i)
    if (!uk::aligned16(Cs[i])) return false;
  return K > 0;
}

}  // namespace

namespace uk {

// C[0..nc) all receive the product; used directly by the multi-GPU path with
// peer pointers (C[0] local).  Shapes must satisfy tc_shape_ok.
int gemm_f16_tc_2sm(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, uint16_t* const* Cs, int nc,
                    int64_t ldc, int M, int N, int K, cudaStream_t st);  // gemm_f16_2sm.cu

// Kernel choice: the SM-pair kernel (256 x 256 tiles over two SMs) needs M
// to have two 128-row blocks.  With one copy of C the solver's argmin decides
// between it and the single-SM kernel; with more copies (the all-gather of
// the N-sharded GEMM over 2-8 GPUs) the pair kernel runs its TMA-store
// epilogue, which hands the accumulator back before the NVLink stores drain.
// UNIKERN_GEMM_F16_PAIR=0 / =1 pins the single-SM / pair kernel (for
// measuring the alternative).
static bool use_pair_kernel(int M, int N, int K, int nc) {
  static int env = -1;  // -1 unread, 0 single, 1 pair, 2 solver
  if (env < 0) {
    const char* e = getenv("UNIKERN_GEMM_F16_PAIR");
    env = e == nullptr || e[0] == 0 ? 2 : e[0] == '0' ? 0 : 1;
  }
  if (env == 0 || M <= 128) return false;
  if (env == 1 || nc > 1) return true;
  return solve_gemm(M, N, K, true, false, sm_count()).family == kFamF16Pair;
}

int gemm_f16_tc(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, uint16_t* const* Cs, int nc,
                int64_t ldc, int M, int N, int K, cudaStream_t st) {
  if (nc < 1 || nc > MAX_OUT) return fail(UK_EINVAL, "gemm_f16: 1..%d outputs, got %d", MAX_OUT, nc);
  if (use_pair_kernel(M, N, K, nc)) {
    note_launch(Candidate{kFamF16Pair, kGemmF16PairTile, 1, 0.0});
    return gemm_f16_tc_2sm(A, lda, B, ldb, Cs, nc, ldc, M, N, K, st);
  }
  note_launch(Candidate{kFamF16Single, kGemmF16Tile, 1, 0.0});
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM)) return rc;
  if (int rc = make_map(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK)) return rc;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_f16_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return fail(UK_ECUDA, "gemm_f16: smem attribute: %s", cudaGetErrorString(e));
    attr_done[dev] = true;
  }
  OutList out{};
  for (int i = 0; i < nc; ++i) out.c[i] = Cs[i];
  out.n = nc;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  k_gemm_f16_tc<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(ta, tb, out, M, N, K, ldc);
  return check_launch("gemm_f16(tcgen05)");
}

bool gemm_f16_tc_ok(const void* A, int64_t lda, const void* B, int64_t ldb, const void* const* Cs, int nc,
                    int64_t ldc, int N, int K) {
  return tc_shape_ok(A, lda, B, ldb, Cs, nc, ldc, N, K);
}

}  // namespace uk

extern "C" int uk_cuda_gemm_f16_ld(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, uint16_t* C,
                                   int64_t ldc, int M, int N, int K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_f16: negative dims %d %d %d", M, N, K);
  if (lda < K || ldb < N || ldc < N)
    return uk::fail(UK_EINVAL, "gemm_f16: leading dimensions lda=%lld ldb=%lld ldc=%lld below K/N", (long long)lda,
                    (long long)ldb, (long long)ldc);
  if (M == 0 || N == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(C, "C")) return rc;
  if (K > 0) {
    if (int rc = uk::check_device_ptr(A, "A")) return rc;
    if (int rc = uk::check_device_ptr(B, "B")) return rc;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const void* cs[1] = {C};
  if (uk::gemm_f16_tc_ok(A, lda, B, ldb, cs, 1, ldc, N, K)) {
    uint16_t* outs[1] = {C};
    return uk::gemm_f16_tc(A, lda, B, ldb, outs, 1, ldc, M, N, K, st);
  }
  if ((M + 31) / 32 > 65535) return uk::fail(UK_EINVAL, "gemm_f16: M=%d exceeds the grid limit", M);
  return uk::gemm_f16_simt((const __half*)A, lda, (const __half*)B, ldb, (__half*)C, ldc, M, N, K, st);
}

extern "C" int uk_cuda_gemm_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                                void* stream) {
  return uk_cuda_gemm_f16_ld(A, K, B, N, C, N, M, N, K, stream);
}

// N-sharded GEMM with the all-gather fused into the epilogue: this rank
// computes columns [col_offset, col_offset + N_shard) of C = A * B from its
// column slice of B, and stores every tile into all n_c copies of C (C_list[0]
// on this GPU, the others peers' buffers opened with uk_cuda_ipc_import).
extern "C" int uk_cuda_gemm_f16_allgather(const uint16_t* A, int64_t lda, const uint16_t* B_shard, int64_t ldb,
                                          uint16_t* const* C_list, int n_c, int64_t ldc, int M, int N_shard, int K,
                                          int64_t col_offset, void* stream) {
  if (M < 0 || N_shard < 0 || K <= 0) return uk::fail(UK_EINVAL, "gemm_f16_allgather: dims %d %d %d", M, N_shard, K);
  if (C_list == nullptr || n_c < 1 || n_c > MAX_OUT)
    return uk::fail(UK_EINVAL, "gemm_f16_allgather: 1..%d outputs, got %d", MAX_OUT, n_c);
  if (col_offset < 0 || col_offset % 8 != 0 || col_offset + N_shard > ldc)
    return uk::fail(UK_EINVAL, "gemm_f16_allgather: column offset %lld (multiple of 8, inside ldc=%lld)",
                    (long long)col_offset, (long long)ldc);
  if (lda < K || ldb < N_shard) return uk::fail(UK_EINVAL, "gemm_f16_allgather: leading dimensions");
  if (M == 0 || N_shard == 0) return UK_OK;
  if (int rc = uk::check_device_ptr(A, "A")) return rc;
  if (int rc = uk::check_device_ptr(B_shard, "B_shard")) return rc;
  if (int rc = uk::check_device_ptr(C_list[0], "C_list[0]")) return rc;
  uint16_t* outs[MAX_OUT];
  for (int i = 0; i < n_c; ++i) {
    if (C_list[i] == nullptr) return uk::fail(UK_EINVAL, "gemm_f16_allgather: C_list[%d] is NULL", i);
    if (i > 0) {
      cudaPointerAttributes a{};
      if (cudaPointerGetAttributes(&a, C_list[i]) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return uk::fail(UK_ERESIDENCY, "gemm_f16_allgather: C_list[%d] is not device memory", i);
      }
    }
    outs[i] = C_list[i] + col_offset;
  }
  const void* cs[MAX_OUT];
  for (int i = 0; i < n_c; ++i) cs[i] = outs[i];
  if (!uk::gemm_f16_tc_ok(A, lda, B_shard, ldb, cs, n_c, ldc, N_shard, K))
    return uk::fail(UK_EINVAL, "gemm_f16_allgather: needs K, N_shard, lda, ldb, ldc multiples of 8 and 16-byte "
                               "aligned pointers");
  return uk::gemm_f16_tc(A, lda, B_shard, ldb, outs, n_c, ldc, M, N_shard, K, (cudaStream_t)stream);
}

namespace uk {
unsigned decode_fault_take();  // decode.cu
unsigned conv_fault_take();    // conv_tc.cu
unsigned fault_take_2sm();     // gemm_f16_2sm.cu
unsigned peer_fault_take();    // peer.cu
}

// the bounded wait of every pipeline, run alone on one mbarrier: when nothing
// arrives it must give up after timeout_ns, record UK_FAULT_SELFTEST and
// return, leaving the context usable
__global__ void k_selftest_wait(int arrive, uint64_t timeout_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    uk_mbar_init(&bar, 1);
    uk_fence_mbar_init();
    if (arrive) uk_mbar_arrive(&bar);
    const bool ok = uk_mbar_wait(&bar, 0, nullptr, timeout_ns);
    if (!ok) atomicOr(&uk::g_fault_word, UK_FAULT_SELFTEST);
    *status = ok ? 1 : 0;
  }
}

extern "C" int uk_cuda_selftest_wait(int arrive, uint64_t timeout_ns, int* status, void* stream) {
  if (timeout_ns < 1000 || timeout_ns > 1000000000ull)
    return uk::fail(UK_EINVAL, "selftest_wait: timeout_ns must be in [1e3, 1e9] (got %llu)",
                    (unsigned long long)timeout_ns);
  if (int rc = uk::check_device_ptr(status, "status")) return rc;
  k_selftest_wait<<<1, 32, 0, (cudaStream_t)stream>>>(arrive, timeout_ns, status);
  return uk::check_launch("selftest_wait");
}

extern "C" unsigned uk_cuda_pipeline_fault(void) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, uk::g_fault_word, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned zero = 0;
  cudaMemcpyToSymbol(uk::g_fault_word, &zero, sizeof(zero));
  return v | uk::decode_fault_take() | uk::conv_fault_take() | uk::fault_take_2sm() | uk::peer_fault_take();
}
