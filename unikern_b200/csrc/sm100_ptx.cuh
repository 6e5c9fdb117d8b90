// sm100_ptx.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a)
// features the tensor-core kernels use: mbarriers, TMA tiled loads (each a
// plain single-CTA load), tcgen05 MMA / TMEM alloc / loads.
//
// Every wait is bounded: uk_mbar_wait gives up after `timeout_ns` of
// %globaltimer (or as soon as another role of the CTA raised the abort flag)
// and returns false; callers record the fault and unwind instead of spinning.
#pragma once

#include <cuda.h>
#include <stdint.h>

// bits of the device fault word (uk_cuda_pipeline_fault)
#define UK_FAULT_PRODUCER 0x1u
#define UK_FAULT_MMA 0x2u
#define UK_FAULT_EPILOGUE 0x4u
#define UK_FAULT_TEARDOWN 0x8u
#define UK_FAULT_SELFTEST 0x10u
#define UK_FAULT_PEER 0x20u

__device__ __forceinline__ uint32_t uk_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t uk_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void uk_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(uk_smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void uk_fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void uk_mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(uk_smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void uk_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(uk_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool uk_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(uk_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with parity `parity` to complete.  Returns false on
// timeout or when *abort was raised by another role of the CTA.
__device__ __forceinline__ bool uk_mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                             uint64_t timeout_ns) {
  if (uk_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = uk_globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (uk_mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (uk_globaltimer() - t0 > timeout_ns) return false;
    }
  }
}

// ---- TMA (tiled, 2-D, single-CTA destination) ------------------------------
__device__ __forceinline__ void uk_tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// x = innermost coordinate (elements; callers keep x * elem_size a multiple
// of 16 bytes), y = row coordinate.
__device__ __forceinline__ void uk_tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          uk_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(uk_smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// TMA tensor store of one 2-D box from this CTA's shared memory to global
// memory (this GPU's or a peer's, through a tensor map of its address),
// tracked in the issuing thread's bulk async-group.  x, y >= 0 (x * elem_size
// a multiple of 16 bytes); the parts of the box outside the tensor are not
// written.  The source must have been made visible to the async proxy
// (uk_fence_proxy_async_smem by every writing thread) before the store.
__device__ __forceinline__ void uk_tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(uk_smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// close the bulk async-group of the stores issued so far by this thread
__device__ __forceinline__ void uk_bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N of this thread's bulk groups still read their shared
// memory sources (the sources of older groups may be rewritten)
template <int N>
__device__ __forceinline__ void uk_bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N of this thread's bulk groups are incomplete (their
// writes performed)
template <int N>
__device__ __forceinline__ void uk_bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---- tcgen05 -----------------------------------------------------------------
__device__ __forceinline__ void uk_tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(uk_smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void uk_tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void uk_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void uk_tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void uk_tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (both operands f16),
// issued by one thread.
__device__ __forceinline__ void uk_umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// mbarrier arrive (count one) once every tcgen05 op issued so far by this
// thread has completed
__device__ __forceinline__ void uk_umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   uk_smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i)
__device__ __forceinline__ void uk_tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void uk_tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit words from registers into TMEM (the
// inverse of uk_tmem_ld32); uk_tmem_st_wait completes this thread's stores
__device__ __forceinline__ void uk_tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      :
      : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void uk_tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// (sm100 descriptor: start >> 4 at [0,14), LBO >> 4 at [16,30), SBO >> 4 at
// [32,46), version 1 at bit 46, layout type 2 = SWIZZLE_128B at [61,64)).
__device__ __forceinline__ uint64_t uk_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: D f32, A and B f16, A K-major,
// B K-major (b_mn_major = 0) or MN-major (1), shape M x N.
__host__ __device__ constexpr uint32_t uk_idesc_f16(int M, int N, int b_mn_major) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor, kind::f16, with both majors chosen: A K-major (0)
// or MN-major (1) at bit 15, B likewise at bit 16.
__host__ __device__ constexpr uint32_t uk_idesc_f16_ab(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 16 consecutive 32-bit columns: thread i gets lane (base + i)
__device__ __forceinline__ void uk_tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// generic-proxy shared-memory writes become visible to the async proxy
// (tensor core operand reads) of this CTA
__device__ __forceinline__ void uk_fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- thread-block clusters ---------------------------------------------------
__device__ __forceinline__ uint32_t uk_cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster arrives (release) and waits
// (acquire).  All threads of each CTA must reach every such barrier.
__device__ __forceinline__ void uk_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t uk_mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float uk_ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 uk_ld_dsmem_f32x4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

// ---- programmatic dependent launch ------------------------------------------
// the next kernel in the stream (launched with programmatic serialization)
// may start its prologue now
__device__ __forceinline__ void uk_pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// block until the preceding kernel in the stream has completed and its
// memory is visible (a no-op without a programmatic dependency)
__device__ __forceinline__ void uk_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- tf32 ----------------------------------------------------------------------
// D[tmem] (+)= A * B, kind::tf32 (both operands tf32: fp32 bit patterns whose
// low 13 mantissa bits the tensor core ignores), K = 8 per instruction.
__device__ __forceinline__ void uk_umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::tf32: D f32 (bits 4-5 = 1), A and B TF32
// (format 2 at bits 7-9 and 10-12), majors at bits 15 / 16, shape M x N.
__host__ __device__ constexpr uint32_t uk_idesc_tf32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// round to tf32, ties away from zero; the low 13 mantissa bits come back zero
__device__ __forceinline__ float uk_tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r & 0xFFFFE000u);
}

// ---- TMA (tiled, 4-D, single-CTA destination) ------------------------------
// c0 = innermost coordinate (elements; callers keep c0 * elem_size a multiple
// of 16 bytes); the outer coordinates may be negative (zero fill).
__device__ __forceinline__ void uk_tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                               int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(uk_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(uk_smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ---- 2-SM (cta_group::2) forms: a CTA pair of a cluster shares one MMA --------
__device__ __forceinline__ void uk_tmem_alloc_cg2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(uk_smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void uk_tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void uk_tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A * B with M = 256 split over the pair: each CTA
// supplies its 128 rows of A and half of B's N columns from the same shared
// memory offsets; issued by one thread of the even (leader) CTA
__device__ __forceinline__ void uk_umma_f16_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive (count one) on the mbarrier at this shared-memory offset in every CTA
// of `cta_mask` once all prior tcgen05 ops of this thread have completed
__device__ __forceinline__ void uk_umma_commit_cg2(uint64_t* bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(uk_smem_u32(bar)),
               "h"(cta_mask)
               : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the pair's leader CTA (bar_cluster: a shared::cluster address)
__device__ __forceinline__ void uk_tma_load_2d_cg2(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                   int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(uk_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// arrive (count one, release at cluster scope) on an mbarrier of another CTA
__device__ __forceinline__ void uk_mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// uk_mbar_wait with cluster-scope acquire: for barriers that other CTAs of the
// cluster (or their tensor-core commits) arrive on
__device__ __forceinline__ bool uk_mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(uk_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool uk_mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                     uint64_t timeout_ns) {
  if (uk_mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = uk_globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (uk_mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (uk_globaltimer() - t0 > timeout_ns) return false;
    }
  }
}

__device__ __forceinline__ void uk_umma_tf32_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void uk_tma_load_4d_cg2(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                   int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(uk_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
