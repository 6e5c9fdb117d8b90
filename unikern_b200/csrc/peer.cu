// peer.cu -- CUDA IPC plumbing for the multi-GPU (one process per GPU) GEMM:
// export a device buffer as an IPC handle, open a peer's handle as a device
// pointer reachable over NVLink.  Handles travel between ranks through the
// caller's process group; this file does no communication itself.  Also the
// device-side barrier of the ranks (uk_cuda_peer_barrier): flags posted into
// every rank's memory over NVLink and waited for with a time limit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "sm100_ptx.cuh"
#include "uk_common.cuh"

namespace uk {
__device__ unsigned int g_fault_word_peer = 0;

unsigned peer_fault_take() {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fault_word_peer, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned zero = 0;
  cudaMemcpyToSymbol(g_fault_word_peer, &zero, sizeof(zero));
  return v;
}
}  // namespace uk

namespace {

// cuMemGetAddressRange from the driver: an IPC handle names a whole
// allocation, so the exporter also reports the offset of `ptr` inside it.
PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuMemGetAddressRange_v3020)p;
  });
  return fn;
}

constexpr int kMaxRanks = 8;

struct FlagList {
  unsigned* f[kMaxRanks];  // every rank's flag array, in rank order (this rank's own included)
};

// One warp: lane r < n posts `epoch` into rank r's array at this rank's slot
// (a release at system scope: everything this GPU wrote before the barrier,
// the sharded GEMM's peer stores included, is visible to rank r first), then
// lane r waits until rank r's post of `epoch` (or a later one) is in this
// rank's own array (an acquire), for at most timeout_ns; on a timeout it
// sets UK_FAULT_PEER and gives up.
__global__ void k_peer_barrier(FlagList fl, int n, int rank, unsigned epoch, uint64_t timeout_ns) {
  const int r = threadIdx.x;
  if (r >= n) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(fl.f[r] + rank), "r"(epoch) : "memory");
  const unsigned* mine = fl.f[rank] + r;
  const uint64_t t0 = uk_globaltimer();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if (uk_globaltimer() - t0 > timeout_ns) {
      atomicOr(&uk::g_fault_word_peer, UK_FAULT_PEER);
      break;
    }
  }
}

}  // namespace

extern "C" {

int uk_cuda_peer_barrier(unsigned* const* flag_list, int n, int rank, unsigned epoch, uint64_t timeout_ns,
                         void* stream) {
  if (flag_list == nullptr || n < 1 || n > kMaxRanks || rank < 0 || rank >= n)
    return uk::fail(UK_EINVAL, "peer_barrier: %d ranks (1..%d), rank %d", n, kMaxRanks, rank);
  if (timeout_ns < 1000ull || timeout_ns > 60000000000ull)
    return uk::fail(UK_EINVAL, "peer_barrier: timeout_ns %llu outside 1 us .. 60 s", (unsigned long long)timeout_ns);
  FlagList fl{};
  for (int i = 0; i < n; ++i) {
    if (flag_list[i] == nullptr || ((uintptr_t)flag_list[i] & 3u) != 0)
      return uk::fail(UK_EINVAL, "peer_barrier: flag array %d is NULL or misaligned", i);
    fl.f[i] = flag_list[i];
  }
  k_peer_barrier<<<1, 32, 0, (cudaStream_t)stream>>>(fl, n, rank, epoch, timeout_ns);
  return uk::check_launch("peer_barrier");
}

int uk_cuda_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (handle_out == nullptr || offset_out == nullptr) return uk::fail(UK_EINVAL, "ipc_export: NULL output");
  if (int rc = uk::check_device_ptr(ptr, "ptr")) return rc;
  auto fn = range_fn();
  if (!fn) return uk::fail(UK_ECUDA, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return uk::fail(UK_ECUDA, "ipc_export: address range failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "ipc_export: %s", cudaGetErrorString(e));
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)((uintptr_t)ptr - (uintptr_t)base);
  return UK_OK;
}

int uk_cuda_ipc_import(const void* handle, uint64_t offset, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return uk::fail(UK_EINVAL, "ipc_import: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "ipc_import: %s", cudaGetErrorString(e));
  *ptr_out = (char*)base + offset;
  return UK_OK;
}

int uk_cuda_ipc_close(void* ptr, uint64_t offset) {
  if (ptr == nullptr) return UK_OK;
  const cudaError_t e = cudaIpcCloseMemHandle((char*)ptr - offset);
  if (e != cudaSuccess) return uk::fail(UK_ECUDA, "ipc_close: %s", cudaGetErrorString(e));
  return UK_OK;
}

size_t uk_cuda_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

}  // extern "C"
