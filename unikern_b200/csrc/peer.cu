// peer.cu -- CUDA IPC plumbing for the multi-GPU (one process per GPU) GEMM:
// export a device buffer as an IPC handle, open a peer's handle as a device
// pointer reachable over NVLink.  Handles travel between ranks through the
// caller's process group; this file does no communication itself.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "uk_common.cuh"

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

}  // namespace

extern "C" {

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
