// uk_common.cu -- error text, residency checks and device attributes.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "uk_common.cuh"

namespace uk {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_device_ptr(const void* p, const char* name) {
  if (p == nullptr) return fail(UK_EINVAL, "%s is NULL", name);
  cudaPointerAttributes a{};
  const cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the non-sticky error
    return fail(UK_ERESIDENCY, "%s is not a CUDA allocation (%s)", name, cudaGetErrorString(e));
  }
  if (a.type != cudaMemoryTypeDevice)
    return fail(UK_ERESIDENCY,
                "%s is not device-resident (memory type %d): host or managed memory "
                "is refused as oversubscription",
                name, (int)a.type);
  int dev = -1;
  cudaGetDevice(&dev);
  if (a.device != dev)
    return fail(UK_ERESIDENCY, "%s lives on device %d, the current device is %d", name, a.device, dev);
  return UK_OK;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return UK_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace uk

extern "C" {

const char* uk_cuda_last_error(void) { return uk::g_last_error.c_str(); }

int uk_cuda_abi_version(void) { return 10000; }

int uk_cuda_device_supported(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

}  // extern "C"
