// uk_common.cu -- error text, residency checks and device attributes.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace uk {

static thread_local std::string g_last_error;
static thread_local Candidate g_last_launch;

void note_launch(const Candidate& c) { g_last_launch = c; }

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

int uk_cuda_solve_plan(int op, int f16, const int64_t* dims, int sms, int allow_tc, int* out8) {
  if (dims == nullptr || out8 == nullptr) return uk::fail(UK_EINVAL, "solve_plan: NULL dims or out8");
  if (op != UK_OP_GEMM) return uk::fail(UK_EINVAL, "solve_plan: the candidate grid covers op=gemm (%d given)", op);
  if (sms < 0 || dims[0] < 0 || dims[1] < 0 || dims[2] < 0) return uk::fail(UK_EINVAL, "solve_plan: negative size");
  const int64_t n_sm = sms > 0 ? sms : uk::sm_count();
  int nf = 0;
  const uk::Candidate c = uk::solve_gemm(dims[0], dims[1], dims[2], f16 != 0, allow_tc != 0, n_sm, &nf);
  out8[0] = c.family;
  out8[1] = c.tile.bm;
  out8[2] = c.tile.bn;
  out8[3] = c.tile.bk;
  out8[4] = c.tile.stages;
  out8[5] = c.ksplit;
  out8[6] = nf;
  out8[7] = (int)(c.us * 1000.0 + 0.5);  // ns
  return UK_OK;
}

int uk_cuda_last_launch(int* out6) {
  if (out6 == nullptr) return uk::fail(UK_EINVAL, "last_launch: NULL out6");
  const uk::Candidate& c = uk::g_last_launch;
  out6[0] = c.family;
  out6[1] = c.tile.bm;
  out6[2] = c.tile.bn;
  out6[3] = c.tile.bk;
  out6[4] = c.tile.stages;
  out6[5] = c.ksplit;
  return UK_OK;
}

int uk_cuda_tile_plan(int op, int f16, const int64_t* dims, int sms, int* out4) {
  if (dims == nullptr || out4 == nullptr) return uk::fail(UK_EINVAL, "tile_plan: NULL dims or out4");
  if (sms < 0) return uk::fail(UK_EINVAL, "tile_plan: sms < 0");
  const int64_t n_sm = sms > 0 ? sms : uk::sm_count();
  uk::Tile t{0, 0, 0, 0};
  switch (op) {
    case UK_OP_GEMM: {  // dims M, N, K: the solver's argmin (the launchers take the same)
      const bool tc16 = f16 && dims[2] % 8 == 0 && dims[1] % 8 == 0;
      t = uk::solve_gemm(dims[0], dims[1], dims[2], tc16, /*allow_tc*/ !f16, n_sm).tile;
      break;
    }
    case UK_OP_CONV: {  // KML dims H, W, C, Kh, Kw, Oc (one image, valid)
      const int64_t npix = (dims[0] - dims[3] + 1) * (dims[1] - dims[4] + 1);
      if (f16) t = uk::kConvPairF16Tile;
      else if (dims[2] >= 32 && dims[2] % 32 == 0) t = uk::kConvPairF32Tile;
      else t = uk::conv_tile(npix, dims[5], n_sm);
      break;
    }
    case UK_OP_REDUCE: {  // dims L: one row of L columns
      const uk::ReducePlan p = uk::plan_reduce(1, dims[0], n_sm);
      t = {1, (int)(p.mode == 3 ? p.chunk : dims[0]), 0, (int)(p.mode == 3 ? p.splits : 1)};
      break;
    }
    case UK_OP_SOFTMAX:
    case UK_OP_RMSNORM: {  // dims L, C: one CTA per row, row in registers
      int th = 0, v = 0;
      const int w = dims[1] % 4 == 0 ? 4 : 1;
      if (uk::rowop_plan(dims[1], w, &th, &v)) t = {1, th * v * w, 0, 1};
      else t = {1, 512 * w, 0, 2};  // two-pass streaming kernel
      break;
    }
    case UK_OP_CHANNELSCALE: {  // dims L, C
      const int w = dims[1] % 4 == 0 ? 4 : 1;
      int th = 0, v = 0;
      if (w == 4 && dims[1] >= 2048 && uk::rowop_plan(dims[1], 4, &th, &v)) {
        t = {1, th * v * 4, 0, 1};  // long rows: one CTA per row
        break;
      }
      // 256 threads over (C/W) column vectors x rows, 4 rows each
      const int64_t ncv = (dims[1] + w - 1) / w;
      const int tx = (int)(ncv < 256 ? ((ncv + 31) / 32) * 32 : 256);
      t = {(256 / tx) * 4, tx * w, 0, 1};
      break;
    }
    default:
      return uk::fail(UK_EINVAL, "tile_plan: unknown op %d", op);
  }
  out4[0] = t.bm;
  out4[1] = t.bn;
  out4[2] = t.bk;
  out4[3] = t.stages;
  return UK_OK;
}

}  // extern "C"
