// uk_common.cuh -- status codes, argument checks and small device helpers
// shared by every translation unit of libunikern_cuda.so.
//
// Status codes keep the meaning of the reference's exit-code protocol
// (src/codegen_hip.cpp:209-293, src/main.cpp:469-539 of UNIKERN):
//   0 ok, 2 invalid argument, 4 CUDA error or refusal,
//   5 a pointer that is not device-resident (managed/host memory is the
//     reference's "oversubscription" signal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "unikern_cuda.h"

namespace uk {

// thread-local text of the last failure, returned by uk_cuda_last_error()
void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);

// 0 when `p` is device memory of the current device; otherwise 2 (NULL) or 5
int check_device_ptr(const void* p, const char* name);
// sticky launch check: returns 4 with the CUDA message on a launch error
int check_launch(const char* what);

int sm_count();  // multiprocessors of the current device (cached per device)

struct Candidate;
// the plan of the last GEMM this thread launched (uk_cuda_last_launch)
void note_launch(const Candidate& c);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace uk

// ---- device helpers ---------------------------------------------------------

__device__ __forceinline__ float uk_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float uk_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Deterministic block-wide reductions (fixed combination order).  `red` must
// hold 33 floats; the call ends with a barrier so `red` can be reused.
template <int THREADS>
__device__ __forceinline__ float uk_block_sum(float v, float* red) {
  constexpr int NW = THREADS / 32;
  v = uk_warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < NW ? red[lane] : 0.f;
    t = uk_warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

template <int THREADS>
__device__ __forceinline__ float uk_block_max(float v, float* red) {
  constexpr int NW = THREADS / 32;
  v = uk_warp_max(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < NW ? red[lane] : -INFINITY;
    t = uk_warp_max(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// W-wide fp32 loads/stores: W = 4 uses 128-bit accesses (caller guarantees
// 16-byte alignment), W = 1 plain scalar accesses.  `cs` = streaming (evict
// first) for data touched once.
template <int W>
__device__ __forceinline__ void uk_ld_cs(float (&d)[W], const float* p) {
  if constexpr (W == 4) {
    const float4 t = __ldcs(reinterpret_cast<const float4*>(p));
    d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
  } else {
    d[0] = __ldcs(p);
  }
}

template <int W>
__device__ __forceinline__ void uk_ld_g(float (&d)[W], const float* p) {
  if constexpr (W == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
  } else {
    d[0] = __ldg(p);
  }
}

template <int W>
__device__ __forceinline__ void uk_st_cs(float* p, const float (&d)[W]) {
  if constexpr (W == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(d[0], d[1], d[2], d[3]));
  } else {
    __stcs(p, d[0]);
  }
}
