// runner_cuda.cpp -- the nvidia:cuda backend of the KML runner (see
// runner_cuda.hpp for the reference interface each part keeps).
//
// run_cuda executes a KML tree in process through the library's own C ABI:
//   1. verify instance: the reference's exact sawtooth operands at its verify
//      shapes (gemm 256^3, conv 32x32x8 -> 16 with 3x3, reduce 2^20 x 2^-6,
//      the row ops at the full declared shape), checked on the GPU by the fp64
//      checker kernels against the dtype's gate (2^-5 fp32, 2^-4 fp16);
//   2. timing at the declared dims: e2e passes (H2D of the inputs from pinned
//      host memory, the launch, D2H of the output) and kernel-only launches,
//      CUDA events on one stream; warm/iters as the reference (2/10, or 1/1
//      when the payload exceeds 2 GiB; the fp16 gemm and the row ops warm once);
//   3. the UNIKERN_RESULT line with the reference's tokens.
// A payload above 0.85 x the device budget (the HCS's device tier, capped by
// the device's own reported memory) runs streamed when it is a GEMM whose B
// fits beside a ring of row blocks (scenario B: verified through the ring,
// mode=streamed on the result line); anything else is refused with
// stream_refused.  The file also holds the solver, the TAB file ledger and
// calibration.
#include "runner_cuda.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <limits>
#include <sstream>
#include <unistd.h>
#include <vector>

#include "runner_dev.h"
#include "unikern_cuda.h"

namespace ukb {

namespace {

int uk_op_of(OpKind k) {
  switch (k) {
    case OpKind::Gemm: return UK_OP_GEMM;
    case OpKind::Conv: return UK_OP_CONV;
    case OpKind::Reduction: return UK_OP_REDUCE;
    case OpKind::Softmax: return UK_OP_SOFTMAX;
    case OpKind::RmsNorm: return UK_OP_RMSNORM;
    case OpKind::ChannelScale: return UK_OP_CHANNELSCALE;
  }
  return -1;
}

std::string perf_string(const KmlTree& t) {
  std::string s;
  for (int i = 0; i < kml_arity(t.op); ++i) s += (i ? "x" : "") + std::to_string(t.dims[i]);
  return s;
}

// bytes the declared tree keeps resident on the device while it is timed
int64_t payload_bytes(const KmlTree& t, size_t op_ws) {  // op_ws: the reduce / conv workspace
  const int64_t* d = nullptr;
  int64_t v[6];
  for (int i = 0; i < 6; ++i) v[i] = t.dims[i];
  d = v;
  const int64_t es = dtype_bytes(t.dtype);
  switch (t.op) {
    case OpKind::Gemm: return (d[0] * d[2] + d[2] * d[1] + d[0] * d[1]) * es;
    case OpKind::Conv:
      return (d[0] * d[1] * d[2] + d[5] * d[3] * d[4] * d[2] + d[5] * (d[0] - d[3] + 1) * (d[1] - d[4] + 1)) * es +
             (int64_t)op_ws;
    case OpKind::Reduction: return d[0] * es + (int64_t)op_ws + es;
    case OpKind::Softmax: return 2 * d[0] * d[1] * es;
    case OpKind::RmsNorm:
    case OpKind::ChannelScale: return (2 * d[0] * d[1] + d[1]) * es;
  }
  return 0;
}

// device allocations of one run, residency-probed like the reference's
// uk_mmalloc (each allocation is one check; a non-device type is a migration)
struct DevArena {
  std::vector<void*> dev, host;
  int checks = 0, migrations = 0;
  std::string err;
  ~DevArena() {
    for (void* p : dev) cudaFree(p);
    for (void* p : host) cudaFreeHost(p);
  }
  void* alloc(size_t bytes, const char* what) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
      cudaGetLastError();
      err = std::string("cudaMalloc ") + what + " (" + std::to_string(bytes) + " B) failed";
      return nullptr;
    }
    dev.push_back(p);
    cudaPointerAttributes a{};
    ++checks;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      ++migrations;
    }
    return p;
  }
  void* pinned(size_t bytes, const char* what) {
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes ? bytes : 16) != cudaSuccess) {
      cudaGetLastError();
      err = std::string("cudaMallocHost ") + what + " (" + std::to_string(bytes) + " B) failed";
      return nullptr;
    }
    host.push_back(p);
    return p;
  }
};

// one op invocation through the C ABI
struct OpCall {
  OpKind op = OpKind::Gemm;
  bool f16 = false;
  int64_t d[6] = {0, 0, 0, 0, 0, 0};
  void* in0 = nullptr;   // A / X
  void* in1 = nullptr;   // B / Wt / W / S (null for softmax, reduce)
  void* out = nullptr;   // C / Y
  void* ws = nullptr;    // reduce / conv / tensor-core fp32 gemm workspace
  size_t ws_bytes = 0;
  bool tc32 = false;     // fp32 gemm on the tensor cores (split-tf32)
  int64_t width = 0;     // reduce: pinned pass-1 width (UK_REDUCE_WIDTH), 0 = the plan
  int launch(cudaStream_t st) const {
    switch (op) {
      case OpKind::Gemm:
        if (f16)
          return uk_cuda_gemm_f16((const uint16_t*)in0, (const uint16_t*)in1, (uint16_t*)out, (int)d[0], (int)d[1],
                                  (int)d[2], st);
        return uk_cuda_gemm_f32_ws((const float*)in0, (const float*)in1, (float*)out, (int)d[0], (int)d[1], (int)d[2],
                                   tc32 ? ws : nullptr, tc32 ? ws_bytes : 0, st);
      case OpKind::Conv:
        if (f16)  // fp16: kind::f16 tensor cores, the KML input read in place
          return uk_cuda_conv2d_f16((const uint16_t*)in0, (const uint16_t*)in1, (uint16_t*)out, 1, (int)d[0],
                                    (int)d[1], (int)d[2], (int)d[3], (int)d[4], (int)d[5], 0, nullptr, UK_CONV_KML,
                                    ws, ws_bytes, st);
        // fp32: tensor cores when C % 32 == 0 (workspace sized for it), else FFMA
        return uk_cuda_conv2d_f32_ws((const float*)in0, (const float*)in1, (float*)out, 1, (int)d[0], (int)d[1],
                                     (int)d[2], (int)d[3], (int)d[4], (int)d[5], 0, nullptr, UK_CONV_KML, ws,
                                     ws_bytes, st);
      case OpKind::Reduction:
        if (f16)  // widening: binary16 in and out, fp32 sums
          return width > 0 ? uk_cuda_reduce_f16_width((const uint16_t*)in0, (uint16_t*)out, 1, d[0], width, ws,
                                                      ws_bytes, st)
                           : uk_cuda_reduce_f16((const uint16_t*)in0, (uint16_t*)out, 1, d[0], ws, ws_bytes, st);
        return width > 0 ? uk_cuda_reduce_f32_width((const float*)in0, (float*)out, 1, d[0], width, ws, ws_bytes, st)
                         : uk_cuda_reduce_f32((const float*)in0, (float*)out, 1, d[0], ws, ws_bytes, st);
      case OpKind::Softmax:
        return f16 ? uk_cuda_softmax_f16((const uint16_t*)in0, (uint16_t*)out, d[0], d[1], st)
                   : uk_cuda_softmax_f32((const float*)in0, (float*)out, d[0], d[1], st);
      case OpKind::RmsNorm:
        // the KML contract's eps (src/codegen_hip.cpp:2162, :2175)
        return f16 ? uk_cuda_rmsnorm_f16((const uint16_t*)in0, (const uint16_t*)in1, (uint16_t*)out, d[0], d[1],
                                         1e-6f, st)
                   : uk_cuda_rmsnorm_f32((const float*)in0, (const float*)in1, (float*)out, d[0], d[1], 1e-6f, st);
      case OpKind::ChannelScale:
        return f16 ? uk_cuda_channelscale_f16((const uint16_t*)in0, (const uint16_t*)in1, (uint16_t*)out, d[0], d[1],
                                              st)
                   : uk_cuda_channelscale_f32((const float*)in0, (const float*)in1, (float*)out, d[0], d[1], st);
    }
    return UK_EINVAL;
  }
  // element counts of in0 / in1 / out
  int64_t n_in0() const {
    switch (op) {
      case OpKind::Gemm: return d[0] * d[2];
      case OpKind::Conv: return d[0] * d[1] * d[2];
      case OpKind::Reduction: return d[0];
      default: return d[0] * d[1];
    }
  }
  int64_t n_in1() const {
    switch (op) {
      case OpKind::Gemm: return d[2] * d[1];
      case OpKind::Conv: return d[5] * d[3] * d[4] * d[2];
      case OpKind::RmsNorm:
      case OpKind::ChannelScale: return d[1];
      default: return 0;
    }
  }
  int64_t n_out() const {
    switch (op) {
      case OpKind::Gemm: return d[0] * d[1];
      case OpKind::Conv: return d[5] * (d[0] - d[3] + 1) * (d[1] - d[4] + 1);
      case OpKind::Reduction: return 1;
      default: return d[0] * d[1];
    }
  }
  size_t es() const { return f16 ? 2 : 4; }
};

// allocate and fill the operands of `c` with the reference's initialisers
bool stage_operands(OpCall* c, DevArena* ar, cudaStream_t st, std::string* err) {
  c->in0 = ar->alloc(c->n_in0() * c->es(), "in0");
  if (c->n_in1() > 0) c->in1 = ar->alloc(c->n_in1() * c->es(), "in1");
  c->out = ar->alloc(c->n_out() * c->es(), "out");
  if (c->op == OpKind::Reduction)
    c->ws_bytes = c->width > 0 ? uk_cuda_reduce_workspace_size_width(1, c->d[0], c->width)
                               : uk_cuda_reduce_workspace_size(1, c->d[0]);
  if (c->op == OpKind::Gemm && c->tc32)
    c->ws_bytes = uk_cuda_gemm_f32_workspace_size((int)c->d[0], (int)c->d[1], (int)c->d[2]);
  if (c->op == OpKind::Conv)
    c->ws_bytes = c->f16 ? uk_cuda_conv2d_f16_workspace_size(1, (int)c->d[0], (int)c->d[1], (int)c->d[2],
                                                             (int)c->d[3], (int)c->d[4], (int)c->d[5], 0, UK_CONV_KML)
                         : uk_cuda_conv2d_workspace_size(1, (int)c->d[0], (int)c->d[1], (int)c->d[2], (int)c->d[3],
                                                         (int)c->d[4], (int)c->d[5], 0, UK_CONV_KML);
  if (c->ws_bytes) c->ws = ar->alloc(c->ws_bytes, "workspace");
  if (!ar->err.empty()) {
    *err = ar->err;
    return false;
  }
  const int k0 = c->op == OpKind::Reduction ? UKR_SAW_CONST : UKR_SAW_A;
  const int k1 = (c->op == OpKind::RmsNorm || c->op == OpKind::ChannelScale) ? UKR_SAW_W : UKR_SAW_B;
  if (ukr_saw_fill(c->in0, c->n_in0(), k0, c->f16, st) != UK_OK ||
      (c->in1 && ukr_saw_fill(c->in1, c->n_in1(), k1, c->f16, st) != UK_OK)) {
    *err = uk_cuda_last_error();
    return false;
  }
  return true;
}

bool cuda_ok(cudaError_t e, const char* what, std::string* err) {
  if (e == cudaSuccess) return true;
  *err = std::string(what) + ": " + cudaGetErrorString(e);
  return false;
}

}  // namespace

// ---- backend descriptor --------------------------------------------------------

bool BackendNvidia::available() const {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return false;
  }
  return uk_cuda_device_supported() != 0;
}

std::string BackendNvidia::capability_gap(const KmlTree& t) const {
  if (t.layout != "NT") return "layout=" + t.layout + " (only NT is implemented)";
  if (t.dtype == DType::I8) return std::string("dtype=int8 for op=") + op_name(t.op) + " (nvidia:cuda runs fp32 ops and the fp16 gemm)";
  if (t.dtype == DType::F16 && t.op == OpKind::Conv && t.dims[2] % 64 != 0)
    return "dtype=fp16 conv with C=" + std::to_string(t.dims[2]) + " (the fp16 conv needs C a multiple of 64)";
  if (!t.children.empty()) return "children (a composite tree executes per op; declare each op on its own)";
  if (t.op == OpKind::Conv && (t.dims[3] > t.dims[0] || t.dims[4] > t.dims[1]))
    return "conv filter larger than the input";
  return "";
}

std::string BackendNvidia::generate(const Solution& s, const Hcs& h, const KmlTree& t) const {
  std::ostringstream os;
  os << "// nvidia:cuda: precompiled sm_100a kernels of libunikern_cuda.so (no source is generated)\n"
     << "// tree " << canonical_form(t) << "\n// device " << h.device << "\n// tile " << s.best.tile_m << "x"
     << s.best.tile_n << " k_block=" << s.best.k_block << " stages=" << s.best.stages << "\n";
  return os.str();
}

// ---- scenario B ----------------------------------------------------------------

// A GEMM whose operands exceed 0.85 x the device budget runs streamed (the
// reference's scenario B, src/codegen_hip.cpp:1485-1500): B stays resident
// and A, C pass through a two-slot ring of row blocks.  Returns the block
// rows (a multiple of 256 where the budget allows, else of 32), or 0 when
// the payload fits (resident), the op is not a GEMM, or B plus the smallest
// ring does not fit the budget.
int64_t stream_block_rows(const KmlTree& t, int64_t payload, double budget_bytes, int* kind_out) {
  if (double(payload) <= 0.85 * budget_bytes || t.op != OpKind::Gemm) return 0;
  const int M = t.dims[0], N = t.dims[1], K = t.dims[2];
  const double room = 0.85 * budget_bytes - double(K) * double(N) * double(dtype_bytes(t.dtype));
  // the largest multiple of 32 rows in [32 * lo, M] whose ring fits, 0 if
  // none (in that range the ring of this kind takes one kernel and grows with
  // the rows)
  auto largest = [&](int kind, int64_t lo) -> int64_t {
    auto fits = [&](int64_t rows) {
      return double(uk_cuda_gemm_streamed_ring_size(M, N, K, kind, (int)rows)) <= room;
    };
    int64_t hi = ((int64_t)M + 31) / 32;
    if (room <= 0 || lo > hi || !fits(lo * 32)) return 0;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) / 2;
      if (fits(mid * 32)) lo = mid;
      else hi = mid - 1;
    }
    return lo * 32;
  };
  auto round256 = [](int64_t r) { return r >= 256 ? r / 256 * 256 : r; };
  if (t.dtype == DType::F16) {
    const int64_t rows = round256(largest(1, 1));
    if (rows == 0) return 0;
    if (kind_out) *kind_out = 1;
    return rows < M ? rows : M;
  }
  // fp32: blocks from the first 256-multiple of rows that gains from the
  // tensor cores (their ring also holds the tf32 pairs of B^T) when such a
  // ring fits, else the FFMA ring
  int64_t rows = 0;
  int kind = 2;
  if (uk_cuda_gemm_f32_prefers_tc(M, N, K)) {
    int64_t r_tc = 256;
    while (r_tc < M && !uk_cuda_gemm_f32_prefers_tc((int)r_tc, N, K)) r_tc += 256;
    const int64_t r = round256(largest(0, std::min<int64_t>(r_tc, M) / 32));
    if (r > 0 && uk_cuda_gemm_f32_prefers_tc((int)std::min<int64_t>(r, M), N, K)) {
      rows = r;
      kind = 0;
    }
  }
  if (rows == 0) rows = round256(largest(2, 1));
  if (rows == 0) return 0;
  if (kind_out) *kind_out = kind;
  return rows < M ? rows : M;
}

// ---- solver ------------------------------------------------------------------

Solution solve_b200(const Hcs& h, const KmlTree& t, int sms) {
  Solution s;
  int64_t dims[6];
  for (int i = 0; i < 6; ++i) dims[i] = t.dims[i];
  int tile[4] = {0, 0, 0, 0};
  if (uk_cuda_tile_plan(uk_op_of(t.op), t.dtype == DType::F16, dims, sms, tile) != UK_OK) return s;
  s.best = {tile[0], tile[1], tile[2], tile[3]};
  s.feasible_count = 1;
  // a GEMM is solved over the candidate grid (kernel family x tile x K split);
  // |X| is the number of feasible candidates, the tile the argmin's
  std::string family;
  int ksplit = 1;
  double device_us = 0;
  if (t.op == OpKind::Gemm) {
    const bool f16 = t.dtype == DType::F16;
    int plan[8] = {0};
    if (uk_cuda_solve_plan(UK_OP_GEMM, f16 && dims[1] % 8 == 0 && dims[2] % 8 == 0, dims, sms, !f16, plan) ==
        UK_OK) {
      static const char* names[] = {"ffma", "tcgen05-1sm", "tcgen05-2sm", "tcgen05-2sm-3xtf32"};
      family = plan[0] >= 0 && plan[0] < 4 ? names[plan[0]] : "?";
      ksplit = plan[5];
      s.feasible_count = plan[6];
      device_us = plan[7] / 1000.0;
    }
  }
  // predicted time: compute or device memory, whichever binds, scaled by the
  // SMs a tile grid leaves idle; plus the host link copies that the measured
  // (end-to-end) time includes
  const Workload w = workload_of(t);
  const double flops = h.flops_gflops * 1e9;
  const double dev_bw = h.tier_bw(h.unified_memory ? "unified" : "vram") * 1e9;
  double comp = flops > 0 ? double(w.ops) / flops * 1e3 : 1e18;
  const double mem = dev_bw > 0 ? double(w.bytes) / dev_bw * 1e3 : 1e18;
  if (t.op == OpKind::Gemm || t.op == OpKind::Conv) {
    const int64_t rows = t.op == OpKind::Gemm ? dims[0] : dims[5];
    const int64_t cols = t.op == OpKind::Gemm ? dims[1] : (dims[0] - dims[3] + 1) * (dims[1] - dims[4] + 1);
    const int64_t ctas = ((rows + tile[0] - 1) / tile[0]) * ((cols + tile[1] - 1) / tile[1]);
    const int64_t units = h.compute_units > 0 ? h.compute_units : 148;
    if (ctas < units) comp *= double(units) / double(ctas > 0 ? ctas : 1);
  }
  const double copy = h.unified_memory || h.link_bw_gbps <= 0 ? 0.0 : double(w.bytes) / (h.link_bw_gbps * 1e9) * 1e3;
  const int64_t payload = payload_bytes(t, 0);
  int kind = 0;
  const int64_t rows = stream_block_rows(t, payload, double(h.device_capacity()), &kind);
  std::ostringstream pr;
  if (rows == 0 && h.device_capacity() > 0 && double(payload) > 0.85 * double(h.device_capacity())) {
    s.c_ms = std::max(comp, mem) + copy;
    pr << "placement: refused on " << h.device << " (the payload exceeds 0.85 x the device tier and only a gemm "
       << "whose B fits streams) path=none";
  } else if (rows > 0) {
    // streamed: the ring overlaps the copies with the block GEMMs
    s.c_ms = std::max(std::max(comp, mem), copy);
    pr << "placement: streamed on " << h.device << " (sm_100a; B resident, A/C in a two-slot ring of " << rows
       << "-row blocks" << (kind == 0 ? ", split-tf32 tensor cores" : kind == 2 ? ", FFMA" : "") << ") tile=" << tile[0] << "x" << tile[1] << " k_block=" << tile[2] << " stages=" << tile[3]
       << " path=pinned-copy";
  } else {
    s.c_ms = std::max(comp, mem) + copy;
    pr << "placement: resident on " << h.device << " (sm_100a) tile=" << tile[0] << "x" << tile[1]
       << " k_block=" << tile[2] << " stages=" << tile[3] << " path=pinned-copy";
  }
  if (!family.empty())
    pr << " kernel=" << family << " k_split=" << ksplit << " predicted_device_us=" << device_us;
  s.placement_record = pr.str();
  return s;
}

// ---- run_cuda ------------------------------------------------------------------

RunOutcome run_cuda(const Solution& sol, const Hcs& hcs, const KmlTree& tree, const std::string& workdir) {
  (void)sol;
  (void)hcs;
  (void)workdir;  // nothing is generated or compiled, so nothing is written
  RunOutcome r;
  std::ostringstream log;
  auto finish = [&]() {
    r.log = log.str();
    return r;
  };
  BackendNvidia be;
  if (!be.available()) {
    log << "nvidia:cuda: no CUDA device of compute capability 10.0 (B200) is visible\n";
    r.exit_code = 4;
    return finish();
  }
  const std::string gap = be.capability_gap(tree);
  if (!gap.empty()) {
    log << "UNSUPPORTED: " << gap << "\n";
    r.exit_code = 2;
    return finish();
  }
  r.built = true;  // the precompiled sm_100a kernels load on this device
  size_t fr = 0, tot = 0;
  cudaMemGetInfo(&fr, &tot);
  r.vram_free = fr;
  r.vram_total = tot;

  OpCall timed;
  timed.op = tree.op;
  timed.f16 = tree.dtype == DType::F16;
  for (int i = 0; i < 6; ++i) timed.d[i] = tree.dims[i];
  // an fp32 gemm large enough to gain from the tensor cores runs split-tf32
  timed.tc32 = tree.op == OpKind::Gemm && !timed.f16 &&
               uk_cuda_gemm_f32_prefers_tc(tree.dims[0], tree.dims[1], tree.dims[2]);
  // measurement knobs, requested through the environment and reported, never
  // silently dropped (src/codegen_hip.cpp:874-908, :1338-1355)
  if (tree.op == OpKind::Reduction) {
    const int64_t n = tree.dims[0];
    const char* pin = std::getenv("UK_REDUCE_WIDTH");
    if (pin != nullptr && *pin != 0) {
      char* end = nullptr;
      const long long pw = std::strtoll(pin, &end, 10);
      if (end == pin || *end != 0 || pw < 256 || pw > n) {
        r.result_line = std::string("UNIKERN_ERROR what=reduce_width_pin_unfit value=") + pin +
                        " needs an integer in [256, n=" + std::to_string(n) + "]; the plan is NOT silently fallen back";
        log << r.result_line << "\n";
        r.exit_code = 2;
        return finish();
      }
      timed.width = pw;
      log << "UNIKERN_INFO reduce_width source=env width=" << pw << " cap=0 n=" << n << "\n";
    } else {
      int out4[4] = {0, 0, 0, 0};
      const int64_t dims[6] = {n, 0, 0, 0, 0, 0};
      const int sms = hcs.compute_units > 0 ? hcs.compute_units : 148;
      uk_cuda_tile_plan(UK_OP_REDUCE, 0, dims, 0, out4);
      log << "UNIKERN_INFO reduce_width source=plan width=" << out4[3] << " cap=" << 8 * sms << " n=" << n << "\n";
    }
  }
  std::string stream_path_src = "plan";
  if (tree.op == OpKind::Gemm) {
    const char* pin = std::getenv("UK_GEMM_STREAM_PATH");
    if (pin != nullptr && *pin != 0 && std::strcmp(pin, "auto") != 0) {
      if (std::strcmp(pin, "pinned") != 0) {
        r.result_line = std::string("UNIKERN_ERROR what=stream_path_pin_unfit val=") + pin +
                        (std::strcmp(pin, "mmap") == 0
                             ? " (nvidia:cuda streams through page-locked copies only; the emulated mmap arm is not built)"
                             : "");
        log << r.result_line << "\n";
        r.exit_code = 2;
        return finish();
      }
      stream_path_src = "env";
    }
  }
  const size_t ws = tree.op == OpKind::Reduction
                        ? (timed.width > 0 ? uk_cuda_reduce_workspace_size_width(1, tree.dims[0], timed.width)
                                           : uk_cuda_reduce_workspace_size(1, tree.dims[0]))
                    : tree.op == OpKind::Conv && tree.dtype == DType::F32
                        ? uk_cuda_conv2d_workspace_size(1, tree.dims[0], tree.dims[1], tree.dims[2], tree.dims[3],
                                                        tree.dims[4], tree.dims[5], 0, UK_CONV_KML)
                    : tree.op == OpKind::Conv
                        ? uk_cuda_conv2d_f16_workspace_size(1, tree.dims[0], tree.dims[1], tree.dims[2], tree.dims[3],
                                                            tree.dims[4], tree.dims[5], 0, UK_CONV_KML)
                    : timed.tc32 ? uk_cuda_gemm_f32_workspace_size(tree.dims[0], tree.dims[1], tree.dims[2])
                                 : 0;
  const int64_t payload = payload_bytes(tree, ws);
  const double payload_mb = double(payload) / (1024.0 * 1024.0);
  // the device budget: the HCS's declared device tier, never more than the
  // device reports (a smaller HCS tier models a smaller device)
  const int64_t declared = hcs.device_capacity();
  const double budget = double(declared > 0 && (uint64_t)declared < tot ? (uint64_t)declared : tot);
  int stream_kind = 0;  // uk_cuda_gemm_streamed's kind
  const int64_t stream_rows = stream_block_rows(tree, payload, budget, &stream_kind);  // > 0: scenario B
  // the streamed fp32 blocks take the tensor cores when the block shape gains
  const bool stream_tc = stream_rows > 0 && stream_kind == 0 &&
                         uk_cuda_gemm_f32_prefers_tc((int)stream_rows, tree.dims[1], tree.dims[2]);
  if (double(payload) > 0.85 * budget) {
    // the streamed operands live in page-locked host memory: at most half of
    // the host's RAM (and of the HCS's host tier where it declares one)
    const int64_t es = dtype_bytes(tree.dtype);
    const double host_need =
        double(tree.dims[0] * tree.dims[2] + tree.dims[2] * tree.dims[1] + tree.dims[0] * tree.dims[1]) * double(es);
    double host_cap = double(sysconf(_SC_PHYS_PAGES)) * double(sysconf(_SC_PAGE_SIZE));
    const int64_t ram = hcs.tier_bytes("ram");
    if (ram > 0 && double(ram) < host_cap) host_cap = double(ram);
    if (stream_rows == 0 || host_need > 0.5 * host_cap) {
      std::ostringstream e;
      e << "UNIKERN_ERROR what=stream_refused payload_mb=" << std::fixed << std::setprecision(6) << payload_mb
        << " vram_total=" << tot << " ("
        << (stream_rows == 0 ? "the payload exceeds 0.85 * the device budget and only a gemm whose B fits streams"
                             : "the streamed operands exceed half of the host's memory")
        << "; nothing ran)";
      r.result_line = e.str();
      log << r.result_line << "\n";
      r.exit_code = 4;
      return finish();
    }
  }
  const bool big = payload > (int64_t(2) << 30);
  const bool warm_once = timed.f16 || tree.op == OpKind::Softmax || tree.op == OpKind::RmsNorm ||
                         tree.op == OpKind::ChannelScale;
  const int warm = big || warm_once ? 1 : 2, iters = big ? 1 : 10;

  cudaStream_t st = nullptr;
  std::string err;
  if (!cuda_ok(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate", &err)) {
    log << err << "\n";
    r.exit_code = 4;
    return finish();
  }
  DevArena ar;
  int rc = UK_OK;
  bool ok = true;

  // ---- 1. verify instance ----
  {
    OpCall v = timed;
    v.tc32 = timed.tc32 && stream_rows == 0;  // a streamed run verifies through the ring
    if (tree.op == OpKind::Gemm) {
      // the reference's 256^3; a streamed fp32 gemm on the tensor cores
      // verifies 2048 x 1024 x 1024 in two 1024-row blocks, the smallest
      // streamed instance whose blocks take them (still exact: every partial
      // sum of the sawtooth operands is representable)
      v.d[0] = v.d[1] = v.d[2] = 256;
      if (stream_tc) v.d[0] = 2048, v.d[1] = v.d[2] = 1024;
    } else if (tree.op == OpKind::Conv) {
      // the reference's instance (32 x 32 x 8 -> 16, 3 x 3); the fp16 conv
      // takes 64-channel steps, so its instance has 64 input channels
      const int64_t vd[6] = {32, 32, timed.f16 ? 64 : 8, 3, 3, 16};
      for (int i = 0; i < 6; ++i) v.d[i] = vd[i];
    } else if (tree.op == OpKind::Reduction) {
      v.d[0] = int64_t(1) << 20;
    }
    double* worst = static_cast<double*>(ar.alloc(sizeof(double), "max_rel"));
    ok = worst && stage_operands(&v, &ar, st, &err) &&
         cuda_ok(cudaMemsetAsync(worst, 0, sizeof(double), st), "memset max_rel", &err);
    if (ok && stream_rows > 0) {
      // scenario B verifies the streamed path itself: the instance through
      // the ring (256^3 in four 64-row blocks, or the tensor-core instance
      // above in two), from and to pinned memory
      const int vm = (int)v.d[0], vn = (int)v.d[1], vk = (int)v.d[2], vr = stream_tc ? 1024 : 64;
      const size_t es = v.es();
      const size_t rb = uk_cuda_gemm_streamed_ring_size(vm, vn, vk, stream_kind, vr);
      void* hA = ar.pinned((size_t)vm * vk * es, "A");
      void* hB = ar.pinned((size_t)vk * vn * es, "B");
      void* hC = ar.pinned((size_t)vm * vn * es, "C");
      void* ring = ar.alloc(rb, "ring");
      ok = ar.err.empty();
      if (!ok) err = ar.err;
      ok = ok && cuda_ok(cudaMemcpyAsync(hA, v.in0, (size_t)vm * vk * es, cudaMemcpyDeviceToHost, st), "stage A", &err) &&
           cuda_ok(cudaMemcpyAsync(hB, v.in1, (size_t)vk * vn * es, cudaMemcpyDeviceToHost, st), "stage B", &err);
      if (ok && uk_cuda_gemm_streamed(hA, hB, hC, v.in1, ring, rb, vm, vn, vk, stream_kind, vr, st) != UK_OK) {
        err = uk_cuda_last_error();
        ok = false;
      }
      ok = ok && cuda_ok(cudaMemcpyAsync(v.out, hC, (size_t)vm * vn * es, cudaMemcpyHostToDevice, st), "return C",
                         &err);
    } else if (ok && (rc = v.launch(st)) != UK_OK) {
      err = uk_cuda_last_error();
      ok = false;
    }
    if (ok) {
      switch (tree.op) {
        case OpKind::Gemm:
          rc = ukr_check_gemm(v.in0, v.in1, v.out, (int)v.d[0], (int)v.d[1], (int)v.d[2], v.f16, worst, st);
          break;
        case OpKind::Conv:
          rc = ukr_check_conv(v.in0, v.in1, v.out, (int)v.d[0], (int)v.d[1], (int)v.d[2], (int)v.d[3],
                              (int)v.d[4], (int)v.d[5], v.f16, worst, st);
          break;
        case OpKind::Reduction:
          rc = ukr_check_rows(UKR_OP_REDUCE, v.in0, nullptr, v.out, 1, v.d[0], 0.0, v.f16, worst, st);
          break;
        case OpKind::Softmax:
          rc = ukr_check_rows(UKR_OP_SOFTMAX, v.in0, nullptr, v.out, v.d[0], v.d[1], 0.0, v.f16, worst, st);
          break;
        case OpKind::RmsNorm:
          rc = ukr_check_rows(UKR_OP_RMSNORM, v.in0, v.in1, v.out, v.d[0], v.d[1], (double)1e-6f, v.f16, worst, st);
          break;
        case OpKind::ChannelScale:
          rc = ukr_check_rows(UKR_OP_CHANNELSCALE, v.in0, v.in1, v.out, v.d[0], v.d[1], 0.0, v.f16, worst, st);
          break;
      }
      if (rc != UK_OK) {
        err = uk_cuda_last_error();
        ok = false;
      }
    }
    double host_worst = 0;
    ok = ok && cuda_ok(cudaMemcpyAsync(&host_worst, worst, sizeof(double), cudaMemcpyDeviceToHost, st),
                       "read max_rel", &err) &&
         cuda_ok(cudaStreamSynchronize(st), "verify", &err);
    if (ok) {
      r.max_rel = host_worst;
      r.verified = host_worst <= tolerance_for(tree.dtype);
    }
    // the verify buffers are released before the timed payload is allocated
    for (void* p : ar.dev) cudaFree(p);
    ar.dev.clear();
  }

  // ---- 2a. scenario B: the GEMM streamed through a ring (B resident) ----
  if (ok && stream_rows > 0) {
    log << "UNIKERN_INFO mode=streamed shards=" << (tree.dims[0] + stream_rows - 1) / stream_rows
        << " shard_rows=" << stream_rows << " prefetch_d=2 stream_path=pinned source=" << stream_path_src
        << " plan=pinned kernel=" << (stream_kind == 1 ? "f16" : stream_tc ? "split-tf32" : "ffma") << "\n";
    const int64_t M = tree.dims[0], N = tree.dims[1], K = tree.dims[2];
    const size_t es = timed.es();
    const size_t ring_bytes = uk_cuda_gemm_streamed_ring_size((int)M, (int)N, (int)K, stream_kind, (int)stream_rows);
    void* dB = ar.alloc((size_t)K * N * es, "B");
    void* ring = ar.alloc(ring_bytes, "ring");
    void* hA = ar.pinned((size_t)M * K * es, "A");
    void* hB = ar.pinned((size_t)K * N * es, "B");
    void* hC = ar.pinned((size_t)M * N * es, "C");
    if (!ar.err.empty()) {
      err = ar.err;
      ok = false;
    }
    // the host operands get the sawtooth values, a ring-sized block at a time
    ok = ok && ukr_saw_fill(dB, K * N, UKR_SAW_B, timed.f16, st) == UK_OK &&
         cuda_ok(cudaMemcpyAsync(hB, dB, (size_t)K * N * es, cudaMemcpyDeviceToHost, st), "stage B", &err);
    for (int64_t r0 = 0; ok && r0 < M; r0 += stream_rows) {
      const int64_t nr = r0 + stream_rows < M ? stream_rows : M - r0;
      ok = ukr_saw_fill_at(ring, nr * K, r0 * K, UKR_SAW_A, timed.f16, st) == UK_OK &&
           cuda_ok(cudaMemcpyAsync((uint8_t*)hA + r0 * K * es, ring, nr * K * es, cudaMemcpyDeviceToHost, st),
                   "stage A", &err) &&
           cuda_ok(cudaStreamSynchronize(st), "stage", &err);
    }
    auto pass = [&]() -> bool {
      if (uk_cuda_gemm_streamed(hA, hB, hC, dB, ring, ring_bytes, (int)M, (int)N, (int)K, stream_kind,
                                (int)stream_rows, st) != UK_OK) {
        err = uk_cuda_last_error();
        return false;
      }
      return true;
    };
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ok) ok = cuda_ok(cudaEventCreate(&e0), "event", &err) && cuda_ok(cudaEventCreate(&e1), "event", &err);
    for (int i = 0; ok && i < warm; ++i) ok = pass();
    double total = 0;
    for (int i = 0; ok && i < iters; ++i) {
      float ms = 0;
      ok = cuda_ok(cudaEventRecord(e0, st), "record", &err) && pass() &&
           cuda_ok(cudaEventRecord(e1, st), "record", &err) && cuda_ok(cudaEventSynchronize(e1), "sync", &err) &&
           cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "elapsed", &err);
      total += ms;
    }
    if (ok) {
      // kernel-only: the device work of one pass (B's pre-pass on the tensor
      // cores, every block's GEMM) without the copies, on the ring's first slot
      r.measured_ms = total / iters;
      float ms = 0;
      ok = cuda_ok(cudaEventRecord(e0, st), "record", &err);
      for (int i = 0; ok && i < iters; ++i)
        if (ukr_gemm_streamed_kernels(dB, ring, ring_bytes, (int)M, (int)N, (int)K, stream_kind, (int)stream_rows,
                                      st) != UK_OK) {
          err = uk_cuda_last_error();
          ok = false;
        }
      ok = ok && cuda_ok(cudaEventRecord(e1, st), "record", &err) &&
           cuda_ok(cudaEventSynchronize(e1), "sync", &err) && cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "elapsed", &err);
      r.kernel_ms = double(ms) / iters;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
  }

  // ---- 2. timing at the declared dims (resident) ----
  if (stream_rows == 0) {
    ok = ok && stage_operands(&timed, &ar, st, &err);
    void *h0 = nullptr, *h1 = nullptr, *hout = nullptr;
    const size_t b0 = timed.n_in0() * timed.es(), b1 = timed.n_in1() * timed.es(), bo = timed.n_out() * timed.es();
    if (ok) {
      h0 = ar.pinned(b0, "in0");
      h1 = b1 ? ar.pinned(b1, "in1") : nullptr;
      hout = ar.pinned(bo, "out");
      if (!ar.err.empty()) {
        err = ar.err;
        ok = false;
      }
    }
    // the host copies hold the same sawtooth values as the device operands
    ok = ok && cuda_ok(cudaMemcpyAsync(h0, timed.in0, b0, cudaMemcpyDeviceToHost, st), "stage in0", &err) &&
         (!b1 || cuda_ok(cudaMemcpyAsync(h1, timed.in1, b1, cudaMemcpyDeviceToHost, st), "stage in1", &err)) &&
         cuda_ok(cudaStreamSynchronize(st), "stage", &err);
    auto pass = [&]() -> bool {
      if (!cuda_ok(cudaMemcpyAsync(timed.in0, h0, b0, cudaMemcpyHostToDevice, st), "H2D in0", &err)) return false;
      if (b1 && !cuda_ok(cudaMemcpyAsync(timed.in1, h1, b1, cudaMemcpyHostToDevice, st), "H2D in1", &err)) return false;
      if (timed.launch(st) != UK_OK) {
        err = uk_cuda_last_error();
        return false;
      }
      return cuda_ok(cudaMemcpyAsync(hout, timed.out, bo, cudaMemcpyDeviceToHost, st), "D2H out", &err);
    };
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ok) ok = cuda_ok(cudaEventCreate(&e0), "event", &err) && cuda_ok(cudaEventCreate(&e1), "event", &err);
    for (int i = 0; ok && i < warm; ++i) ok = pass();
    if (ok) ok = cuda_ok(cudaStreamSynchronize(st), "warm", &err);
    double total = 0;
    for (int i = 0; ok && i < iters; ++i) {
      float ms = 0;
      ok = cuda_ok(cudaEventRecord(e0, st), "record", &err) && pass() &&
           cuda_ok(cudaEventRecord(e1, st), "record", &err) && cuda_ok(cudaEventSynchronize(e1), "sync", &err) &&
           cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "elapsed", &err);
      total += ms;
    }
    if (ok) {
      r.measured_ms = total / iters;
      float ms = 0;
      ok = cuda_ok(cudaEventRecord(e0, st), "record", &err);
      for (int i = 0; ok && i < iters; ++i)
        if (timed.launch(st) != UK_OK) {
          err = uk_cuda_last_error();
          ok = false;
        }
      ok = ok && cuda_ok(cudaEventRecord(e1, st), "record", &err) && cuda_ok(cudaEventSynchronize(e1), "sync", &err) &&
           cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "elapsed", &err);
      r.kernel_ms = double(ms) / iters;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
  }
  const unsigned fault = uk_cuda_pipeline_fault();
  if (ok && fault != 0) {
    err = "a bounded wait inside a tensor-core pipeline expired (fault word " + std::to_string(fault) + ")";
    ok = false;
  }
  cudaStreamSynchronize(st);
  cudaStreamDestroy(st);
  r.checks = ar.checks;
  r.migrations = ar.migrations;
  if (!ok) {
    log << "nvidia:cuda run failed: " << err << "\n";
    r.verified = false;
    r.exit_code = r.migrations > 0 ? 5 : 4;
    return finish();
  }
  r.ran = true;
  r.stream_path = "pinned";  // the only host data path: page-locked copies
  r.exit_code = r.verified ? 0 : 1;
  std::ostringstream res;
  res << "UNIKERN_RESULT backend=nvidia:cuda verify=" << (r.verified ? "PASS" : "FAIL") << " max_rel=" << std::scientific
      << std::setprecision(6) << r.max_rel << std::fixed << std::setprecision(6) << " measured_ms=" << r.measured_ms
      << " kernel_ms=" << r.kernel_ms << " mode=" << (stream_rows > 0 ? "streamed" : "resident")
      << " stream_path=pinned payload_mb=" << payload_mb << " perf=" << perf_string(tree)
      << (timed.f16 ? " dtype=fp16" : "") << " migrations=" << r.migrations << " checks=" << r.checks
      << " vram_free=" << r.vram_free << " vram_total=" << r.vram_total;
  r.result_line = res.str();
  log << r.result_line << "\n";
  return finish();
}

// ---- calibration -----------------------------------------------------------------

double calibrated_link_bw(const std::vector<MeasuredRow>& rows, std::string* detail) {
  std::vector<double> bws;
  std::ostringstream log;
  for (const MeasuredRow& r : rows) {
    if (r.measured_ms <= 0 || r.kernel_ms <= 0 || r.measured_ms <= r.kernel_ms) continue;  // no copy time known
    // rebuild the tree from "op:dtype:d0xd1x..." (the signature keeps the
    // leading dims only; a gemm row is exact)
    const size_t c1 = r.op_sig.find(':'), c2 = c1 == std::string::npos ? c1 : r.op_sig.find(':', c1 + 1);
    if (c2 == std::string::npos) continue;
    const auto op = op_from_name(r.op_sig.substr(0, c1));
    const auto dt = dtype_from_name(r.op_sig.substr(c1 + 1, c2 - c1 - 1));
    if (!op || !dt) continue;
    KmlTree t;
    t.op = *op;
    t.dtype = *dt;
    bool bad = false;
    std::stringstream ds(r.op_sig.substr(c2 + 1));
    std::string tok;
    for (int i = 0; i < 6 && std::getline(ds, tok, 'x'); ++i) {
      try {
        t.dims[i] = std::stoi(tok);
      } catch (...) {
        bad = true;
        break;
      }
    }
    if (bad) continue;
    if (t.op == OpKind::Reduction)
      for (int i = 1; i < 6; ++i) t.dims[i] = 0;
    const Workload w = workload_of(t);
    if (w.bytes <= 0) continue;
    const double copy_ms = r.measured_ms - r.kernel_ms;
    const double bw = double(w.bytes) / (copy_ms * 1e6);
    bws.push_back(bw);
    log << r.op_sig << " bytes=" << w.bytes << " copy_ms=" << copy_ms << " eff_bw=" << bw << "GB/s; ";
  }
  if (bws.empty()) {
    if (detail) *detail = "no usable rows (need measured_ms > kernel_ms > 0)";
    return 0;
  }
  std::sort(bws.begin(), bws.end());
  const size_t n = bws.size();
  const double med = n % 2 ? bws[n / 2] : 0.5 * (bws[n / 2 - 1] + bws[n / 2]);
  if (detail)
    *detail = "usable_rows=" + std::to_string(n) + " median_link_bw=" + std::to_string(med) + "GB/s [" + log.str() + "]";
  return med;
}

int calibrate(const std::string& hcs_json, const std::string& ledger_path, bool allow_unified, std::string* hcs_out,
              std::string* transcript) {
  std::ostringstream out;
  auto done = [&](int rc) {
    if (transcript) *transcript = out.str();
    return rc;
  };
  std::string err;
  const std::optional<Hcs> hcs = hcs_import(hcs_json, &err);
  if (!hcs) {
    out << "HCS rejected: " << err << "\n";
    return done(2);
  }
  // on a unified-memory device measured - kernel is dispatch overhead, not a
  // copy: refused before the ledger is read unless explicitly allowed
  if (hcs->unified_memory && !allow_unified) {
    out << "CALIBRATE SKIP: scenario A (unified memory, zero-copy) -- measured_ms-kernel_ms is host dispatch "
           "overhead, not link copy time; link_bw_gbps is a scenario-B constant. Pass allow_unified to force it.\n";
    return done(3);
  }
  const std::string fp = hcs_fingerprint(*hcs);
  std::string lerr;
  const std::unique_ptr<Ledger> ledger = make_ledger(ledger_path, &lerr);
  if (!ledger) {
    out << "LEDGER " << lerr << "\n";
    return done(2);
  }
  const std::vector<MeasuredRow> rows = ledger->measured_rows(fp);
  if (rows.empty()) {
    out << "CALIBRATE SKIP: no measured rows for hcs_fp=" << fp.substr(0, 8) << " (run first, then calibrate)\n";
    return done(3);
  }
  std::string detail;
  const double bw = calibrated_link_bw(rows, &detail);
  if (bw <= 0) {
    out << "CALIBRATE SKIP: " << detail << "\n";
    return done(3);
  }
  Hcs cal = *hcs;
  cal.link_bw_gbps = bw;
  cal.constants_version = hcs->constants_version + 1;
  if (hcs_out) *hcs_out = hcs_export(cal);
  const KmlTree demo;  // the default 4096^3 fp32 gemm
  const int sms = hcs->compute_units > 0 ? hcs->compute_units : 148;
  out << "CALIBRATED link_bw_gbps " << hcs->link_bw_gbps << " -> " << bw << " constants_version "
      << hcs->constants_version << " -> " << cal.constants_version << "\n"
      << detail << "\n"
      << "PREDICTED demo c_ms " << solve_b200(*hcs, demo, sms).c_ms << " -> " << solve_b200(cal, demo, sms).c_ms
      << "\n";
  return done(0);
}

// ---- cmd_solve's nvidia branch ---------------------------------------------------

int solve_kml(const std::string& hcs_json, const std::string& kml_json, const std::string& ledger_path,
              bool write_ledger, int sms, std::string* transcript) {
  std::ostringstream out;
  auto done = [&](int rc) {
    if (transcript) *transcript = out.str();
    return rc;
  };
  std::string err;
  const std::optional<Hcs> hcs = hcs_import(hcs_json, &err);
  if (!hcs) {
    out << "HCS " << err << "\n";
    return done(2);
  }
  const std::optional<KmlTree> tree = kml_import(kml_json, &err);
  if (!tree) {
    out << "KML " << err << "\n";
    return done(2);
  }
  BackendNvidia be;
  const std::string gap = be.capability_gap(*tree);
  if (!gap.empty()) {
    out << "UNSUPPORTED: " << gap << " - solve writes no ledger row for this tree. [backend=" << be.name() << "]\n";
    return done(2);
  }
  const LedgerKey key = ledger_key_parts(*hcs, *tree);
  std::unique_ptr<Ledger> ledger;
  if (!ledger_path.empty()) {
    ledger = make_ledger(ledger_path, &err);
    if (!ledger) {
      out << "LEDGER " << err << "\n";
      return done(2);
    }
    if (auto hit = ledger->lookup(key)) {
      out << "LEDGER HIT  c_cached_ms=" << hit->c_ms << "  tile=" << hit->best.tile_m << "x" << hit->best.tile_n
          << "\n"
          << hit->placement_record << "\n";
      return done(0);
    }
  }
  const int n_sm = sms > 0 ? sms : (hcs->compute_units > 0 ? hcs->compute_units : 148);
  const Solution sol = solve_b200(*hcs, *tree, n_sm);
  if (sol.feasible_count == 0) {
    out << "INFEASIBLE: no tile for " << canonical_form(*tree) << "\n";
    return done(3);
  }
  out << "SOLVED  x* tile=" << sol.best.tile_m << "x" << sol.best.tile_n << "  c_ms=" << sol.c_ms
      << "  |X|=" << sol.feasible_count << "  hcs_fp=" << key.hcs_fp.substr(0, 8) << "\n"
      << sol.placement_record << "\n";
  if (write_ledger && ledger) {
    // solve has no measurement: measured_ms is seeded with c_ms, and a run
    // of the same key overwrites it (src/main.cpp:332-335)
    if (!ledger->commit(key, sol, sol.c_ms, 0.0, &err)) {
      out << "LEDGER " << err << "\n";
      return done(2);
    }
  }
  return done(0);
}

// ---- cmd_run's nvidia branch -------------------------------------------------

int run_kml(const std::string& hcs_json, const std::string& kml_json, const std::string& ledger_path,
            bool write_ledger, std::string* transcript) {
  std::ostringstream out;
  auto done = [&](int rc) {
    if (transcript) *transcript = out.str();
    return rc;
  };
  std::string err;
  const std::optional<Hcs> hcs = hcs_import(hcs_json, &err);
  if (!hcs) {
    out << "HCS " << err << "\n";
    return done(2);
  }
  const std::optional<KmlTree> tree = kml_import(kml_json, &err);
  if (!tree) {
    out << "KML " << err << "\n";
    return done(2);
  }
  BackendNvidia be;
  const std::string gap = be.capability_gap(*tree);
  if (!gap.empty()) {
    out << "UNSUPPORTED: " << gap << " - run/verify execute nothing and write no ledger row for this tree. [backend="
        << be.name() << "]\n";
    return done(2);
  }
  const LedgerKey key = ledger_key_parts(*hcs, *tree);
  std::unique_ptr<Ledger> ledger;
  if (!ledger_path.empty()) {
    std::string lerr;
    ledger = make_ledger(ledger_path, &lerr);
    if (!ledger) {
      out << "LEDGER " << lerr << "\n";
      return done(2);
    }
  }
  Solution sol;
  if (auto rec = ledger ? ledger->lookup(key) : std::nullopt) {
    sol = *rec;
    out << "LEDGER HIT  c_cached_ms=" << sol.c_ms << "  tile=" << sol.best.tile_m << "x" << sol.best.tile_n
        << "  (from ledger)\n"
        << sol.placement_record << "\n";
  } else {
    int sms = 0;
    if (!be.available()) sms = hcs->compute_units > 0 ? hcs->compute_units : 148;
    sol = solve_b200(*hcs, *tree, sms);
    if (sol.feasible_count == 0) {
      out << "INFEASIBLE: no tile for " << canonical_form(*tree) << "\n";
      return done(3);
    }
  }
  RunOutcome r = run_cuda(sol, *hcs, *tree, "");
  out << r.log;
  out << "RUN " << be.name() << " built=" << (r.built ? "yes" : "no") << " ran=" << (r.ran ? "yes" : "no")
      << " verified=" << (r.verified ? "PASS" : "FAIL") << " max_rel=" << r.max_rel
      << " measured_ms=" << r.measured_ms;
  if (r.migrations >= 0) out << " migrations=" << r.migrations;
  if (r.checks >= 0) out << " checks=" << r.checks;
  out << "\n";
  if (r.migrations > 0 || r.exit_code == 5) {
    const double rate = r.checks > 0 ? double(r.migrations) / r.checks : 1.0;
    out << "UNIKERN_VIOLATION what=migration_rate rate=" << rate << " threshold=0 migrations=" << r.migrations
        << " checks=" << r.checks << " exit=" << r.exit_code << " vram_free=" << r.vram_free
        << " vram_total=" << r.vram_total << " committed=no\n";
    std::string werr;
    if (write_ledger && ledger && !ledger->record_violation(key, rate, 0.0, r.migrations, r.checks, r.vram_free, &werr))
      out << "LEDGER " << werr << "\n";
    // cudaMalloc memory does not migrate on this device, so a violation means
    // something outside the plan's control: record it and stop
    out << "RESOLVE STOP: nvidia:cuda allocates device memory only; violation recorded, nothing committed.\n";
    return done(5);
  }
  if (!r.built || !r.ran || !r.verified) {
    out << "RUN FAILED; solution NOT committed to ledger\n";
    return done(1);
  }
  if (!write_ledger || !ledger) {
    out << "VERIFY PASS (no ledger write)\n";
    return done(0);
  }
  std::string werr;
  if (!ledger->commit(key, sol, r.measured_ms, r.kernel_ms, &werr)) {
    out << "LEDGER " << werr << "; solution NOT committed\n";
    return done(1);
  }
  const double eps_abs = std::fabs(r.measured_ms - sol.c_ms);
  out << "LEDGER COMMIT predicted_ms=" << sol.c_ms << " measured_ms=" << r.measured_ms << " epsilon_abs=" << eps_abs
      << " epsilon_rel=" << eps_abs / std::max(sol.c_ms, 1e-9) << "\n";
  return done(0);
}

}  // namespace ukb
