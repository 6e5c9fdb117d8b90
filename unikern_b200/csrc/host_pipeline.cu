// host_pipeline.cu -- the f16 GEMM from and to host memory, with the PCIe
// copies overlapped against the tensor-core GEMM.
//
// The reference measures its GEMM end to end: upload A and B, run, download
// C, one after the other (src/codegen_hip.cpp:692-744).  On a B200 the GEMM
// itself is a small part of that (0.8 ms of ~8 ms at 8192^3): the copies
// dominate.  This entry point keeps the same inputs and outputs but runs the
// three phases as a pipeline over row blocks of A and C:
//
//   copy-in stream   B, then A block 0, A block 1, ...        (host -> device)
//   caller's stream  GEMM block i once A block i (and B) landed
//   copy-out stream  C block i once GEMM block i finished      (device -> host)
//
// so the device-to-host direction runs concurrently with the uploads and the
// GEMM hides behind them; what remains exposed is the upload of both operands
// plus the last block's GEMM and download.  The two copy streams and the
// events are created once per device on first use and kept (no device memory
// is allocated); the caller provides the device buffers.
#include <mutex>

#include "uk_common.cuh"

extern "C" int uk_cuda_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K, void* stream);
extern "C" int uk_cuda_gemm_f32_prefers_tc(int M, int N, int K);

namespace uk {  // the tensor-core fp32 GEMM's stages (conv_tc.cu)
size_t gemm_f32_tc_b_bytes(int N, int K);
size_t gemm_f32_tc_a_bytes(int M, int K);
int gemm_f32_tc_prep_b(const float* B, void* bws, int N, int K, cudaStream_t st);
int gemm_f32_tc_run(const float* A, const void* bws, void* aws, float* C, int M, int N, int K, cudaStream_t st,
                    float* part, size_t part_room);
}  // namespace uk

namespace {

constexpr int MAX_CHUNKS = 64;
constexpr int MAX_DEV = 64;

struct DevPipe {
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, b_ready = nullptr, done = nullptr;
  cudaEvent_t a_ready[MAX_CHUNKS] = {}, c_ready[MAX_CHUNKS] = {};
  bool ok = false;
};

DevPipe g_pipe[MAX_DEV];
std::mutex g_pipe_mu;

int get_pipe(DevPipe** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEV)
    return uk::fail(UK_ECUDA, "gemm_f16_host: no current device");
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  DevPipe& p = g_pipe[dev];
  if (!p.ok) {
    const unsigned ef = cudaEventDisableTiming;
    bool ok = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.start, ef) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.b_ready, ef) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.done, ef) == cudaSuccess;
    for (int i = 0; ok && i < MAX_CHUNKS; ++i)
      ok = cudaEventCreateWithFlags(&p.a_ready[i], ef) == cudaSuccess &&
           cudaEventCreateWithFlags(&p.c_ready[i], ef) == cudaSuccess;
    if (!ok) return uk::check_launch("gemm_f16_host: stream/event creation");
    p.ok = true;
  }
  *out = &p;
  return UK_OK;
}

int check_host(const void* p, const char* name) {
  if (p == nullptr) return uk::fail(UK_EINVAL, "%s is NULL", name);
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return uk::fail(UK_EINVAL, "%s is not page-locked host memory", name);
  }
  if (a.type != cudaMemoryTypeHost) return uk::fail(UK_EINVAL, "%s is not page-locked host memory", name);
  return UK_OK;
}

}  // namespace

extern "C" int uk_cuda_gemm_f16_host(const uint16_t* hA, const uint16_t* hB, uint16_t* hC, uint16_t* dA,
                                     uint16_t* dB, uint16_t* dC, int M, int N, int K, int chunks, void* stream) {
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_f16_host: negative dims %d %d %d", M, N, K);
  if (chunks < 0 || chunks > MAX_CHUNKS) return uk::fail(UK_EINVAL, "gemm_f16_host: chunks %d (0..%d)", chunks, MAX_CHUNKS);
  if (M == 0 || N == 0) return UK_OK;
  if (int rc = check_host(hA, "hA")) return rc;
  if (int rc = check_host(hB, "hB")) return rc;
  if (int rc = check_host(hC, "hC")) return rc;
  if (int rc = uk::check_device_ptr(dA, "dA")) return rc;
  if (int rc = uk::check_device_ptr(dB, "dB")) return rc;
  if (int rc = uk::check_device_ptr(dC, "dC")) return rc;
  DevPipe* p = nullptr;
  if (int rc = get_pipe(&p)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;

  // row blocks of A / C: multiples of 256 rows (whole SM-pair tiles)
  if (chunks == 0) chunks = 8;
  int64_t rows = ((int64_t)M + chunks - 1) / chunks;
  rows = (rows + 255) / 256 * 256;
  const int nblk = (int)((M + rows - 1) / rows);

  // everything is ordered after the work already queued on `stream`
  if (cudaEventRecord(p->start, st) != cudaSuccess || cudaStreamWaitEvent(p->in, p->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(p->out, p->start, 0) != cudaSuccess)
    return uk::check_launch("gemm_f16_host: ordering");
  if (cudaMemcpyAsync(dB, hB, (size_t)K * N * 2, cudaMemcpyHostToDevice, p->in) != cudaSuccess ||
      cudaEventRecord(p->b_ready, p->in) != cudaSuccess)
    return uk::check_launch("gemm_f16_host: upload B");
  for (int i = 0; i < nblk; ++i) {
    const int64_t r0 = (int64_t)i * rows, r1 = r0 + rows < M ? r0 + rows : M;
    if (cudaMemcpyAsync(dA + r0 * K, hA + r0 * K, (size_t)(r1 - r0) * K * 2, cudaMemcpyHostToDevice, p->in) !=
            cudaSuccess ||
        cudaEventRecord(p->a_ready[i], p->in) != cudaSuccess)
      return uk::check_launch("gemm_f16_host: upload A");
  }
  for (int i = 0; i < nblk; ++i) {
    const int64_t r0 = (int64_t)i * rows, r1 = r0 + rows < M ? r0 + rows : M;
    if ((i == 0 && cudaStreamWaitEvent(st, p->b_ready, 0) != cudaSuccess) ||
        cudaStreamWaitEvent(st, p->a_ready[i], 0) != cudaSuccess)
      return uk::check_launch("gemm_f16_host: wait");
    if (int rc = uk_cuda_gemm_f16_ld(dA + r0 * K, K, dB, N, dC + r0 * N, N, (int)(r1 - r0), N, K, stream)) return rc;
    if (cudaEventRecord(p->c_ready[i], st) != cudaSuccess || cudaStreamWaitEvent(p->out, p->c_ready[i], 0) != cudaSuccess ||
        cudaMemcpyAsync(hC + r0 * N, dC + r0 * N, (size_t)(r1 - r0) * N * 2, cudaMemcpyDeviceToHost, p->out) !=
            cudaSuccess)
      return uk::check_launch("gemm_f16_host: download C");
  }
  // the caller's stream completes when the last block of C is home
  if (cudaEventRecord(p->done, p->out) != cudaSuccess || cudaStreamWaitEvent(st, p->done, 0) != cudaSuccess)
    return uk::check_launch("gemm_f16_host: join");
  return UK_OK;
}

// ---- row ops from and to host memory ------------------------------------------
// The same pipeline for the row ops (their rows are independent): the copy-in
// stream uploads W (RMSNorm's gamma, channelscale's S), then the row blocks of
// X; the caller's stream runs the op on each block once it landed; the
// copy-out stream brings each block of Y home while later blocks upload, so
// the two PCIe directions run at once instead of one after the other.
extern "C" int uk_cuda_rmsnorm_f32(const float* X, const float* W, float* Y, int64_t L, int64_t C, float eps,
                                   void* stream);
extern "C" int uk_cuda_softmax_f32(const float* X, float* Y, int64_t L, int64_t C, void* stream);
extern "C" int uk_cuda_channelscale_f32(const float* X, const float* S, float* Y, int64_t L, int64_t C,
                                        void* stream);
extern "C" int uk_cuda_reduce_f32(const float* X, float* Y, int64_t rows, int64_t cols, void* workspace,
                                  size_t workspace_bytes, void* stream);

extern "C" int uk_cuda_rowop_host(int op, const float* hX, const float* hW, float* hY, float* dX, float* dW,
                                  float* dY, int64_t L, int64_t C, float eps, int chunks, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (op != UK_OP_REDUCE && op != UK_OP_SOFTMAX && op != UK_OP_RMSNORM && op != UK_OP_CHANNELSCALE)
    return uk::fail(UK_EINVAL, "rowop_host: op %d is not reduce, softmax, rmsnorm or channelscale", op);
  if (L < 0 || C < 0) return uk::fail(UK_EINVAL, "rowop_host: negative size L=%lld C=%lld", (long long)L, (long long)C);
  if (chunks < 0 || chunks > MAX_CHUNKS) return uk::fail(UK_EINVAL, "rowop_host: chunks %d (0..%d)", chunks, MAX_CHUNKS);
  if (L == 0) return UK_OK;
  const bool has_w = op == UK_OP_RMSNORM || op == UK_OP_CHANNELSCALE;
  if (int rc = check_host(hX, "hX")) return rc;
  if (int rc = check_host(hY, "hY")) return rc;
  if (has_w)
    if (int rc = check_host(hW, "hW")) return rc;
  if (int rc = uk::check_device_ptr(dX, "dX")) return rc;
  if (int rc = uk::check_device_ptr(dY, "dY")) return rc;
  if (has_w)
    if (int rc = uk::check_device_ptr(dW, "dW")) return rc;
  DevPipe* p = nullptr;
  if (int rc = get_pipe(&p)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  if (chunks == 0) chunks = 8;
  const int64_t rows = (L + chunks - 1) / chunks;
  const int nblk = (int)((L + rows - 1) / rows);
  const int64_t ycols = op == UK_OP_REDUCE ? 1 : C;  // Y per row: one sum, or a row
  if (cudaEventRecord(p->start, st) != cudaSuccess || cudaStreamWaitEvent(p->in, p->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(p->out, p->start, 0) != cudaSuccess)
    return uk::check_launch("rowop_host: ordering");
  if (has_w && (cudaMemcpyAsync(dW, hW, (size_t)C * 4, cudaMemcpyHostToDevice, p->in) != cudaSuccess ||
                cudaEventRecord(p->b_ready, p->in) != cudaSuccess))
    return uk::check_launch("rowop_host: upload W");
  for (int i = 0; i < nblk; ++i) {
    const int64_t r0 = (int64_t)i * rows, r1 = r0 + rows < L ? r0 + rows : L;
    if (cudaMemcpyAsync(dX + r0 * C, hX + r0 * C, (size_t)(r1 - r0) * C * 4, cudaMemcpyHostToDevice, p->in) !=
            cudaSuccess ||
        cudaEventRecord(p->a_ready[i], p->in) != cudaSuccess)
      return uk::check_launch("rowop_host: upload X");
  }
  for (int i = 0; i < nblk; ++i) {
    const int64_t r0 = (int64_t)i * rows, r1 = r0 + rows < L ? r0 + rows : L, n = r1 - r0;
    if ((i == 0 && has_w && cudaStreamWaitEvent(st, p->b_ready, 0) != cudaSuccess) ||
        cudaStreamWaitEvent(st, p->a_ready[i], 0) != cudaSuccess)
      return uk::check_launch("rowop_host: wait");
    int rc = UK_OK;
    float* x = dX + r0 * C;
    float* y = dY + r0 * ycols;
    switch (op) {
      case UK_OP_SOFTMAX: rc = uk_cuda_softmax_f32(x, y, n, C, stream); break;
      case UK_OP_RMSNORM: rc = uk_cuda_rmsnorm_f32(x, dW, y, n, C, eps, stream); break;
      case UK_OP_CHANNELSCALE: rc = uk_cuda_channelscale_f32(x, dW, y, n, C, stream); break;
      default: rc = uk_cuda_reduce_f32(x, y, n, C, workspace, workspace_bytes, stream); break;
    }
    if (rc != UK_OK) return rc;
    if (cudaEventRecord(p->c_ready[i], st) != cudaSuccess || cudaStreamWaitEvent(p->out, p->c_ready[i], 0) != cudaSuccess ||
        cudaMemcpyAsync(hY + r0 * ycols, y, (size_t)n * ycols * 4, cudaMemcpyDeviceToHost, p->out) != cudaSuccess)
      return uk::check_launch("rowop_host: download Y");
  }
  if (cudaEventRecord(p->done, p->out) != cudaSuccess || cudaStreamWaitEvent(st, p->done, 0) != cudaSuccess)
    return uk::check_launch("rowop_host: join");
  return UK_OK;
}

// ---- fp32 conv from and to host memory ------------------------------------------
// Images are independent: the copy-in stream uploads the weights (and the
// scale), then the blocks of images of X; the caller's stream runs the
// convolution (uk_cuda_conv2d_f32_ws, NCHW) on each block once it landed; the
// copy-out stream brings each block of Y home while later blocks upload, so
// both directions of the host link run at once.
extern "C" size_t uk_cuda_conv2d_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc, int pad,
                                                int layout);
extern "C" int uk_cuda_conv2d_f32_ws(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh,
                                     int Kw, int Oc, int pad, const float* scale, int layout, void* workspace,
                                     size_t workspace_bytes, void* stream);

extern "C" size_t uk_cuda_conv2d_f32_host_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc, int pad,
                                                         int chunks) {
  if (N <= 0 || chunks < 0 || chunks > MAX_CHUNKS) return 0;
  if (chunks == 0) chunks = 8;
  const int per = (N + chunks - 1) / chunks;
  return uk_cuda_conv2d_workspace_size(per, H, W, C, Kh, Kw, Oc, pad, UK_CONV_NCHW);
}

extern "C" int uk_cuda_conv2d_f32_host(const float* hX, const float* hW, const float* hS, float* hY, float* dX,
                                       float* dW, float* dS, float* dY, int N, int H, int W, int C, int Kh, int Kw,
                                       int Oc, int pad, int chunks, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (N < 0 || H <= 0 || W <= 0 || C <= 0 || Kh <= 0 || Kw <= 0 || Oc <= 0 || pad < 0)
    return uk::fail(UK_EINVAL, "conv2d_host: invalid dims N=%d H=%d W=%d C=%d Kh=%d Kw=%d Oc=%d pad=%d", N, H, W, C,
                    Kh, Kw, Oc, pad);
  if (chunks < 0 || chunks > MAX_CHUNKS) return uk::fail(UK_EINVAL, "conv2d_host: chunks %d (0..%d)", chunks, MAX_CHUNKS);
  const int Ho = H + 2 * pad - Kh + 1, Wo = W + 2 * pad - Kw + 1;
  if (Ho <= 0 || Wo <= 0) return uk::fail(UK_EINVAL, "conv2d_host: the filter is larger than the padded input");
  if (N == 0) return UK_OK;
  if ((hS == nullptr) != (dS == nullptr))
    return uk::fail(UK_EINVAL, "conv2d_host: the scale needs both its host (hS) and device (dS) buffer, or neither");
  if (int rc = check_host(hX, "hX")) return rc;
  if (int rc = check_host(hW, "hW")) return rc;
  if (int rc = check_host(hY, "hY")) return rc;
  if (hS)
    if (int rc = check_host(hS, "hS")) return rc;
  if (int rc = uk::check_device_ptr(dX, "dX")) return rc;
  if (int rc = uk::check_device_ptr(dW, "dW")) return rc;
  if (int rc = uk::check_device_ptr(dY, "dY")) return rc;
  if (dS)
    if (int rc = uk::check_device_ptr(dS, "dS")) return rc;
  DevPipe* p = nullptr;
  if (int rc = get_pipe(&p)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  if (chunks == 0) chunks = 8;
  const int per = (N + chunks - 1) / chunks;
  const int nblk = (N + per - 1) / per;
  const size_t ximg = (size_t)C * H * W, yimg = (size_t)Oc * Ho * Wo;
  if (cudaEventRecord(p->start, st) != cudaSuccess || cudaStreamWaitEvent(p->in, p->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(p->out, p->start, 0) != cudaSuccess)
    return uk::check_launch("conv2d_host: ordering");
  if (cudaMemcpyAsync(dW, hW, (size_t)Oc * C * Kh * Kw * 4, cudaMemcpyHostToDevice, p->in) != cudaSuccess ||
      (hS && cudaMemcpyAsync(dS, hS, (size_t)Oc * 4, cudaMemcpyHostToDevice, p->in) != cudaSuccess) ||
      cudaEventRecord(p->b_ready, p->in) != cudaSuccess)
    return uk::check_launch("conv2d_host: upload weights");
  for (int i = 0; i < nblk; ++i) {
    const int n0 = i * per, nb = n0 + per < N ? per : N - n0;
    if (cudaMemcpyAsync(dX + n0 * ximg, hX + n0 * ximg, (size_t)nb * ximg * 4, cudaMemcpyHostToDevice, p->in) !=
            cudaSuccess ||
        cudaEventRecord(p->a_ready[i], p->in) != cudaSuccess)
      return uk::check_launch("conv2d_host: upload X");
  }
  for (int i = 0; i < nblk; ++i) {
    const int n0 = i * per, nb = n0 + per < N ? per : N - n0;
    if ((i == 0 && cudaStreamWaitEvent(st, p->b_ready, 0) != cudaSuccess) ||
        cudaStreamWaitEvent(st, p->a_ready[i], 0) != cudaSuccess)
      return uk::check_launch("conv2d_host: wait");
    if (int rc = uk_cuda_conv2d_f32_ws(dX + n0 * ximg, dW, dY + n0 * yimg, nb, H, W, C, Kh, Kw, Oc, pad, dS,
                                       UK_CONV_NCHW, workspace, workspace_bytes, stream))
      return rc;
    if (cudaEventRecord(p->c_ready[i], st) != cudaSuccess || cudaStreamWaitEvent(p->out, p->c_ready[i], 0) != cudaSuccess ||
        cudaMemcpyAsync(hY + n0 * yimg, dY + n0 * yimg, (size_t)nb * yimg * 4, cudaMemcpyDeviceToHost, p->out) !=
            cudaSuccess)
      return uk::check_launch("conv2d_host: download Y");
  }
  if (cudaEventRecord(p->done, p->out) != cudaSuccess || cudaStreamWaitEvent(st, p->done, 0) != cudaSuccess)
    return uk::check_launch("conv2d_host: join");
  return UK_OK;
}

// ---- streamed GEMM (payload larger than the device) -------------------------
// Only B is resident; A and C pass through a two-slot ring of row blocks in
// the caller's device buffer.  Block i uses slot i % 2: its upload waits until
// block i-2's GEMM has finished reading the slot's A rows, its GEMM waits
// until block i-2's C rows have left the slot.  Device memory: K*N elements
// for B plus 2 * block_rows * (K + N) for the ring, and for an fp32 GEMM on
// the tensor cores (split-tf32) 2 * (K*N + block_rows*K) more for the tf32
// pairs of B^T and of one block of A.
namespace {

struct StreamPipe {
  cudaEvent_t a_ready[2] = {}, gemm_done[2] = {}, c_home[2] = {};
  bool ok = false;
};
StreamPipe g_spipe[MAX_DEV];

int get_stream_pipe(StreamPipe** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEV)
    return uk::fail(UK_ECUDA, "gemm_streamed: no current device");
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  StreamPipe& p = g_spipe[dev];
  if (!p.ok) {
    bool ok = true;
    for (int i = 0; ok && i < 2; ++i)
      ok = cudaEventCreateWithFlags(&p.a_ready[i], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&p.gemm_done[i], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&p.c_home[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) return uk::check_launch("gemm_streamed: event creation");
    p.ok = true;
  }
  *out = &p;
  return UK_OK;
}

// ring layout (each part 256-byte aligned from the first aligned address):
// A slot 0, A slot 1, C slot 0, C slot 1, and for an fp32 GEMM on the tensor
// cores the tf32 pairs of B^T (made once per call) and of one A block
struct RingLayout {
  int64_t rows = 0;
  size_t a_slot = 0, c_slot = 0, b_split = 0, a_split = 0, total = 0;
  bool tc = false;
};

// kind: 1 binary16; 0 fp32, on the tensor cores where a block gains; 2 fp32
// on the FFMA kernel (no tf32 pairs, the smallest ring)
RingLayout ring_layout(int M, int N, int K, int kind, int block_rows) {
  RingLayout r;
  if (M <= 0 || N <= 0 || K <= 0 || block_rows <= 0 || kind < 0 || kind > 2) return r;
  const int f16 = kind == 1;
  auto align = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t es = f16 ? 2 : 4;
  r.rows = block_rows < M ? block_rows : M;
  r.a_slot = align((size_t)r.rows * K * es);
  r.c_slot = align((size_t)r.rows * N * es);
  r.tc = kind == 0 && uk_cuda_gemm_f32_prefers_tc((int)r.rows, N, K);
  if (r.tc) {
    r.b_split = uk::gemm_f32_tc_b_bytes(N, K);
    r.a_split = uk::gemm_f32_tc_a_bytes((int)r.rows, K);
  }
  r.total = 255 + 2 * r.a_slot + 2 * r.c_slot + r.b_split + r.a_split;
  return r;
}

}  // namespace

extern "C" size_t uk_cuda_gemm_streamed_ring_size(int M, int N, int K, int kind, int block_rows) {
  return ring_layout(M, N, K, kind, block_rows).total;
}

namespace {

// the device work of one streamed call over data already in the ring: B's
// pre-pass (tensor-core fp32) and one GEMM per block, all on slot 0
int streamed_block_gemms(const RingLayout& L, void* dB, uint8_t* base, int M, int N, int K, int f16,
                         cudaStream_t st, bool prep_b) {
  // f16: the data type (kind 1); the fp32 kernel choice is L.tc
  uint8_t* b_split = base + 2 * L.a_slot + 2 * L.c_slot;
  if (L.tc && prep_b)
    if (int rc = uk::gemm_f32_tc_prep_b((const float*)dB, b_split, N, K, st)) return rc;
  const int nblk = (int)((M + L.rows - 1) / L.rows);
  for (int i = 0; i < nblk; ++i) {
    const int nr = (int)(i == nblk - 1 ? M - (int64_t)(nblk - 1) * L.rows : L.rows);
    uint8_t* a = base;
    uint8_t* c = base + 2 * L.a_slot;
    const int rc = f16 ? uk_cuda_gemm_f16_ld((const uint16_t*)a, K, (const uint16_t*)dB, N, (uint16_t*)c, N, nr, N,
                                             K, st)
                   : L.tc ? uk::gemm_f32_tc_run((const float*)a, b_split, b_split + L.b_split, (float*)c, nr, N, K,
                                                st, nullptr, 0)
                          : uk_cuda_gemm_f32((const float*)a, (const float*)dB, (float*)c, nr, N, K, st);
    if (rc != UK_OK) return rc;
  }
  return UK_OK;
}

}  // namespace

// kernel-only timing aid of the runner (declared in host/runner_dev.h)
extern "C" int ukr_gemm_streamed_kernels(void* dB, void* ring, size_t ring_bytes, int M, int N, int K, int kind,
                                         int block_rows, void* stream) {
  const RingLayout L = ring_layout(M, N, K, kind, block_rows);
  if (L.total == 0 || ring_bytes < L.total) return uk::fail(UK_EINVAL, "gemm_streamed: ring too small");
  uint8_t* base = (uint8_t*)(((uintptr_t)ring + 255) & ~(uintptr_t)255);
  return streamed_block_gemms(L, dB, base, M, N, K, kind == 1, (cudaStream_t)stream, true);
}

extern "C" int uk_cuda_gemm_streamed(const void* hA, const void* hB, void* hC, void* dB, void* ring,
                                     size_t ring_bytes, int M, int N, int K, int kind, int block_rows, void* stream) {
  if (M < 0 || N < 0 || K < 0) return uk::fail(UK_EINVAL, "gemm_streamed: negative dims %d %d %d", M, N, K);
  if (kind < 0 || kind > 2) return uk::fail(UK_EINVAL, "gemm_streamed: kind must be 0, 1 or 2 (got %d)", kind);
  const int f16 = kind == 1;
  if (block_rows <= 0) return uk::fail(UK_EINVAL, "gemm_streamed: block_rows must be positive");
  if (M == 0 || N == 0) return UK_OK;
  if (int rc = check_host(hA, "hA")) return rc;
  if (int rc = check_host(hB, "hB")) return rc;
  if (int rc = check_host(hC, "hC")) return rc;
  if (int rc = uk::check_device_ptr(dB, "dB")) return rc;
  if (int rc = uk::check_device_ptr(ring, "ring")) return rc;
  const RingLayout L = ring_layout(M, N, K, kind, block_rows);
  if (ring_bytes < L.total)
    return uk::fail(UK_EINVAL, "gemm_streamed: the ring needs %zu bytes (uk_cuda_gemm_streamed_ring_size), got %zu",
                    L.total, ring_bytes);
  DevPipe* p = nullptr;
  StreamPipe* q = nullptr;
  if (int rc = get_pipe(&p)) return rc;
  if (int rc = get_stream_pipe(&q)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  const size_t es = f16 ? 2 : 4;
  const int64_t rows = L.rows;
  const int nblk = (int)((M + rows - 1) / rows);
  uint8_t* base = (uint8_t*)(((uintptr_t)ring + 255) & ~(uintptr_t)255);
  uint8_t* a_buf[2] = {base, base + L.a_slot};
  uint8_t* c_buf[2] = {base + 2 * L.a_slot, base + 2 * L.a_slot + L.c_slot};
  uint8_t* b_split = base + 2 * L.a_slot + 2 * L.c_slot;
  uint8_t* a_split = b_split + L.b_split;

  if (cudaEventRecord(p->start, st) != cudaSuccess || cudaStreamWaitEvent(p->in, p->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(p->out, p->start, 0) != cudaSuccess)
    return uk::check_launch("gemm_streamed: ordering");
  if (cudaMemcpyAsync(dB, hB, (size_t)K * N * es, cudaMemcpyHostToDevice, p->in) != cudaSuccess ||
      cudaEventRecord(p->b_ready, p->in) != cudaSuccess || cudaStreamWaitEvent(st, p->b_ready, 0) != cudaSuccess)
    return uk::check_launch("gemm_streamed: upload B");
  if (L.tc)  // B^T as tf32 pairs, once for every block
    if (int rc = uk::gemm_f32_tc_prep_b((const float*)dB, b_split, N, K, st)) return rc;
  for (int i = 0; i < nblk; ++i) {
    const int slot = i & 1;
    const int64_t r0 = (int64_t)i * rows, r1 = r0 + rows < M ? r0 + rows : M, nr = r1 - r0;
    // upload: after block i-2's GEMM released the slot's A rows
    if ((i >= 2 && cudaStreamWaitEvent(p->in, q->gemm_done[slot], 0) != cudaSuccess) ||
        cudaMemcpyAsync(a_buf[slot], (const uint8_t*)hA + r0 * K * es, nr * K * es, cudaMemcpyHostToDevice, p->in) !=
            cudaSuccess ||
        cudaEventRecord(q->a_ready[slot], p->in) != cudaSuccess)
      return uk::check_launch("gemm_streamed: upload A");
    // GEMM: after its A rows landed and block i-2's C rows left the slot
    if (cudaStreamWaitEvent(st, q->a_ready[slot], 0) != cudaSuccess ||
        (i >= 2 && cudaStreamWaitEvent(st, q->c_home[slot], 0) != cudaSuccess))
      return uk::check_launch("gemm_streamed: wait");
    const int rc = f16 ? uk_cuda_gemm_f16_ld((const uint16_t*)a_buf[slot], K, (const uint16_t*)dB, N,
                                             (uint16_t*)c_buf[slot], N, (int)nr, N, K, stream)
                   : L.tc ? uk::gemm_f32_tc_run((const float*)a_buf[slot], b_split, a_split, (float*)c_buf[slot],
                                                (int)nr, N, K, st, nullptr, 0)
                          : uk_cuda_gemm_f32((const float*)a_buf[slot], (const float*)dB, (float*)c_buf[slot],
                                             (int)nr, N, K, stream);
    if (rc != UK_OK) return rc;
    if (cudaEventRecord(q->gemm_done[slot], st) != cudaSuccess ||
        cudaStreamWaitEvent(p->out, q->gemm_done[slot], 0) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t*)hC + r0 * N * es, c_buf[slot], nr * N * es, cudaMemcpyDeviceToHost, p->out) !=
            cudaSuccess ||
        cudaEventRecord(q->c_home[slot], p->out) != cudaSuccess)
      return uk::check_launch("gemm_streamed: download C");
  }
  if (cudaEventRecord(p->done, p->out) != cudaSuccess || cudaStreamWaitEvent(st, p->done, 0) != cudaSuccess)
    return uk::check_launch("gemm_streamed: join");
  return UK_OK;
}
