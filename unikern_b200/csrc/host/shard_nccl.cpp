// shard_nccl.cpp -- the N-sharded f16 GEMM across the GPUs of one node from a
// C or C++ host, over a caller's NCCL communicator (one process per GPU), with
// failure detection that ends in an error status, never a hang.
//
//   uk_nccl_comm_init      ncclCommInitRankConfig with a non-blocking config,
//                          polled with ncclCommGetAsyncError against a time
//                          limit; a rank that never joins ends the wait with
//                          ncclCommAbort and UK_ECUDA
//   uk_shard_gemm_f16_*    the fused GEMM + all-gather of gemm_f16_2sm.cu
//                          (each rank's kernel stores its column block of C
//                          into every rank's C over NVLink); the IPC handles
//                          of the ranks' C travel once over NCCL, and every
//                          step is bracketed by two one-float all-reduces:
//                          one that proves every peer alive and past its
//                          previous step BEFORE this rank's kernel stores into
//                          their memory, one after it that orders the ranks
//                          before C is read.  A host wait on each, bounded by
//                          the caller's limit and polling the communicator's
//                          asynchronous error, turns a rank that left, stalled
//                          or failed into ncclCommAbort + UK_ECUDA.
// The reference is single-GPU; its failure protocol is an exit code per
// outcome (src/main.cpp:469-539), which this keeps: 4 for a lost peer.
//
// NCCL is resolved at run time: the process's already-loaded libnccl (the one
// that made the caller's communicator) when there is one, else libnccl.so.2,
// so the library links no NCCL of its own.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "unikern_cuda.h"

namespace uk {
int fail(int code, const char* fmt, ...);
}

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = RTLD_DEFAULT;
    if (dlsym(h, "ncclCommInitRankConfig") == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    get(api.get_unique_id, "ncclGetUniqueId");
    get(api.init_rank_config, "ncclCommInitRankConfig");
    get(api.async_error, "ncclCommGetAsyncError");
    get(api.abort, "ncclCommAbort");
    get(api.destroy, "ncclCommDestroy");
    get(api.all_gather, "ncclAllGather");
    get(api.all_reduce, "ncclAllReduce");
    get(api.error_string, "ncclGetErrorString");
    api.ok = all;
  });
  return api;
}

int need_nccl(const char* what) {
  if (nccl().ok) return UK_OK;
  return uk::fail(UK_ECUDA, "%s: NCCL is not available (libnccl.so.2 not found)", what);
}

using Clock = std::chrono::steady_clock;

// communicators this library aborted after a failure: their handles are
// dead, and uk_nccl_comm_destroy must not touch them again
std::mutex g_aborted_mu;
std::set<ncclComm_t> g_aborted;

void abort_comm(ncclComm_t comm) {
  std::lock_guard<std::mutex> lock(g_aborted_mu);
  if (g_aborted.insert(comm).second) nccl().abort(comm);
}

bool was_aborted(ncclComm_t comm) {
  std::lock_guard<std::mutex> lock(g_aborted_mu);
  return g_aborted.count(comm) != 0;
}

// Poll until `done()` or the communicator reports an error or the limit
// passes; on error or timeout the communicator is aborted (which also ends
// any NCCL kernel of it still waiting on the device) and UK_ECUDA returned.
template <class Done>
int bounded_wait(ncclComm_t comm, uint64_t timeout_ns, const char* what, Done done) {
  const auto& n = nccl();
  const auto t0 = Clock::now();
  for (;;) {
    ncclResult_t ar = ncclSuccess;
    if (n.async_error(comm, &ar) != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
      abort_comm(comm);
      return uk::fail(UK_ECUDA, "%s: NCCL reported %s; communicator aborted", what,
                      n.error_string(ar != ncclSuccess ? ar : ncclInternalError));
    }
    const int d = done();
    if (d < 0) {
      abort_comm(comm);
      return uk::fail(UK_ECUDA, "%s: CUDA error while waiting; communicator aborted", what);
    }
    if (d > 0 && ar == ncclSuccess) return UK_OK;
    const uint64_t waited = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now() - t0).count();
    if (waited > timeout_ns) {
      abort_comm(comm);
      return uk::fail(UK_ECUDA,
                      "%s: a peer did not arrive within %.3f s (it left, stalled or failed); communicator aborted",
                      what, timeout_ns * 1e-9);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// 1 when the stream's work is complete, 0 while it runs, -1 on a CUDA error
int stream_done(cudaStream_t st) {
  const cudaError_t e = cudaStreamQuery(st);
  if (e == cudaSuccess) return 1;
  if (e == cudaErrorNotReady) return 0;
  return -1;
}

}  // namespace

struct uk_shard_gemm {
  ncclComm_t comm = nullptr;
  int rank = 0, nranks = 1;
  int M = 0, N = 0, K = 0;
  int64_t ldc = 0, n0 = 0, n1 = 0;
  std::vector<uint16_t*> c_list;  // this rank's C first, then the peers' around the ring
  std::vector<std::pair<void*, uint64_t>> opened;
  float* flag = nullptr;  // one float for the barrier all-reduces
};

extern "C" {

size_t uk_nccl_unique_id_size(void) { return sizeof(ncclUniqueId); }

int uk_nccl_get_unique_id(void* out) {
  if (out == nullptr) return uk::fail(UK_EINVAL, "nccl_get_unique_id: NULL out");
  if (int rc = need_nccl("nccl_get_unique_id")) return rc;
  ncclUniqueId id;
  const ncclResult_t r = nccl().get_unique_id(&id);
  if (r != ncclSuccess) return uk::fail(UK_ECUDA, "ncclGetUniqueId: %s", nccl().error_string(r));
  std::memcpy(out, &id, sizeof(id));
  return UK_OK;
}

int uk_nccl_comm_init(const void* unique_id, int nranks, int rank, uint64_t timeout_ns, void** comm_out) {
  if (unique_id == nullptr || comm_out == nullptr || nranks < 1 || rank < 0 || rank >= nranks)
    return uk::fail(UK_EINVAL, "nccl_comm_init: bad arguments (rank %d of %d)", rank, nranks);
  if (int rc = need_nccl("nccl_comm_init")) return rc;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // return at once; completion is polled below
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nccl().init_rank_config(&comm, nranks, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm != nullptr) abort_comm(comm);
    return uk::fail(UK_ECUDA, "ncclCommInitRankConfig: %s", nccl().error_string(r));
  }
  if (int rc = bounded_wait(comm, timeout_ns, "nccl_comm_init", [] { return 1; })) return rc;
  *comm_out = comm;
  return UK_OK;
}

int uk_nccl_comm_destroy(void* comm) {
  if (comm == nullptr) return UK_OK;
  if (int rc = need_nccl("nccl_comm_destroy")) return rc;
  // abort frees the communicator with no collective with the peers (which may
  // be gone); one this library already aborted after a failure is left alone
  abort_comm((ncclComm_t)comm);
  return UK_OK;
}

int uk_shard_gemm_f16_create(void* comm, int rank, int nranks, uint16_t* C, int64_t ldc, int M, int N, int K,
                             uint64_t timeout_ns, uk_shard_gemm** out) {
  if (comm == nullptr || C == nullptr || out == nullptr || nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks)
    return uk::fail(UK_EINVAL, "shard_gemm_create: bad arguments (rank %d of %d; 1..8 ranks)", rank, nranks);
  if (M <= 0 || N <= 0 || K <= 0 || ldc < N || N % 8 != 0 || ldc % 8 != 0)
    return uk::fail(UK_EINVAL, "shard_gemm_create: M=%d N=%d K=%d ldc=%lld (N, ldc multiples of 8)", M, N, K,
                    (long long)ldc);
  if (int rc = need_nccl("shard_gemm_create")) return rc;
  auto* h = new uk_shard_gemm;
  h->comm = (ncclComm_t)comm;
  h->rank = rank;
  h->nranks = nranks;
  h->M = M;
  h->N = N;
  h->K = K;
  h->ldc = ldc;
  // this rank's column block: multiples of 8 columns, as even as possible
  const int64_t units = (N + 7) / 8, per = units / nranks, extra = units % nranks;
  const int64_t u0 = rank * per + (rank < extra ? rank : extra), u1 = u0 + per + (rank < extra ? 1 : 0);
  h->n0 = u0 * 8 < N ? u0 * 8 : N;
  h->n1 = u1 * 8 < N ? u1 * 8 : N;
  auto undo = [&](int rc) {
    for (auto& o : h->opened) uk_cuda_ipc_close(o.first, o.second);
    if (h->flag) cudaFree(h->flag);
    delete h;
    return rc;
  };
  // every rank's (IPC handle, offset) of C, gathered over NCCL once
  const size_t hs = uk_cuda_ipc_handle_size(), rec = (hs + 8 + 15) / 16 * 16;
  std::vector<uint8_t> mine(rec, 0), all(rec * nranks, 0);
  uint64_t off = 0;
  if (int rc = uk_cuda_ipc_export(C, mine.data(), &off)) return undo(rc);
  std::memcpy(mine.data() + hs, &off, 8);
  void* dbuf = nullptr;
  if (cudaMalloc(&dbuf, rec * (nranks + 1)) != cudaSuccess || cudaMalloc(&h->flag, sizeof(float)) != cudaSuccess) {
    if (dbuf) cudaFree(dbuf);
    return undo(uk::fail(UK_ECUDA, "shard_gemm_create: device buffers for the handle exchange"));
  }
  cudaMemset(h->flag, 0, sizeof(float));
  cudaStream_t st = nullptr;
  cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  uint8_t* dsend = (uint8_t*)dbuf + rec * nranks;
  cudaMemcpyAsync(dsend, mine.data(), rec, cudaMemcpyHostToDevice, st);
  const ncclResult_t r = nccl().all_gather(dsend, dbuf, rec, ncclUint8, h->comm, st);
  int rc = r == ncclSuccess || r == ncclInProgress ? UK_OK : uk::fail(UK_ECUDA, "ncclAllGather: %s", nccl().error_string(r));
  if (rc == UK_OK)
    rc = bounded_wait(h->comm, timeout_ns, "shard_gemm_create (handle exchange)", [st] { return stream_done(st); });
  if (rc == UK_OK) cudaMemcpy(all.data(), dbuf, rec * nranks, cudaMemcpyDeviceToHost);
  cudaStreamDestroy(st);
  cudaFree(dbuf);
  if (rc != UK_OK) return undo(rc);
  // the copies in store order: local first, then around the ring
  for (int i = 0; i < nranks; ++i) {
    const int r2 = (rank + i) % nranks;
    if (r2 == rank) {
      h->c_list.push_back(C);
      continue;
    }
    uint64_t o = 0;
    std::memcpy(&o, all.data() + rec * r2 + hs, 8);
    void* p = nullptr;
    if (int e = uk_cuda_ipc_import(all.data() + rec * r2, o, &p)) return undo(e);
    h->opened.push_back({p, o});
    h->c_list.push_back((uint16_t*)p);
  }
  *out = h;
  return UK_OK;
}

int uk_shard_gemm_f16_columns(const uk_shard_gemm* h, int64_t* n0, int64_t* n1) {
  if (h == nullptr || n0 == nullptr || n1 == nullptr) return uk::fail(UK_EINVAL, "shard_gemm_columns: NULL argument");
  *n0 = h->n0;
  *n1 = h->n1;
  return UK_OK;
}

int uk_shard_gemm_f16_run(uk_shard_gemm* h, const uint16_t* A, int64_t lda, const uint16_t* B_shard, int64_t ldb,
                          void* stream, uint64_t timeout_ns) {
  if (h == nullptr || A == nullptr || B_shard == nullptr) return uk::fail(UK_EINVAL, "shard_gemm_run: NULL argument");
  if (h->comm == nullptr || was_aborted(h->comm))
    return uk::fail(UK_ECUDA, "shard_gemm_run: the communicator was aborted by an earlier failure");
  const cudaStream_t st = (cudaStream_t)stream;
  const auto& n = nccl();
  auto barrier = [&](const char* what, bool wait) -> int {
    const ncclResult_t r = n.all_reduce(h->flag, h->flag, 1, ncclFloat32, ncclSum, h->comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
      abort_comm(h->comm);
      h->comm = nullptr;
      return uk::fail(UK_ECUDA, "%s: ncclAllReduce: %s; communicator aborted", what, n.error_string(r));
    }
    if (!wait) return UK_OK;
    const int rc = bounded_wait(h->comm, timeout_ns, what, [st] { return stream_done(st); });
    if (rc != UK_OK) h->comm = nullptr;
    return rc;
  };
  const bool bounded = timeout_ns > 0;
  // 1. every peer alive and past its previous step (so its C exists and no
  //    one still reads it) before this rank's kernel stores into it
  if (int rc = barrier("shard_gemm_run (peers alive)", bounded)) return rc;
  // 2. this rank's column block, stored into every rank's C
  const int rc = uk_cuda_gemm_f16_allgather(A, lda, B_shard, ldb, h->c_list.data(), h->nranks, h->ldc, h->M,
                                            (int)(h->n1 - h->n0), h->K, h->n0, stream);
  if (rc != UK_OK) return rc;
  // 3. every rank's stores landed before anyone reads C
  return barrier("shard_gemm_run (stores complete)", bounded);
}

int uk_shard_gemm_f16_destroy(uk_shard_gemm* h) {
  if (h == nullptr) return UK_OK;
  for (auto& o : h->opened) uk_cuda_ipc_close(o.first, o.second);
  if (h->flag) cudaFree(h->flag);
  delete h;
  return UK_OK;
}

}  // extern "C"
