/*
 * unikern_cuda.h -- C ABI of libunikern_cuda.so, the B200 (sm_100a) path of
 * the UNIKERN KML operator set.
 *
 * Conventions
 *   - All tensors are caller-owned DEVICE memory of the current device
 *     (cudaMalloc'd or equivalent).  Host, managed or another device's memory
 *     is refused with UK_ERESIDENCY (the reference refuses non-device-resident
 *     allocations as oversubscription, src/codegen_hip.cpp:209-293).
 *   - Every call is stream-ordered on `stream` (a cudaStream_t; NULL = the
 *     legacy default stream) and returns before the kernel finishes.
 *   - No call allocates or frees memory.  Calls that need scratch memory take
 *     a caller-provided workspace whose size a *_workspace_size() call gives.
 *   - Return value: UK_OK (0) or an error code; uk_cuda_last_error() gives
 *     the text of the last failure on the calling thread.
 *   - Layouts are the KML contract's "NT" tag: row-major A[M][K], B[K][N],
 *     C[M][N] (src/codegen.hpp codegen_layout_supported, src/codegen_hip.cpp:72).
 *   - Reentrant across streams; the library keeps no per-call state except
 *     the thread-local error text and per-device cached attributes.
 *
 * Each entry point replaces the device kernel(s) the reference generates for
 * the op (file:line within the UNIKERN project).
 */
#ifndef UNIKERN_CUDA_H
#define UNIKERN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UK_OK 0
#define UK_EVERIFY 1    /* runner level: result outside the tolerance */
#define UK_EINVAL 2     /* invalid argument (sizes, NULL, alignment) */
#define UK_ECUDA 4      /* CUDA error, or a refused configuration */
#define UK_ERESIDENCY 5 /* pointer is not device-resident on this device */

/* text of the last failure on this thread ("" if none) */
const char* uk_cuda_last_error(void);
/* ABI version: major * 10000 + minor * 100 + patch */
int uk_cuda_abi_version(void);
/* 1 when the current device is an sm_100 part this library can run on */
int uk_cuda_device_supported(void);

/* ---- launch plan -----------------------------------------------------------
 * The tile this library launches for a KML op, given its KML dims (gemm M,N,K;
 * conv H,W,C,Kh,Kw,Oc; reduce L; softmax/rmsnorm/channelscale L,C), on a part
 * with `sms` multiprocessors (0 = the current device).  out4 = {tile_m,
 * tile_n, k_block, stages}: outputs per CTA (rows x columns; for the row ops
 * one row x the columns one register pass covers), the K depth of a pipeline
 * step (0 for the row ops), and the pipeline stages (reduce: row splits;
 * softmax/rmsnorm: 2 when the row streams from HBM twice).  Host only; with
 * sms > 0 it needs no GPU.  Replaces emit_tile_for / the solver's tile choice
 * (src/codegen_hip.cpp:58-68, src/solver.cpp:14-186): these are the tm/tn the
 * runner records in the ledger row. */
#define UK_OP_GEMM 0
#define UK_OP_CONV 1
#define UK_OP_REDUCE 2
#define UK_OP_SOFTMAX 3
#define UK_OP_RMSNORM 4
#define UK_OP_CHANNELSCALE 5
int uk_cuda_tile_plan(int op, int f16, const int64_t* dims, int sms, int* out4);

/* The GEMM solve behind that plan (op = UK_OP_GEMM; dims M, N, K): the
 * re-target of the reference's solver (src/solver.cpp:14-186: candidate
 * grid, feasibility, pure cost, lexicographic argmin) to this library's
 * kernels.  Candidates are kernel families with their tile and K split:
 * the FFMA tiles 128x128, 64x64 and 32x64 (the last with K split over 2, 4 or
 * 8 CTAs), and for fp32 with allow_tc the split-tf32 pair kernel (K % 32,
 * N % 64, from 2^30 multiply-adds); for f16 (the tensor-core shape rules
 * hold) the single-SM 128x256 and SM-pair 256x256 tcgen05 kernels.  Cost =
 * predicted device time from wave counts at each family's measured
 * efficiency, pre-passes, folds and launches.  out8 = {family (0 FFMA, 1
 * tcgen05 single-SM, 2 tcgen05 pair, 3 split-tf32 pair), tile_m, tile_n,
 * k_block, stages, k_split, feasible candidates, predicted ns}.  The GEMM
 * launchers take the same argmin.  Host only; with sms > 0 it needs no GPU. */
int uk_cuda_solve_plan(int op, int f16, const int64_t* dims, int sms, int allow_tc, int* out8);
/* The plan of the last GEMM launched on the calling thread, as out6 =
 * {family, tile_m, tile_n, k_block, stages, k_split} (family -1 before any):
 * how a caller sees the solver's choice reach the launcher.  Families beyond
 * the solver's: 6 the decode chain's skinny GEMM (tile = 128 weight columns x
 * 32 token rows, k_split = its K-split cluster size), 7 the FFMA 32 x 64 tile
 * with K split over warp groups of one CTA (k_split = the groups). */
int uk_cuda_last_launch(int* out6);

/* ---- channelscale ----------------------------------------------------------
 * Y[i*C + c] = X[i*C + c] * S[c] for i < L, c < C.  Bit-exact to the reference.
 * Replaces uk_channelscale (src/codegen_hip.cpp:2329-2335). */
int uk_cuda_channelscale_f32(const float* X, const float* S, float* Y, int64_t L,
                             int64_t C, void* stream);

/* ---- reduce ----------------------------------------------------------------
 * Y[r] = sum_c X[r*cols + c] (fp32) for r < rows.  rows = 1 is the KML
 * `reduce` op (a length-L vector to one scalar); cols = 0 writes zeros.
 * Deterministic: the same inputs give the same bits on every call.
 * Replaces uk_reduce_part + uk_reduce_sum (src/codegen_hip.cpp:818-833) and
 * the width plan uk_reduce_width_plan (:874-908). */
size_t uk_cuda_reduce_workspace_size(int64_t rows, int64_t cols);
int uk_cuda_reduce_f32(const float* X, float* Y, int64_t rows, int64_t cols,
                       void* workspace, size_t workspace_bytes, void* stream);

/* The same reduce with the pass-1 width pinned: each row is cut into chunks of
 * ceil(cols / width) elements, one partial sum per chunk, folded in a fixed
 * order (the reference's UK_REDUCE_WIDTH knob, src/codegen_hip.cpp:874-908;
 * the runner validates a pin against the reference's range [256, cols]).
 * width >= 1; the partial count is ceil(cols / ceil(cols / width)), which is
 * width whenever width divides the chunking exactly.  Workspace:
 * uk_cuda_reduce_workspace_size_width(rows, cols, width) bytes. */
size_t uk_cuda_reduce_workspace_size_width(int64_t rows, int64_t cols, int64_t width);
int uk_cuda_reduce_f32_width(const float* X, float* Y, int64_t rows, int64_t cols, int64_t width,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Row sums of binary16 rows (fp32 accumulation, one rounding into the
 * binary16 result Y[rows]); the same plans, workspace sizes and determinism
 * as the fp32 reduce.  The reference refuses fp16 for reduce
 * (src/codegen_hip.cpp:81-89); this widens the dtype interval. */
int uk_cuda_reduce_f16(const uint16_t* X, uint16_t* Y, int64_t rows, int64_t cols, void* workspace,
                       size_t workspace_bytes, void* stream);
int uk_cuda_reduce_f16_width(const uint16_t* X, uint16_t* Y, int64_t rows, int64_t cols, int64_t width,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Reduce without a workspace: the same result as uk_cuda_reduce_f32 (same
 * kernels, same plan), for callers that cannot allocate device memory -- a
 * plugin inside a host application that owns every device allocation through
 * its own pool or budget, or a caller that must not risk an allocation's
 * implicit synchronisation or out-of-memory failure in the middle of a run --
 * and so have no workspace to pass.  This call allocates nothing: the partial
 * sums of the split-row plan go to a 32 KiB array (8192 floats) inside the
 * library, which every GPU that loads the library holds until the process
 * exits.  Limit: a shape whose plan needs more than 8192 partial sums is
 * rejected with UK_EINVAL (on a 148-SM B200 the plan never needs more than
 * about 1800, so every shape fits).  The first call on each device looks up
 * the array's device address with that device current (and looks it up again
 * after that device's context changed, e.g. after cudaDeviceReset); make that
 * first call before any stream capture.  All calls share the one array: calls that
 * overlap on the GPU (different streams, or threads, on the same device)
 * race and must be serialised, e.g. on one stream.  The array keeps the last
 * call's contents; nothing in it has to start at zero.
 * No counterpart in the reference (its reduce always allocates its partials). */
int uk_cuda_reduce_f32_noalloc(const float* X, float* Y, int64_t rows, int64_t cols, void* stream);

/* ---- rmsnorm ---------------------------------------------------------------
 * Y[l][c] = X[l][c] * (1 / sqrt(sum_c X[l][c]^2 / C + eps)) * W[c].
 * The reference hard-codes eps = 1e-6 (src/codegen_hip.cpp:2162, :2175);
 * pass 1e-6f for the KML contract.  Replaces uk_rmsnorm (:2154-2164). */
int uk_cuda_rmsnorm_f32(const float* X, const float* W, float* Y, int64_t L,
                        int64_t C, float eps, void* stream);

/* ---- softmax ---------------------------------------------------------------
 * Y[l][c] = exp(X[l][c] - max_l) / sum_c exp(X[l][c] - max_l).
 * Replaces uk_softmax (src/codegen_hip.cpp:1985-1996). */
int uk_cuda_softmax_f32(const float* X, float* Y, int64_t L, int64_t C, void* stream);

/* ---- fp16 row ops ------------------------------------------------------------
 * softmax / RMSNorm / channelscale on IEEE binary16 rows (uint16_t bit
 * patterns in and out, fp32 arithmetic, one rounding to f16 per output), with
 * the formulas and operation order of the fp32 entry points above.  W (the
 * RMSNorm weight) and S (the channel scale) are f16 too.  Deterministic.
 * The reference refuses fp16 for these ops (src/codegen_hip.cpp:81-89); these
 * widen the dtype interval with the same algorithms. */
int uk_cuda_softmax_f16(const uint16_t* X, uint16_t* Y, int64_t L, int64_t C, void* stream);
int uk_cuda_rmsnorm_f16(const uint16_t* X, const uint16_t* W, uint16_t* Y, int64_t L, int64_t C, float eps,
                        void* stream);
int uk_cuda_channelscale_f16(const uint16_t* X, const uint16_t* S, uint16_t* Y, int64_t L, int64_t C,
                             void* stream);

/* ---- gemm f32 --------------------------------------------------------------
 * C = A * B, fp32 FFMA (no TF32), fp32 accumulation.  Any M, N, K >= 0.
 * Replaces uk_gemm (src/codegen_hip.cpp:1089-1120). */
int uk_cuda_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K,
                     void* stream);

/* The same GEMM on the tcgen05 tensor cores at fp32 accuracy: every operand
 * is carried as a tf32 (hi, lo) pair and each product as lo*hi + hi*lo +
 * hi*hi in the fp32 accumulator ("3xTF32"), so results agree with the FFMA
 * kernel to a few ulps of the output scale (exactly, where every partial sum
 * is representable).  C = A * B runs as the 1 x 1 convolution of B^T's pixels
 * with A's rows as filters, on the convolution's kernels.
 * uk_cuda_gemm_f32_workspace_size returns the workspace (2 (N + M) K fp32 plus
 * alignment) when the shape can take the tensor cores (K % 32 == 0 and
 * N % 64 == 0), else 0; uk_cuda_gemm_f32_prefers_tc says whether it gains
 * from them (M N K >= 2^30: below, the FFMA kernel is as fast).
 * uk_cuda_gemm_f32_ws with a workspace of at least that size runs the
 * tensor-core path; with workspace NULL or 0 bytes it is uk_cuda_gemm_f32. */
size_t uk_cuda_gemm_f32_workspace_size(int M, int N, int K);
int uk_cuda_gemm_f32_prefers_tc(int M, int N, int K);
int uk_cuda_gemm_f32_ws(const float* A, const float* B, float* C, int M, int N, int K, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ---- gemm f16 --------------------------------------------------------------
 * C(f16) = A(f16) * B(f16) with fp32 accumulation on the tcgen05 tensor
 * cores; A, B, C are IEEE binary16 bit patterns (uint16_t).  Row-major A[M][K],
 * B[K][N], C[M][N] with leading dimensions lda >= K, ldb >= N, ldc >= N
 * (in elements).  The tensor-core path needs K % 8 == 0, N % 8 == 0, the
 * leading dimensions multiples of 8 and 16-byte aligned pointers; other
 * shapes run a CUDA-core kernel with the same numerics.
 * Replaces uk_gemm_h (src/codegen_hip.cpp:1777-1808). */
int uk_cuda_gemm_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N,
                     int K, void* stream);
int uk_cuda_gemm_f16_ld(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb,
                        uint16_t* C, int64_t ldc, int M, int N, int K, void* stream);

/* The same GEMM from and to HOST memory: hA[M][K], hB[K][N] in, hC[M][N] out
 * (page-locked host memory; anything else is refused with UK_EINVAL), through
 * the caller's device buffers dA, dB, dC of the same shapes.  The copies are
 * pipelined against the GEMM over `chunks` row blocks of A and C (0 = 8):
 * B uploads first, then each block of A; a block's GEMM starts when its rows
 * have landed, and its rows of C download while later blocks compute.  The
 * call is asynchronous on `stream` and complete, C included, when `stream`
 * is.  Two copy streams and their events are created per device on first use
 * and kept; calls on one device from different host threads must not
 * overlap.  This is the reference's end-to-end measurement (upload, run,
 * download: src/codegen_hip.cpp:692-744) with the phases overlapped. */
int uk_cuda_gemm_f16_host(const uint16_t* hA, const uint16_t* hB, uint16_t* hC, uint16_t* dA,
                          uint16_t* dB, uint16_t* dC, int M, int N, int K, int chunks, void* stream);

/* The row ops from and to HOST memory (page-locked hX[L][C], hW[C] for
 * RMSNorm's gamma or channelscale's S, hY[L][C] -- or hY[L] for the reduce),
 * through the caller's device buffers dX, dW, dY of the same shapes: op is
 * UK_OP_REDUCE, UK_OP_SOFTMAX, UK_OP_RMSNORM (eps) or UK_OP_CHANNELSCALE.
 * The copies are pipelined over `chunks` row blocks (0 = 8): W uploads
 * first, then each block of X; a block's op runs once its rows landed and its
 * rows of Y download while later blocks upload, so both directions of the
 * host link run at once.  The reduce takes the workspace of
 * uk_cuda_reduce_workspace_size(rows, C) for a block's rows (NULL when that
 * is 0).  Asynchronous on `stream`, complete (Y included) when `stream` is;
 * shares the copy streams of uk_cuda_gemm_f16_host.  The reference measures
 * each op end to end (upload, run, download: src/codegen_hip.cpp:2036-2126);
 * this overlaps those phases. */
int uk_cuda_rowop_host(int op, const float* hX, const float* hW, float* hY, float* dX, float* dW, float* dY,
                       int64_t L, int64_t C, float eps, int chunks, void* workspace, size_t workspace_bytes,
                       void* stream);

/* The fp32 NCHW convolution (uk_cuda_conv2d_f32_ws) from and to page-locked
 * host memory: hX [N][C][H][W], hW [Oc][C][Kh][Kw], hS [Oc] (or NULL, with dS
 * NULL), hY [N][Oc][Ho][Wo], each with a device buffer of the same size (dX,
 * dW, dS, dY).  Images are independent: the weights upload first, then the
 * images in `chunks` blocks (0: 8); each block's convolution runs once it
 * landed and its Y downloads while later blocks upload, so both directions
 * of the host link run at once.  The workspace is that of one block's
 * images: uk_cuda_conv2d_f32_host_workspace_size(N, ..., chunks) bytes (the
 * split tail is used when it has room, as for the device call).
 * Asynchronous on `stream`, complete (Y included) when `stream` is; shares
 * the copy streams of uk_cuda_gemm_f16_host.  The reference measures its
 * conv end to end (upload, run, download: measured_ms,
 * src/codegen_hip.cpp:692-744); this overlaps those phases. */
size_t uk_cuda_conv2d_f32_host_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc,
                                              int pad, int chunks);
int uk_cuda_conv2d_f32_host(const float* hX, const float* hW, const float* hS, float* hY, float* dX,
                            float* dW, float* dS, float* dY, int N, int H, int W, int C, int Kh,
                            int Kw, int Oc, int pad, int chunks, void* workspace,
                            size_t workspace_bytes, void* stream);

/* GEMM larger than the device (the reference's streamed scenario B,
 * src/codegen_hip.cpp:1143-1238): C = A * B from and to page-locked host
 * memory with only B resident (dB, K*N elements) and A, C passing through a
 * two-slot ring of block_rows-row blocks in `ring` (at least
 * uk_cuda_gemm_streamed_ring_size(M, N, K, kind, block_rows) bytes of device
 * memory).  Block i's upload, GEMM and download overlap blocks i+-1; a slot is
 * reused only after its previous block's GEMM and download finished.  kind:
 *   1  binary16 data on the tensor cores;
 *   0  fp32, on the tensor cores (split-tf32, uk_cuda_gemm_f32_ws) when a
 *      block gains from them, the ring then also holding the tf32 pairs of
 *      B^T (made once per call) and of one block of A; else FFMA;
 *   2  fp32 on the FFMA kernel (the smallest ring).
 * Asynchronous on `stream`; shares the copy streams of uk_cuda_gemm_f16_host. */
size_t uk_cuda_gemm_streamed_ring_size(int M, int N, int K, int kind, int block_rows);
int uk_cuda_gemm_streamed(const void* hA, const void* hB, void* hC, void* dB, void* ring, size_t ring_bytes,
                          int M, int N, int K, int kind, int block_rows, void* stream);

/* ---- multi-GPU f16 GEMM (one process per GPU, NVLink peers) ----------------
 * N-sharded GEMM with the all-gather fused into the store: computes columns
 * [col_offset, col_offset + N_shard) of C = A * B from this rank's column
 * slice of B (B_shard[K][N_shard], leading dimension ldb) and writes every
 * output tile into all n_c (<= 8) copies of the full C[M][ldc]:
 * C_list[0] on this GPU, C_list[1..] other GPUs' buffers opened with
 * uk_cuda_ipc_import.  The caller orders ranks after the call (a stream-
 * ordered barrier) before reading C.  Tensor-core shapes only (K, N_shard,
 * lda, ldb, ldc, col_offset multiples of 8).  No reference counterpart (the
 * reference is single-GPU); the column split and all-gather are the north
 * star's multi-GPU plan. */
int uk_cuda_gemm_f16_allgather(const uint16_t* A, int64_t lda, const uint16_t* B_shard, int64_t ldb,
                               uint16_t* const* C_list, int n_c, int64_t ldc, int M, int N_shard, int K,
                               int64_t col_offset, void* stream);
/* ---- decode layer: RMSNorm -> skinny f16 GEMM ----------------------------
 * For B <= 32 token rows X[B][K] (fp32, contiguous) and this rank's column
 * block W[K][N_shard] (f16, leading dimension ldw) of the layer weight:
 *   Y[b][col_offset + n] = f16( sum_k f16((X[b][k] * rms_b) * gamma[k]) * W[k][n] ),
 *   rms_b = 1 / sqrt(sum_k X[b][k]^2 / K + eps),  fp32 accumulation,
 * written into all n_y (<= 8) copies Y_list[i][B][ldy] (Y_list[0] on this GPU,
 * the others peers' buffers from uk_cuda_ipc_import: the weight-column
 * sharding of the decode layer with its all-gather fused into the store).
 * The normalised f16 rows go to the caller's workspace of
 * uk_cuda_decode_workspace_size(B, K) bytes.  Needs K a multiple of 8, ldw a
 * multiple of 8, X, gamma, W and the workspace 16-byte aligned.
 * Deterministic.  Two kernels (the norm, then tcgen05 tiles of W streamed by
 * TMA, K split over a thread-block cluster when N_shard is narrow) overlapped
 * by programmatic dependent launch.  Replaces the RMSNorm -> fp16 GEMM steps
 * of the decode chain (uk_rmsnorm src/codegen_hip.cpp:2154-2164 and uk_gemm_h
 * :1777-1808 run back to back). */
size_t uk_cuda_decode_workspace_size(int B, int K);
int uk_cuda_decode_rmsnorm_gemm_f16(const float* X, const float* gamma, float eps, const uint16_t* W, int64_t ldw,
                                    uint16_t* const* Y_list, int n_y, int64_t ldy, int B, int N_shard, int K,
                                    int64_t col_offset, void* workspace, size_t workspace_bytes, void* stream);

/* ---- multi-GPU from a C/C++ host, over NCCL (one process per GPU) ----------
 * NCCL is resolved at run time (the process's loaded libnccl, else
 * libnccl.so.2); these calls return UK_ECUDA when it is absent.
 * uk_nccl_get_unique_id: rank 0's id (uk_nccl_unique_id_size() bytes), which
 *   the caller hands to every rank (file, socket, MPI ...).
 * uk_nccl_comm_init: ncclCommInitRankConfig with a non-blocking config,
 *   polled (ncclCommGetAsyncError) for at most timeout_ns: a rank that never
 *   joins ends it with ncclCommAbort and UK_ECUDA instead of a hang.
 * uk_nccl_comm_destroy: aborts (frees) the communicator without a collective
 *   (the peers may be gone); a communicator this library already aborted
 *   after a failure is left alone.
 * uk_shard_gemm_f16_create: for C[M][ldc] on this rank (the full C), this
 *   rank's column block of the N-sharded GEMM (multiples of 8 columns, as
 *   even as possible: uk_shard_gemm_f16_columns) and every rank's C opened
 *   over CUDA IPC, the handles exchanged once with an NCCL all-gather (bounded
 *   by timeout_ns).  Set-up, not a hot call: it allocates a few bytes.
 * uk_shard_gemm_f16_run: one step on `stream`: a one-float NCCL all-reduce
 *   that proves every peer alive and past its previous step, the GEMM of this
 *   rank's column block with its all-gather fused into the store (every
 *   tile into every rank's C, uk_cuda_gemm_f16_allgather), then a second
 *   all-reduce after which every rank's C is complete.  With timeout_ns > 0
 *   the host waits on each all-reduce for at most timeout_ns, polling the
 *   communicator's asynchronous error: a peer that left, stalled or failed
 *   is caught before this rank's kernel stores into its memory, and the call
 *   aborts the communicator and returns UK_ECUDA (the runner's exit code 4)
 *   -- never a hang.  With timeout_ns = 0 the step is enqueued asynchronously.
 *   B_shard is this rank's [K][n1 - n0] column block of B (leading dim ldb).
 * No reference counterpart (the reference is single-GPU; its failure
 * protocol, an exit code per outcome, src/main.cpp:469-539, is kept). */
size_t uk_nccl_unique_id_size(void);
int uk_nccl_get_unique_id(void* out);
int uk_nccl_comm_init(const void* unique_id, int nranks, int rank, uint64_t timeout_ns, void** comm_out);
int uk_nccl_comm_destroy(void* comm);
typedef struct uk_shard_gemm uk_shard_gemm;
int uk_shard_gemm_f16_create(void* comm, int rank, int nranks, uint16_t* C, int64_t ldc, int M, int N, int K,
                             uint64_t timeout_ns, uk_shard_gemm** out);
int uk_shard_gemm_f16_columns(const uk_shard_gemm* h, int64_t* n0, int64_t* n1);
int uk_shard_gemm_f16_run(uk_shard_gemm* h, const uint16_t* A, int64_t lda, const uint16_t* B_shard, int64_t ldb,
                          void* stream, uint64_t timeout_ns);
int uk_shard_gemm_f16_destroy(uk_shard_gemm* h);

/* CUDA IPC: export a device buffer (handle of uk_cuda_ipc_handle_size() bytes
 * plus the offset of `ptr` inside its allocation), open a peer's export as a
 * pointer on this device, close it.  No reference counterpart. */
size_t uk_cuda_ipc_handle_size(void);
int uk_cuda_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
int uk_cuda_ipc_import(const void* handle, uint64_t offset, void** ptr_out);
int uk_cuda_ipc_close(void* ptr, uint64_t offset);

/* Device-side barrier of the ranks of one node (one process per GPU): a
 * one-warp kernel on `stream` posts `epoch` into every rank's flag array at
 * this rank's slot (flag_list[r] = rank r's array of n unsigned ints, in rank
 * order, this rank's own included; peers' arrays opened with
 * uk_cuda_ipc_import), with a system-scope release that makes everything this
 * GPU wrote earlier on the stream (the sharded GEMM's peer stores included)
 * visible first; it then waits until every rank's post of `epoch` (or a later
 * one) is in its own array.  Epochs only grow (the caller counts steps from
 * 1; arrays start at 0).  A wait longer than timeout_ns (1 us .. 60 s) gives
 * up and sets bit 32 of uk_cuda_pipeline_fault: an error status, never a
 * hang.  Each rank runs it on its own GPU: ranks that share a GPU must not use
 * it.  No reference counterpart (the reference is single-GPU). */
int uk_cuda_peer_barrier(unsigned* const* flag_list, int n, int rank, unsigned epoch, uint64_t timeout_ns,
                         void* stream);

/* Fault word of the tensor-core pipelines: 0 when no bounded wait inside a
 * kernel of this library expired since the last call, otherwise a bit mask
 * (1 producer, 2 MMA issuer, 4 epilogue, 8 teardown, 16 self-test, 32 peer
 * wait).  Synchronises with the device and clears the word.  A kernel whose
 * wait expires unwinds and leaves its outputs undefined instead of hanging.
 * No reference counterpart (the reference has no device-side waits). */
unsigned uk_cuda_pipeline_fault(void);

/* Failure detection check: one CTA runs the pipelines' bounded mbarrier wait
 * (the one every producer, MMA and epilogue wait uses) on a barrier that
 * nothing completes unless `arrive` != 0.  Without the arrival the wait gives
 * up after timeout_ns (1 us .. 1 s), sets bit 16 of the fault word and writes
 * *status = 0; with it *status = 1.  The context stays usable either way.
 * status is one device int. */
int uk_cuda_selftest_wait(int arrive, uint64_t timeout_ns, int* status, void* stream);

/* ---- conv2d ----------------------------------------------------------------
 * layout UK_CONV_KML: the KML conv contract, one image, valid padding:
 *   X[H][W][C], Wt[Oc][Kh][Kw][C], Y[Oc][Ho][Wo], Ho = H-Kh+1, Wo = W-Kw+1;
 *   N must be 1 and pad 0 (src/reference.cpp:6-22, src/codegen_hip.cpp:337-411).
 * layout UK_CONV_NCHW: X[N][C][H][W], Wt[Oc][C][Kh][Kw], Y[N][Oc][Ho][Wo],
 *   zero padding `pad`, stride 1, Ho = H+2pad-Kh+1.
 * scale (may be NULL): per-output-channel factor s[Oc] applied in the
 * epilogue (the fused channelscale).  fp32 FFMA implicit GEMM. */
#define UK_CONV_KML 0
#define UK_CONV_NCHW 1
int uk_cuda_conv2d_f32(const float* X, const float* Wt, float* Y, int N, int H, int W,
                       int C, int Kh, int Kw, int Oc, int pad, const float* scale,
                       int layout, void* stream);

/* The same convolution on the tcgen05 tensor cores, at fp32 accuracy: the
 * operands are split into tf32 (hi, lo) pairs and each step accumulates
 * lo*hi + hi*lo + hi*hi in fp32 (within a few ulps of the output scale of
 * an fp32 FFMA result; the fp32 gate, 1e-4 against fp64, holds).  The split
 * operands (and, for NCHW, the input transposed to NHWC) live in a caller
 * workspace of uk_cuda_conv2d_workspace_size(...) bytes (16-byte aligned).
 * The size includes room for the fp32 partial tiles of the last round of
 * tiles, which the kernel then splits along K over the SM pairs that round
 * would leave idle (summed by a second, deterministic kernel); a smaller
 * workspace that still holds the operand pairs runs without the split.
 * Takes the tensor cores when C is a multiple of 32; other shapes run the
 * FFMA kernel of uk_cuda_conv2d_f32 (the size query then returns 0 and the
 * workspace may be NULL).  Replaces uk_conv<OCB>/uk_conv_g
 * (src/codegen_hip.cpp:337-411) at the sizes where the tensor cores pay. */
size_t uk_cuda_conv2d_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc,
                                     int pad, int layout);

/* fp16 convolution on the tcgen05 tensor cores (kind::f16 MMAs over SM
 * pairs): X, Wt, scale and Y are IEEE binary16 (uint16_t bit patterns) in the
 * layouts of uk_cuda_conv2d_f32; fp32 accumulation, the scale applied in
 * fp32, one rounding to f16.  Needs C a multiple of 64.  The KML layout (HWC
 * input, [Oc][Kh][Kw][C] weights) is read in place and runs without a
 * workspace; NCHW takes a workspace of uk_cuda_conv2d_f16_workspace_size(...)
 * bytes for the NHWC copy of X and the permuted weights.  For either layout
 * the size also covers the last round's split partial tiles (as for fp32),
 * used when the workspace passed has room for them.  The reference refuses fp16
 * conv (src/codegen_hip.cpp:81-89); this widens the dtype interval. */
size_t uk_cuda_conv2d_f16_workspace_size(int N, int H, int W, int C, int Kh, int Kw, int Oc,
                                         int pad, int layout);
int uk_cuda_conv2d_f16(const uint16_t* X, const uint16_t* Wt, uint16_t* Y, int N, int H, int W,
                       int C, int Kh, int Kw, int Oc, int pad, const uint16_t* scale, int layout,
                       void* workspace, size_t workspace_bytes, void* stream);
int uk_cuda_conv2d_f32_ws(const float* X, const float* Wt, float* Y, int N, int H, int W,
                          int C, int Kh, int Kw, int Oc, int pad, const float* scale,
                          int layout, void* workspace, size_t workspace_bytes, void* stream);

/* The NCHW tensor-core fp32 conv (uk_cuda_conv2d_f32_ws, C a multiple of 32)
 * with its output stored into n_y (<= 8) copies of Y: Y_list[0] on this GPU,
 * Y_list[1..] other GPUs' buffers opened with uk_cuda_ipc_import, each
 * pointing at the same place (this rank's first image).  That is the
 * batch-sharded conv with its all-gather fused into the store: rank r passes
 * its image block X[b0:b1] (N = b1 - b0) and every rank's Y + b0 * Oc * Ho * Wo,
 * and orders the ranks after the call (uk_cuda_peer_barrier) before reading
 * Y.  Same workspace as uk_cuda_conv2d_f32_ws.  No reference counterpart (the
 * reference is single-GPU); the batch split and all-gather are the north
 * star's multi-GPU plan for the conv. */
int uk_cuda_conv2d_f32_allgather(const float* X, const float* Wt, float* const* Y_list, int n_y, int N, int H, int W,
                                 int C, int Kh, int Kw, int Oc, int pad, const float* scale, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ---- KML runner (host side; the nvidia branch of `unikern run`) -----------
 * uk_kml_describe: the KML contract for one declaration, no GPU needed.
 *   Writes "key=value" lines to out: canonical= (canonical_form), signature=
 *   (op_signature), ops= / bytes= (workload_of), tolerance= (the verify gate of
 *   the dtype), gap= (empty when nvidia:cuda runs the tree), and with an HCS
 *   also hcs_fingerprint=, ledger_key=, tile=, k_block=, stages=, c_ms=,
 *   placement= (the solver, on `sms` multiprocessors; 0 = the HCS's
 *   compute_units), then export= and the exported JSON.  A rejected
 *   declaration returns UK_EINVAL with the reference's "rejected (N
 *   violations): ..." text in out.
 *   Replaces kml_import / canonical_form / op_signature / workload_of /
 *   hcs_fingerprint / the ledger key (src/kml_front.cpp:75-251,
 *   src/kml.cpp:60-177, src/hcs.cpp:52-115, src/main.cpp:217-219).
 * uk_run_kml: import the HCS and the KML tree, look the ledger key up in the
 *   ledger (a hit reuses the recorded tile), solve on a
 *   miss, run the tree on the current device (verify instance checked on the
 *   GPU in fp64 against the dtype's gate, then e2e and kernel-only timing at
 *   the declared dims), and commit a verified run when write_ledger != 0.
 *   The transcript (LEDGER HIT, UNIKERN_RESULT backend=nvidia:cuda ..., RUN
 *   ..., LEDGER COMMIT ...) goes to out.  Returns cmd_run's exit code: 0 ok,
 *   1 run failed or verify FAIL, 2 bad input / unsupported tree, 3
 *   infeasible, 5 residency violation.  ledger_path may be NULL (no ledger).
 *   Replaces cmd_run's execute branch + run_ocl/run_hip (src/main.cpp:346-570,
 *   src/runner_ocl.cpp); allocates its own device and pinned buffers (this is
 *   the runner, not a hot call).
 * Ledgers (both entry points, and uk_calibrate): a path ending in ".jsonl"
 *   is the reference's TAB-separated file ledger (src/runtime.cpp:20-170);
 *   any other path is an SQLite database with the reference's solutions /
 *   violations tables, one row per key, each write in BEGIN IMMEDIATE ..
 *   COMMIT (src/sqlite_ledger.cpp:44-133; the choice is src/main.cpp:61-70's).
 *   The SQLite engine is the system's libsqlite3.so.0, loaded on first use;
 *   without it a non-.jsonl path is refused with exit code 2.
 * uk_solve_kml: `unikern solve`'s nvidia branch (src/main.cpp:276-343): the
 *   gap check, a ledger lookup (LEDGER HIT reuses the recorded tile) or the
 *   solver on `sms` multiprocessors (0 = the HCS's compute_units), and, when
 *   write_ledger != 0, a solve-time row (measured_ms = c_ms, kernel_ms = 0; a
 *   later run of the same key overwrites it).  Transcript (LEDGER HIT ... or
 *   SOLVED  x* tile=MxN  c_ms=...) to out.  Returns 0, 2 bad input /
 *   unsupported tree / ledger error, 3 infeasible.  No GPU needed. */
int uk_kml_describe(const char* kml_json, const char* hcs_json, int sms, char* out, size_t out_cap);
int uk_solve_kml(const char* hcs_json, const char* kml_json, const char* ledger_path, int write_ledger, int sms,
                 char* out, size_t out_cap);
int uk_run_kml(const char* hcs_json, const char* kml_json, const char* ledger_path, int write_ledger, char* out,
               size_t out_cap);

/* run_cuda as a C call: run one tree on the current device exactly as
 * uk_run_kml does (verify instance checked in fp64 on the GPU against the
 * dtype's gate, then e2e and kernel-only timing at the declared dims, the
 * UNIKERN_RESULT line), without the ledger and without solving: tile_m /
 * tile_n are the caller's solution's tile, reported on the result line.  The
 * fields of *out are RunOutcome's (include/unikern/codegen.hpp:49-83), so a
 * reference-side run_cuda(Solution, Hcs, KmlTree, workdir) fills its
 * RunOutcome from them field by field (src/runner.cpp:195-237 parses the
 * same values from a HIP program's result line).  migrations / checks are -1
 * when the run never reached a result line; stream_path is "pinned" once it
 * ran.  log gets the transcript (UNIKERN_INFO / UNIKERN_RESULT lines, or the
 * reason it did not run).  Returns UK_OK when *out was filled (the run's own
 * status is out->exit_code: 0 pass, 1 verify FAIL, 2 unsupported tree, 4 no
 * usable device or a CUDA error, 5 residency violation), UK_EINVAL when the
 * HCS or KML is rejected (log gets the reason). */
typedef struct uk_run_outcome {
  int built, ran, verified;
  double max_rel, measured_ms, kernel_ms;
  int migrations, checks;
  unsigned long long vram_free, vram_total;
  int exit_code;
  char stream_path[16];
} uk_run_outcome;
int uk_run_cuda(const char* hcs_json, const char* kml_json, int tile_m, int tile_n, uk_run_outcome* out, char* log,
                size_t log_cap);

/* `unikern calibrate` (src/main.cpp:573-652, src/solver.cpp:188-245): read the
 * rows the ledger at ledger_path measured under the HCS's fingerprint, take
 * per usable row (measured_ms > kernel_ms > 0) the compulsory bytes of its
 * signature's tree over measured_ms - kernel_ms, and write the HCS with
 * link_bw_gbps = the median and constants_version + 1 (flat JSON that
 * round-trips through the importer) to hcs_out; the report ("CALIBRATED
 * link_bw_gbps a -> b constants_version ...", the per-row detail, "PREDICTED
 * demo c_ms ...") or the skip reason goes to out.  Returns 0 calibrated, 2 bad
 * input, 3 skipped: a unified-memory HCS without allow_unified (checked before
 * the ledger is read), no measured rows, or none usable.  No GPU needed. */
int uk_calibrate(const char* hcs_json, const char* ledger_path, int allow_unified, char* hcs_out, size_t hcs_cap,
                 char* out, size_t out_cap);

#ifdef __cplusplus
}
#endif

#endif /* UNIKERN_CUDA_H */
