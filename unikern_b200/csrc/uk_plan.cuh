// uk_plan.cuh -- launch-plan rules of every kernel family, in one place so the
// launchers and the plan query (uk_cuda_tile_plan, which the runner's solver
// and the ledger's tile_m/tile_n columns read) can never disagree.
//
// This is the Blackwell re-target of the reference's tile choice
// (emit_tile_for, src/codegen_hip.cpp:58-68, which clamps the solver's
// tm/tn to 32-96, and uk_conv_plan / uk_reduce_width_plan, :420-599,
// :874-908): tiles are sized so that a 148-SM part gets at least one CTA per
// SM, and the f16 GEMM uses the one tcgen05 tile the tensor-core kernel is
// built for.  Pure host functions of the shape and the SM count.
#pragma once

#include <stdint.h>

namespace uk {

struct Tile {
  int bm, bn, bk, stages;
};

// f16 tensor-core GEMM: 128 x 256 UMMA tile, 64-deep K blocks, 4-stage ring
// (single SM); and the SM-pair kernel's 256 x 256 tile (128 rows per SM,
// 6-stage ring), which runs whenever M > 128
constexpr Tile kGemmF16Tile = {128, 256, 64, 4};
constexpr Tile kGemmF16PairTile = {256, 256, 64, 6};

// f32 FFMA GEMM (and the CUDA-core f16 path): the largest tile that still
// gives every SM a CTA; double-buffered shared memory (2 stages)
inline Tile sgemm_tile(int64_t M, int64_t N, int64_t sms) {
  auto ctas = [&](int bm, int bn) { return ((M + bm - 1) / bm) * ((N + bn - 1) / bn); };
  if (ctas(128, 128) >= sms) return {128, 128, 8, 2};
  if (ctas(64, 64) >= sms) return {64, 64, 8, 2};
  return {32, 64, 16, 2};
}

// K split of the smallest f32 tile (32 x 64): CTAs per tile (a cluster along
// K) so that up to UK_SGEMM_SPLIT_CAP CTAs per SM run, each keeping >= 64 of K
#ifndef UK_SGEMM_SPLIT_CAP
#define UK_SGEMM_SPLIT_CAP 4
#endif
inline int sgemm_ksplit(int64_t M, int64_t N, int64_t K, int64_t sms) {
  const int64_t ctas = ((M + 31) / 32) * ((N + 63) / 64);
  int ks = 1;
  while (ks < 8 && ctas * ks * 2 <= UK_SGEMM_SPLIT_CAP * sms && K / (ks * 2) >= 64) ks *= 2;
  return ks;
}

// the tensor-core convolutions on SM pairs (also the fp32 GEMM run as a 1 x 1
// convolution): 256 output channels x 256 pixels per pair, 32 fp32 channels
// (split-tf32, 3 stages) or 64 fp16 channels (6 stages) per k-step
constexpr Tile kConvPairF32Tile{256, 256, 32, 3};
constexpr Tile kConvPairF16Tile{256, 256, 64, 6};

// implicit-GEMM FFMA conv: rows = output channels, columns = output pixels
inline Tile conv_tile(int64_t npix, int64_t Oc, int64_t sms) {
  auto ctas = [&](int bm, int bn) { return ((npix + bn - 1) / bn) * ((Oc + bm - 1) / bm); };
  if (ctas(128, 128) >= sms && Oc > 64) return {128, 128, 8, 2};
  if (ctas(64, 64) >= sms || Oc <= 32) return {64, 64, 8, 2};
  return {32, 64, 16, 2};
}

// RMSNorm / softmax with the row in registers: the fewest threads that keep at
// most 8 (vec4) or 8 (scalar) vectors per thread.  false = the row is too long
// for registers and the two-pass streaming kernel runs instead.
inline bool rowop_plan(int64_t C, int W, int* threads, int* vpt) {
  static const int v4[][2] = {{32, 1}, {32, 2}, {64, 2}, {128, 2}, {128, 4},
                              {256, 4}, {256, 8}, {512, 8}, {512, 16}};
  static const int v1[][2] = {{32, 1}, {64, 2}, {128, 4}, {256, 4}, {256, 8}};
  const int64_t nv = C / W;
  const int(*t)[2] = W == 4 ? v4 : v1;
  const int n = W == 4 ? 9 : 5;
  for (int i = 0; i < n; ++i)
    if (nv <= (int64_t)t[i][0] * t[i][1]) {
      *threads = t[i][0];
      *vpt = t[i][1];
      return true;
    }
  *threads = 512;
  *vpt = 0;
  return false;
}

// reduce: 0 zero-fill (cols = 0), 1 CTA per row, 2 warp per row, 3 each row
// split into `splits` chunks of `chunk` columns (partials + a fixed-order fold)
struct ReducePlan {
  int mode;
  int64_t splits, chunk;
};

inline ReducePlan plan_reduce(int64_t rows, int64_t cols, int64_t sms) {
  if (cols == 0) return {0, 0, 0};
  const int64_t target = sms * 8;
  if (rows >= target / 2 || cols < 16384) return {cols >= 1024 ? 1 : 2, 1, cols};
  int64_t splits = (target + rows - 1) / rows;
  const int64_t cap = cols / 4096;
  if (splits > cap) splits = cap;
  if (splits <= 1) return {1, 1, cols};
  int64_t chunk = (cols + splits - 1) / splits;
  chunk = (chunk + 3) / 4 * 4;
  splits = (cols + chunk - 1) / chunk;
  return {3, splits, chunk};
}

}  // namespace uk
