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

#include <cmath>

namespace uk {

struct Tile {
  int bm, bn, bk, stages;
};

// f16 tensor-core GEMM: 128 x 256 UMMA tile, 64-deep K blocks, 4-stage ring
// (single SM); and the SM-pair kernel's 256 x 256 tile (128 rows per SM,
// 6-stage ring), which runs whenever M > 128
constexpr Tile kGemmF16Tile = {128, 256, 64, 4};
constexpr Tile kGemmF16PairTile = {256, 256, 64, 6};

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

// ---- solve: the Blackwell candidate grid ---------------------------------------
//
// The re-target of the reference's solver (src/solver.cpp): sketch a grid of
// candidates (:14-47), keep the feasible ones (:54-77), cost each with a pure
// function of the shape and the machine (:81-120), and take the lexicographic
// argmin of (cost, candidate key) (:153-179).  Here a candidate is a kernel
// family with its tile, K split and stage count, and the cost is device time:
//   waves x (work one SM does per wave) / (its peak x the family's measured
//   efficiency), plus the fixed latency of a tile, the pre-passes the family
//   needs, the split fold and one launch per kernel;
// and never less than the compulsory bytes over HBM bandwidth.  The launchers
// call the same argmin, so the solver's choice is the kernel that runs, and
// uk_cuda_tile_plan / the ledger's tm, tn report it.

enum Family : int {
  kFamSgemm = 0,      // FFMA register-blocked GEMM (gemm_f32.cu)
  kFamF16Single = 1,  // tcgen05 cta_group::1, 128 x 256 per SM (gemm_f16.cu)
  kFamF16Pair = 2,    // tcgen05 cta_group::2, 256 x 256 per SM pair (gemm_f16_2sm.cu)
  kFamTf32x3 = 3,     // fp32 as split-tf32 on the conv pair kernel (conv_tc.cu)
  kFamConvFfma = 4,   // FFMA implicit-GEMM conv (conv_f32.cu)
  kFamConvPair = 5,   // tcgen05 conv on SM pairs, split-tf32 or f16 (conv_tc.cu)
  kFamSkinny = 6,     // tcgen05 skinny GEMM of the decode chain, K split over a cluster (decode.cu)
  kFamSgemmGroups = 7,  // FFMA 32 x 64 tile with K split over warp groups of one CTA (gemm_f32.cu)
};

inline const char* family_name(int f) {
  switch (f) {
    case kFamSgemm: return "ffma";
    case kFamF16Single: return "tcgen05-1sm";
    case kFamF16Pair: return "tcgen05-2sm";
    case kFamTf32x3: return "tcgen05-2sm-3xtf32";
    case kFamConvFfma: return "ffma-conv";
    case kFamConvPair: return "tcgen05-2sm-conv";
    case kFamSkinny: return "tcgen05-skinny";
    case kFamSgemmGroups: return "ffma-kgroups";
  }
  return "?";
}

struct Candidate {
  int family = -1;
  Tile tile{0, 0, 0, 0};
  int ksplit = 1;
  double us = 0;  // predicted device time
};

// The machine model: a B200 at 1965 MHz.  Peaks: the measured dense f16
// tensor rate and copy bandwidth of this pool's B200s, the nominal FFMA rate.
// Efficiencies are the measured fraction of peak each family sustains in
// steady state: the tcgen05 kernels' tensor-pipe activity in ncu (92 % for
// the pair GEMM, 91 % for the split-tf32 pair kernel) and the single-SM GEMM's
// measured rate at 8192^3 (86 %); the FFMA tiles' rates from a sweep of every
// compiled tile and K split on a B200 (128 x 128: 60 % of the nominal FFMA
// peak, 64 x 64: 42 %, 32 x 64: 45 % once 16 warps per SM hide latency,
// falling with the square root of the warps below that; a K-split fold costs
// about 0.6 us per CTA of the cluster); a tile's fixed cost (pipeline fill,
// epilogue drain) is 1-2 us, a launch 2 us.
struct CostModel {
  double f16_tflops_sm = 1620.0 / 148;  // per SM (a part with fewer SMs has proportionally less)
  double ffma_tflops_sm = 74.4 / 148;
  double hbm_gbs = 6544.0;
  double launch_us = 2.0;
};

namespace detail {

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// time of `units` equal work items of `flops` each on `slots` processors
// (SMs or SM pairs), each slot at `rate` flop/s; items go round-robin
inline double waves_us(int64_t units, int64_t slots, double flops, double rate, double lat_us) {
  const int64_t waves = cdiv(units, slots > 0 ? slots : 1);
  return (double)waves * (flops / rate * 1e6 + lat_us);
}

// FFMA tile shapes the sgemm kernel is compiled for: {bm, bn, bk, threads}
// with the measured fraction of the FFMA peak one SM reaches with it, and the
// K splits (over a cluster) compiled for it as a bit mask of ks in {1,2,4,8}.
// The 64 x 64 tile comes twice: 4 x 4 per thread (256 threads, whole K) and
// 8 x 8 per thread (64 threads, twice the FFMAs per shared-memory load, K
// split 4 or 8 ways); its 0.58 is fitted to one B200's times of every plan at
// 256^3 .. 2048^3 and 1000 x 3000 x 700 with the L2 flushed before each run.
struct SgemmShape {
  int bm, bn, bk, threads;
  double eff;
  unsigned splits;  // bit (log2 ks) set when that split is compiled
};
constexpr SgemmShape kSgemmShapes[] = {{128, 128, 8, 256, 0.60, 0x1},
                                       {64, 64, 8, 256, 0.42, 0x1},
                                       {64, 64, 16, 64, 0.58, 0x4 | 0x8},
                                       {32, 64, 16, 128, 0.45, 0x1 | 0x2 | 0x4 | 0x8}};

}  // namespace detail

// f32 / CUDA-core GEMM on the FFMA pipes: every compiled tile with each K
// split compiled for it (a cluster of up to 8 CTAs, each keeping >= 64 of K)
inline void sgemm_candidates(int64_t M, int64_t N, int64_t K, int64_t sms, const CostModel& cm,
                             Candidate* out, int* n) {
  const double sm_rate = cm.ffma_tflops_sm * 1e12;
  for (const auto& s : detail::kSgemmShapes) {
    const int64_t tiles = detail::cdiv(M, s.bm) * detail::cdiv(N, s.bn);
    for (int ks = 1, lg = 0; ks <= 8; ks *= 2, ++lg) {
      if (!(s.splits & (1u << lg)) || (ks > 1 && K / ks < 64)) continue;
      const int64_t ctas = tiles * ks;
      // resident CTAs per SM: 2048 threads, at most 16 CTAs; a wave is one
      // round of resident CTAs, and too few warps per SM cost latency hiding:
      // 16 warps for a 4 x 4 micro-tile, fewer in proportion for larger ones
      // (an 8 x 8 micro-tile has four times the independent FFMAs per load)
      const int64_t per_sm = 2048 / s.threads < 16 ? 2048 / s.threads : 16;
      const int64_t load = detail::cdiv(ctas, sms);  // CTAs the busiest SM runs
      const int64_t warps = (load < per_sm ? load : per_sm) * s.threads / 32;
      const double need = 16.0 * 16.0 / ((double)s.bm * s.bn / s.threads);
      const double hide = warps >= need ? 1.0 : std::sqrt((double)warps / need);
      const double flops_sm = (double)load * 2.0 * s.bm * s.bn * (double)K / ks;
      double us = flops_sm / (sm_rate * s.eff * hide) * 1e6 + 1.0 * detail::cdiv(load, per_sm);
      if (ks > 1) us += 0.6 * ks;  // the cluster barrier and distributed-shared-memory fold
      us += cm.launch_us;
      out[(*n)++] = Candidate{kFamSgemm, Tile{s.bm, s.bn, s.bk, 2}, ks, us};
    }
  }
}

// f16 GEMM on the tensor cores: the single-SM and the SM-pair kernel (the
// pair needs two 128-row blocks of M)
inline void f16_gemm_candidates(int64_t M, int64_t N, int64_t K, int64_t sms, const CostModel& cm,
                                Candidate* out, int* n) {
  const double sm_rate = cm.f16_tflops_sm * 1e12;
  {
    const Tile t = kGemmF16Tile;
    const int64_t tiles = detail::cdiv(M, t.bm) * detail::cdiv(N, t.bn);
    const double us = detail::waves_us(tiles, sms, 2.0 * t.bm * t.bn * K, sm_rate * 0.86, 1.5) + cm.launch_us;
    out[(*n)++] = Candidate{kFamF16Single, t, 1, us};
  }
  if (M > 128) {
    const Tile t = kGemmF16PairTile;
    const int64_t tiles = detail::cdiv(M, t.bm) * detail::cdiv(N, t.bn);
    const double us =
        detail::waves_us(tiles, sms / 2, 2.0 * t.bm * t.bn * K, 2.0 * sm_rate * 0.92, 1.5) + cm.launch_us;
    out[(*n)++] = Candidate{kFamF16Pair, t, 1, us};
  }
}

// fp32 GEMM as the 1 x 1 convolution on the split-tf32 pair kernel (K % 32,
// N % 64): the tf32 (hi, lo) pre-passes of A and B^T, then 256 x 256 tiles at a
// sixth of the f16 rate (three tf32 MMAs at half rate), the last round of
// tiles split along K over the pairs it would leave idle
inline void tf32x3_gemm_candidates(int64_t M, int64_t N, int64_t K, int64_t sms, const CostModel& cm,
                                   Candidate* out, int* n) {
  if (K % 32 != 0 || N % 64 != 0) return;
  const Tile t = kConvPairF32Tile;
  const double pair_rate = 2.0 * cm.f16_tflops_sm * 1e12 / 6.0 * 0.91;
  const int64_t tiles = detail::cdiv(M, t.bm) * detail::cdiv(N, t.bn);
  const int64_t pairs = sms / 2;
  const int64_t full = tiles / pairs, last = tiles % pairs;
  const double tile_us = 2.0 * t.bm * t.bn * K / pair_rate * 1e6 + 2.0;
  double us = (double)full * tile_us;
  if (last > 0) us += tile_us * (double)last / (double)pairs + 2.0 + cm.launch_us;  // split last round + its fold
  const double prepass_bytes = 3.0 * (double)(M + N) * (double)K * 4.0;
  us += prepass_bytes / (cm.hbm_gbs * 1e9) * 1e6 + 3.0 * cm.launch_us;
  out[(*n)++] = Candidate{kFamTf32x3, t, 1, us};
}

// a candidate's key for the lexicographic tie-break (src/solver.cpp:153-179)
inline bool candidate_less(const Candidate& a, const Candidate& b) {
  if (a.us != b.us) return a.us < b.us;
  if (a.family != b.family) return a.family < b.family;
  if (a.tile.bm != b.tile.bm) return a.tile.bm < b.tile.bm;
  if (a.tile.bn != b.tile.bn) return a.tile.bn < b.tile.bn;
  return a.ksplit < b.ksplit;
}

inline Candidate argmin(const Candidate* c, int n) {
  Candidate best{};
  for (int i = 0; i < n; ++i)
    if (best.family < 0 || candidate_less(c[i], best)) best = c[i];
  return best;
}

constexpr int kMaxCandidates = 16;

// The GEMM solve.  f16: the tensor-core families (the caller checks the
// tensor-core shape rules).  fp32: the FFMA candidates, and with allow_tc the
// split-tf32 one, which is taken only from 2^30 multiply-adds (below that its
// pre-passes and launches are never repaid on a B200: measured).
inline Candidate solve_gemm(int64_t M, int64_t N, int64_t K, bool f16, bool allow_tc, int64_t sms,
                            int* n_feasible = nullptr, const CostModel& cm = CostModel{}) {
  Candidate c[kMaxCandidates];
  int n = 0;
  if (f16) {
    f16_gemm_candidates(M, N, K, sms, cm, c, &n);
  } else {
    sgemm_candidates(M, N, K, sms, cm, c, &n);
    if (allow_tc && M * N * K >= ((int64_t)1 << 30)) tf32x3_gemm_candidates(M, N, K, sms, cm, c, &n);
  }
  if (n_feasible) *n_feasible = n;
  return argmin(c, n);
}

}  // namespace uk
