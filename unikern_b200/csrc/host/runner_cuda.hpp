// runner_cuda.hpp -- the nvidia:cuda backend of the KML runner: solve (tile
// choice re-targeted to the B200 kernels), run_cuda (verify instance + timing
// + result line, in process), the file ledger, and the backend descriptor.
//
// Reference shapes it keeps (UNIKERN, file:line):
//   RunOutcome ............ include/unikern/codegen.hpp:49-83
//   run_cuda .............. same signature as run_ocl, :104-106; protocol of
//                           src/runner_ocl.cpp (verify instance, warm/iters,
//                           e2e and kernel-only spans, result line :834-841)
//   BackendNvidia ......... IBackend, include/unikern/components.hpp:14-33
//   ledger ................ ledger.hpp: TAB file ledger for .jsonl paths
//                           (src/runtime.cpp:20-170), SQLite for the rest
//                           (src/sqlite_ledger.cpp, src/main.cpp:61-70)
//   solve ................. cmd_solve, src/main.cpp:276-343
//   run flow .............. cmd_run, src/main.cpp:346-570
//   scenario B ............ src/codegen_hip.cpp:1143-1238, :1485-1500
//   calibrate ............. cmd_calibrate, src/main.cpp:573-652;
//                           calibrated_link_bw, src/solver.cpp:188-245
#pragma once

#include <optional>
#include <string>
#include <vector>

#include "kml.hpp"
#include "ledger.hpp"

namespace ukb {

// Pure function of (hcs, tree, sms): the tile the library launches for the
// tree (uk_cuda_tile_plan) and its predicted cost from the HCS constants.
Solution solve_b200(const Hcs& h, const KmlTree& t, int sms);

struct RunOutcome {
  bool built = false, ran = false, verified = false;
  double max_rel = 0, measured_ms = 0, kernel_ms = 0;
  int migrations = -1, checks = -1;
  unsigned long long vram_free = 0, vram_total = 0;
  int exit_code = 0;
  std::string stream_path;  // the host data path of a run: "pinned" (page-locked copies) once it ran
  std::string result_line;  // the UNIKERN_RESULT line (or the UNIKERN_ERROR line)
  std::string log;
};

RunOutcome run_cuda(const Solution& sol, const Hcs& hcs, const KmlTree& tree, const std::string& workdir);

class BackendNvidia {
 public:
  const char* vendor() const { return "nvidia"; }
  const char* name() const { return "nvidia:cuda"; }
  bool available() const;  // a CUDA device of compute capability 10.0
  // provenance text: no source is generated, the kernels are precompiled
  std::string generate(const Solution& s, const Hcs& h, const KmlTree& t) const;
  bool supports_streaming() const { return true; }  // gemm operands, with B resident
  std::string capability_gap(const KmlTree& t) const;  // "" = supported
};

// The effective host link bandwidth (GB/s) from measured rows: per row the
// compulsory bytes of its signature's tree over measured_ms - kernel_ms, and
// the median over usable rows (the mean of the middle two for an even
// count); 0 when no row is usable (src/solver.cpp:188-245 of UNIKERN).
double calibrated_link_bw(const std::vector<MeasuredRow>& rows, std::string* detail);

// cmd_calibrate (src/main.cpp:573-652 of UNIKERN): reads the rows measured
// under the HCS's fingerprint, writes the HCS with the calibrated
// link_bw_gbps and constants_version + 1 to *hcs_out, and the report to
// *transcript.  Returns 0 calibrated, 2 bad HCS, 3 skipped (a unified-memory
// HCS without allow_unified, no measured rows, or no usable row).
int calibrate(const std::string& hcs_json, const std::string& ledger_path, bool allow_unified,
              std::string* hcs_out, std::string* transcript);

// cmd_solve's nvidia branch (src/main.cpp:276-343): ledger lookup (a hit
// reuses the recorded tile) or solve_b200 on `sms` multiprocessors (0 = the
// HCS's compute_units), then a solve-time row (measured_ms seeded with c_ms,
// kernel_ms 0; a later run overwrites it) when write_ledger.  No GPU needed.
// Returns 0 solved or hit, 2 bad input / unsupported tree / ledger error,
// 3 infeasible; the transcript (LEDGER HIT / SOLVED lines) goes to *transcript.
int solve_kml(const std::string& hcs_json, const std::string& kml_json, const std::string& ledger_path,
              bool write_ledger, int sms, std::string* transcript);

// cmd_run's nvidia branch (run: write_ledger = true; verify: false).  Returns
// cmd_run's exit code: 0 committed / verified, 1 run failed, 2 bad input or
// unsupported tree, 3 infeasible, 5 residency violation.  Everything cmd_run
// would print goes to *transcript.
int run_kml(const std::string& hcs_json, const std::string& kml_json, const std::string& ledger_path,
            bool write_ledger, std::string* transcript);

}  // namespace ukb
