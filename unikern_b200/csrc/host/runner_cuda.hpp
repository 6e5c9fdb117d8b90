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
//   FileLedger ............ src/runtime.cpp:20-170 (TAB rows, #VIOLATION events)
//   run flow .............. cmd_run, src/main.cpp:346-570
#pragma once

#include <optional>
#include <string>

#include "kml.hpp"

namespace ukb {

struct Instance {
  int tile_m = 0, tile_n = 0, k_block = 0, stages = 0;
};

struct Solution {
  Instance best;
  double c_ms = 0;  // predicted end-to-end time (roofline + host link copies)
  int feasible_count = 0;
  bool from_ledger = false;
  std::string placement_record;
};

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
  bool supports_streaming() const { return false; }
  std::string capability_gap(const KmlTree& t) const;  // "" = supported
};

class FileLedger {
 public:
  explicit FileLedger(std::string path) : path_(std::move(path)) {}
  std::optional<Solution> lookup(const std::string& key) const;
  void commit(const std::string& key, const Solution& s, double measured_ms, double kernel_ms) const;
  void record_violation(const std::string& key, double rate, double threshold, int migrations, int checks,
                        unsigned long long vram_free) const;
  int size() const;

 private:
  std::string path_;
};

// cmd_run's nvidia branch (run: write_ledger = true; verify: false).  Returns
// cmd_run's exit code: 0 committed / verified, 1 run failed, 2 bad input or
// unsupported tree, 3 infeasible, 5 residency violation.  Everything cmd_run
// would print goes to *transcript.
int run_kml(const std::string& hcs_json, const std::string& kml_json, const std::string& ledger_path,
            bool write_ledger, std::string* transcript);

}  // namespace ukb
