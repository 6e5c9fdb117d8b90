// kml_abi.cpp -- C entry points of the host runner (declared in
// include/unikern_cuda.h): the KML contract queries and `solve` (no GPU
// needed), and the nvidia branch of the reference's `run`/`verify` flow.
#include <cstdio>
#include <cstring>
#include <sstream>
#include <string>

#include "kml.hpp"
#include "runner_cuda.hpp"
#include "unikern_cuda.h"

namespace {

// copy `s` into out[cap] (always NUL-terminated); UK_EINVAL when it does not fit
int put(const std::string& s, char* out, size_t cap) {
  if (out == nullptr || cap == 0) return UK_EINVAL;
  const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
  std::memcpy(out, s.data(), n);
  out[n] = '\0';
  return s.size() < cap ? UK_OK : UK_EINVAL;
}

}  // namespace

extern "C" {

int uk_kml_describe(const char* kml_json, const char* hcs_json, int sms, char* out, size_t out_cap) {
  if (kml_json == nullptr) {
    put("kml_json is NULL", out, out_cap);
    return UK_EINVAL;
  }
  std::string err;
  const auto tree = ukb::kml_import(kml_json, &err);
  if (!tree) {
    put(err, out, out_cap);
    return UK_EINVAL;
  }
  std::ostringstream os;
  const ukb::Workload w = ukb::workload_of(*tree);
  os << "canonical=" << ukb::canonical_form(*tree) << "\n"
     << "signature=" << ukb::op_signature(*tree) << "\n"
     << "ops=" << w.ops << "\n"
     << "bytes=" << w.bytes << "\n"
     << "tolerance=" << ukb::tolerance_for(tree->dtype) << "\n";
  ukb::BackendNvidia be;
  os << "gap=" << be.capability_gap(*tree) << "\n";
  if (hcs_json != nullptr) {
    const auto hcs = ukb::hcs_import(hcs_json, &err);
    if (!hcs) {
      put("HCS " + err, out, out_cap);
      return UK_EINVAL;
    }
    os << "hcs_fingerprint=" << ukb::hcs_fingerprint(*hcs) << "\n"
       << "ledger_key=" << ukb::ledger_key(*hcs, *tree) << "\n";
    if (be.capability_gap(*tree).empty()) {
      const ukb::Solution s = ukb::solve_b200(*hcs, *tree, sms > 0 ? sms : (hcs->compute_units > 0 ? hcs->compute_units : 148));
      os.precision(17);
      os << "tile=" << s.best.tile_m << "x" << s.best.tile_n << "\n"
         << "k_block=" << s.best.k_block << "\n"
         << "stages=" << s.best.stages << "\n"
         << "c_ms=" << s.c_ms << "\n"
         << "placement=" << s.placement_record << "\n";
    }
  }
  os << "export=" << ukb::kml_export(*tree);
  return put(os.str(), out, out_cap);
}

int uk_run_kml(const char* hcs_json, const char* kml_json, const char* ledger_path, int write_ledger, char* out,
               size_t out_cap) {
  if (hcs_json == nullptr || kml_json == nullptr) {
    put("hcs_json and kml_json are required", out, out_cap);
    return 2;
  }
  std::string transcript;
  const int rc = ukb::run_kml(hcs_json, kml_json, ledger_path ? ledger_path : "", write_ledger != 0, &transcript);
  if (out != nullptr && out_cap > 0) put(transcript, out, out_cap);
  return rc;
}

int uk_solve_kml(const char* hcs_json, const char* kml_json, const char* ledger_path, int write_ledger, int sms,
                 char* out, size_t out_cap) {
  if (hcs_json == nullptr || kml_json == nullptr) {
    put("hcs_json and kml_json are required", out, out_cap);
    return 2;
  }
  std::string transcript;
  const int rc =
      ukb::solve_kml(hcs_json, kml_json, ledger_path ? ledger_path : "", write_ledger != 0, sms, &transcript);
  if (out != nullptr && out_cap > 0) put(transcript, out, out_cap);
  return rc;
}

int uk_run_cuda(const char* hcs_json, const char* kml_json, int tile_m, int tile_n, uk_run_outcome* out, char* log,
                size_t log_cap) {
  if (hcs_json == nullptr || kml_json == nullptr || out == nullptr) {
    put("hcs_json, kml_json and out are required", log, log_cap);
    return UK_EINVAL;
  }
  std::string err;
  const auto hcs = ukb::hcs_import(hcs_json, &err);
  if (!hcs) {
    put("HCS " + err, log, log_cap);
    return UK_EINVAL;
  }
  const auto tree = ukb::kml_import(kml_json, &err);
  if (!tree) {
    put("KML " + err, log, log_cap);
    return UK_EINVAL;
  }
  ukb::Solution sol;
  sol.best.tile_m = tile_m;
  sol.best.tile_n = tile_n;
  sol.feasible_count = 1;
  const ukb::RunOutcome r = ukb::run_cuda(sol, *hcs, *tree, "");
  *out = uk_run_outcome{};
  out->built = r.built;
  out->ran = r.ran;
  out->verified = r.verified;
  out->max_rel = r.max_rel;
  out->measured_ms = r.measured_ms;
  out->kernel_ms = r.kernel_ms;
  out->migrations = r.migrations;
  out->checks = r.checks;
  out->vram_free = r.vram_free;
  out->vram_total = r.vram_total;
  out->exit_code = r.exit_code;
  std::snprintf(out->stream_path, sizeof out->stream_path, "%s", r.stream_path.c_str());
  if (log != nullptr && log_cap > 0) put(r.log, log, log_cap);
  return UK_OK;
}

int uk_calibrate(const char* hcs_json, const char* ledger_path, int allow_unified, char* hcs_out, size_t hcs_cap,
                 char* out, size_t out_cap) {
  if (hcs_json == nullptr || ledger_path == nullptr) {
    put("hcs_json and ledger_path are required", out, out_cap);
    return 2;
  }
  std::string cal, transcript;
  const int rc = ukb::calibrate(hcs_json, ledger_path, allow_unified != 0, &cal, &transcript);
  if (out != nullptr && out_cap > 0) put(transcript, out, out_cap);
  if (rc == 0 && hcs_out != nullptr && hcs_cap > 0 && put(cal, hcs_out, hcs_cap) != UK_OK) return 2;
  return rc;
}

}  // extern "C"
