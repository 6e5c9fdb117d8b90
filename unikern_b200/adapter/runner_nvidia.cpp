// runner_nvidia.cpp -- the reference-side nvidia backend over the C ABI of
// libunikern_cuda.so (include/unikern_cuda.h).  Trees and HCS values cross
// the boundary as the reference's own flat JSON (kml_export / hcs_export,
// src/kml_front.cpp:246, src/hcs.cpp:121), which the library imports with
// the same rules; results come back as the RunOutcome fields.
#include "runner_nvidia.hpp"

#include <sstream>

#include "unikern_cuda.h"

namespace unikern {

namespace {

// the "gap=" line of uk_kml_describe ("" when the library runs the tree)
std::string library_gap(const KmlTree& tree) {
  std::string out(1 << 14, '\0');
  const int rc = uk_kml_describe(kml_export(tree).c_str(), nullptr, 0, out.data(), out.size());
  out.resize(out.find('\0'));
  if (rc != UK_OK) return "declaration refused by nvidia:cuda: " + out;
  const size_t g = out.find("\ngap=");
  if (g == std::string::npos) return "nvidia:cuda gave no capability answer";
  const size_t e = out.find('\n', g + 5);
  return out.substr(g + 5, e == std::string::npos ? std::string::npos : e - g - 5);
}

}  // namespace

RunOutcome run_cuda(const Solution& sol, const Hcs& hcs, const KmlTree& tree, const std::string& workdir) {
  (void)workdir;  // nothing is generated or compiled
  RunOutcome r;
  uk_run_outcome o{};
  std::string log(1 << 16, '\0');
  const int rc = uk_run_cuda(hcs_export(hcs).c_str(), kml_export(tree).c_str(), sol.best.tile_m, sol.best.tile_n, &o,
                             log.data(), log.size());
  log.resize(log.find('\0'));
  r.log = log;
  if (rc != UK_OK) {
    r.exit_code = 2;
    return r;
  }
  r.built = o.built != 0;
  r.ran = o.ran != 0;
  r.verified = o.verified != 0;
  r.max_rel = o.max_rel;
  r.measured_ms = o.measured_ms;
  r.kernel_ms = o.kernel_ms;
  r.migrations = o.migrations;
  r.checks = o.checks;
  r.vram_free = o.vram_free;
  r.vram_total = o.vram_total;
  r.exit_code = o.exit_code;
  r.stream_path = o.stream_path;
  return r;
}

bool BackendNvidia::available() const { return uk_cuda_device_supported() != 0; }

std::string BackendNvidia::generate(const Solution& sol, const Hcs& hcs, const KmlTree& tree) const {
  const int v = uk_cuda_abi_version();
  std::ostringstream os;
  os << "// nvidia:cuda: precompiled sm_100a kernels of libunikern_cuda.so (ABI " << v / 10000 << "."
     << v / 100 % 100 << "." << v % 100 << "); no source is generated\n"
     << "// tree " << canonical_form(tree) << "\n// device " << hcs.device << "\n// tile " << sol.best.tile_m << "x"
     << sol.best.tile_n << "\n";
  return os.str();
}

std::string BackendNvidia::capability_gap(const KmlTree& tree) const {
  // the library's own answer (it refuses other layouts as the shared
  // predicate does), so that this backend, the runner and the ledger gate
  // cannot disagree about what nvidia:cuda runs
  return library_gap(tree);
}

std::vector<std::unique_ptr<IBackend>> make_backends_with_nvidia() {
  std::vector<std::unique_ptr<IBackend>> v = make_backends();
  v.push_back(std::make_unique<BackendNvidia>());
  return v;
}

}  // namespace unikern
