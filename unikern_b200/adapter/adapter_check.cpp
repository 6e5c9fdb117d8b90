// adapter_check.cpp -- TEST INFRASTRUCTURE: drives the reference-side nvidia
// backend (runner_nvidia.cpp) with the reference's own front end and solver,
// as cmd_run would (src/main.cpp:348-436): kml_import / hcs_import, solve,
// then run_cuda; prints one JSON object per line for tests/test_adapter.py.
//
//   adapter_check backends <kml-json>...     the four backends' answers
//   adapter_check run <hcs-json> <kml-json>... RunOutcome of each tree
#include <cstdio>
#include <string>

#include "runner_nvidia.hpp"

using namespace unikern;

namespace {

std::string esc(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\', o += c;
    else if (c == '\n') o += "\\n";
    else if ((unsigned char)c < 0x20) o += ' ';
    else o += c;
  }
  return o;
}

int backends(int argc, char** argv) {
  const auto all = make_backends_with_nvidia();
  for (const auto& b : all)
    std::printf("{\"backend\":\"%s\",\"vendor\":%d,\"available\":%s,\"streaming\":%s}\n", b->name().c_str(),
                (int)b->vendor(), b->available() ? "true" : "false", b->supports_streaming() ? "true" : "false");
  for (int i = 0; i < argc; ++i) {
    std::string err;
    const auto t = kml_import(argv[i], &err);
    if (!t) {
      std::printf("{\"kml\":\"%s\",\"rejected\":\"%s\"}\n", esc(argv[i]).c_str(), esc(err).c_str());
      continue;
    }
    std::printf("{\"kml\":\"%s\",\"gaps\":{", esc(argv[i]).c_str());
    for (size_t k = 0; k < all.size(); ++k)
      std::printf("%s\"%s\":\"%s\"", k ? "," : "", all[k]->name().c_str(), esc(all[k]->capability_gap(*t)).c_str());
    std::printf("}}\n");
  }
  return 0;
}

int run(const char* hcs_json, int argc, char** argv) {
  std::string err;
  const auto hcs = hcs_import(hcs_json, &err);
  if (!hcs) {
    std::printf("{\"hcs_rejected\":\"%s\"}\n", esc(err).c_str());
    return 2;
  }
  BackendNvidia be;
  for (int i = 0; i < argc; ++i) {
    const auto tree = kml_import(argv[i], &err);
    if (!tree) {
      std::printf("{\"kml\":\"%s\",\"rejected\":\"%s\"}\n", esc(argv[i]).c_str(), esc(err).c_str());
      continue;
    }
    const Solution sol = solve(*hcs, *tree);
    const RunOutcome r = run_cuda(sol, *hcs, *tree, "");
    std::printf(
        "{\"kml\":\"%s\",\"gap\":\"%s\",\"tile\":\"%dx%d\",\"built\":%d,\"ran\":%d,\"verified\":%d,"
        "\"max_rel\":%.9g,\"measured_ms\":%.9g,\"kernel_ms\":%.9g,\"migrations\":%d,\"checks\":%d,"
        "\"vram_free\":%llu,\"vram_total\":%llu,\"exit_code\":%d,\"stream_path\":\"%s\",\"log\":\"%s\"}\n",
        esc(argv[i]).c_str(), esc(be.capability_gap(*tree)).c_str(), sol.best.tile_m, sol.best.tile_n, r.built,
        r.ran, r.verified, r.max_rel, r.measured_ms, r.kernel_ms, r.migrations, r.checks, r.vram_free, r.vram_total,
        r.exit_code, esc(r.stream_path).c_str(), esc(r.log).c_str());
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 2 && std::string(argv[1]) == "backends") return backends(argc - 2, argv + 2);
  if (argc >= 3 && std::string(argv[1]) == "run") return run(argv[2], argc - 3, argv + 3);
  std::fprintf(stderr, "usage: adapter_check backends <kml>... | run <hcs-json> <kml>...\n");
  return 2;
}
