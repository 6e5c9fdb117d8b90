// ref_shim.cpp -- extern "C" entry points over the UNIKERN reference's own
// C++ sources, compiled unchanged from the reference tree into
// oracle/_ref/libukref.so by oracle/build.py.
//
// TEST INFRASTRUCTURE ONLY.  The shim adds no arithmetic: every call forwards
// to a reference function so tests can compare the restated oracle and the
// product's host logic against the reference itself:
//   cpu_conv / cpu_reduce / cpu_reduce_blocked ... src/reference.cpp:6-48
//   tolerance_for .................................. src/runtime.cpp:182-190
//   kml_import / canonical_form / op_signature ..... src/kml_front.cpp:203,
//     src/kml.cpp:60-121, ledger key src/main.cpp:217-219
//   hcs_import / hcs_fingerprint ................... src/hcs.cpp:52-115
//   workload_of .................................... src/kml.cpp:125-177
//   hip_runnable_program (emitted CPU references) .. src/codegen_hip.cpp:132
//   make_file_ledger / make_sqlite_ledger .......... src/runtime.cpp,
//     src/sqlite_ledger.cpp, chosen by suffix as src/main.cpp:61-70 does
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "unikern/codegen.hpp"
#include "unikern/components.hpp"
#include "unikern/core.hpp"

using namespace unikern;

namespace {
int put(const std::string& s, char* out, int cap) {
  if (!out || cap <= 0) return (int)s.size();
  const size_t n = s.size() < (size_t)(cap - 1) ? s.size() : (size_t)(cap - 1);
  std::memcpy(out, s.data(), n);
  out[n] = 0;
  return (int)s.size();
}
}  // namespace

extern "C" {

void ref_cpu_conv(const float* x, const float* wt, float* y, int H, int W, int C,
                  int Kh, int Kw, int Oc) {
  cpu_conv(x, wt, y, H, W, C, Kh, Kw, Oc);
}

float ref_cpu_reduce(const float* x, long long n) {
  float y = 0.f;
  cpu_reduce(x, &y, n);
  return y;
}

float ref_cpu_reduce_blocked(const float* x, long long n, int width) {
  float y = 0.f;
  cpu_reduce_blocked(x, &y, n, width);
  return y;
}

int ref_basis_width(void) { return kRefReduceWidth; }

double ref_tolerance_for(int dtype) {
  return tolerance_for(dtype == 1 ? DType::F16 : dtype == 2 ? DType::I8 : DType::F32);
}

// 0 = accepted (out gets canonical_form), 2 = rejected (out gets the message)
int ref_kml_check(const char* json, char* out, int cap) {
  std::string err;
  auto t = kml_import(json, &err);
  if (!t) {
    put(err, out, cap);
    return 2;
  }
  put(canonical_form(*t), out, cap);
  return 0;
}

int ref_kml_export(const char* json, char* out, int cap) {
  auto t = kml_import(json, nullptr);
  if (!t) return -1;
  return put(kml_export(*t), out, cap);
}

// ledger key "op_sig|hcs_fp|tree_hash" (src/main.cpp:217-219 joined as in
// src/runtime.cpp key_str)
int ref_ledger_key(const char* kml_json, const char* hcs_json, char* out, int cap) {
  auto t = kml_import(kml_json, nullptr);
  auto h = hcs_import(hcs_json, nullptr);
  if (!t || !h) return -1;
  const std::string k = op_signature(*t) + "|" + hcs_fingerprint(*h) + "|" +
                        fnv1a_hex(canonical_form(*t));
  return put(k, out, cap);
}

int ref_hcs_check(const char* json, char* out, int cap) {
  std::string err;
  auto h = hcs_import(json, &err);
  if (!h) {
    put(err, out, cap);
    return 2;
  }
  put(hcs_fingerprint(*h), out, cap);
  return 0;
}

int ref_workload(const char* kml_json, long long* ops, long long* bytes) {
  auto t = kml_import(kml_json, nullptr);
  if (!t) return -1;
  const Workload w = workload_of(*t);
  *ops = w.ops;
  *bytes = w.bytes;
  return 0;
}

int ref_solve_tile(const char* kml_json, const char* hcs_json, int* tm, int* tn) {
  auto t = kml_import(kml_json, nullptr);
  auto h = hcs_import(hcs_json, nullptr);
  if (!t || !h) return -1;
  const Solution s = solve(*h, *t);
  *tm = s.best.tile_m;
  *tn = s.best.tile_n;
  return s.feasible_count;
}

namespace {
std::unique_ptr<ILedger> open_ledger(const std::string& path) {
  const std::string sfx = ".jsonl";
  if (path.size() >= sfx.size() && path.compare(path.size() - sfx.size(), sfx.size(), sfx) == 0)
    return make_file_ledger(path);
  return make_sqlite_ledger(path);
}
Key key_of(const KmlTree& t, const Hcs& h) {
  return Key{op_signature(t), hcs_fingerprint(h), fnv1a_hex(canonical_form(t))};
}
}  // namespace

// The reference ledger's lookup of a tree's key: 1 hit (out gets
// "c_ms tm tn placement"), 0 miss, -1 bad input or an unopenable ledger.
int ref_ledger_lookup(const char* path, const char* kml_json, const char* hcs_json, char* out, int cap) {
  auto t = kml_import(kml_json, nullptr);
  auto h = hcs_import(hcs_json, nullptr);
  if (!t || !h) return -1;
  try {
    auto l = open_ledger(path);
    auto hit = l->lookup(key_of(*t, *h));
    if (!hit) return 0;
    char num[64];
    std::snprintf(num, sizeof num, "%.17g", hit->c_ms);
    put(std::string(num) + " " + std::to_string(hit->best.tile_m) + " " + std::to_string(hit->best.tile_n) + " " +
            hit->placement_record,
        out, cap);
    return 1;
  } catch (...) {
    return -1;
  }
}

// The reference's solve of the tree committed to its ledger: measured_ms < 0
// commits a solve-time row (measured = c_ms, as cmd_solve does), otherwise a
// run's row with the given measured / kernel times.  0 ok, -1 error.
int ref_ledger_commit(const char* path, const char* kml_json, const char* hcs_json, double measured_ms,
                      double kernel_ms) {
  auto t = kml_import(kml_json, nullptr);
  auto h = hcs_import(hcs_json, nullptr);
  if (!t || !h) return -1;
  try {
    auto l = open_ledger(path);
    const Solution s = solve(*h, *t);
    l->commit(key_of(*t, *h), s, measured_ms < 0 ? s.c_ms : measured_ms, kernel_ms);
    return 0;
  } catch (...) {
    return -1;
  }
}

// rows (solutions) and violation events in the reference ledger's view; -1 error
int ref_ledger_counts(const char* path, int* violations) {
  try {
    auto l = open_ledger(path);
    *violations = l->violation_count();
    return l->size();
  } catch (...) {
    return -1;
  }
}

// The emitted AMD program text; its embedded CPU references are extracted by
// oracle/build.py and compiled on their own.
int ref_emit_program(const char* kml_json, const char* hcs_json, char* out, int cap) {
  auto t = kml_import(kml_json, nullptr);
  auto h = hcs_import(hcs_json, nullptr);
  if (!t || !h) return -1;
  const Solution s = solve(*h, *t);
  return put(hip_runnable_program(s, *h, *t), out, cap);
}

}  // extern "C"
