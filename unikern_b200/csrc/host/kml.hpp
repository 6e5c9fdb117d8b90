// kml.hpp -- the KML op contract on the host side: the op declaration, its
// canonical form and ledger key, the roofline workload, and the hardware
// capability spec (HCS) as far as the runner and the ledger key need it.
//
// The behaviour follows the UNIKERN reference so that a tree declared for the
// reference means the same work here and lands under the same ledger key:
//   OpKind / DType / KmlTree ...... include/unikern/core.hpp:11-31
//   kml_import / kml_export ....... src/kml_front.cpp:75-251 (strict flat
//                                   JSON, complete violation list, same texts)
//   canonical_form / op_signature / fnv1a_hex / kml_arity / workload_of
//                                   src/kml.cpp:60-177
//   hcs_import / hcs_fingerprint .. src/hcs.cpp:52-115
//   ledger key .................... src/main.cpp:217-219
// The string formats are interfaces and are kept identical; the code is this
// project's own.
#pragma once

#include <stdint.h>

#include <optional>
#include <string>
#include <vector>

namespace ukb {

enum class OpKind { Gemm, Conv, Reduction, Softmax, RmsNorm, ChannelScale };
enum class DType { F32, F16, I8 };

const char* op_name(OpKind k);
const char* dtype_name(DType d);
std::optional<OpKind> op_from_name(const std::string& s);
std::optional<DType> dtype_from_name(const std::string& s);
int dtype_bytes(DType d);
int kml_arity(OpKind op);
const char* kml_dim_spec(OpKind op);

struct KmlTree {
  OpKind op = OpKind::Gemm;
  DType dtype = DType::F32;
  int dims[6] = {4096, 4096, 4096, 0, 0, 0};
  int tile_m = 64;
  int tile_n = 128;
  std::string layout = "NT";
  std::vector<KmlTree> children;
};

// nullopt + *err = "rejected (N violations):\n  ..." on a bad declaration
std::optional<KmlTree> kml_import(const std::string& json, std::string* err);
std::string kml_export(const KmlTree& t);

std::string canonical_form(const KmlTree& t);
std::string fnv1a_hex(const std::string& data);
std::string op_signature(const KmlTree& t);

struct Workload {
  int64_t ops = 0;
  int64_t bytes = 0;
};
Workload workload_of(const KmlTree& t);

struct Tier {
  std::string name;
  int64_t bytes = 0;
  double bw_gbps = 0;
  std::string confidence = "official";  // provenance: official | measured | predicted
};

struct Hcs {
  std::string vendor, device, toolchain;
  bool unified_memory = false;
  double link_bw_gbps = 0, flops_gflops = 0;
  int compute_units = 0;
  int constants_version = 1;
  std::string confidence = "official";  // provenance, outside the fingerprint
  std::vector<Tier> tiers;
  int64_t tier_bytes(const std::string& name) const;
  double tier_bw(const std::string& name) const;
  int64_t device_capacity() const;
};

std::optional<Hcs> hcs_import(const std::string& json, std::string* err);
std::string hcs_fingerprint(const Hcs& h);
// flat JSON that round-trips through hcs_import, doubles to max_digits10
// (src/hcs.cpp:117-148 of UNIKERN); calibration writes its HCS with it
std::string hcs_export(const Hcs& h);

// the ledger key (src/main.cpp:217-219): its three parts, and the composite
// "op_sig|hcs_fp|tree_hash" both ledger formats file a row under
struct LedgerKey {
  std::string op_sig, hcs_fp, tree_hash;
  std::string str() const { return op_sig + "|" + hcs_fp + "|" + tree_hash; }
};
LedgerKey ledger_key_parts(const Hcs& h, const KmlTree& t);
std::string ledger_key(const Hcs& h, const KmlTree& t);

// tolerance gate of the verify instance, by declared dtype (2^-5, 2^-4, 0)
double tolerance_for(DType d);

}  // namespace ukb
