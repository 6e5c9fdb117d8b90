// kml.cpp -- host side of the KML op contract (see kml.hpp for the reference
// behaviour each function keeps).
#include "kml.hpp"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <sstream>

namespace ukb {

// ---- names -------------------------------------------------------------------

const char* op_name(OpKind k) {
  switch (k) {
    case OpKind::Gemm: return "gemm";
    case OpKind::Conv: return "conv";
    case OpKind::Reduction: return "reduce";
    case OpKind::Softmax: return "softmax";
    case OpKind::RmsNorm: return "rmsnorm";
    case OpKind::ChannelScale: return "channelscale";
  }
  return "?";
}

const char* dtype_name(DType d) {
  switch (d) {
    case DType::F32: return "fp32";
    case DType::F16: return "fp16";
    case DType::I8: return "int8";
  }
  return "?";
}

std::optional<OpKind> op_from_name(const std::string& s) {
  static const OpKind all[] = {OpKind::Gemm, OpKind::Conv, OpKind::Reduction,
                               OpKind::Softmax, OpKind::RmsNorm, OpKind::ChannelScale};
  for (OpKind k : all)
    if (s == op_name(k)) return k;
  return std::nullopt;
}

std::optional<DType> dtype_from_name(const std::string& s) {
  for (DType d : {DType::F32, DType::F16, DType::I8})
    if (s == dtype_name(d)) return d;
  return std::nullopt;
}

int dtype_bytes(DType d) { return d == DType::F16 ? 2 : d == DType::I8 ? 1 : 4; }

int kml_arity(OpKind op) {
  switch (op) {
    case OpKind::Gemm: return 3;
    case OpKind::Conv: return 6;
    case OpKind::Reduction: return 1;
    default: return 2;  // softmax / rmsnorm / channelscale: L, C
  }
}

const char* kml_dim_spec(OpKind op) {
  switch (op) {
    case OpKind::Gemm: return "3 dims (M,N,K)";
    case OpKind::Conv: return "6 dims (H,W,C,Kh,Kw,outC)";
    case OpKind::Reduction: return "1 dim (L)";
    default: return "2 dims (L,C)";
  }
}

// ---- a flat JSON scanner (scalars, strings, one level of arrays) -------------

namespace {

std::string trim(const std::string& s) {
  const size_t a = s.find_first_not_of(" \t\r\n");
  if (a == std::string::npos) return "";
  const size_t b = s.find_last_not_of(" \t\r\n");
  return s.substr(a, b - a + 1);
}

bool has_key(const std::string& j, const std::string& key) { return j.find("\"" + key + "\"") != std::string::npos; }

// value of the first "key": as raw text (strings without their quotes)
std::optional<std::string> field(const std::string& j, const std::string& key) {
  const std::string q = "\"" + key + "\"";
  const size_t k = j.find(q);
  if (k == std::string::npos) return std::nullopt;
  size_t p = j.find(':', k + q.size());
  if (p == std::string::npos) return std::nullopt;
  for (++p; p < j.size() && (j[p] == ' ' || j[p] == '\t'); ++p) {
  }
  if (p >= j.size()) return std::nullopt;
  if (j[p] == '"') {
    const size_t e = j.find('"', p + 1);
    if (e == std::string::npos) return std::nullopt;
    return j.substr(p + 1, e - p - 1);
  }
  size_t e = j.find_first_of(",}\n", p);
  if (e == std::string::npos) e = j.size();
  return trim(j.substr(p, e - p));
}

// the {...} bodies inside "key": [ ... ]
std::vector<std::string> objects(const std::string& j, const std::string& key) {
  std::vector<std::string> out;
  const std::string q = "\"" + key + "\"";
  const size_t k = j.find(q);
  if (k == std::string::npos) return out;
  const size_t open = j.find('[', k + q.size());
  if (open == std::string::npos) return out;
  int depth = 0;
  size_t start = 0;
  for (size_t p = open + 1; p < j.size(); ++p) {
    if (j[p] == '{') {
      if (depth++ == 0) start = p;
    } else if (j[p] == '}') {
      if (--depth == 0) out.push_back(j.substr(start, p - start + 1));
    } else if (j[p] == ']' && depth == 0) {
      break;
    }
  }
  return out;
}

// the comma-separated tokens of "key": [ a, b, c ]
std::vector<std::string> number_tokens(const std::string& j, const std::string& key) {
  std::vector<std::string> out;
  const std::string q = "\"" + key + "\"";
  const size_t k = j.find(q);
  if (k == std::string::npos) return out;
  const size_t open = j.find('[', k + q.size());
  const size_t close = open == std::string::npos ? open : j.find(']', open);
  if (close == std::string::npos) return out;
  std::stringstream ss(j.substr(open + 1, close - open - 1));
  std::string tok;
  while (std::getline(ss, tok, ',')) {
    tok = trim(tok);
    if (!tok.empty()) out.push_back(tok);
  }
  return out;
}

// keys of the outermost object, in text order
std::vector<std::string> top_keys(const std::string& j) {
  std::vector<std::string> keys;
  int depth = 0;
  for (size_t p = 0; p < j.size(); ++p) {
    const char c = j[p];
    if (c == '"') {
      size_t e = p + 1;
      std::string s;
      for (; e < j.size() && j[e] != '"'; ++e) {
        if (j[e] == '\\' && e + 1 < j.size()) s.push_back(j[e++]);
        s.push_back(j[e]);
      }
      size_t n = e + 1;
      while (n < j.size() && std::isspace((unsigned char)j[n])) ++n;
      if (depth == 1 && n < j.size() && j[n] == ':') keys.push_back(s);
      p = e;
    } else if (c == '{' || c == '[') {
      ++depth;
    } else if (c == '}' || c == ']') {
      --depth;
    }
  }
  return keys;
}

// wide integer parse: optional '-', digits only, no overflow
bool parse_wide(const std::string& tok, long long* out) {
  size_t i = (!tok.empty() && tok[0] == '-') ? 1 : 0;
  if (i >= tok.size()) return false;
  for (; i < tok.size(); ++i)
    if (!std::isdigit((unsigned char)tok[i])) return false;
  errno = 0;
  char* end = nullptr;
  const long long v = std::strtoll(tok.c_str(), &end, 10);
  if (errno == ERANGE || end == tok.c_str()) return false;
  *out = v;
  return true;
}

// remove the "children": [ ... ] span (its keys must not answer for the parent)
void take_children(std::string* body, std::vector<std::string>* kids) {
  const size_t k = body->find("\"children\"");
  if (k == std::string::npos) return;
  const size_t open = body->find('[', k);
  if (open == std::string::npos) return;
  int depth = 0;
  size_t close = body->size();
  for (size_t p = open; p < body->size(); ++p) {
    if ((*body)[p] == '[') ++depth;
    if ((*body)[p] == ']' && --depth == 0) {
      close = p;
      break;
    }
  }
  *kids = objects(*body, "children");
  body->erase(k, close - k + 1);
}

void parse_node(const std::string& text, const std::string& path, KmlTree* t, std::vector<std::string>* errs) {
  auto bad = [&](const std::string& m) { errs->push_back(path + m); };
  std::string own = text;
  std::vector<std::string> kids;
  take_children(&own, &kids);

  static const char* allowed[] = {"op", "dtype", "dims", "tile_m", "tile_n", "layout"};
  for (const std::string& k : top_keys(own)) {
    bool ok = false;
    for (const char* a : allowed) ok = ok || k == a;
    if (!ok) bad("unknown field '" + k + "' (typo would otherwise be ignored)");
  }

  bool op_ok = false;
  if (auto v = field(own, "op")) {
    if (auto k = op_from_name(*v)) {
      t->op = *k;
      op_ok = true;
    } else {
      bad("op='" + *v + "' not one of gemm|conv|reduce");
    }
  } else {
    bad("missing op (one of gemm|conv|reduce)");
  }

  if (auto v = field(own, "dtype")) {
    if (auto d = dtype_from_name(*v)) t->dtype = *d;
    else bad("dtype='" + *v + "' not one of fp32|fp16|int8");
  } else {
    bad("missing dtype (one of fp32|fp16|int8)");
  }

  if (!has_key(own, "dims")) {
    bad("missing dims");
  } else {
    const std::vector<std::string> toks = number_tokens(own, "dims");
    bool vals_ok = true;
    int vals[6] = {0, 0, 0, 0, 0, 0};
    if (toks.size() > 6) {
      bad("dims has " + std::to_string(toks.size()) + " entries, max 6");
      vals_ok = false;
    }
    for (size_t i = 0; i < toks.size() && i < 6; ++i) {
      const std::string idx = "dims[" + std::to_string(i) + "]";
      long long w = 0;
      if (!parse_wide(toks[i], &w)) {
        bad(idx + "='" + toks[i] + "' is not an integer");
        vals_ok = false;
      } else if (w > INT_MAX) {
        bad(idx + "=" + toks[i] + " exceeds " + std::to_string(INT_MAX) +
            ", the largest element index the generated kernels can address");
        vals_ok = false;
      } else if (w <= 0) {
        bad(idx + "=" + std::to_string((int)w) + " must be positive");
        vals_ok = false;
      } else {
        vals[i] = (int)w;
      }
    }
    if (op_ok && vals_ok) {
      if ((int)toks.size() != kml_arity(t->op)) {
        bad(std::string("dims: ") + op_name(t->op) + " needs " + kml_dim_spec(t->op) + ", got " +
            std::to_string(toks.size()));
      } else {
        for (int i = 0; i < 6; ++i) t->dims[i] = vals[i];
      }
    }
  }

  for (const char* key : {"tile_m", "tile_n"}) {
    auto v = field(own, key);
    if (!v) continue;
    long long w = 0;
    if (!parse_wide(*v, &w) || w <= 0 || w > INT_MAX) {
      bad(std::string(key) + "='" + *v + "' must be a positive integer");
    } else if (std::string(key) == "tile_m") {
      t->tile_m = (int)w;
    } else {
      t->tile_n = (int)w;
    }
  }

  if (auto v = field(own, "layout")) {
    t->layout = *v;
    if (*v != "NT")
      bad("layout='" + *v + "' is not implemented by kernel generation (only NT: A/B/C row-major indexing)");
  }

  for (size_t i = 0; i < kids.size(); ++i) {
    KmlTree child;
    const size_t before = errs->size();
    parse_node(kids[i], path + "children[" + std::to_string(i) + "].", &child, errs);
    if (errs->size() == before) t->children.push_back(child);
  }
}

void export_node(std::ostringstream& os, const KmlTree& t, bool nested) {
  const char* ind = nested ? "    " : "  ";
  os << (nested ? "    {" : "{") << "\n";
  os << ind << "\"op\": \"" << op_name(t.op) << "\",\n";
  os << ind << "\"dtype\": \"" << dtype_name(t.dtype) << "\",\n";
  os << ind << "\"dims\": [";
  for (int i = 0; i < kml_arity(t.op); ++i) os << (i ? "," : "") << t.dims[i];
  os << "],\n";
  os << ind << "\"tile_m\": " << t.tile_m << ",\n";
  os << ind << "\"tile_n\": " << t.tile_n << ",\n";
  os << ind << "\"layout\": \"" << t.layout << "\"";
  if (!t.children.empty()) {
    os << ",\n" << ind << "\"children\": [";
    for (size_t i = 0; i < t.children.size(); ++i) {
      os << (i ? "," : "") << "\n";
      export_node(os, t.children[i], true);
    }
    os << "]\n";
  } else {
    os << "\n";
  }
  os << (nested ? "    " : "") << "}";
}

}  // namespace

std::optional<KmlTree> kml_import(const std::string& json, std::string* err) {
  KmlTree t;
  std::vector<std::string> errs;
  parse_node(json, "", &t, &errs);
  if (errs.empty()) return t;
  if (err) {
    std::ostringstream os;
    os << "rejected (" << errs.size() << " violations):";
    for (const auto& e : errs) os << "\n  " << e;
    *err = os.str();
  }
  return std::nullopt;
}

std::string kml_export(const KmlTree& t) {
  std::ostringstream os;
  export_node(os, t, false);
  os << "\n";
  return os.str();
}

// ---- canonical form, signature, workload --------------------------------------

std::string canonical_form(const KmlTree& t) {
  std::string s = std::string("(") + op_name(t.op) + ":" + dtype_name(t.dtype) + " dims=";
  for (int i = 0; i < kml_arity(t.op); ++i) s += (i ? "," : "") + std::to_string(t.dims[i]);
  s += " tile=" + std::to_string(t.tile_m) + "x" + std::to_string(t.tile_n) + " layout=" + t.layout;
  std::vector<std::string> kids;
  for (const auto& c : t.children) kids.push_back(canonical_form(c));
  std::sort(kids.begin(), kids.end());
  for (const auto& k : kids) s += " " + k;
  return s + ")";
}

std::string fnv1a_hex(const std::string& data) {
  // The reference's ledger keys start from 1469598103934665603, which is the
  // published FNV-1a 64-bit offset basis (14695981039346656037) with its last
  // digit dropped.  Kept as is: any other basis files the same tree under a
  // different key and a shared ledger would never hit.
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : data) {
    h ^= c;
    h *= 1099511628211ull;  // FNV prime
  }
  char buf[17];
  std::snprintf(buf, sizeof buf, "%016llx", (unsigned long long)h);
  return buf;
}

std::string op_signature(const KmlTree& t) {
  std::string s = std::string(op_name(t.op)) + ":" + dtype_name(t.dtype) + ":";
  for (int i = 0; i < kml_arity(t.op); ++i) s += (i ? "x" : "") + std::to_string(t.dims[i]);
  return s;
}

Workload workload_of(const KmlTree& t) {
  const int64_t es = dtype_bytes(t.dtype);
  const int64_t* d = nullptr;
  int64_t v[6];
  for (int i = 0; i < 6; ++i) v[i] = t.dims[i];
  d = v;
  Workload w;
  switch (t.op) {
    case OpKind::Gemm:
      w.ops = 2 * d[0] * d[1] * d[2];
      w.bytes = (d[0] * d[2] + d[2] * d[1] + d[0] * d[1]) * es;
      break;
    case OpKind::Conv: {
      const int64_t kh = d[3] ? d[3] : 3, kw = d[4] ? d[4] : 3, oc = d[5] ? d[5] : 64;
      w.ops = 2 * d[0] * d[1] * d[2] * kh * kw * oc;  // the reference counts H*W outputs
      w.bytes = (d[0] * d[1] * d[2] + kh * kw * d[2] * oc + d[0] * d[1] * oc) * es;
      break;
    }
    case OpKind::Reduction:
      w.ops = d[0];
      w.bytes = 2 * d[0] * es;
      break;
    case OpKind::Softmax:
      w.ops = 5 * d[0] * d[1];
      w.bytes = 3 * d[0] * d[1] * es;
      break;
    case OpKind::RmsNorm:
      w.ops = 7 * d[0] * d[1];
      w.bytes = 3 * d[0] * d[1] * es;
      break;
    case OpKind::ChannelScale:
      w.ops = d[0] * d[1];
      w.bytes = 3 * d[0] * d[1] * es;
      break;
  }
  return w;
}

// ---- HCS ---------------------------------------------------------------------

int64_t Hcs::tier_bytes(const std::string& name) const {
  for (const auto& t : tiers)
    if (t.name == name) return t.bytes;
  return 0;
}

double Hcs::tier_bw(const std::string& name) const {
  for (const auto& t : tiers)
    if (t.name == name) return t.bw_gbps;
  return 0;
}

int64_t Hcs::device_capacity() const { return tier_bytes(unified_memory ? "unified" : "vram"); }

std::optional<Hcs> hcs_import(const std::string& json, std::string* err) {
  auto num = [&](const std::string& key, const char* dflt) {
    return field(json, key).value_or(dflt);
  };
  Hcs h;
  try {
    h.vendor = field(json, "vendor").value_or("");
    h.device = field(json, "device").value_or("");
    h.unified_memory = field(json, "unified_memory").value_or("false") == "true";
    h.link_bw_gbps = std::stod(num("link_bw_gbps", "0"));
    h.flops_gflops = std::stod(num("flops_gflops", "0"));
    h.compute_units = std::stoi(num("compute_units", "0"));
    h.toolchain = field(json, "toolchain").value_or("");
    for (const std::string& body : objects(json, "tiers")) {
      Tier t;
      t.name = field(body, "name").value_or("");
      if (t.name.empty()) continue;
      t.bytes = std::stoll(field(body, "bytes").value_or("0"));
      t.bw_gbps = std::stod(field(body, "bw_gbps").value_or("0"));
      t.confidence = field(body, "confidence").value_or("official");
      h.tiers.push_back(t);
    }
    if (h.tiers.empty()) {  // legacy flat form
      const char* nm = h.unified_memory ? "unified" : "vram";
      h.tiers.push_back({nm, std::stoll(num(h.unified_memory ? "unified_bytes" : "vram_bytes", "0")),
                         std::stod(num("mem_bw_gbps", "0"))});
    }
    h.constants_version = std::stoi(num("constants_version", "1"));
    if (h.constants_version < 1) h.constants_version = 1;
    // the top-level confidence: looked up outside the tiers array, whose
    // entries carry their own
    std::string top = json;
    const size_t tk = top.find("\"tiers\"");
    if (tk != std::string::npos) {
      const size_t close = top.find(']', tk);
      top.erase(tk, close == std::string::npos ? std::string::npos : close - tk + 1);
    }
    h.confidence = field(top, "confidence").value_or("official");
  } catch (const std::exception&) {
    if (err) *err = "malformed numeric field";
    return std::nullopt;
  }
  std::vector<std::string> missing;
  if (h.vendor.empty()) missing.push_back("vendor");
  if (h.device.empty()) missing.push_back("device");
  if (h.device_capacity() <= 0) missing.push_back(h.unified_memory ? "tiers[unified].bytes" : "tiers[vram].bytes");
  if (h.tier_bw(h.unified_memory ? "unified" : "vram") <= 0) missing.push_back("tiers[device].bw_gbps");
  if (h.link_bw_gbps <= 0) missing.push_back("link_bw_gbps");
  if (h.flops_gflops <= 0) missing.push_back("flops_gflops");
  if (h.compute_units <= 0) missing.push_back("compute_units");
  if (!missing.empty()) {
    if (err) {
      std::string m = "missing required fields:";
      for (const auto& s : missing) m += " " + s;
      *err = m;
    }
    return std::nullopt;
  }
  return h;
}

std::string hcs_fingerprint(const Hcs& h) {
  // the modelled capability fields in a fixed order (ostream default number
  // formatting, as the key format requires); provenance fields are excluded
  std::ostringstream os;
  os << "vendor=" << h.vendor << ";device=" << h.device << ";unified=" << (h.unified_memory ? 1 : 0)
     << ";linkbw=" << h.link_bw_gbps << ";flops=" << h.flops_gflops << ";cu=" << h.compute_units;
  for (const auto& t : h.tiers) os << ";tier=" << t.name << ":" << t.bytes << ":" << t.bw_gbps;
  os << ";schema=2";
  return fnv1a_hex(os.str());
}

std::string hcs_export(const Hcs& h) {
  std::ostringstream os;
  os.precision(std::numeric_limits<double>::max_digits10);
  os << "{\n  \"vendor\": \"" << h.vendor << "\",\n  \"device\": \"" << h.device << "\",\n  \"unified_memory\": "
     << (h.unified_memory ? "true" : "false") << ",\n  \"link_bw_gbps\": " << h.link_bw_gbps
     << ",\n  \"flops_gflops\": " << h.flops_gflops << ",\n  \"compute_units\": " << h.compute_units
     << ",\n  \"toolchain\": \"" << h.toolchain << "\",\n  \"constants_version\": " << h.constants_version
     << ",\n  \"confidence\": \"" << h.confidence << "\",\n  \"tiers\": [\n";
  for (size_t i = 0; i < h.tiers.size(); ++i) {
    const Tier& t = h.tiers[i];
    os << "    { \"name\": \"" << t.name << "\", \"bytes\": " << t.bytes << ", \"bw_gbps\": " << t.bw_gbps
       << ", \"confidence\": \"" << t.confidence << "\" }" << (i + 1 < h.tiers.size() ? "," : "") << "\n";
  }
  os << "  ]\n}\n";
  return os.str();
}

LedgerKey ledger_key_parts(const Hcs& h, const KmlTree& t) {
  return LedgerKey{op_signature(t), hcs_fingerprint(h), fnv1a_hex(canonical_form(t))};
}

std::string ledger_key(const Hcs& h, const KmlTree& t) { return ledger_key_parts(h, t).str(); }

double tolerance_for(DType d) { return d == DType::F16 ? 0.0625 : d == DType::I8 ? 0.0 : 0.03125; }

}  // namespace ukb
