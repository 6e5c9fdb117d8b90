// ledger.hpp -- the kernel solution ledger of the runner, in both record
// formats of the UNIKERN reference:
//   * a path ending in ".jsonl": the TAB-separated file ledger
//     (src/runtime.cpp:20-170: rows `key c_ms measured_ms kernel_ms tm tn
//     placement`, `#VIOLATION` event rows);
//   * any other path (the reference's default is ledger.sqlite3): an SQLite
//     database with the reference's tables (src/sqlite_ledger.cpp:44-66)
//       solutions(key TEXT PRIMARY KEY, op_sig TEXT, hcs_fp TEXT,
//                 tree_hash TEXT, c_ms REAL, measured_ms REAL, tm INTEGER,
//                 tn INTEGER, placement TEXT, kernel_ms REAL NOT NULL DEFAULT 0)
//       violations(id INTEGER PRIMARY KEY AUTOINCREMENT, key TEXT, rate REAL,
//                  threshold REAL, migrations INTEGER, checks INTEGER,
//                  vram_free INTEGER, ts TEXT)
//     one row per key (INSERT OR REPLACE), each write in its own
//     BEGIN IMMEDIATE .. COMMIT (src/sqlite_ledger.cpp:99-133), so either tool
//     reads the other's rows.
// The choice by suffix is the reference's make_ledger (src/main.cpp:61-70).
// The interface follows ILedger (include/unikern/components.hpp:102-128).
// The SQLite engine is the system's libsqlite3.so.0, loaded at run time: the
// library needs no SQLite headers or link, and a process without it gets a
// clear error for non-.jsonl paths instead of rows in the wrong format.
#pragma once

#include <memory>
#include <optional>
#include <string>
#include <vector>

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

// one measured ledger row under an HCS fingerprint (calibration input)
struct MeasuredRow {
  std::string op_sig;      // carries the dims, e.g. "gemm:fp32:1024x1024x1024"
  double c_ms = 0;         // predicted at record time
  double measured_ms = 0;  // end to end per pass
  double kernel_ms = 0;    // kernel only; 0 in rows that predate it
};

class Ledger {
 public:
  virtual ~Ledger() = default;
  // a recorded solution for the key (from_ledger = true), or nullopt
  virtual std::optional<Solution> lookup(const LedgerKey& key) = 0;
  // rows with a measurement (> 0) recorded under hcs_fp, in record order
  virtual std::vector<MeasuredRow> measured_rows(const std::string& hcs_fp) = 0;
  // false + *err when the row could not be written (nothing half-written)
  virtual bool commit(const LedgerKey& key, const Solution& s, double measured_ms, double kernel_ms,
                      std::string* err) = 0;
  virtual bool record_violation(const LedgerKey& key, double rate, double threshold, int migrations, int checks,
                                unsigned long long vram_free, std::string* err) = 0;
  virtual int size() = 0;
  virtual int violation_count() = 0;
};

// true for paths that take the TAB file ledger (".jsonl" suffix)
bool is_file_ledger_path(const std::string& path);

// The ledger at `path` in the format its suffix selects; nullptr + *err when
// an SQLite ledger cannot be opened or created (or libsqlite3 is missing).
std::unique_ptr<Ledger> make_ledger(const std::string& path, std::string* err);

}  // namespace ukb
