// ledger.cpp -- the TAB file ledger and the SQLite ledger (see ledger.hpp for
// the record formats each keeps and the reference lines they follow).
#include "ledger.hpp"

#include <dlfcn.h>

#include <fstream>
#include <limits>
#include <mutex>
#include <sstream>
#include <type_traits>

namespace ukb {

bool is_file_ledger_path(const std::string& path) {
  static const std::string suffix = ".jsonl";
  return path.size() >= suffix.size() && path.compare(path.size() - suffix.size(), suffix.size(), suffix) == 0;
}

// ---- TAB file ledger (src/runtime.cpp:20-170) ----------------------------------

namespace {

const char kSep = '\t';
const char* kViolation = "#VIOLATION";

std::vector<std::string> split_tabs(const std::string& line) {
  std::vector<std::string> f;
  size_t pos = 0;
  while (true) {
    const size_t tab = line.find(kSep, pos);
    f.push_back(line.substr(pos, tab == std::string::npos ? std::string::npos : tab - pos));
    if (tab == std::string::npos) break;
    pos = tab + 1;
  }
  return f;
}

class FileLedger final : public Ledger {
 public:
  explicit FileLedger(std::string path) : path_(std::move(path)) {}

  std::optional<Solution> lookup(const LedgerKey& k) override {
    const std::string key = k.str();
    std::ifstream in(path_);
    std::string line;
    while (std::getline(in, line)) {
      const std::vector<std::string> f = split_tabs(line);
      if (f.size() < 4 || f[0] != key) continue;
      Solution s;
      try {
        s.c_ms = std::stod(f[1]);
        if (f.size() >= 7) {  // key c_ms measured kernel tm tn placement
          s.best.tile_m = std::stoi(f[4]);
          s.best.tile_n = std::stoi(f[5]);
          s.placement_record = f[6];
        } else if (f.size() >= 6) {  // key c_ms measured tm tn placement
          s.best.tile_m = std::stoi(f[3]);
          s.best.tile_n = std::stoi(f[4]);
          s.placement_record = f[5];
        } else {
          s.placement_record = f[3];
        }
      } catch (...) {
        continue;  // a corrupt row is skipped, never surfaced as a solution
      }
      s.from_ledger = true;
      s.feasible_count = 1;
      return s;
    }
    return std::nullopt;
  }

  std::vector<MeasuredRow> measured_rows(const std::string& hcs_fp) override {
    std::vector<MeasuredRow> out;
    std::ifstream in(path_);
    std::string line;
    while (std::getline(in, line)) {
      const std::vector<std::string> f = split_tabs(line);
      if (f.size() < 4) continue;
      // key = op_sig|hcs_fp|tree_hash (violation rows start with their marker)
      const size_t b1 = f[0].find('|'), b2 = b1 == std::string::npos ? b1 : f[0].find('|', b1 + 1);
      if (b2 == std::string::npos || f[0].compare(b1 + 1, b2 - b1 - 1, hcs_fp) != 0) continue;
      MeasuredRow r;
      r.op_sig = f[0].substr(0, b1);
      try {
        r.c_ms = std::stod(f[1]);
        r.measured_ms = std::stod(f[2]);
        if (f.size() >= 7) r.kernel_ms = std::stod(f[3]);  // only the 7-field row carries it
      } catch (...) {
        continue;  // a corrupt row is no calibration material
      }
      if (r.measured_ms > 0) out.push_back(r);
    }
    return out;
  }

  bool commit(const LedgerKey& k, const Solution& s, double measured_ms, double kernel_ms,
              std::string* err) override {
    std::ofstream out(path_, std::ios::app);
    out.precision(std::numeric_limits<double>::max_digits10);
    out << k.str() << kSep << s.c_ms << kSep << measured_ms << kSep << kernel_ms << kSep << s.best.tile_m << kSep
        << s.best.tile_n << kSep << s.placement_record << "\n";
    out.flush();
    if (!out) {
      if (err) *err = "cannot append to " + path_;
      return false;
    }
    return true;
  }

  bool record_violation(const LedgerKey& k, double rate, double threshold, int migrations, int checks,
                        unsigned long long vram_free, std::string* err) override {
    std::ofstream out(path_, std::ios::app);
    out.precision(std::numeric_limits<double>::max_digits10);
    out << kViolation << kSep << k.str() << kSep << rate << kSep << threshold << kSep << migrations << kSep
        << checks << kSep << vram_free << "\n";
    out.flush();
    if (!out) {
      if (err) *err = "cannot append to " + path_;
      return false;
    }
    return true;
  }

  int size() override { return count(false); }
  int violation_count() override { return count(true); }

 private:
  int count(bool violations) {
    std::ifstream in(path_);
    std::string line;
    int n = 0;
    while (std::getline(in, line))
      if (!line.empty() && (line.rfind(kViolation, 0) == 0) == violations) ++n;
    return n;
  }
  std::string path_;
};

// ---- SQLite ledger (src/sqlite_ledger.cpp:44-236) -------------------------------
//
// The few entry points of the SQLite C API this writer uses, resolved from the
// system's libsqlite3.so.0 when the first SQLite ledger opens.  Handles are
// opaque; the constants are the API's published values.

struct sqlite3;
struct sqlite3_stmt;
constexpr int kSqliteOk = 0, kSqliteRow = 100, kSqliteDone = 101;
constexpr int kOpenReadWrite = 0x2, kOpenCreate = 0x4;
using Destructor = void (*)(void*);
const Destructor kTransient = reinterpret_cast<Destructor>(-1);

struct SqliteApi {
  int (*open_v2)(const char*, sqlite3**, int, const char*) = nullptr;
  int (*close)(sqlite3*) = nullptr;
  int (*exec)(sqlite3*, const char*, int (*)(void*, int, char**, char**), void*, char**) = nullptr;
  void (*free)(void*) = nullptr;
  const char* (*errmsg)(sqlite3*) = nullptr;
  int (*busy_timeout)(sqlite3*, int) = nullptr;
  int (*prepare_v2)(sqlite3*, const char*, int, sqlite3_stmt**, const char**) = nullptr;
  int (*step)(sqlite3_stmt*) = nullptr;
  int (*finalize)(sqlite3_stmt*) = nullptr;
  int (*bind_text)(sqlite3_stmt*, int, const char*, int, Destructor) = nullptr;
  int (*bind_double)(sqlite3_stmt*, int, double) = nullptr;
  int (*bind_int)(sqlite3_stmt*, int, int) = nullptr;
  int (*bind_int64)(sqlite3_stmt*, int, long long) = nullptr;
  const unsigned char* (*column_text)(sqlite3_stmt*, int) = nullptr;
  double (*column_double)(sqlite3_stmt*, int) = nullptr;
  int (*column_int)(sqlite3_stmt*, int) = nullptr;
  bool ok = false;
  std::string why;
};

const SqliteApi& sqlite_api() {
  static SqliteApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libsqlite3.so.0", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) h = dlopen("libsqlite3.so", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) {
      api.why = "libsqlite3.so.0 not found";
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    get(api.open_v2, "sqlite3_open_v2");
    get(api.close, "sqlite3_close");
    get(api.exec, "sqlite3_exec");
    get(api.free, "sqlite3_free");
    get(api.errmsg, "sqlite3_errmsg");
    get(api.busy_timeout, "sqlite3_busy_timeout");
    get(api.prepare_v2, "sqlite3_prepare_v2");
    get(api.step, "sqlite3_step");
    get(api.finalize, "sqlite3_finalize");
    get(api.bind_text, "sqlite3_bind_text");
    get(api.bind_double, "sqlite3_bind_double");
    get(api.bind_int, "sqlite3_bind_int");
    get(api.bind_int64, "sqlite3_bind_int64");
    get(api.column_text, "sqlite3_column_text");
    get(api.column_double, "sqlite3_column_double");
    get(api.column_int, "sqlite3_column_int");
    api.ok = all;
    if (!all) api.why = "libsqlite3.so.0 lacks an entry point this ledger uses";
  });
  return api;
}

// A prepared statement, finalized on every path out.
class Stmt {
 public:
  Stmt(const SqliteApi& a, sqlite3* db, const char* sql) : a_(a) {
    if (a_.prepare_v2(db, sql, -1, &st_, nullptr) != kSqliteOk) st_ = nullptr;
  }
  ~Stmt() {
    if (st_) a_.finalize(st_);
  }
  Stmt(const Stmt&) = delete;
  Stmt& operator=(const Stmt&) = delete;
  explicit operator bool() const { return st_ != nullptr; }
  sqlite3_stmt* get() const { return st_; }
  void text(int i, const std::string& s) { a_.bind_text(st_, i, s.c_str(), -1, kTransient); }

 private:
  const SqliteApi& a_;
  sqlite3_stmt* st_ = nullptr;
};

class SqliteLedger final : public Ledger {
 public:
  // nullptr-equivalent state (db_ == nullptr) + *err when it cannot open
  SqliteLedger(const std::string& path, std::string* err) : a_(sqlite_api()), path_(path) {
    if (!a_.ok) {
      if (err) *err = "SQLite ledger " + path + " unavailable: " + a_.why + " (a .jsonl path takes the file ledger)";
      return;
    }
    if (a_.open_v2(path.c_str(), &db_, kOpenReadWrite | kOpenCreate, nullptr) != kSqliteOk) {
      if (err) *err = "sqlite ledger open failed (" + path + "): " + (db_ ? a_.errmsg(db_) : "no handle");
      if (db_) a_.close(db_);
      db_ = nullptr;
      return;
    }
    a_.busy_timeout(db_, 5000);
    // the reference's schema; a database it created without kernel_ms gains
    // the column the same way it migrates one
    std::string e;
    if (!exec("CREATE TABLE IF NOT EXISTS solutions(key TEXT PRIMARY KEY, op_sig TEXT, hcs_fp TEXT, "
              "tree_hash TEXT, c_ms REAL, measured_ms REAL, tm INTEGER, tn INTEGER, placement TEXT, "
              "kernel_ms REAL NOT NULL DEFAULT 0)",
              &e) ||
        !ensure_kernel_column(&e) ||
        !exec("CREATE TABLE IF NOT EXISTS violations(id INTEGER PRIMARY KEY AUTOINCREMENT, key TEXT, rate REAL, "
              "threshold REAL, migrations INTEGER, checks INTEGER, vram_free INTEGER, ts TEXT)",
              &e)) {
      if (err) *err = "sqlite ledger schema (" + path + "): " + e;
      a_.close(db_);
      db_ = nullptr;
    }
  }
  ~SqliteLedger() override {
    if (db_) a_.close(db_);
  }
  bool is_open() const { return db_ != nullptr; }

  std::optional<Solution> lookup(const LedgerKey& k) override {
    Stmt st(a_, db_, "SELECT c_ms, tm, tn, placement FROM solutions WHERE key = ?1");
    if (!st) return std::nullopt;  // an unreadable database reads as a miss: re-solve
    st.text(1, k.str());
    if (a_.step(st.get()) != kSqliteRow) return std::nullopt;
    Solution s;
    s.c_ms = a_.column_double(st.get(), 0);
    s.best.tile_m = a_.column_int(st.get(), 1);
    s.best.tile_n = a_.column_int(st.get(), 2);
    const unsigned char* place = a_.column_text(st.get(), 3);
    s.placement_record = place ? reinterpret_cast<const char*>(place) : "";
    s.from_ledger = true;
    s.feasible_count = 1;
    return s;
  }

  std::vector<MeasuredRow> measured_rows(const std::string& hcs_fp) override {
    std::vector<MeasuredRow> out;
    Stmt st(a_, db_,
            "SELECT op_sig, c_ms, measured_ms, kernel_ms FROM solutions WHERE hcs_fp = ?1 AND measured_ms > 0 "
            "ORDER BY rowid");
    if (!st) return out;
    st.text(1, hcs_fp);
    while (a_.step(st.get()) == kSqliteRow) {
      MeasuredRow r;
      const unsigned char* sig = a_.column_text(st.get(), 0);
      r.op_sig = sig ? reinterpret_cast<const char*>(sig) : "";
      r.c_ms = a_.column_double(st.get(), 1);
      r.measured_ms = a_.column_double(st.get(), 2);
      r.kernel_ms = a_.column_double(st.get(), 3);
      out.push_back(r);
    }
    return out;
  }

  bool commit(const LedgerKey& k, const Solution& s, double measured_ms, double kernel_ms,
              std::string* err) override {
    return in_transaction(
        "INSERT OR REPLACE INTO solutions(key, op_sig, hcs_fp, tree_hash, c_ms, measured_ms, tm, tn, placement, "
        "kernel_ms) VALUES(?1,?2,?3,?4,?5,?6,?7,?8,?9,?10)",
        [&](Stmt& st) {
          st.text(1, k.str());
          st.text(2, k.op_sig);
          st.text(3, k.hcs_fp);
          st.text(4, k.tree_hash);
          a_.bind_double(st.get(), 5, s.c_ms);
          a_.bind_double(st.get(), 6, measured_ms);
          a_.bind_int(st.get(), 7, s.best.tile_m);
          a_.bind_int(st.get(), 8, s.best.tile_n);
          st.text(9, s.placement_record);
          a_.bind_double(st.get(), 10, kernel_ms);
        },
        err);
  }

  bool record_violation(const LedgerKey& k, double rate, double threshold, int migrations, int checks,
                        unsigned long long vram_free, std::string* err) override {
    return in_transaction(
        "INSERT INTO violations(key, rate, threshold, migrations, checks, vram_free, ts) "
        "VALUES(?1,?2,?3,?4,?5,?6,datetime('now'))",
        [&](Stmt& st) {
          st.text(1, k.str());
          a_.bind_double(st.get(), 2, rate);
          a_.bind_double(st.get(), 3, threshold);
          a_.bind_int(st.get(), 4, migrations);
          a_.bind_int(st.get(), 5, checks);
          a_.bind_int64(st.get(), 6, (long long)vram_free);
        },
        err);
  }

  int size() override { return count("SELECT count(*) FROM solutions"); }
  int violation_count() override { return count("SELECT count(*) FROM violations"); }

 private:
  bool exec(const char* sql, std::string* err) {
    char* msg = nullptr;
    if (a_.exec(db_, sql, nullptr, nullptr, &msg) == kSqliteOk) return true;
    if (err) *err = msg ? msg : "sqlite3_exec failed";
    if (msg) a_.free(msg);
    return false;
  }

  bool ensure_kernel_column(std::string* err) {
    bool has = false;
    {
      Stmt st(a_, db_, "PRAGMA table_info(solutions)");
      if (!st) return false;
      while (a_.step(st.get()) == kSqliteRow) {
        const unsigned char* name = a_.column_text(st.get(), 1);
        has = has || (name && std::string(reinterpret_cast<const char*>(name)) == "kernel_ms");
      }
    }
    return has || exec("ALTER TABLE solutions ADD COLUMN kernel_ms REAL NOT NULL DEFAULT 0", err);
  }

  // one statement inside BEGIN IMMEDIATE .. COMMIT: all or nothing
  template <class Bind>
  bool in_transaction(const char* sql, Bind bind, std::string* err) {
    if (!exec("BEGIN IMMEDIATE", err)) return false;
    bool ok = false;
    {
      Stmt st(a_, db_, sql);
      if (st) {
        bind(st);
        ok = a_.step(st.get()) == kSqliteDone;
      }
      if (!ok && err) *err = std::string("sqlite ledger write (") + path_ + "): " + a_.errmsg(db_);
    }
    if (!ok) {
      exec("ROLLBACK", nullptr);
      return false;
    }
    return exec("COMMIT", err);
  }

  int count(const char* sql) {
    Stmt st(a_, db_, sql);
    if (!st || a_.step(st.get()) != kSqliteRow) return 0;
    return a_.column_int(st.get(), 0);
  }

  const SqliteApi& a_;
  std::string path_;
  sqlite3* db_ = nullptr;
};

}  // namespace

std::unique_ptr<Ledger> make_ledger(const std::string& path, std::string* err) {
  if (is_file_ledger_path(path)) return std::make_unique<FileLedger>(path);
  auto db = std::make_unique<SqliteLedger>(path, err);
  if (!db->is_open()) return nullptr;
  return db;
}

}  // namespace ukb
