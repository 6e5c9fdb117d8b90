"""Build recipe for the CPU oracle and for the reference-compiled checker.

TEST INFRASTRUCTURE ONLY.  Outputs:

* ``oracle/_build/liboracle.so``  -- the C restatement ``uk_oracle.c``
  (gcc, -O2 -ffp-contract=off, OpenMP over outer indices).  Built here and
  carried to the GPU box with the snapshot.
* ``oracle/_ref/libukref.so``  -- the UNIKERN reference's own C++ sources
  (``src/reference.cpp``, ``src/kml.cpp``, ``src/kml_front.cpp``,
  ``src/json_flat.cpp``, ``src/runtime.cpp``, ``src/hcs.cpp``,
  ``src/solver.cpp``, ``src/codegen_hip.cpp``, ``src/sqlite_ledger.cpp``,
  and the backend registry ``src/backends.cpp`` with the runners and
  emitters it links: ``src/runner.cpp``, ``src/runner_ocl.cpp``,
  ``src/runner_metal_stub.cpp``, ``src/codegen_other.cpp``) compiled unchanged with g++ straight from the reference tree (the SQLite
  ledger against the reference's vendored ``sqlite3.h``, linked to the
  system's ``libsqlite3.so.0``), plus ``ref_shim.cpp`` (extern "C"
  forwarding only).  Nothing is copied into the repository.
* ``oracle/_ref/libukemit.so``  -- the CPU reference functions that the
  reference embeds as text in its generated programs (gemm ``cpu_ref``,
  ``cpu_softmax``, ``cpu_rmsnorm``, ``cpu_channelscale``, ``cpu_conv_ref``,
  ``cpu_reduce_ref`` and the sawtooth initialisers), cut out of the program
  text that ``libukref.so`` emits and compiled on their own.

The ``_ref`` libraries need the reference tree, named by the environment
variable ``UK_REFERENCE_TREE`` (the UNIKERN project root), and are only built
where it is set and exists; they are git-ignored but travel with the
snapshot.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"


def reference_tree():
    """The UNIKERN source tree named by UK_REFERENCE_TREE (its project root,
    holding src/ and include/), or None: there is no default location."""
    t = os.environ.get("UK_REFERENCE_TREE")
    return Path(t) if t else None


CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-fopenmp"]
REF_SOURCES = ["reference", "kml", "kml_front", "json_flat", "runtime", "hcs",
               "solver", "codegen_hip", "sqlite_ledger",
               # the backend registry (make_backends) and what it links: the
               # runners (the OpenCL and Metal ones compile to their stubs
               # without those SDKs) and the other emitters
               "backends", "runner", "runner_ocl", "runner_metal_stub", "codegen_other"]
# the reference's SQLite ledger is compiled against its vendored sqlite3.h and
# linked to the system's SQLite library (the same engine the product loads)
SQLITE_LIB = "-l:libsqlite3.so.0"


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: %s\n%s%s" % (" ".join(map(str, cmd)), r.stdout, r.stderr))


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_oracle(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    out = BUILD / "liboracle.so"
    deps = [HERE / "uk_oracle.c", HERE / "uk_oracle.h"]
    if force or _stale(out, deps):
        _run(["gcc", "-std=c11", *CFLAGS, "-shared", str(HERE / "uk_oracle.c"),
              "-o", str(out), "-lm"])
    return out


# --- reference-compiled checker -------------------------------------------

# name -> (sample declaration, functions to cut out of the emitted program)
_EMIT = {
    "gemm": ('{"op":"gemm","dtype":"fp32","dims":[256,256,256],"layout":"NT"}',
             ["initA", "initB", "cpu_ref"]),
    "gemm_f16": ('{"op":"gemm","dtype":"fp16","dims":[256,256,256],"layout":"NT"}',
                 ["cpu_ref"]),
    "conv": ('{"op":"conv","dtype":"fp32","dims":[32,32,8,3,3,16],"layout":"NT"}',
             ["cpu_conv_ref"]),
    "reduce": ('{"op":"reduce","dtype":"fp32","dims":[1048576],"layout":"NT"}',
               ["cpu_reduce_ref"]),
    "softmax": ('{"op":"softmax","dtype":"fp32","dims":[64,256]}',
                ["initX", "cpu_softmax"]),
    "rmsnorm": ('{"op":"rmsnorm","dtype":"fp32","dims":[64,256]}',
                ["initW", "cpu_rmsnorm"]),
    "channelscale": ('{"op":"channelscale","dtype":"fp32","dims":[64,256]}',
                     ["initS", "cpu_channelscale"]),
}

# extern "C" forwarding written here (the cut-out functions take std::vector)
_WRAPPERS = r'''
static std::vector<float> g_B;
static int g_K = 0, g_N = 0;
extern "C" {
// timing form: B is held once so that each call computes `rows` full rows of C
void emit_gemm_set_B(const float* B, int K, int N) {
  g_B.assign(B, B + (size_t)K * N);
  g_K = K;
  g_N = N;
}
void emit_gemm_f16_rows(const float* A, float* C, int rows) {
  std::vector<float> a(A, A + (size_t)rows * g_K), c((size_t)rows * g_N);
  ns_gemm_f16::cpu_ref(a, g_B, c, rows, g_N, g_K);
  std::copy(c.begin(), c.end(), C);
}
void emit_gemm_rows(const float* A, float* C, int rows) {
  std::vector<float> a(A, A + (size_t)rows * g_K), c((size_t)rows * g_N);
  ns_gemm::cpu_ref(a, g_B, c, rows, g_N, g_K);
  std::copy(c.begin(), c.end(), C);
}
float emit_initA(int i) { return ns_gemm::initA(i); }
float emit_initB(int i) { return ns_gemm::initB(i); }
float emit_initX(int i) { return ns_softmax::initX(i); }
float emit_initW(int i) { return ns_rmsnorm::initW(i); }
float emit_initS(int i) { return ns_channelscale::initS(i); }
void emit_gemm_cpu_ref(const float* A, const float* B, float* C, int M, int N, int K) {
  std::vector<float> a(A, A + (size_t)M * K), b(B, B + (size_t)K * N), c((size_t)M * N);
  ns_gemm::cpu_ref(a, b, c, M, N, K);
  std::copy(c.begin(), c.end(), C);
}
void emit_gemm_f16_cpu_ref(const float* A, const float* B, float* C, int M, int N, int K) {
  std::vector<float> a(A, A + (size_t)M * K), b(B, B + (size_t)K * N), c((size_t)M * N);
  ns_gemm_f16::cpu_ref(a, b, c, M, N, K);
  std::copy(c.begin(), c.end(), C);
}
void emit_conv(const float* X, const float* Wt, float* Y, int H, int W, int C, int Kh, int Kw, int Oc) {
  std::vector<float> x(X, X + (size_t)H * W * C), w(Wt, Wt + (size_t)Oc * Kh * Kw * C);
  std::vector<float> y((size_t)Oc * (H - Kh + 1) * (W - Kw + 1));
  ns_conv::cpu_conv_ref(x, w, y, H, W, C, Kh, Kw, Oc);
  std::copy(y.begin(), y.end(), Y);
}
float emit_reduce(const float* X, long long n) {
  std::vector<float> x(X, X + n);
  float y = 0.f;
  ns_reduce::cpu_reduce_ref(x, &y);
  return y;
}
void emit_softmax(const float* X, float* Y, int L, int C) {
  std::vector<float> x(X, X + (size_t)L * C), y((size_t)L * C);
  ns_softmax::cpu_softmax(x, y, L, C);
  std::copy(y.begin(), y.end(), Y);
}
void emit_rmsnorm(const float* X, const float* W, float* Y, int L, int C) {
  std::vector<float> x(X, X + (size_t)L * C), w(W, W + C), y((size_t)L * C);
  ns_rmsnorm::cpu_rmsnorm(x, w, y, L, C);
  std::copy(y.begin(), y.end(), Y);
}
void emit_channelscale(const float* X, const float* S, float* Y, int L, int C) {
  std::vector<float> x(X, X + (size_t)L * C), s(S, S + C), y((size_t)L * C);
  ns_channelscale::cpu_channelscale(x, s, y, L, C);
  std::copy(y.begin(), y.end(), Y);
}
}
'''


def _cut_function(text: str, name: str) -> str:
    """Return the full definition of `static ... name(...) {...}` (brace matched),
    plus any `static const` constant it names that precedes it."""
    m = re.search(r"^static [^\n(]*\b%s\(" % re.escape(name), text, re.M)
    if not m:
        raise RuntimeError("emitted program has no function %s" % name)
    i = text.index("{", m.end())
    depth = 0
    for j in range(i, len(text)):
        if text[j] == "{":
            depth += 1
        elif text[j] == "}":
            depth -= 1
            if depth == 0:
                body = text[m.start():j + 1]
                break
    consts = []
    for cm in re.finditer(r"^static const int (UK_[A-Z_]+) = [^;]+;", text, re.M):
        if cm.group(1) in body:
            consts.append(cm.group(0))
    return "\n".join(consts + [body])


def build_ref(force: bool = False) -> bool:
    """Compile the reference's sources (only where the reference tree exists)."""
    REFERENCE = reference_tree()
    if REFERENCE is None or not (REFERENCE / "src" / "reference.cpp").exists():
        return False
    src = REFERENCE / "src"
    REF_OUT.mkdir(exist_ok=True)
    objdir = REF_OUT / "obj"
    objdir.mkdir(exist_ok=True)
    inc = ["-I", str(REFERENCE / "include"), "-I", str(src), "-I", str(REFERENCE / "third_party" / "sqlite")]
    objs = []
    for name in REF_SOURCES:
        s = src / (name + ".cpp")
        o = objdir / (name + ".o")
        if force or _stale(o, [s]):
            _run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fPIC", *inc, "-c", str(s), "-o", str(o)])
        objs.append(str(o))
    shim = HERE / "ref_shim.cpp"
    lib = REF_OUT / "libukref.so"
    if force or _stale(lib, objs + [str(shim)]):
        _run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fPIC", "-shared", *inc,
              str(shim), *objs, "-o", str(lib), SQLITE_LIB])

    emit_lib = REF_OUT / "libukemit.so"
    if not force and not _stale(emit_lib, [str(lib), __file__]):
        return True
    ref = ctypes.CDLL(str(lib))
    ref.ref_emit_program.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    hcs = (REFERENCE / "samples" / "hcs_amd.json").read_bytes()
    parts = ["// cut out of the programs emitted by the UNIKERN reference generator",
             "#include <algorithm>", "#include <cmath>", "#include <cstddef>",
             "#include <vector>", "using std::size_t;"]
    for op, (kml, funcs) in _EMIT.items():
        n = ref.ref_emit_program(kml.encode(), hcs, None, 0)
        if n < 0:
            raise RuntimeError("reference emitter refused %s" % op)
        buf = ctypes.create_string_buffer(n + 1)
        ref.ref_emit_program(kml.encode(), hcs, buf, n + 1)
        text = buf.value.decode()
        (REF_OUT / ("emitted_%s.hip" % op)).write_text(text)
        parts.append("namespace ns_%s {" % op)
        parts.extend(_cut_function(text, f) for f in funcs)
        parts.append("}  // namespace ns_%s" % op)
    parts.append(_WRAPPERS)
    cpp = REF_OUT / "emitted_refs.cpp"
    cpp.write_text("\n".join(parts) + "\n")
    _run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared", str(cpp), "-o", str(emit_lib)])
    return True


def main(argv=None):
    force = "--force" in (argv or sys.argv[1:])
    print("oracle:", build_oracle(force))
    print("reference checker:", "built" if build_ref(force) else "skipped (no reference tree)")


if __name__ == "__main__":
    main()
