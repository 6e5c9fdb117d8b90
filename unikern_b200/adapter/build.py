"""Build recipe for the reference-side nvidia backend (runner_nvidia.cpp)
and its check driver, against the UNIKERN reference's own headers.

    UK_REFERENCE_TREE=<UNIKERN project root> python -m unikern_b200.adapter.build

The adapter is the translation unit a maintainer adds to the reference tree;
here it is compiled against the reference's unmodified include/ and linked
with the reference compiled from its sources (oracle/_ref/libukref.so, built
by oracle/build.py) and with libunikern_cuda.so.  Outputs go to
unikern_b200/adapter/_build/ (git-ignored; they travel with the snapshot and
find both libraries through relative rpaths).  Where the reference tree or
oracle/_ref is absent the build is skipped.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build"
REF_LIB = ROOT / "oracle" / "_ref" / "libukref.so"
UK_LIB = ROOT / "unikern_b200" / "_lib" / "libunikern_cuda.so"


def _stale(out: Path, deps) -> bool:
    return not out.exists() or any(Path(d).stat().st_mtime > out.stat().st_mtime for d in deps)


def build(force: bool = False):
    """The check driver's path, or None when the reference is not here."""
    sys.path.insert(0, str(ROOT))
    from oracle import build as ob
    tree = ob.reference_tree()
    if tree is None or not (tree / "include" / "unikern" / "components.hpp").exists() or not REF_LIB.exists() \
            or not UK_LIB.exists():
        return None
    OUT.mkdir(exist_ok=True)
    exe = OUT / "adapter_check"
    srcs = [HERE / "runner_nvidia.cpp", HERE / "adapter_check.cpp"]
    deps = srcs + [HERE / "runner_nvidia.hpp", ROOT / "include" / "unikern_cuda.h", REF_LIB, UK_LIB]
    if force or _stale(exe, deps):
        cmd = ["g++", "-std=c++20", "-O2", "-Wall", "-I", str(tree / "include"), "-I", str(ROOT / "include"),
               *map(str, srcs), "-o", str(exe),
               "-L", str(REF_LIB.parent), "-l:libukref.so", "-L", str(UK_LIB.parent), "-l:libunikern_cuda.so",
               "-Wl,-rpath,$ORIGIN/../../../oracle/_ref", "-Wl,-rpath,$ORIGIN/../../_lib"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("adapter build failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return exe


if __name__ == "__main__":
    print(build(force="--force" in sys.argv[1:]))
