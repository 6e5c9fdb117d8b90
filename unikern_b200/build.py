"""Build libunikern_cuda.so in-tree for sm_100a (nvcc; no PyTorch involved).

    python -m unikern_b200.build [--force] [-v]

Every ``csrc/*.cu`` and ``csrc/host/*.cpp`` file is compiled to an object under
``unikern_b200/_build`` (in parallel) and linked into
``unikern_b200/_lib/libunikern_cuda.so`` with a static CUDA runtime, so the
library does not depend on which libcudart a host process has loaded.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libunikern_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", "-I", str(ROOT / "include")]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted((CSRC / "host").glob("*.cpp"))
    return cu, cpp


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((CSRC / "host").glob("*.h*")) + \
        sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, verbose: bool):
    obj = OBJ / (src.stem + (".cu.o" if src.suffix == ".cu" else ".o"))
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, None
    if src.suffix == ".cu":
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXX_FLAGS, "-I", "/usr/local/cuda/include", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return obj, (r.stdout + r.stderr) if verbose else None


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    if force:
        for o in OBJ.glob("*.o"):
            o.unlink()
    cu, cpp = _sources()
    srcs = cu + cpp
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", *map(str, objs), "-o", str(LIB), "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return LIB


def ptxas_report(src: str) -> str:
    """Registers / spills / shared memory per kernel (-Xptxas -v) for one source."""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-c", str(CSRC / src), "-o", os.devnull]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.stdout + r.stderr


if __name__ == "__main__":
    args = sys.argv[1:]
    print(build(force="--force" in args, verbose="-v" in args))
