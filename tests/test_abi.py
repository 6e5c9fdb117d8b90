"""The C-ABI library loads and exports what include/*.h declares (CPU only).

No test here launches a kernel: argument validation runs before any CUDA
call, so invalid-argument paths are checked without a GPU.
"""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(uk_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    import unikern_b200.abi as abi
    return abi.lib()


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 12
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_prototypes_cover_the_header():
    import unikern_b200.abi as abi
    assert set(declared_symbols()) <= set(abi.PROTOTYPES), set(declared_symbols()) - set(abi.PROTOTYPES)


def test_abi_version(lib):
    assert lib.uk_cuda_abi_version() >= 10000


@pytest.mark.parametrize("call", [
    lambda l: l.uk_cuda_gemm_f32(None, None, None, -1, 4, 4, None),
    lambda l: l.uk_cuda_gemm_f16(None, None, None, 4, -4, 4, None),
    lambda l: l.uk_cuda_gemm_f16_ld(None, 2, None, 4, None, 4, 4, 4, 4, None),  # lda < K
    lambda l: l.uk_cuda_channelscale_f32(None, None, None, -5, 3, None),
    lambda l: l.uk_cuda_softmax_f32(None, None, 4, -1, None),
    lambda l: l.uk_cuda_rmsnorm_f32(None, None, None, 1 << 40, 4, 1e-6, None),
    lambda l: l.uk_cuda_reduce_f32(None, None, -1, 5, None, 0, None),
    lambda l: l.uk_cuda_conv2d_f32(None, None, None, 1, 8, 8, 3, 3, 3, 4, 0, None, 7, None),  # layout
    lambda l: l.uk_cuda_conv2d_f32(None, None, None, 2, 8, 8, 3, 3, 3, 4, 0, None, 0, None),  # KML N=2
    lambda l: l.uk_cuda_conv2d_f32(None, None, None, 1, 2, 2, 3, 3, 3, 4, 0, None, 1, None),  # filter > input
])
def test_invalid_arguments_return_2_with_text(lib, call):
    assert call(lib) == 2
    assert lib.uk_cuda_last_error().decode()


def test_empty_shapes_are_no_ops(lib):
    # zero-sized work returns before touching any pointer or device
    assert lib.uk_cuda_gemm_f32(None, None, None, 0, 4, 4, None) == 0
    assert lib.uk_cuda_softmax_f32(None, None, 0, 7, None) == 0
    assert lib.uk_cuda_channelscale_f32(None, None, None, 3, 0, None) == 0
    assert lib.uk_cuda_reduce_workspace_size(0, 100) == 0


def test_product_does_not_link_the_oracle():
    import subprocess
    out = subprocess.run(["nm", "-D", str(ROOT / "unikern_b200" / "_lib" / "libunikern_cuda.so")],
                         capture_output=True, text=True).stdout
    assert "or_" not in " ".join(l.split()[-1] for l in out.splitlines() if " U " in l)
    assert "oracle" not in (ROOT / "unikern_b200" / "abi.py").read_text().split('"""')[-1]
