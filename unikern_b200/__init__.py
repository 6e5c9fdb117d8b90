"""unikern_b200 -- the UNIKERN KML operator set on NVIDIA B200 (sm_100a).

The product is the C-ABI library ``_lib/libunikern_cuda.so`` (declared in
``include/unikern_cuda.h``).  This package only locates and binds it:
``abi`` holds the ctypes prototypes and thin wrappers that take torch CUDA
tensors (torch is used for device memory and streams, nothing else).

Importing fails loudly when the library has not been built; there is no CPU
fallback.
"""
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libunikern_cuda.so"

from .abi import lib, UkError  # noqa: E402,F401

__all__ = ["lib", "UkError", "LIB_PATH"]
