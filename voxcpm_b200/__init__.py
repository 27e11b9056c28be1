"""voxcpm_b200: a B200-native (sm_100a) VoxCPM2 per-patch generation path.

The implementation is the CUDA shared library libvoxcpm_b200.so behind the C
ABI in include/voxcpm_b200.h. This package binds it with ctypes and mirrors
the reference's C++ interfaces (gemm.hpp, kernels/*.hpp, transformer.hpp,
generator.hpp) for Python callers and tests. The library is loaded on first
use; every entry point raises if it is missing (there is no fallback).
"""

from ._lib import LIBRARY, VxError, load

__all__ = ["LIBRARY", "VxError", "load"]
