"""Bf16Gemm: product dispatch by weight format and row count (gemm.hpp:49-72),
over the C ABI (vx_gemm_*)."""

from __future__ import annotations

import ctypes

import torch

from ._lib import MatmulShape, TuningBucket, check, load  # noqa: F401 (re-exported)
from .kernels import _ptr, _stream


class Matrix:
    """A weight matrix on the device (matrix.hpp:15-19): format + data."""

    def __init__(self, fmt: int, data: torch.Tensor):
        self.format = fmt
        self.data = data


class Bf16Gemm:
    """One instance per stream (gemm.hpp:49-72)."""

    def __init__(self, stream=None):
        self._lib = load()
        self._handle = self._lib.vx_gemm_create(_stream(stream))
        if not self._handle:
            raise RuntimeError("vx_gemm_create failed")

    def Linear(self, x: torch.Tensor, w: Matrix, y: torch.Tensor, rows: int, columns: int, out: int,
               accumulate: bool) -> None:
        """y[rows][out] (+)= x[rows][columns] * w^T (gemm.hpp:51-58)."""
        check(self._lib.vx_gemm_linear(self._handle, _ptr(x), w.format, _ptr(w.data), _ptr(y),
                                       rows, columns, out, int(accumulate)))

    def LinearEx(self, x: torch.Tensor, w: Matrix, y: torch.Tensor, rows: int, columns: int, out: int,
                 flags: int = 0) -> None:
        """Linear with the output type of `y` (float32 or bfloat16) and
        flags (PRODUCT_ACCUMULATE): vx_gemm_linear_ex."""
        from ._lib import OUT_BF16, OUT_F32

        dtype = OUT_BF16 if y.dtype == torch.bfloat16 else OUT_F32
        check(self._lib.vx_gemm_linear_ex(self._handle, _ptr(x), w.format, _ptr(w.data), _ptr(y), dtype,
                                          rows, columns, out, flags))

    def Matmul(self, shape, representative, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> None:
        """Column-major C (+)= op(A) op(B) of bf16 a and b into float32 c
        (gemm.hpp:60-63). `shape` and `representative` are MatmulShape; the
        representative may be None (one kernel serves every shape)."""
        rep = ctypes.byref(representative) if representative is not None else None
        check(self._lib.vx_gemm_matmul(self._handle, ctypes.byref(shape), rep, _ptr(a), _ptr(b),
                                       _ptr(c)))

    def close(self) -> None:
        if self._handle:
            self._lib.vx_gemm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
