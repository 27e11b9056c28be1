"""Product launchers over torch device tensors, named after the reference's
kernels/wmma_products.hpp and kernels/skinny_gemm.hpp. Each call goes through
the C ABI of libvoxcpm_b200.so; torch only supplies device memory and streams.

Launchers return False where the reference's return false (the shape does
not suit the kernels, nothing launched) and raise VxError on other failures.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import WmmaPlan, SplitScratch, check, load

kTileRows = 16
kTileColumns = 32
kQ8TileBytes = 16 * 32 + 16 * 2
kBf16TileBytes = 16 * 32 * 2


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("device tensor expected")
    if not t.is_contiguous():
        raise ValueError("contiguous tensor expected")
    return t.data_ptr()


def _stream(stream=None) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def Q8TilesBytes(rows: int, columns: int) -> int:
    """kernels/wmma_products.hpp:29-33"""
    return load().vx_q8_tiles_bytes(rows, columns)


def Bf16TilesBytes(rows: int, columns: int) -> int:
    """kernels/wmma_products.hpp:34-38"""
    return load().vx_bf16_tiles_bytes(rows, columns)


def Q8_0ToTiles(blocks: torch.Tensor, rows: int, columns: int, output: torch.Tensor, stream=None) -> None:
    """GGML Q8_0 blocks -> Q8 tiles (kernels/wmma_products.hpp:55-59)."""
    check(load().vx_q8_0_to_tiles(_ptr(blocks), rows, columns, _ptr(output), _stream(stream)))


def Bf16ToTiles(weights: torch.Tensor, rows: int, columns: int, output: torch.Tensor, stream=None) -> None:
    """kernels/wmma_products.hpp:61-63"""
    check(load().vx_bf16_to_tiles(_ptr(weights), rows, columns, _ptr(output), _stream(stream)))


def Q8TilesToBf16(tiles: torch.Tensor, rows: int, columns: int, output: torch.Tensor, stream=None) -> None:
    """kernels/wmma_products.hpp:65-68"""
    check(load().vx_q8_tiles_to_bf16(_ptr(tiles), rows, columns, _ptr(output), _stream(stream)))


def Bf16TilesToRows(tiles: torch.Tensor, rows: int, columns: int, output: torch.Tensor, stream=None) -> None:
    """kernels/wmma_products.hpp:70-72"""
    check(load().vx_bf16_tiles_to_rows(_ptr(tiles), rows, columns, _ptr(output), _stream(stream)))


def PlanWmma(rows: int, columns: int, out: int, target_waves: int = 0) -> WmmaPlan:
    """kernels/wmma_products.hpp:83-85 (target_waves: about that many CTAs)."""
    return load().vx_plan_wmma(rows, columns, out, target_waves)


def _plan_arg(plan: WmmaPlan | None):
    return ctypes.byref(plan) if plan is not None else None


def _scratch_arg(scratch: SplitScratch | None):
    return ctypes.byref(scratch) if scratch is not None else None


def WmmaQ8(x, w, y, rows, columns, out, accumulate, plan=None, scratch=None, stream=None) -> bool:
    """kernels/wmma_products.hpp:87-93"""
    return check(
        load().vx_wmma_q8(_ptr(x), _ptr(w), _ptr(y), rows, columns, out, int(accumulate),
                          _plan_arg(plan), _scratch_arg(scratch), _stream(stream)),
        unsupported_ok=True,
    )


def WmmaBf16(x, w, y, rows, columns, out, accumulate, plan=None, scratch=None, stream=None) -> bool:
    """kernels/wmma_products.hpp:95-99"""
    return check(
        load().vx_wmma_bf16(_ptr(x), _ptr(w), _ptr(y), rows, columns, out, int(accumulate),
                            _plan_arg(plan), _scratch_arg(scratch), _stream(stream)),
        unsupported_ok=True,
    )


def SkinnyGemm(x, w, y, rows, columns, out, accumulate, stream=None) -> bool:
    """kernels/skinny_gemm.hpp:18-24"""
    return check(
        load().vx_skinny_gemm(_ptr(x), _ptr(w), _ptr(y), rows, columns, out, int(accumulate),
                              _stream(stream)),
        unsupported_ok=True,
    )


def SkinnyGemmWith(vec, x, w, y, rows, columns, out, accumulate, stream=None) -> bool:
    """kernels/skinny_gemm.hpp:26-30 (vec selects the kernel variant)."""
    return check(
        load().vx_skinny_gemm_with(vec, _ptr(x), _ptr(w), _ptr(y), rows, columns, out,
                                   int(accumulate), _stream(stream)),
        unsupported_ok=True,
    )


def Product(fmt: int, x, w, y, rows, columns, out, accumulate=False, plan=None, stream=None) -> bool:
    """Any weight format; y float32 or bfloat16 (the bf16-output epilogue)."""
    if y.dtype == torch.float32:
        out_dtype = _lib.OUT_F32
    elif y.dtype == torch.bfloat16:
        out_dtype = _lib.OUT_BF16
    else:
        raise ValueError("y must be float32 or bfloat16")
    return check(
        load().vx_product(fmt, _ptr(x), _ptr(w), _ptr(y), out_dtype, rows, columns, out,
                          int(accumulate), _plan_arg(plan), _stream(stream)),
        unsupported_ok=True,
    )


def ReadProbe(data: torch.Tensor, pieces: int, blocks: int, sink: torch.Tensor, stream=None) -> None:
    """kernels/skinny_gemm.hpp:32-34"""
    check(load().vx_read_probe(_ptr(data), pieces, blocks, _ptr(sink), _stream(stream)))


def DeviceError() -> int:
    """Reads and clears the kernels' timeout bits (synchronizes)."""
    bits = ctypes.c_uint(0)
    check(load().vx_device_error(ctypes.byref(bits)))
    return bits.value


def SetProgrammaticLaunch(enabled: bool) -> None:
    load().vx_set_programmatic_launch(int(enabled))


def ProductVariants() -> list[tuple[int, int, int, int]]:
    lib = load()
    shapes = []
    for v in range(lib.vx_product_variants()):
        a, b, c, d = (ctypes.c_int() for _ in range(4))
        lib.vx_product_variant_shape(v, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), ctypes.byref(d))
        shapes.append((a.value, b.value, c.value, d.value))
    return shapes


def RandomQ8_0(seed: int, tensor: int, rows: int, columns: int, scale_std: float = 0.02 / 127):
    """Host GGML Q8_0 blocks (numpy uint8 [rows * columns / 32 * 34])."""
    import numpy as np

    out = np.empty(rows * (columns // 32) * 34, dtype=np.uint8)
    check(load().vx_random_q8_0(seed, tensor, rows, columns, scale_std, out.ctypes.data))
    return out


def RandomBf16(seed: int, tensor: int, count: int, mean: float = 0.0, std: float = 0.02):
    """Host bf16 bit patterns (numpy uint16 [count])."""
    import numpy as np

    out = np.empty(count, dtype=np.uint16)
    check(load().vx_random_bf16(seed, tensor, count, mean, std, out.ctypes.data))
    return out
