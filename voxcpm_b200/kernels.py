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


def _any_ptr(t: torch.Tensor) -> int:
    """A device tensor, or a page-locked host tensor (reachable from the
    device at the same address)."""
    if not t.is_contiguous():
        raise ValueError("contiguous tensor expected")
    if not t.is_cuda and not t.is_pinned():
        raise ValueError("device or page-locked host tensor expected")
    return t.data_ptr()


def _host_ptr(t: torch.Tensor) -> int:
    if t.is_cuda or not t.is_pinned():
        raise ValueError("page-locked host tensor expected")
    return _any_ptr(t)


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


def PlanSpread(fmt: int, rows: int, columns: int, out: int) -> WmmaPlan:
    """The spread plan (vx_plan_spread): CTA count, longest run and the split
    scratch it needs (kernels/wmma_products.hpp:83-85 extended)."""
    return load().vx_plan_spread(fmt, rows, columns, out)


class SpreadScratch:
    """Device split scratch for spread plans (kernels/wmma_products.hpp:62-68):
    zeroed counters; kernels leave them zero."""

    def __init__(self, plan: WmmaPlan, device="cuda"):
        import torch

        self.partials = torch.empty(max(int(plan.partial_floats), 1), dtype=torch.float32, device=device)
        self.counters = torch.zeros(max(int(plan.counters), 1), dtype=torch.int32, device=device)
        self.c = SplitScratch(self.partials.data_ptr(), int(plan.partial_floats),
                              self.counters.data_ptr(), int(plan.counters))


def _plan_arg(plan: WmmaPlan | None):
    return ctypes.byref(plan) if plan is not None else None


def _scratch_arg(scratch):
    if scratch is None:
        return None
    if isinstance(scratch, SpreadScratch):
        scratch = scratch.c
    return ctypes.byref(scratch)


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


def ProductEx(fmt: int, x, w, y, rows, columns, out, flags: int = 0, plan=None, stream=None) -> bool:
    """vx_product_ex: `flags` of PRODUCT_ACCUMULATE and PRODUCT_INDEPENDENT."""
    if y.dtype == torch.float32:
        out_dtype = _lib.OUT_F32
    elif y.dtype == torch.bfloat16:
        out_dtype = _lib.OUT_BF16
    else:
        raise ValueError("y must be float32 or bfloat16")
    return check(
        load().vx_product_ex(fmt, _ptr(x), _ptr(w), _ptr(y), out_dtype, rows, columns, out,
                             int(flags), _plan_arg(plan), _stream(stream)),
        unsupported_ok=True,
    )


def ProductHost(fmt: int, x_host, x_dev, w, y_dev, y_host, rows, columns, out, flags: int = 0,
                plan=None, stream=None) -> bool:
    """vx_product_host: x_host and y_host page-locked host tensors, x_dev and
    y_dev device tensors of the same shapes (staging and product output)."""
    if y_dev.dtype != y_host.dtype:
        raise ValueError("y_dev and y_host must have one dtype")
    if y_dev.dtype == torch.float32:
        out_dtype = _lib.OUT_F32
    elif y_dev.dtype == torch.bfloat16:
        out_dtype = _lib.OUT_BF16
    else:
        raise ValueError("y must be float32 or bfloat16")
    return check(
        load().vx_product_host(fmt, _host_ptr(x_host), _ptr(x_dev), _ptr(w), _ptr(y_dev), _host_ptr(y_host),
                               out_dtype, rows, columns, out, int(flags), _plan_arg(plan),
                               _stream(stream)),
        unsupported_ok=True,
    )


def Stage(dst, src, nbytes: int, stream=None) -> None:
    """vx_stage: copy `nbytes` between device or page-locked host tensors with
    SM loads and stores, ordered on the stream."""
    if nbytes > min(dst.numel() * dst.element_size(), src.numel() * src.element_size()):
        raise ValueError("nbytes exceeds a tensor")
    check(load().vx_stage(_any_ptr(dst), _any_ptr(src), nbytes, _stream(stream)))


def SetProgrammaticLaunch(enabled: bool) -> None:
    load().vx_set_programmatic_launch(int(enabled))


TENSOR_CORE_VARIANT = 100  # VX_TENSOR_CORE_VARIANT


def SetTensorCoreProducts(enabled: bool) -> None:
    """Q8_0 products of 9..32 rows planned onto the tcgen05 kernel, or
    (default) onto the mma.sync kernels."""
    load().vx_set_tensor_core_products(int(enabled))


def TensorCoreProducts() -> bool:
    return bool(load().vx_tensor_core_products())


TENSOR_CORE_WIDE_VARIANT = 101  # VX_TENSOR_CORE_WIDE_VARIANT


def SetWideTensorCoreProducts(enabled: bool) -> None:
    """Q8_0 products without a plan onto the wide tcgen05 kernel where it
    measured faster (more than 64 rows, in <= 1024, out >= 3072; default on),
    or always onto the mma.sync planner."""
    load().vx_set_wide_tensor_core_products(int(enabled))


def WideTensorCoreProducts() -> bool:
    return bool(load().vx_wide_tensor_core_products())


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


# ---------------------------------------------------------------- stack kernels
# Named after kernels/generator_kernels.hpp; tensors are device tensors
# (bf16 as int16/bfloat16 bit patterns), None for null pointers.

def Embed(table, ids, text_mask, output, rows, width, scale, stream=None) -> None:
    check(load().vx_embed(_ptr(table), _ptr(ids), _ptr(text_mask), _ptr(output), rows, width, scale,
                          _stream(stream)))


def ScatterRows(input, indices, output, rows, width, stream=None) -> None:
    check(load().vx_scatter_rows(_ptr(input), _ptr(indices), _ptr(output), rows, width, _stream(stream)))


def GatherRows(input, indices, output, rows, width, stream=None) -> None:
    check(load().vx_gather_rows(_ptr(input), _ptr(indices), _ptr(output), rows, width, _stream(stream)))


def RmsNorm(input, weight, output, output_f32, rows, width, epsilon, stream=None) -> None:
    check(load().vx_rms_norm(_ptr(input), _ptr(weight), _ptr(output), _ptr(output_f32), rows, width,
                             epsilon, _stream(stream)))


def QkvRope(qkv, cos_sin, positions, cache_rows, q, k_cache, v_cache, rows, heads, kv_heads, head_dim,
            capacity, cache_type=_lib.CACHE_F32, stream=None) -> None:
    check(load().vx_qkv_rope(_ptr(qkv), _ptr(cos_sin), _ptr(positions), _ptr(cache_rows), _ptr(q),
                             _ptr(k_cache), _ptr(v_cache), cache_type, rows, heads, kv_heads, head_dim,
                             capacity, _stream(stream)))


def Attention(q, k_cache, v_cache, output, rows, rows_per_sequence, keys_per_sequence, past, causal,
              heads, kv_heads, head_dim, capacity, cache_type=_lib.CACHE_F32, past_device=None,
              max_keys=0, stream=None) -> None:
    check(load().vx_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), cache_type, _ptr(output), rows,
                              rows_per_sequence, keys_per_sequence, past, _ptr(past_device), int(causal),
                              heads, kv_heads, head_dim, capacity, max_keys, _stream(stream)))


def SwiGlu(gate_up, output, rows, width, stream=None) -> None:
    check(load().vx_swiglu(_ptr(gate_up), _ptr(output), rows, width, _stream(stream)))


def AddBias(data, bias, rows, width, stream=None) -> None:
    check(load().vx_add_bias(_ptr(data), _ptr(bias), rows, width, _stream(stream)))


def ToBf16(input, output, count, silu=False, stream=None) -> None:
    check(load().vx_to_bf16(_ptr(input), _ptr(output), count, int(silu), _stream(stream)))


def ConcatRows(a, a_scale, a_width, b, b_scale, b_width, output, rows, stream=None) -> None:
    check(load().vx_concat_rows(_ptr(a), _ptr(a_scale), a_width, _ptr(b), _ptr(b_scale), b_width,
                                _ptr(output), rows, _stream(stream)))


def Quantize(input, output, count, scale, stream=None) -> None:
    check(load().vx_quantize(_ptr(input), _ptr(output), count, scale, _stream(stream)))


def SelectRows(quantized, plain, mask, output, rows, width, stream=None) -> None:
    check(load().vx_select_rows(_ptr(quantized), _ptr(plain), _ptr(mask), _ptr(output), rows, width,
                                _stream(stream)))


def PrependSpecial(rows_in, special, output, patches, patch_size, width, stream=None) -> None:
    check(load().vx_prepend_special(_ptr(rows_in), _ptr(special), _ptr(output), patches, patch_size, width,
                                    _stream(stream)))


def AssembleDit(mu, time, cond, x, output, patch_size, width, stream=None) -> None:
    check(load().vx_assemble_dit(_ptr(mu), _ptr(time), _ptr(cond), _ptr(x), _ptr(output), patch_size, width,
                                 _stream(stream)))


def GuidedEuler(velocity, x, count, cfg, dt, stream=None) -> None:
    check(load().vx_guided_euler(_ptr(velocity), _ptr(x), count, cfg, dt, _stream(stream)))
