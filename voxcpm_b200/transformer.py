"""transformer.hpp over the C ABI: KvCache, ForwardStack and Project
(transformer.hpp:17-76) for callers that run a MiniCPM4 stack themselves."""

from __future__ import annotations

import ctypes

import torch

from ._lib import (AttentionLayoutC, LayerWeightsC, ProjectionC, StackConfig, StackScratchC,  # noqa: F401
                   StackWeightsC, check, load)
from .kernels import _ptr, _stream


class KvCache:
    """Keys and values [layer][kv_head][capacity][head_dim], zeroed
    (transformer.hpp:17-36); `cache_type` is _lib.CACHE_F32 or CACHE_BF16."""

    def __init__(self, config: StackConfig, capacity: int, cache_type: int):
        self._lib = load()
        self._handle = self._lib.vx_kv_cache_create(ctypes.byref(config), capacity, cache_type)
        if not self._handle:
            raise RuntimeError(self._lib.vx_last_error().decode(errors="replace"))

    @property
    def handle(self) -> int:
        return self._handle

    def capacity(self) -> int:
        return self._lib.vx_kv_cache_capacity(self._handle)

    def keys(self, layer: int) -> int:
        return self._lib.vx_kv_cache_keys(self._handle, layer) or 0

    def values(self, layer: int) -> int:
        return self._lib.vx_kv_cache_values(self._handle, layer) or 0

    def close(self) -> None:
        if self._handle:
            self._lib.vx_kv_cache_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def StackScratchElements(config: StackConfig, rows: int) -> list[int]:
    """Elements of each StackScratch buffer (normed, qkv, q, attention,
    gate_up, activation) for `rows` rows."""
    counts = (ctypes.c_size_t * 6)()
    check(load().vx_stack_scratch_elements(ctypes.byref(config), rows, counts))
    return list(counts)


def ForwardStack(stack: StackWeightsC, rope: torch.Tensor | None, layout: AttentionLayoutC, cache: KvCache,
                 hidden: torch.Tensor, output: torch.Tensor, rows: int, scratch: StackScratchC,
                 stream=None) -> None:
    """transformer.hpp:68-71: `hidden` [rows][width] fp32 updated in place,
    the final norm's fp32 output into `output`."""
    check(load().vx_forward_stack(ctypes.byref(stack), _ptr(rope), ctypes.byref(layout), cache.handle,
                                  _ptr(hidden), _ptr(output), rows, ctypes.byref(scratch), _stream(stream)))


def Project(projection: ProjectionC, x: torch.Tensor, y: torch.Tensor, rows: int, stream=None) -> None:
    """transformer.hpp:73-76: y = x W^T + b for bf16 x."""
    check(load().vx_project(ctypes.byref(projection), _ptr(x), _ptr(y), rows, _stream(stream)))
