"""ModelFiles: the generator's checkpoint files (model_files.hpp:45-83) over
the C ABI (vx_model_files_*), and ParseConfig (config.hpp:89-98).

A path is a Hugging Face directory (config.json, model.safetensors,
tokenizer.json when present) or an audio.cpp VoxCPM2 GGUF file. Tensors are
views of the library's read-only mapping: `Tensor.raw()` copies the bytes
out as numpy uint8.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import COMPONENT_MODEL, COMPONENT_VAE, DTYPE_NAMES, ModelConfig, TensorInfo, VxError, check, load


@dataclass(frozen=True)
class Tensor:
    """One tensor (safetensors.hpp:23-34); `shape` outermost first."""

    name: str
    dtype: str
    shape: tuple
    bytes: int
    offset: int
    _data: int

    def raw(self) -> np.ndarray:
        """The tensor's bytes (a copy)."""
        if self.bytes == 0:
            return np.empty(0, np.uint8)
        return np.frombuffer(ctypes.string_at(self._data, self.bytes), np.uint8).copy()


def _tensor(info: TensorInfo) -> Tensor:
    return Tensor(info.name.decode(), DTYPE_NAMES[info.dtype], tuple(info.shape[: info.rank]),
                  int(info.bytes), int(info.offset), info.data or 0)


class ModelFiles:
    """ModelFiles::Open (model_files.cpp:111-180); raises VxError on a
    missing or malformed file."""

    def __init__(self, path):
        self._lib = load()
        self._handle = self._lib.vx_model_files_open(str(path).encode())
        if not self._handle:
            raise VxError(_lib.VX_INVALID, self._lib.vx_last_error().decode(errors="replace"))

    @staticmethod
    def IsVoxCpm2Gguf(path) -> bool:
        return bool(load().vx_model_files_is_voxcpm2_gguf(str(path).encode()))

    @property
    def handle(self) -> int:
        return self._handle

    def gguf(self) -> bool:
        return bool(self._lib.vx_model_files_is_gguf(self._handle))

    def config(self) -> str:
        return self._lib.vx_model_files_config(self._handle).decode()

    def tokenizer(self) -> str:
        return self._lib.vx_model_files_tokenizer(self._handle).decode()

    def _tensors(self, component: int) -> list[Tensor]:
        out = []
        for i in range(self._lib.vx_model_files_count(self._handle, component)):
            info = TensorInfo()
            check(self._lib.vx_model_files_tensor(self._handle, component, i, ctypes.byref(info)))
            out.append(_tensor(info))
        return out

    def model_tensors(self) -> list[Tensor]:
        return self._tensors(COMPONENT_MODEL)

    def vae_tensors(self) -> list[Tensor]:
        return self._tensors(COMPONENT_VAE)

    def _find(self, component: int, name: str) -> Tensor | None:
        info = TensorInfo()
        if self._lib.vx_model_files_find(self._handle, component, name.encode(), ctypes.byref(info)) != 0:
            return None
        return _tensor(info)

    def Model(self, name: str) -> Tensor | None:
        return self._find(COMPONENT_MODEL, name)

    def Vae(self, name: str) -> Tensor | None:
        return self._find(COMPONENT_VAE, name)

    def close(self) -> None:
        if self._handle:
            self._lib.vx_model_files_close(self._handle)
            self._handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ParseConfig(text: str) -> ModelConfig:
    """config.json text -> the generator's configuration, checked against
    what the kernels serve (config.cpp:149-301); raises VxError."""
    data = text.encode()
    c = ModelConfig()
    check(load().vx_parse_config(data, len(data), ctypes.byref(c)))
    return c
