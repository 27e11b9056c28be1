"""Generator: VoxCPM2's per-patch generation on one GPU (generator.hpp:58-179),
over the C ABI (vx_generator_*). Host arrays are numpy float32 / int32."""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import ModelConfig, StackConfig, check, load


def released_config() -> ModelConfig:
    """The released checkpoint's shapes (tests/config_test.cpp:36-67)."""
    c = ModelConfig()
    load().vx_model_config_released(ctypes.byref(c))
    return c


def small_config(layers: int = 2, max_length: int = 256, vocab: int = 64) -> ModelConfig:
    """The released widths with fewer layers (fast parity tests)."""
    c = released_config()
    for stack in (c.lm, c.residual_lm, c.encoder, c.dit):
        stack.layers = layers
    c.max_length = max_length
    c.vocab = vocab
    return c


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def EulerSchedule(timesteps: int, sway: float = 1.0):
    """(t, dt, evaluate) of the sway-sampled Euler steps (generator.hpp:43-44)."""
    t = np.empty(timesteps, np.float32)
    dt = np.empty(timesteps, np.float32)
    ev = np.empty(timesteps, np.int32)
    n = load().vx_euler_schedule(timesteps, sway, t.ctypes.data, dt.ctypes.data, ev.ctypes.data, timesteps)
    return t[:n], dt[:n], ev[:n].astype(bool)


class Generator:
    """generator.hpp:58-179: seeded weights from the constructor, checkpoint
    files from Create."""

    def __init__(self, config: ModelConfig, seed: int = 0, checkpoint: int = _lib.CHECKPOINT_Q8,
                 cache_type: int = _lib.CACHE_F32):
        self._lib = load()
        self.config = config
        self._handle = self._lib.vx_generator_create(ctypes.byref(config), seed, checkpoint, cache_type)
        if not self._handle:
            raise _lib.VxError(_lib.VX_CUDA_ERROR, self._lib.vx_last_error().decode())

    @classmethod
    def Create(cls, config: ModelConfig, files, cache_type: int = _lib.CACHE_F32) -> "Generator":
        """Generator::Create(config, files) (generator.hpp:60-62): the weights
        of a ModelFiles (model_files.py)."""
        self = cls.__new__(cls)
        self._lib = load()
        self.config = config
        self._handle = self._lib.vx_generator_create_from_files(ctypes.byref(config), files.handle, cache_type)
        if not self._handle:
            raise _lib.VxError(_lib.VX_CUDA_ERROR, self._lib.vx_last_error().decode())
        return self

    @property
    def patch_values(self) -> int:
        return self.config.patch_size * self.config.feat_dim

    def Prefill(self, tokens, text_mask, audio_mask, feats) -> None:
        tokens, text_mask, audio_mask = _i32(tokens), _i32(text_mask), _i32(audio_mask)
        feats = _f32(feats)
        check(self._lib.vx_generator_prefill(self._handle, tokens.ctypes.data, text_mask.ctypes.data,
                                             audio_mask.ctypes.data, feats.ctypes.data, tokens.size))

    def Step(self, noise, timesteps: int = 10, cfg: float = 2.0):
        """Returns (latent [patch][feat], stop_logits [2])."""
        noise = _f32(noise)
        latent = np.empty(self.patch_values, np.float32)
        stop = np.empty(2, np.float32)
        check(self._lib.vx_generator_step(self._handle, noise.ctypes.data, timesteps, cfg,
                                          latent.ctypes.data, stop.ctypes.data))
        return latent.reshape(self.config.patch_size, self.config.feat_dim), stop

    def Velocity(self, mu, cond, x, t: float) -> np.ndarray:
        mu, cond, x = _f32(mu), _f32(cond), _f32(x)
        v = np.empty(2 * self.patch_values, np.float32)
        check(self._lib.vx_generator_velocity(self._handle, mu.ctypes.data, cond.ctypes.data, x.ctypes.data,
                                              t, v.ctypes.data))
        return v.reshape(2, self.config.patch_size, self.config.feat_dim)

    def DitPatch(self, mu, cond, noise, timesteps: int = 10, cfg: float = 2.0, download: bool = True):
        mu, cond, noise = _f32(mu), _f32(cond), _f32(noise)
        latent = np.empty(self.patch_values, np.float32) if download else None
        check(self._lib.vx_generator_dit_patch(self._handle, mu.ctypes.data, cond.ctypes.data,
                                               noise.ctypes.data, timesteps, cfg,
                                               latent.ctypes.data if download else None))
        return None if latent is None else latent.reshape(self.config.patch_size, self.config.feat_dim)

    def ReplayDitPatch(self) -> None:
        check(self._lib.vx_generator_replay_dit_patch(self._handle))

    def State(self, name: str, count: int) -> np.ndarray:
        out = np.empty(count, np.float32)
        check(self._lib.vx_generator_state(self._handle, name.encode(), out.ctypes.data, count))
        return out

    def SetState(self, name: str, values) -> None:
        values = _f32(np.atleast_1d(values))
        check(self._lib.vx_generator_set_state(self._handle, name.encode(), values.ctypes.data, values.size))

    def SetGraphs(self, enabled: bool) -> None:
        check(self._lib.vx_generator_set_graphs(self._handle, int(enabled)))

    def SetPersistent(self, enabled: bool) -> None:
        """The DiT patch as one persistent kernel (VoxCPM2's DiT shape) or as
        the per-kernel sequence."""
        check(self._lib.vx_generator_set_persistent(self._handle, int(enabled)))

    def persistent(self) -> bool:
        return bool(self._lib.vx_generator_persistent(self._handle))

    def position(self) -> int:
        return self._lib.vx_generator_position(self._handle)

    def latent(self) -> int:
        """Device address of the last patch's latent [patch][feat], valid
        until the step after next; 0 before the first step of a sequence
        (generator.hpp:78-84)."""
        return self._lib.vx_generator_latent(self._handle) or 0

    def latent_event(self) -> int:
        """The cudaEvent_t recorded after the last step (generator.hpp:84)."""
        return self._lib.vx_generator_latent_event(self._handle) or 0

    def weight_bytes(self) -> int:
        return self._lib.vx_generator_weight_bytes(self._handle)

    def stream(self) -> int:
        return self._lib.vx_generator_stream(self._handle) or 0

    def close(self) -> None:
        if self._handle:
            self._lib.vx_generator_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GeneratorBatch:
    """Several requests per GPU (vx_generator_batch_*): `slots` generators
    sharing one set of weights and one stream; a step advances every active
    slot by one patch with one DiT pass for all of them. Batches the
    per-request loop of synthesizer.cpp:283-307."""

    def __init__(self, config: ModelConfig, slots: int, seed: int = 0, checkpoint: int = _lib.CHECKPOINT_Q8,
                 cache_type: int = _lib.CACHE_F32, files=None):
        self._lib = load()
        self.config = config
        if files is not None:
            self._handle = self._lib.vx_generator_batch_create_from_files(ctypes.byref(config), files.handle,
                                                                          cache_type, slots)
        else:
            self._handle = self._lib.vx_generator_batch_create(ctypes.byref(config), seed, checkpoint, cache_type,
                                                               slots)
        if not self._handle:
            raise _lib.VxError(_lib.VX_CUDA_ERROR, self._lib.vx_last_error().decode())
        self.slots = slots

    @property
    def patch_values(self) -> int:
        return self.config.patch_size * self.config.feat_dim

    def Prefill(self, slot: int, tokens, text_mask, audio_mask, feats) -> None:
        tokens, text_mask, audio_mask = _i32(tokens), _i32(text_mask), _i32(audio_mask)
        feats = _f32(feats)
        check(self._lib.vx_generator_batch_prefill(self._handle, slot, tokens.ctypes.data, text_mask.ctypes.data,
                                                   audio_mask.ctypes.data, feats.ctypes.data, tokens.size))

    def Step(self, noise, active=None, timesteps: int = 10, cfg: float = 2.0):
        """noise [slots][patch][feat]; returns (latents [slots][patch][feat],
        stop logits [slots][2]); rows of inactive slots are zero."""
        active = _i32(np.ones(self.slots) if active is None else active)
        noise = _f32(noise)
        latents = np.zeros((self.slots, self.config.patch_size, self.config.feat_dim), np.float32)
        stop = np.zeros((self.slots, 2), np.float32)
        check(self._lib.vx_generator_batch_step(self._handle, active.ctypes.data, noise.ctypes.data, timesteps, cfg,
                                                latents.ctypes.data, stop.ctypes.data))
        return latents, stop

    def State(self, slot: int, name: str, count: int) -> np.ndarray:
        out = np.empty(count, np.float32)
        check(self._lib.vx_generator_batch_state(self._handle, slot, name.encode(), out.ctypes.data, count))
        return out

    def position(self, slot: int) -> int:
        return self._lib.vx_generator_batch_position(self._handle, slot)

    def SetGraphs(self, enabled: bool) -> None:
        check(self._lib.vx_generator_batch_set_graphs(self._handle, int(enabled)))

    def stream(self) -> int:
        return self._lib.vx_generator_batch_stream(self._handle) or 0

    def close(self) -> None:
        if self._handle:
            self._lib.vx_generator_batch_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
