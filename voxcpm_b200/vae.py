"""AudioVae: the AudioVAE V2 decoder on its own stream (vae.hpp:25-79), over
the C ABI (vx_audio_vae_*). Host arrays are numpy float32."""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import VaeConfig, check, load


def default_vae_config() -> VaeConfig:
    """The released AudioVAE V2's decoder: latent 64, decoder 2048, rates
    8 6 5 2 2 2, 48 kHz out, rate boundaries 20000 30000 40000."""
    c = VaeConfig()
    load().vx_vae_config_default(ctypes.byref(c))
    return c


def vae_config(latent_dim: int, decoder_dim: int, decoder_rates, out_sample_rate: int = 48000,
               sr_bin_boundaries=(20000, 30000, 40000)) -> VaeConfig:
    c = VaeConfig()
    c.latent_dim, c.decoder_dim, c.out_sample_rate = latent_dim, decoder_dim, out_sample_rate
    c.decoder_rate_count = len(decoder_rates)
    for i, r in enumerate(decoder_rates):
        c.decoder_rates[i] = r
    c.sr_bin_boundary_count = len(sr_bin_boundaries)
    for i, b in enumerate(sr_bin_boundaries):
        c.sr_bin_boundaries[i] = b
    return c


class AudioVae:
    """AudioVae (vae.hpp:25-79), decoding: Reset, Decode, Enqueue, Collect,
    with the seeded AudioVAE checkpoint of `seed`."""

    def __init__(self, config: VaeConfig, seed: int = 0):
        self._lib = load()
        self.config = config
        self._handle = self._lib.vx_audio_vae_create(ctypes.byref(config), seed)
        if not self._handle:
            raise _lib.VxError(_lib.VX_INVALID, self._lib.vx_last_error().decode())
        self.decode_hop = self._lib.vx_audio_vae_decode_hop(self._handle)
        self.pending = 0

    def Reset(self) -> None:
        check(self._lib.vx_audio_vae_reset(self._handle))

    def Decode(self, latents) -> np.ndarray:
        """latents [frames][latent_dim] -> frames * decode_hop samples."""
        latents = np.ascontiguousarray(latents, dtype=np.float32).reshape(-1, self.config.latent_dim)
        audio = np.empty(latents.shape[0] * self.decode_hop, np.float32)
        check(self._lib.vx_audio_vae_decode(self._handle, latents.ctypes.data, latents.shape[0],
                                            audio.ctypes.data))
        return audio

    def Enqueue(self, latents: int, frames: int, ready: int = 0) -> None:
        """Device latents (an address) once the event `ready` (0: none) has
        completed, on the AudioVAE's own stream."""
        check(self._lib.vx_audio_vae_enqueue(self._handle, latents, frames, ready or None))
        self.pending = frames * self.decode_hop

    def Collect(self) -> np.ndarray:
        audio = np.empty(max(self.pending, 1), np.float32)
        samples = ctypes.c_size_t(0)
        check(self._lib.vx_audio_vae_collect(self._handle, audio.ctypes.data, audio.size, ctypes.byref(samples)))
        self.pending = 0
        return audio[:samples.value]

    def stream(self) -> int:
        return self._lib.vx_audio_vae_stream(self._handle) or 0

    def close(self) -> None:
        if self._handle:
            self._lib.vx_audio_vae_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
