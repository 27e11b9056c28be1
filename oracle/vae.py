"""The oracle's AudioVAE V2 decoder — TEST INFRASTRUCTURE ONLY (the checker of
the AudioVAE parity tests): the reference's streaming decoder (vae.cpp:415-
516, AudioVae::Run; kernels/vae_kernels.hip:19-100) restated in numpy
float32, time-major ([frames][channels]), with the state of every causal
convolution carried between calls. Weights are the library's seeded
AudioVAE checkpoint, regenerated here from the same rule (bf16 values of the
seeded hash, widened to float32; tensor id = FNV-1a of the name) in the
layouts the reference packs at load (weight norm folded; the transposed
convolution as one matrix per input frame, current and previous).
"""

from __future__ import annotations

import numpy as np

from . import bf16_value, random_bf16
from .model import tensor_id

KERNEL = 7                # the residual units' and the outer convolutions' width
DILATIONS = (1, 3, 9)


class VaeConfig:
    """AudioVaeConfig (config.hpp:55-72), the decoder's fields."""

    def __init__(self, latent_dim=64, decoder_dim=2048, decoder_rates=(8, 6, 5, 2, 2, 2),
                 out_sample_rate=48000, sr_bin_boundaries=(20000, 30000, 40000)):
        self.latent_dim = latent_dim
        self.decoder_dim = decoder_dim
        self.decoder_rates = tuple(decoder_rates)
        self.out_sample_rate = out_sample_rate
        self.sr_bin_boundaries = tuple(sr_bin_boundaries)

    def decode_hop(self) -> int:
        """Output samples per latent frame (config.cpp:264-267)."""
        return int(np.prod(self.decoder_rates))

    def rate_bucket(self) -> int:
        """torch.bucketize of the output rate, right=False (config.cpp:269-275)."""
        bucket = 0
        while bucket < len(self.sr_bin_boundaries) and self.sr_bin_boundaries[bucket] < self.out_sample_rate:
            bucket += 1
        return bucket


def _seeded(seed, name, count, mean, std):
    return bf16_value(random_bf16(seed, tensor_id("audio_vae." + name), count, mean, std)).astype(np.float32)


class VaeWeights:
    """The seeded decoder weights, drawn in the checkpoint's layouts and
    packed as the reference packs at load (AudioVae::Create, vae.cpp:222-
    291): the same names, counts and distributions as the library's
    (vae.cu SeededVaeWeights), packed here by numpy reshapes."""

    def __init__(self, c: VaeConfig, seed: int):
        latent, width = c.latent_dim, c.decoder_dim
        self.in_depthwise = _seeded(seed, "in.depthwise", latent * KERNEL, 0.0, 0.3).reshape(latent, KERNEL)
        self.in_depthwise_bias = _seeded(seed, "in.depthwise_bias", latent, 0.0, 0.02)
        self.in_pointwise = _seeded(seed, "in.pointwise", width * latent, 0.0, latent ** -0.5).reshape(width, latent)
        self.in_pointwise_bias = _seeded(seed, "in.pointwise_bias", width, 0.0, 0.02)
        self.blocks = []
        channels = width
        buckets = len(c.sr_bin_boundaries) + 1
        bucket = c.rate_bucket()
        for b, s in enumerate(c.decoder_rates):
            out = channels // 2
            p = f"block{b}."
            # The rate conditioning's embedding tables [buckets][in]; the
            # output rate's bucket selects one row (vae.cpp:250-261).
            scale = _seeded(seed, p + "scale_embed", buckets * channels, 1.0, 0.05).reshape(buckets, channels)
            bias = _seeded(seed, p + "bias_embed", buckets * channels, 0.0, 0.05).reshape(buckets, channels)
            # ConvTranspose1d weight [in][out][2s] (vae.cpp:263-275), packed
            # as two [s * out][in] matrices: row r * out + o holds tap r (for
            # the current frame) and tap r + s (for the previous one).
            up = _seeded(seed, p + "up", channels * out * 2 * s, 0.0, (2 * channels) ** -0.5).reshape(
                channels, out, 2 * s)
            previous = up[:, :, s:].transpose(2, 1, 0).reshape(s * out, channels)
            current = up[:, :, :s].transpose(2, 1, 0).reshape(s * out, channels)
            block = dict(
                stride=s, inp=channels, out=out,
                scale=np.ascontiguousarray(scale[bucket]),
                bias=np.ascontiguousarray(bias[bucket]),
                alpha=_seeded(seed, p + "alpha", channels, 1.0, 0.1),
                up_weight=up,
                up_current=np.ascontiguousarray(current),
                up_previous=np.ascontiguousarray(previous),
                up_bias=np.tile(_seeded(seed, p + "up_bias", out, 0.0, 0.02), s),
                units=[])
            for u, d in enumerate(DILATIONS):
                q = p + f"unit{u}."
                block["units"].append(dict(
                    dilation=d,
                    alpha_in=_seeded(seed, q + "alpha_in", out, 1.0, 0.1),
                    depthwise=_seeded(seed, q + "depthwise", out * KERNEL, 0.0, 0.3).reshape(out, KERNEL),
                    depthwise_bias=_seeded(seed, q + "depthwise_bias", out, 0.0, 0.02),
                    alpha_out=_seeded(seed, q + "alpha_out", out, 1.0, 0.1),
                    pointwise=_seeded(seed, q + "pointwise", out * out, 0.0, 0.5 * out ** -0.5).reshape(out, out),
                    pointwise_bias=_seeded(seed, q + "pointwise_bias", out, 0.0, 0.02)))
            self.blocks.append(block)
            channels = out
        self.out_channels = channels
        self.out_alpha = _seeded(seed, "out.alpha", channels, 1.0, 0.1)
        self.out_conv = _seeded(seed, "out.conv", channels * KERNEL, 0.0, (KERNEL * channels) ** -0.5).reshape(
            channels, KERNEL)
        self.out_bias = np.float32(0.01)


def snake(x: np.ndarray, alpha: np.ndarray, scale=None, bias=None) -> np.ndarray:
    """kernels/vae_kernels.hip:19-33: y (* scale + bias), then
    y + sin(alpha y)^2 / (alpha + 1e-9), per channel."""
    y = x.astype(np.float32)
    if scale is not None:
        y = (y * scale + bias).astype(np.float32)
    s = np.sin(alpha * y).astype(np.float32)
    return (y + (np.float32(1.0) / (alpha + np.float32(1e-9))) * (s * s)).astype(np.float32)


def depthwise(work: np.ndarray, weight: np.ndarray, bias: np.ndarray, frames: int, dilation: int) -> np.ndarray:
    """kernels/vae_kernels.hip:35-50: out[t][c] = bias[c] + sum_j
    weight[c][j] work[t + j * dilation][c], over frames t of the history-
    padded `work`."""
    out = np.broadcast_to(bias, (frames, bias.size)).astype(np.float32).copy()
    for j in range(weight.shape[1]):
        out += weight[:, j] * work[j * dilation: j * dilation + frames]
    return out.astype(np.float32)


def to_mono(work: np.ndarray, weight: np.ndarray, bias: np.float32, frames: int) -> np.ndarray:
    """kernels/vae_kernels.hip:67-89: tanh(bias + sum_{c, j} weight[c][j]
    work[t + j][c])."""
    total = np.zeros(frames, np.float64)
    for j in range(weight.shape[1]):
        total += work[j: j + frames].astype(np.float64) @ weight[:, j].astype(np.float64)
    return np.tanh(total + np.float64(bias)).astype(np.float32)


class OracleVae:
    """AudioVae's decoder (vae.hpp:25-79) on the CPU: Reset, then Decode
    calls that continue one stream."""

    def __init__(self, c: VaeConfig, seed: int):
        self.c = c
        self.w = VaeWeights(c, seed)
        self.reset()

    def reset(self):
        """vae.cpp:363-368 (the states of vae.cpp:334-342, in decoding
        order, zeroed)."""
        w = self.w
        self.states = [np.zeros((KERNEL - 1, self.c.latent_dim), np.float32)]
        for block in w.blocks:
            self.states.append(np.zeros((1, block["inp"]), np.float32))
            for unit in block["units"]:
                self.states.append(np.zeros(((KERNEL - 1) * unit["dilation"], block["out"]), np.float32))
        self.states.append(np.zeros((KERNEL - 1, w.out_channels), np.float32))

    def decode(self, latents: np.ndarray) -> np.ndarray:
        """vae.cpp:382-393 (Decode) and 415-516 (Run): latents
        [frames][latent_dim] -> frames * decode_hop samples."""
        w = self.w
        latents = np.asarray(latents, np.float32).reshape(-1, self.c.latent_dim)
        frames = latents.shape[0]
        state = iter(range(len(self.states)))

        def window(new: np.ndarray) -> np.ndarray:
            """state ++ new; the next state keeps the window's last rows."""
            i = next(state)
            work = np.concatenate([self.states[i], new]).astype(np.float32)
            rows = self.states[i].shape[0]
            self.states[i] = work[work.shape[0] - rows:].copy()
            return work

        work = window(latents)
        h = depthwise(work, w.in_depthwise, w.in_depthwise_bias, frames, 1)
        hidden = (h @ w.in_pointwise.T + w.in_pointwise_bias).astype(np.float32)
        t = frames
        for block in w.blocks:
            work = window(snake(hidden, block["alpha"], block["scale"], block["bias"]))
            s, out = block["stride"], block["out"]
            # ConvTranspose1d (kernel 2s, stride s, causal) as the reference
            # computes it (vae.cpp:473-479): frame t of the input gives output
            # frames t * s + r from the current frame's taps r and the
            # previous frame's taps r + s.
            hidden = (work[1:t + 1] @ block["up_current"].T).astype(np.float32)
            hidden = (hidden + work[0:t] @ block["up_previous"].T).astype(np.float32)
            hidden = (hidden + block["up_bias"]).astype(np.float32).reshape(t * s, out)
            t *= s
            for unit in block["units"]:
                work = window(snake(hidden, unit["alpha_in"]))
                sc = depthwise(work, unit["depthwise"], unit["depthwise_bias"], t, unit["dilation"])
                sc = snake(sc, unit["alpha_out"])
                hidden = (hidden + (sc @ unit["pointwise"].T + unit["pointwise_bias"])).astype(np.float32)
        work = window(snake(hidden, w.out_alpha))
        return to_mono(work, w.out_conv, w.out_bias, t)
