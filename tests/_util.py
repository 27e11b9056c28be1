"""Helpers shared by the GPU parity tests (device buffers, comparisons)."""

from __future__ import annotations

import numpy as np
import torch


def to_dev(a: np.ndarray) -> torch.Tensor:
    """A device copy of a numpy array (uint16 travels as int16 bits)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if t.dtype == torch.uint16:
        t = t.view(torch.int16)
    return t.cuda()


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.float32)


def bf16_ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 units in the last place between two bit arrays of
    finite values (sign-magnitude mapped to a monotone integer line)."""
    def line(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(line(a) - line(b))


def assert_bf16_close(got: np.ndarray, ref: np.ndarray, max_ulps: int = 1, min_exact: float = 0.98,
                      what: str = ""):
    """bf16 outputs of the same fp32 arithmetic in a different order: every
    value within `max_ulps` bf16 ulps of the reference, or (for values that
    cancel towards zero, where an ulp is tiny) within 2^-8 of the output's
    root-mean-square; at least `min_exact` of them bit-equal."""
    got = np.asarray(got).reshape(-1)
    ref = np.asarray(ref).reshape(-1)
    assert got.shape == ref.shape, what
    d = bf16_ulps(got, ref)
    exact = float(np.mean(d == 0))
    gv = (got.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    rv = (ref.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    scale = float(np.sqrt(np.mean(rv * rv))) if rv.size else 0.0
    ok = (d <= max_ulps) | (np.abs(gv - rv) <= 2.0 ** -8 * scale)
    worst = int(np.argmin(ok)) if not ok.all() else -1
    assert ok.all(), (f"{what}: value {worst} {gv[worst]:.6g} vs {rv[worst]:.6g} ({int(d[worst])} ulps, "
                      f"rms {scale:.3g}, exact {exact:.4f})")
    assert exact >= min_exact, f"{what}: only {exact:.4f} bit-equal"


def assert_f32_close(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float, what: str = ""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    worst = float(np.max(err - bound)) if err.size else -1.0
    assert worst <= 0, f"{what}: max excess {worst:.3e} (max err {float(err.max()):.3e})"


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
