"""CPU oracle of the VoxCPM2 per-patch path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs use it, as the checker or the timed CPU baseline. The product
(voxcpm_b200, libvoxcpm_b200.so) never imports or links it.

The arithmetic lives in vxoracle.c (plain C, one function per reference
kernel, each citing the reference file:line it restates); this module loads
it with ctypes and wraps numpy arrays. model.py composes the primitives into
the reference's ForwardStack / DiT evaluation / generation step.

Parity status: UNPINNED against OpenBMB's outputs (the golden tensors need the
absent checkpoint); pinned on the weight-free pieces (see vxoracle.h).
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_size_t, c_uint16, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "libvxoracle.so"

BF16_ROWS = 0
Q8_0 = 2


def build(force: bool = False) -> Path:
    """Compiles vxoracle.c with gcc (oracle/Makefile)."""
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < (HERE / "vxoracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "-B" if force else "libvxoracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIBRARY


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIBRARY))
        P = c_void_p
        sig = {
            "vxo_bf16_bits": (c_uint16, [c_float]),
            "vxo_bf16_value": (c_float, [c_uint16]),
            "vxo_half_value": (c_float, [c_uint16]),
            "vxo_half_bits": (c_uint16, [c_float]),
            "vxo_to_bf16_array": (None, [P, P, c_size_t]),
            "vxo_hash": (c_uint64, [c_uint64, c_uint64, c_uint64]),
            "vxo_random_q8_0": (None, [c_uint64, c_uint64, c_size_t, c_size_t, c_float, P]),
            "vxo_random_bf16": (None, [c_uint64, c_uint64, c_size_t, c_float, c_float, P]),
            "vxo_q8_0_to_tiles": (None, [P, c_size_t, c_size_t, P]),
            "vxo_bf16_to_tiles": (None, [P, c_size_t, c_size_t, P]),
            "vxo_q8_0_dequant": (None, [P, c_size_t, c_size_t, P]),
            "vxo_product_exact": (None, [P, c_int, P, P, P, P, c_size_t, c_size_t, c_size_t, c_int]),
            "vxo_linear": (None, [P, c_int, P, P, c_size_t, c_size_t, c_size_t, c_int, c_int]),
            "vxo_rms_norm": (None, [P, P, P, P, c_size_t, c_size_t, c_float]),
            "vxo_rope_table": (None, [c_double, c_size_t, P, c_double, c_size_t, P]),
            "vxo_qkv_rope": (None, [P, P, P, P, P, P, P, c_size_t, c_size_t, c_size_t, c_size_t, c_size_t]),
            "vxo_attention": (None, [P, P, P, P, c_size_t, c_size_t, c_size_t, c_size_t, c_int,
                                     c_size_t, c_size_t, c_size_t, c_size_t]),
            "vxo_swiglu": (None, [P, P, c_size_t, c_size_t]),
            "vxo_add_bias": (None, [P, P, c_size_t, c_size_t]),
            "vxo_to_bf16": (None, [P, P, c_size_t, c_int]),
            "vxo_concat_rows": (None, [P, P, c_size_t, P, P, c_size_t, P, c_size_t]),
            "vxo_quantize": (None, [P, P, c_size_t, c_float]),
            "vxo_prepend_special": (None, [P, P, P, c_size_t, c_size_t, c_size_t]),
            "vxo_assemble_dit": (None, [P, P, P, P, P, c_size_t, c_size_t]),
            "vxo_gather_rows": (None, [P, P, P, c_size_t, c_size_t]),
            "vxo_guided_euler": (None, [P, P, c_size_t, c_float, c_float]),
            "vxo_euler_schedule": (c_size_t, [c_size_t, c_float, P, P, P, c_size_t]),
            "vxo_linspace": (None, [c_float, c_float, c_size_t, P]),
            "vxo_sinusoid": (None, [c_float, c_size_t, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "contiguous array expected"
    return a.ctypes.data


# ---------------------------------------------------------------- numerics

def bf16_bits(values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(values.shape, dtype=np.uint16)
    lib().vxo_to_bf16_array(_p(values), _p(out), values.size)
    return out


def bf16_value(bits: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def half_value(bits: int) -> float:
    return lib().vxo_half_value(bits)


def half_bits(value: float) -> int:
    return lib().vxo_half_bits(value)


# ---------------------------------------------------------------- weights

def random_q8_0(seed: int, tensor: int, rows: int, columns: int, scale_std: float = 0.02 / 127) -> np.ndarray:
    out = np.empty(rows * (columns // 32) * 34, dtype=np.uint8)
    lib().vxo_random_q8_0(seed, tensor, rows, columns, scale_std, _p(out))
    return out


def random_bf16(seed: int, tensor: int, count: int, mean: float = 0.0, std: float = 0.02) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib().vxo_random_bf16(seed, tensor, count, mean, std, _p(out))
    return out


def q8_0_to_tiles(blocks: np.ndarray, rows: int, columns: int) -> np.ndarray:
    out = np.empty((rows + 15) // 16 * (columns // 32) * 544, dtype=np.uint8)
    lib().vxo_q8_0_to_tiles(_p(blocks), rows, columns, _p(out))
    return out


def bf16_to_tiles(w: np.ndarray, rows: int, columns: int) -> np.ndarray:
    out = np.empty((rows + 15) // 16 * (columns // 32) * 512, dtype=np.uint16)
    lib().vxo_bf16_to_tiles(_p(np.ascontiguousarray(w)), rows, columns, _p(out))
    return out


def q8_0_dequant(blocks: np.ndarray, rows: int, columns: int) -> np.ndarray:
    out = np.empty(rows * columns, dtype=np.float64)
    lib().vxo_q8_0_dequant(_p(blocks), rows, columns, _p(out))
    return out.reshape(rows, columns)


# ---------------------------------------------------------------- products

def product_exact(x: np.ndarray, fmt: int, w: np.ndarray, rows: int, columns: int, out: int,
                  before: np.ndarray | None = None, threads: int = 0):
    """(exact, magnitude) in double: tests/products_test.cpp:115-145."""
    exact = np.empty(rows * out, dtype=np.float64)
    magnitude = np.empty(rows * out, dtype=np.float64)
    b = None if before is None else np.ascontiguousarray(before, dtype=np.float32)
    lib().vxo_product_exact(_p(np.ascontiguousarray(x, dtype=np.uint16)), fmt, _p(w), _p(b), _p(exact),
                            _p(magnitude), rows, columns, out, threads)
    return exact.reshape(rows, out), magnitude.reshape(rows, out)


def linear(x: np.ndarray, fmt: int, w: np.ndarray, rows: int, columns: int, out: int,
           y: np.ndarray | None = None, accumulate: bool = False, threads: int = 0) -> np.ndarray:
    """float32 transcription of the device products (y (+)= x W^T)."""
    if y is None:
        y = np.zeros((rows, out), dtype=np.float32)
    assert y.dtype == np.float32 and y.flags["C_CONTIGUOUS"]
    lib().vxo_linear(_p(np.ascontiguousarray(x, dtype=np.uint16)), fmt, _p(w), _p(y), rows, columns, out,
                     int(accumulate), threads)
    return y


def matmul_exact(a: np.ndarray, b: np.ndarray, c: np.ndarray | None, transpose_a: bool, transpose_b: bool,
                 m: int, n: int, k: int, lda: int, ldb: int, ldc: int, stride_a: int = 0, stride_b: int = 0,
                 stride_c: int = 0, batch: int = 1):
    """(exact, magnitude) in double of the column-major BLAS product
    C[m][n] (+)= op(A)[m][k] op(B)[k][n] per batch (gemm.hpp:16-38;
    gemm.cpp:338-361 runs it with alpha 1 and beta = accumulate). `a`, `b`
    are bf16 bits, `c` the float32 C before the call (None: beta 0). Both
    results are flat arrays laid out as C: element (i, j) of batch t at
    t * stride_c + i + j * ldc; entries outside the product are NaN."""
    av, bv = bf16_value(a).astype(np.float64), bf16_value(b).astype(np.float64)
    size = (batch - 1) * stride_c + (n - 1) * ldc + m if m and n and batch else 0
    exact = np.full(max(size, 0 if c is None else c.size), np.nan)
    magnitude = np.full_like(exact, np.nan)
    i = np.arange(m)[:, None]
    ll = np.arange(k)[None, :]
    for t in range(batch):
        ia = t * stride_a + (ll + i * lda if transpose_a else i + ll * lda)  # op(A)[i][l]
        j = np.arange(n)[None, :]
        lb = np.arange(k)[:, None]
        ib = t * stride_b + (j + lb * ldb if transpose_b else lb + j * ldb)  # op(B)[l][j]
        opa, opb = av[ia], bv[ib]
        prod = opa @ opb
        mag = np.abs(opa) @ np.abs(opb)
        ic = t * stride_c + np.arange(m)[:, None] + np.arange(n)[None, :] * ldc
        if c is not None:
            before = c.astype(np.float64)[ic]
            prod = prod + before
            mag = mag + np.abs(before)
        exact[ic] = prod
        magnitude[ic] = mag
    return exact, magnitude


def relative_error(y: np.ndarray, exact: np.ndarray, magnitude: np.ndarray) -> float:
    """max |y - exact| / sum |x w| (tests/products_test.cpp:115-145)."""
    return float(np.max(np.abs(y.astype(np.float64) - exact) / np.maximum(magnitude, 1e-30)))


# ---------------------------------------------------------------- schedule / time

def linspace(start: float, end: float, steps: int) -> np.ndarray:
    out = np.empty(steps, dtype=np.float32)
    lib().vxo_linspace(start, end, steps, _p(out))
    return out


def euler_schedule(timesteps: int, sway: float = 1.0):
    cap = timesteps + 1
    t = np.empty(cap, np.float32)
    dt = np.empty(cap, np.float32)
    ev = np.empty(cap, np.int32)
    n = lib().vxo_euler_schedule(timesteps, sway, _p(t), _p(dt), _p(ev), cap)
    return t[:n].copy(), dt[:n].copy(), ev[:n].astype(bool)


def sinusoid(t: float, width: int) -> np.ndarray:
    out = np.empty(width, np.float32)
    lib().vxo_sinusoid(t, width, _p(out))
    return out


# ---------------------------------------------------------------- stack kernels

def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, want_f32: bool = False):
    """kernels/generator_kernels.hip:91-108 -> (bf16 bits, fp32 or None)."""
    x = _f32(x)
    rows, width = x.shape
    out = np.empty((rows, width), np.uint16)
    out32 = np.empty((rows, width), np.float32) if want_f32 else None
    lib().vxo_rms_norm(_p(x), _p(_u16(weight)), _p(out), _p(out32), rows, width, eps)
    return out, out32


def rope_table(theta: float, dim: int, factors: np.ndarray, scaling: float, positions: int) -> np.ndarray:
    table = np.empty((positions, dim), np.float32)
    lib().vxo_rope_table(theta, dim, _p(np.ascontiguousarray(factors, np.float64)), scaling, positions,
                         _p(table))
    return table


def qkv_rope(qkv, cos_sin, positions, cache_rows, k_cache, v_cache, heads, kv_heads, head_dim):
    """kernels/generator_kernels.hip:110-158; k_cache/v_cache [kv][capacity][d]
    float32 arrays updated in place. Returns q [rows][heads][d]."""
    qkv = _f32(qkv)
    rows = qkv.shape[0]
    q = np.empty((rows, heads, head_dim), np.float32)
    capacity = k_cache.shape[1]
    lib().vxo_qkv_rope(_p(qkv), _p(None if cos_sin is None else _f32(cos_sin)), _p(_i32(positions)),
                       _p(_i32(cache_rows)), _p(q), _p(k_cache), _p(v_cache), rows, heads, kv_heads,
                       head_dim, capacity)
    return q


def attention(q, k_cache, v_cache, rows_per_sequence, keys_per_sequence, past, causal, heads, kv_heads,
              head_dim):
    """kernels/generator_kernels.hip:160-241 -> bf16 bits [rows][heads*d]."""
    q = _f32(q)
    rows = q.shape[0]
    out = np.empty((rows, heads * head_dim), np.uint16)
    lib().vxo_attention(_p(q), _p(_f32(k_cache)), _p(_f32(v_cache)), _p(out), rows, rows_per_sequence,
                        keys_per_sequence, past, int(causal), heads, kv_heads, head_dim, k_cache.shape[1])
    return out


def swiglu(gate_up: np.ndarray) -> np.ndarray:
    gate_up = _f32(gate_up)
    rows, width2 = gate_up.shape
    out = np.empty((rows, width2 // 2), np.uint16)
    lib().vxo_swiglu(_p(gate_up), _p(out), rows, width2 // 2)
    return out


def add_bias(data: np.ndarray, bias: np.ndarray) -> np.ndarray:
    data = _f32(data).copy()
    rows, width = data.shape
    lib().vxo_add_bias(_p(data), _p(_u16(bias)), rows, width)
    return data


def to_bf16(x: np.ndarray, silu: bool = False) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().vxo_to_bf16(_p(x), _p(out), x.size, int(silu))
    return out


def concat_rows(a, b, a_scale=None, b_scale=None) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    rows = a.shape[0]
    out = np.empty((rows, a.shape[1] + b.shape[1]), np.uint16)
    lib().vxo_concat_rows(_p(a), _p(None if a_scale is None else _f32(a_scale)), a.shape[1], _p(b),
                          _p(None if b_scale is None else _f32(b_scale)), b.shape[1], _p(out), rows)
    return out


def quantize(x: np.ndarray, scale: float) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().vxo_quantize(_p(x), _p(out), x.size, scale)
    return out


def prepend_special(rows_in: np.ndarray, special: np.ndarray, patches: int, patch_size: int) -> np.ndarray:
    rows_in = _f32(rows_in)
    width = rows_in.shape[-1]
    out = np.empty((patches * (patch_size + 1), width), np.float32)
    lib().vxo_prepend_special(_p(rows_in), _p(_u16(special)), _p(out), patches, patch_size, width)
    return out


def assemble_dit(mu, time, cond, x, patch_size: int) -> np.ndarray:
    width = time.shape[-1]
    out = np.empty((2 * (3 + 2 * patch_size), width), np.float32)
    lib().vxo_assemble_dit(_p(_f32(mu)), _p(_f32(time)), _p(_f32(cond)), _p(_f32(x)), _p(out), patch_size,
                           width)
    return out


def gather_rows(x: np.ndarray, indices) -> np.ndarray:
    x = _f32(x)
    idx = _i32(indices)
    out = np.empty((idx.size, x.shape[1]), np.float32)
    lib().vxo_gather_rows(_p(x), _p(idx), _p(out), idx.size, x.shape[1])
    return out


def guided_euler(velocity: np.ndarray, x: np.ndarray, cfg: float, dt: float) -> np.ndarray:
    x = _f32(x).copy()
    lib().vxo_guided_euler(_p(_f32(velocity)), _p(x), x.size, cfg, dt)
    return x
