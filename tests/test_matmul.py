"""Bf16Gemm::Matmul (gemm.hpp:16-38, 60-63; gemm.cpp:338-361): the general
column-major product C (+)= op(A) op(B) with bf16 operands and float32 C.

The reference runs it through hipBLASLt (hipBLAS as the fallback) with
alpha 1 and beta = accumulate. The oracle is the double-precision product of
the same bf16 operands; the metric and limit are the products' (max
|c - exact| / sum |a b| per entry, 1e-5; tests/products_test.cpp:115-145).
Entries of C outside the product (ldc above m, gaps between batches) must
keep their values."""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200.gemm import Bf16Gemm, MatmulShape, TuningBucket

LIMIT = 1e-5


def padded(v: np.ndarray, size: int) -> np.ndarray:
    out = np.full(size, np.nan)
    out[: min(size, v.size)] = v[:size]
    return out


def shape_of(ta, tb, m, n, k, lda, ldb, ldc, sa=0, sb=0, sc=0, batch=1, accumulate=False):
    return MatmulShape(int(ta), int(tb), m, n, k, lda, ldb, ldc, sa, sb, sc, batch, int(accumulate))


def test_oracle_matches_column_major_definition():
    """The oracle's indexing against numpy on explicitly column-major
    (Fortran-order) operands, every transpose pair."""
    rng = np.random.default_rng(3)
    m, n, k = 5, 4, 7
    for ta in (False, True):
        for tb in (False, True):
            a_mat = rng.normal(size=(k, m) if ta else (m, k)).astype(np.float32)
            b_mat = rng.normal(size=(n, k) if tb else (k, n)).astype(np.float32)
            a = oracle.bf16_bits(a_mat.reshape(-1, order="F").copy())
            b = oracle.bf16_bits(b_mat.reshape(-1, order="F").copy())
            av = oracle.bf16_value(a).reshape(a_mat.shape, order="F").astype(np.float64)
            bv = oracle.bf16_value(b).reshape(b_mat.shape, order="F").astype(np.float64)
            want = (av.T if ta else av) @ (bv.T if tb else bv)
            exact, magnitude = oracle.matmul_exact(a, b, None, ta, tb, m, n, k,
                                                   a_mat.shape[0], b_mat.shape[0], m)
            assert np.allclose(exact.reshape((m, n), order="F"), want, rtol=0, atol=1e-12)
            assert np.all(magnitude >= np.abs(exact) - 1e-12)


def test_tuning_bucket():
    assert [TuningBucket(v) for v in (0, 1, 128, 129, 300)] == [0, 128, 128, 256, 384]


def test_matmul_rejects_bad_shapes():
    """Argument checks happen before any launch (no device needed)."""
    lib = _lib.load()
    bad = [
        shape_of(False, False, 64, 8, 32, 63, 32, 64),      # lda < m
        shape_of(True, False, 64, 8, 32, 31, 32, 64),       # transposed A: lda < k
        shape_of(False, True, 64, 8, 32, 64, 7, 64),        # transposed B: ldb < n
        shape_of(False, False, 64, 8, 32, 64, 32, 60),      # ldc < m
        shape_of(False, False, 64, 8, 32, 64, 32, 64, batch=70000),
        shape_of(False, False, 1 << 31, 8, 32, 1 << 31, 32, 1 << 31),
    ]
    for shape in bad:
        assert lib.vx_matmul(ctypes.byref(shape), None, None, None, None, None) == _lib.VX_INVALID
        assert lib.vx_last_error()
    assert lib.vx_matmul(None, None, None, None, None, None) == _lib.VX_INVALID
    # Nothing to compute: no launch, no operands read.
    empty = shape_of(False, False, 0, 8, 32, 1, 32, 1)
    assert lib.vx_matmul(ctypes.byref(empty), None, None, None, None, None) == _lib.VX_OK


CASES = [
    # (ta, tb, m, n, k, pads, batch)
    (False, False, 200, 72, 300, (3, 1, 5), 1),
    (True, False, 130, 64, 96, (0, 2, 0), 2),    # ldb not a multiple of 8: general kernel
    (True, False, 200, 72, 296, (8, 0, 5), 2),   # reduction-contiguous kernel, ragged tiles
    (True, False, 257, 300, 1024, (0, 0, 3), 1),  # reduction-contiguous kernel, several tiles
    (False, True, 64, 129, 33, (1, 0, 2), 3),
    (True, True, 77, 50, 1024, (4, 4, 4), 1),
    (True, False, 1, 1, 1, (0, 0, 0), 1),
    (False, False, 33, 17, 0, (0, 1, 0), 1),  # k = 0: C = beta C
]


@pytest.mark.gpu
@pytest.mark.parametrize("ta,tb,m,n,k,pads,batch", CASES)
def test_matmul_against_oracle(cuda, ta, tb, m, n, k, pads, batch):
    rng = np.random.default_rng(m * 1000 + n + k)
    lda = (k if ta else m) + pads[0]
    ldb = (n if tb else k) + pads[1]
    ldc = m + pads[2]
    cols_a, cols_b = (m if ta else k), (k if tb else n)
    # Batch gaps of 8 elements keep the reduction-contiguous layout's 16-byte
    # alignment; odd gaps elsewhere.
    gap = 8 if (ta and not tb) else 3
    sa, sb, sc = lda * cols_a + gap, ldb * cols_b + gap, ldc * n + 7
    a = oracle.bf16_bits(rng.normal(0, 1, size=max(1, sa * batch)).astype(np.float32))
    b = oracle.bf16_bits(rng.normal(0, 1, size=max(1, sb * batch)).astype(np.float32))
    c0 = rng.normal(0, 1, size=sc * batch).astype(np.float32)
    a_dev = torch.from_numpy(a.view(np.int16)).cuda()
    b_dev = torch.from_numpy(b.view(np.int16)).cuda()
    gemm = Bf16Gemm()
    for accumulate in (False, True):
        shape = shape_of(ta, tb, m, n, k, lda, ldb, ldc, sa, sb, sc, batch, accumulate)
        rep = shape_of(ta, tb, m, TuningBucket(n), k, lda, ldb, ldc, sa, sb, sc, batch, accumulate)
        c_dev = torch.from_numpy(c0.copy()).cuda()
        gemm.Matmul(shape, rep, a_dev, b_dev, c_dev)
        torch.cuda.synchronize()
        c = c_dev.cpu().numpy()
        exact, magnitude = oracle.matmul_exact(a, b, c0 if accumulate else None, ta, tb, m, n, k,
                                               lda, ldb, ldc, sa, sb, sc, batch)
        exact, magnitude = padded(exact, c.size), padded(magnitude, c.size)
        inside = ~np.isnan(exact)
        err = oracle.relative_error(c[inside], exact[inside], magnitude[inside])
        assert err <= LIMIT, f"accumulate {accumulate}: {err:.3e}"
        assert np.array_equal(c[~inside], c0[~inside]), "entries outside the product changed"
    gemm.close()


@pytest.mark.gpu
def test_matmul_as_linear_rows(cuda):
    """The reference's LinearRows shape (gemm.cpp:324-335): y[rows][out] =
    x W^T as C = W^T x^T in column-major form (transpose_a, m = out, n = rows,
    k = in), here at 256 rows, against the exact product and against
    Bf16Gemm::Linear over bf16 rows."""
    from voxcpm_b200 import kernels as K
    from voxcpm_b200.gemm import Matrix

    rng = np.random.default_rng(11)
    rows, columns, out = 256, 2048, 1024
    w = oracle.bf16_bits(rng.normal(0, 0.02, size=(out, columns)).astype(np.float32))
    x = oracle.bf16_bits(rng.normal(0, 1, size=(rows, columns)).astype(np.float32))
    w_dev = torch.from_numpy(w.view(np.int16)).cuda()
    x_dev = torch.from_numpy(x.view(np.int16)).cuda()
    shape = shape_of(True, False, out, rows, columns, columns, columns, out)
    y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    gemm = Bf16Gemm()
    gemm.Matmul(shape, None, w_dev, x_dev, y)
    y_linear = torch.empty_like(y)
    gemm.Linear(x_dev, Matrix(_lib.WEIGHTS_BF16, w_dev), y_linear, rows, columns, out, False)
    torch.cuda.synchronize()
    exact, magnitude = oracle.product_exact(x, oracle.BF16_ROWS, w.reshape(-1), rows, columns, out)
    assert oracle.relative_error(y.cpu().numpy(), exact, magnitude) <= LIMIT
    assert oracle.relative_error(y_linear.cpu().numpy(), exact, magnitude) <= LIMIT
    assert K.DeviceError() == 0
    gemm.close()
