"""The spread product (one wave of CTAs over the (panel, block) units, cut
panels added in part order through split scratch) against the CPU oracle,
on a B200, through the C ABI.

The same operands, shapes, row counts and metric as tests/test_products.py
(the reference's tests/products_test.cpp:59-145: max |y - exact| / sum |x w|
per output, limit 1e-5), on all three weight formats, plain and
accumulating; plus what the split scratch promises: counters left at zero,
results independent of launch order and repeatable bit for bit.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K
from voxcpm_b200.gemm import Bf16Gemm, Matrix

from test_products import SHAPES, make_activations, prepare, from_dev_u16, to_dev

pytestmark = pytest.mark.gpu

LIMIT = 1e-5

FORMATS = ("q8", "bf16 tiles")


def spread_plan(fmt, rows, columns, out):
    plan = K.PlanSpread(fmt, rows, columns, out)
    return plan if plan.splits > 0 else None


@pytest.mark.parametrize("columns,out,row_counts", SHAPES)
def test_spread_shape(cuda, columns, out, row_counts):
    rng = np.random.default_rng(4321 + columns * 7 + out)
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    host_dequant = from_dev_u16(dequant)
    served = 0
    for rows in row_counts:
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        for accumulate in (False, True):
            for name, fn, fmt, weights, ref_fmt, ref_w in (
                ("q8", K.WmmaQ8, _lib.WEIGHTS_Q8_TILES, q8_tiles, oracle.Q8_0, blocks),
                ("bf16 tiles", K.WmmaBf16, _lib.WEIGHTS_BF16_TILES, bf16_tiles, oracle.BF16_ROWS,
                 host_dequant),
            ):
                plan = spread_plan(fmt, rows, columns, out)
                if plan is None:
                    continue
                served += 1
                assert plan.variant == _lib.SPREAD_VARIANT
                scratch = K.SpreadScratch(plan)
                exact = oracle.product_exact(x, ref_fmt, ref_w, rows, columns, out,
                                             before if accumulate else None)
                y.copy_(torch.from_numpy(before))
                assert fn(x_dev, weights, y, rows, columns, out, accumulate, plan, scratch), name
                torch.cuda.synchronize()
                err = oracle.relative_error(y.cpu().numpy(), *exact)
                assert err <= LIMIT, f"{name} rows {rows} acc {accumulate}: {err:.3e}"
                assert int(scratch.counters.abs().sum()) == 0, "counters not left at zero"
    assert K.DeviceError() == 0
    # Every shape with at least one panel per CTA's run is served.
    assert served > 0 or out * columns < 128 * 32 * 4


@pytest.fixture
def spread_on():
    lib = _lib.load()
    before = lib.vx_spread_products()
    lib.vx_set_spread_products(1)
    yield
    lib.vx_set_spread_products(before)


def test_spread_rows_through_linear(cuda, spread_on):
    """With the switch on, bf16 rows (SkinnyGemm's format) take the spread
    kernel through Bf16Gemm::Linear's own scratch; the result matches the
    oracle."""
    rng = np.random.default_rng(77)
    gemm = Bf16Gemm()
    for columns, out in ((1024, 2560), (2048, 6144), (6144, 2048), (2048, 2)):
        _, _, dequant, _ = prepare(out, columns, rng)
        host_dequant = from_dev_u16(dequant)
        for rows in (1, 5, 22, 32):
            x = make_activations(rows, columns, rng)
            x_dev = to_dev(x)
            before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
            for accumulate in (False, True):
                exact = oracle.product_exact(x, oracle.BF16_ROWS, host_dequant, rows, columns, out,
                                             before if accumulate else None)
                y = torch.from_numpy(before).cuda()
                gemm.Linear(x_dev, Matrix(_lib.WEIGHTS_BF16, dequant), y, rows, columns, out, accumulate)
                torch.cuda.synchronize()
                err = oracle.relative_error(y.cpu().numpy(), *exact)
                assert err <= LIMIT, f"rows {rows} {columns}->{out} acc {accumulate}: {err:.3e}"
    gemm.close()
    assert K.DeviceError() == 0


def test_spread_config0_bf16_output_and_repeat(cuda, spread_on):
    """Config 0 through Linear with the bf16 epilogue: bf16 of the fp32
    spread sums, bit for bit; repeated launches (each resetting the counters
    for the next) give the same bits; the cluster plan agrees within the
    limit."""
    rng = np.random.default_rng(2024)
    rows, columns, out = 22, 2048, 6144
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng, std=1.0)
    x_dev = to_dev(x)
    gemm = Bf16Gemm()
    w = Matrix(_lib.WEIGHTS_Q8_TILES, q8_tiles)
    y32 = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    gemm.Linear(x_dev, w, y32, rows, columns, out, False)
    firsts = []
    for _ in range(3):
        y16 = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
        gemm.LinearEx(x_dev, w, y16, rows, columns, out)
        firsts.append(y16)
    torch.cuda.synchronize()
    expect = oracle.bf16_bits(y32.cpu().numpy())
    for y16 in firsts:
        assert np.array_equal(y16.cpu().view(torch.int16).numpy().view(np.uint16), expect)
    exact, mag = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    assert oracle.relative_error(y32.cpu().numpy(), exact, mag) <= LIMIT
    # The same product on the cluster plan (no scratch): within the limit.
    y_cluster = torch.empty_like(y32)
    assert K.WmmaQ8(x_dev, q8_tiles, y_cluster, rows, columns, out, False)
    torch.cuda.synchronize()
    assert oracle.relative_error(y_cluster.cpu().numpy(), exact, mag) <= LIMIT
    gemm.close()
    assert K.DeviceError() == 0


def test_spread_chain_in_graph(cuda, spread_on):
    """A dependent chain of spread products on rotating weights, captured
    in a CUDA graph and replayed (the benchmark's form): every output is
    the same as an eager launch of that product."""
    rng = np.random.default_rng(5)
    rows, columns, out = 22, 2048, 6144
    copies = []
    for c in range(3):
        _, q8_tiles, _, _ = prepare(out, columns, rng)
        copies.append(q8_tiles)
    x = make_activations(rows, columns, rng, std=1.0)
    x_dev = to_dev(x)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        gemm = Bf16Gemm(stream)
        eager = []
        for c in range(3):
            y = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
            gemm.LinearEx(x_dev, Matrix(_lib.WEIGHTS_Q8_TILES, copies[c]), y, rows, columns, out)
            eager.append(y)
        stream.synchronize()
        ys = [torch.empty(rows, out, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(9):
                gemm.LinearEx(x_dev, Matrix(_lib.WEIGHTS_Q8_TILES, copies[i % 3]), ys[i % 3], rows,
                              columns, out)
        for _ in range(3):
            g.replay()
        stream.synchronize()
    for c in range(3):
        assert torch.equal(ys[c], eager[c])
    del g
    gemm.close()
    assert K.DeviceError() == 0


def test_spread_plan_needs_scratch(cuda):
    """A spread plan without scratch, or with too little, is refused with
    nothing launched."""
    rows, columns, out = 22, 2048, 6144
    plan = K.PlanSpread(_lib.WEIGHTS_Q8_TILES, rows, columns, out)
    x = torch.zeros(rows * columns, dtype=torch.int16, device="cuda")
    w = torch.zeros(K.Q8TilesBytes(out, columns), dtype=torch.uint8, device="cuda")
    y = torch.zeros(rows * out, dtype=torch.float32, device="cuda")
    lib = _lib.load()
    import ctypes

    status = lib.vx_wmma_q8(x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, columns, out, 0,
                            ctypes.byref(plan), None, None)
    assert status == _lib.VX_INVALID
    small = _lib.SplitScratch(y.data_ptr(), 16, y.data_ptr(), 1)
    status = lib.vx_wmma_q8(x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, columns, out, 0,
                            ctypes.byref(plan), ctypes.byref(small), None)
    assert status == _lib.VX_INVALID
