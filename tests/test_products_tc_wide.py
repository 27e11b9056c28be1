"""The tcgen05 product for 33..128 rows (products_tc_wide.cu) against the
CPU oracle, on a B200: the metric and operands of test_products.py (the
reference's tests/products_test.cpp: max |y - exact| / sum |x w| <= 1e-5
against a double-precision sum). Covers the three MMA widths (64, 96, 128
rows) and row counts just past each, the DiT's batched row counts (22 per
request), the config-1 shapes, partial 128-row panels, odd block counts and
slices that end inside a ring stage, one to eight cluster splits,
accumulating and bf16 outputs, the planner switch, and repeatability. Every
call goes through the C ABI.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K

from test_products import LIMIT, make_activations, make_q8_blocks, to_dev

pytestmark = pytest.mark.gpu

WIDE = K.TENSOR_CORE_WIDE_VARIANT


def tiles_of(blocks, out, columns):
    t = torch.zeros(K.Q8TilesBytes(out, columns), dtype=torch.uint8, device="cuda")
    K.Q8_0ToTiles(to_dev(blocks), out, columns, t)
    return t


def run(x_dev, tiles, y, rows, columns, out, accumulate=False, plan=None, independent=False):
    flags = (_lib.PRODUCT_ACCUMULATE if accumulate else 0) | \
        (_lib.PRODUCT_INDEPENDENT if independent else 0)
    ok = K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, tiles, y, rows, columns, out, flags, plan)
    torch.cuda.synchronize()
    return ok


def wide_plan(columns, splits):
    k_blocks = columns // 32
    bps = -(-k_blocks // splits)
    return _lib.WmmaPlan(-(-k_blocks // bps), bps, 0, 0, WIDE)


# (in, out, rows, splits)
CASES = [
    (1024, 2560, [33, 44, 64], 2),
    (1024, 2560, [65, 88, 96, 97, 110, 128], 2),
    (2048, 1024, [44, 88, 128], 4),
    (4096, 1024, [88, 128], 8),
    (1024, 8192, [88], 1),
    (2048, 6144, [64, 128], 2),
    (6144, 2048, [64, 128], 6),
    (1056, 1040, [40, 100], 3),   # 33 blocks, 65 tile groups (partial panel)
    (1024, 72, [50], 1),          # 5 of 8 groups in the only panel
    (320, 256, [128], 1),         # 10 blocks: a slice ending inside a stage
]


@pytest.mark.parametrize("columns,out,row_counts,splits", CASES)
def test_wide_shape(cuda, columns, out, row_counts, splits):
    rng = np.random.default_rng(7000 + columns + out)
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    plan = wide_plan(columns, splits)
    worst = 0.0
    for rows in row_counts:
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        for accumulate in (False, True):
            exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out,
                                         before if accumulate else None)
            y.copy_(torch.from_numpy(before))
            assert run(x_dev, tiles, y, rows, columns, out, accumulate, plan)
            err = oracle.relative_error(y.cpu().numpy(), *exact)
            worst = max(worst, err)
            assert err <= LIMIT, f"rows {rows} splits {plan.splits} acc {accumulate}: {err:.3e}"
    assert K.DeviceError() == 0
    print(f"wide in {columns} out {out}: worst {worst:.3e}")


def test_wide_splits_and_repeat(cuda):
    """One to eight splits give the same sums within the limit; a launch
    repeats bit for bit; the independent flag changes nothing; bf16 output is
    one rounding of the fp32 sums."""
    rng = np.random.default_rng(77)
    rows, columns, out = 88, 2048, 1024
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    x = make_activations(rows, columns, rng, std=1.0)
    x_dev = to_dev(x)
    exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    for splits in (1, 2, 3, 5, 8):
        y.fill_(float("nan"))
        plan = wide_plan(columns, splits)
        assert run(x_dev, tiles, y, rows, columns, out, plan=plan)
        err = oracle.relative_error(y.cpu().numpy(), *exact)
        assert err <= LIMIT, f"splits {splits}: {err:.3e}"
    plan = wide_plan(columns, 4)
    first = torch.empty_like(y)
    assert run(x_dev, tiles, first, rows, columns, out, plan=plan)
    again = torch.empty_like(y)
    assert run(x_dev, tiles, again, rows, columns, out, plan=plan, independent=True)
    assert torch.equal(first, again)
    y16 = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
    assert run(x_dev, tiles, y16, rows, columns, out, plan=plan)
    got = y16.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, oracle.bf16_bits(first.cpu().numpy()))
    assert K.DeviceError() == 0


@pytest.mark.parametrize("columns,out", [(1024, 8192), (1024, 3072), (4096, 1024)])
def test_wide_planner_switch(cuda, columns, out):
    """Products launched without a plan, with the switch on (default: the
    wide kernel where it pays, 65..128 rows of 1024 -> 3072 or more) and off
    (the mma.sync planner or 32-row launches), match the oracle either way."""
    rng = np.random.default_rng(5 + columns + out)
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    assert K.WideTensorCoreProducts()
    try:
        for enabled in (True, False):
            K.SetWideTensorCoreProducts(enabled)
            for rows in (32, 33, 88, 128):
                x = make_activations(rows, columns, rng)
                y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
                assert run(to_dev(x), tiles, y, rows, columns, out)
                exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
                assert oracle.relative_error(y.cpu().numpy(), *exact) <= LIMIT, (enabled, rows)
    finally:
        K.SetWideTensorCoreProducts(True)
    assert K.DeviceError() == 0
