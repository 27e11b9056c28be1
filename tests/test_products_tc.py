"""The tensor-core (tcgen05) Q8_0 product against the CPU oracle, on a B200.

Same operands and metric as test_products.py (the reference's
tests/products_test.cpp: GGML Q8_0 blocks with q uniform in [-128, 127] and
fp16 scale bits in [0x1000, 0x1C00], bf16 x ~ N(0, 2); max |y - exact| /
sum |x w| <= 1e-5 against a double-precision sum). Covers every activation
row count the kernel takes (9..32, its three read-back widths), partial
128-row panels, odd block counts, one to eight cluster splits, plain and
accumulating products, fp32 and bf16 outputs, the independent-launch flag,
and bit-for-bit repeatability. Every call goes through the C ABI.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K

from test_products import LIMIT, make_activations, make_q8_blocks, to_dev

pytestmark = pytest.mark.gpu

TC = K.TENSOR_CORE_VARIANT


@pytest.fixture(autouse=True)
def tensor_core_planner(cuda):
    """The planner hands 9..32-row Q8_0 products to the tensor-core kernel
    for these tests (it is off by default)."""
    K.SetTensorCoreProducts(True)
    yield
    K.SetTensorCoreProducts(False)


def tiles_of(blocks, out, columns):
    t = torch.zeros(K.Q8TilesBytes(out, columns), dtype=torch.uint8, device="cuda")
    K.Q8_0ToTiles(to_dev(blocks), out, columns, t)
    return t


def run(x_dev, tiles, y, rows, columns, out, accumulate, plan, independent=False):
    flags = (_lib.PRODUCT_ACCUMULATE if accumulate else 0) | \
        (_lib.PRODUCT_INDEPENDENT if independent else 0)
    ok = K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, tiles, y, rows, columns, out, flags, plan)
    torch.cuda.synchronize()
    return ok


def tc_plan(rows, columns, out):
    plan = K.PlanWmma(rows, columns, out, 0)
    assert plan.variant == TC, f"rows {rows} ({columns}, {out}) planned variant {plan.variant}"
    return plan


# (in, out, rows): VoxCPM2's 22-row DiT products, the config-0 and config-1
# shapes, a partial last panel (out = 72: 5 of 8 groups; out = 1040: 65
# groups), an odd block count (in = 1056: 33 blocks).
CASES = [
    (2048, 6144, [9, 16, 17, 22, 24, 25, 32]),
    (1024, 2560, [11, 22]),
    (2048, 1024, [22]),
    (1024, 8192, [22]),
    (4096, 1024, [22, 32]),
    (6144, 2048, [22]),
    (1024, 3072, [22]),
    (2048, 2560, [22]),
    (1024, 72, [22]),
    (1056, 1040, [13, 22]),
]


@pytest.mark.parametrize("columns,out,row_counts", CASES)
def test_tensor_core_shape(cuda, columns, out, row_counts):
    rng = np.random.default_rng(4321 + columns * 3 + out)
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    worst = 0.0
    for rows in row_counts:
        plan = tc_plan(rows, columns, out)
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
    print(f"tensor core in {columns} out {out}: worst {worst:.3e}")


def test_tensor_core_splits(cuda):
    """One to eight cluster splits of the reduction, uneven last slices."""
    rng = np.random.default_rng(17)
    rows = 22
    for columns, out, splits_list in ((2048, 1024, (3, 4, 5, 8)), (512, 2048, (1, 2, 3)),
                                      (6144, 2048, (8,))):
        blocks = make_q8_blocks(out, columns, rng)
        tiles = tiles_of(blocks, out, columns)
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        k_blocks = columns // 32
        for splits in splits_list:
            bps = -(-k_blocks // splits)
            assert bps <= 24 and -(-k_blocks // bps) == splits
            plan = _lib.WmmaPlan(splits, bps, 0, 0, TC)
            y.fill_(float("nan"))
            assert run(x_dev, tiles, y, rows, columns, out, False, plan)
            err = oracle.relative_error(y.cpu().numpy(), *exact)
            assert err <= LIMIT, f"({columns}, {out}) splits {splits}: {err:.3e}"
    # A slice longer than 24 blocks is not taken.
    plan = _lib.WmmaPlan(2, 32, 0, 0, TC)
    assert not run(x_dev, tiles, y, rows, 2048, 1024, False, plan)
    assert K.DeviceError() == 0


def test_tensor_core_matches_mma_path(cuda):
    """Both kernels sum the same operands within the limit, bf16 output is
    one rounding of the fp32 sums, the independent flag changes nothing,
    and repeated launches agree bit for bit."""
    rng = np.random.default_rng(23)
    rows, columns, out = 22, 2048, 6144
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    x = make_activations(rows, columns, rng, std=1.0)
    x_dev = to_dev(x)
    exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    plan = tc_plan(rows, columns, out)
    y_tc = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    assert run(x_dev, tiles, y_tc, rows, columns, out, False, plan)
    K.SetTensorCoreProducts(False)
    try:
        mma_plan = K.PlanWmma(rows, columns, out, 0)
        assert mma_plan.variant != TC
        y_mma = torch.empty_like(y_tc)
        assert run(x_dev, tiles, y_mma, rows, columns, out, False, mma_plan)
    finally:
        K.SetTensorCoreProducts(True)
    assert K.TensorCoreProducts()
    for name, y in (("tcgen05", y_tc), ("mma.sync", y_mma)):
        err = oracle.relative_error(y.cpu().numpy(), *exact)
        assert err <= LIMIT, f"{name}: {err:.3e}"
    again = torch.empty_like(y_tc)
    assert run(x_dev, tiles, again, rows, columns, out, False, plan, independent=True)
    assert torch.equal(again, y_tc), "independent launch or repeat differs"
    y16 = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
    assert run(x_dev, tiles, y16, rows, columns, out, False, plan)
    got = y16.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, oracle.bf16_bits(y_tc.cpu().numpy()))
    # bf16 output, accumulating: bf16(bf16 y + fp32 sum).
    base = torch.randn(rows, out, device="cuda").to(torch.bfloat16)
    y16.copy_(base)
    assert run(x_dev, tiles, y16, rows, columns, out, True, plan)
    expect = oracle.bf16_bits(base.float().cpu().numpy() + y_tc.cpu().numpy())
    assert np.array_equal(y16.cpu().view(torch.int16).numpy().view(np.uint16), expect)
    assert K.DeviceError() == 0


def test_tensor_core_plan_for_bf16_weights(cuda):
    """A tensor-core plan passed with bf16 weights runs the mma.sync kernel
    for that format (the reference's PlanWmma serves both formats)."""
    rng = np.random.default_rng(31)
    rows, columns, out = 22, 1024, 2560
    blocks = make_q8_blocks(out, columns, rng)
    tiles = tiles_of(blocks, out, columns)
    dequant = torch.empty(out * columns, dtype=torch.int16, device="cuda")
    K.Q8TilesToBf16(tiles, out, columns, dequant)
    bf16_tiles = torch.zeros(K.Bf16TilesBytes(out, columns) // 2, dtype=torch.int16, device="cuda")
    K.Bf16ToTiles(dequant, out, columns, bf16_tiles)
    x = make_activations(rows, columns, rng)
    plan = tc_plan(rows, columns, out)
    y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    assert K.WmmaBf16(to_dev(x), bf16_tiles, y, rows, columns, out, False, plan)
    torch.cuda.synchronize()
    host = dequant.cpu().numpy().view(np.uint16)
    exact = oracle.product_exact(x, oracle.BF16_ROWS, host, rows, columns, out)
    assert oracle.relative_error(y.cpu().numpy(), *exact) <= LIMIT
