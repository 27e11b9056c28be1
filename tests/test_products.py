"""The products and their weight tiles against the CPU oracle, on a B200.

Mirrors the reference's tests/products_test.cpp: random GGML Q8_0 blocks
(q uniform in [-128, 127], fp16 scale bits uniform in [0x1000, 0x1C00]) and
bf16 activations ~N(0, 2) at VoxCPM2's shapes and odd ones, every row count
the reference tests, plans of one, the planner's and many splits, plain and
accumulating products, compared with a double-precision sum of the same
operands. Metric: max |y - exact| / sum |x w| per output, limit 1e-5
(products_test.cpp:115-145, :229-237). Every call goes through the C ABI.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import kernels as K
from voxcpm_b200 import _lib
from voxcpm_b200.gemm import Bf16Gemm, Matrix

pytestmark = pytest.mark.gpu

LIMIT = 1e-5

ALL_ROWS = [1, 2, 4, 5, 8, 11, 16, 22, 32]
# products_test.cpp:326-338: VoxCPM2's shapes and odd ones.
SHAPES = [
    (64, 1024, [4, 8]),
    (512, 1024, [1, 4]),
    (1024, 2560, ALL_ROWS),
    (2048, 1024, [1, 5, 22]),
    (4096, 1024, [1, 5, 22]),
    (2048, 2048, [1, 5]),
    (6144, 2048, [1, 3]),
    (8192, 512, [1, 22]),
    (1024, 72, [3, 22]),  # rows not a multiple of 16
    (2048, 2, [1]),
]


def make_q8_blocks(out, columns, rng):
    """GGML Q8_0 blocks as products_test.cpp:59-84 draws them."""
    blocks = out * columns // 32
    raw = np.empty((blocks, 34), dtype=np.uint8)
    scale_bits = rng.integers(0x1000, 0x1C01, size=blocks).astype(np.uint16)
    raw[:, 0] = scale_bits & 0xFF
    raw[:, 1] = scale_bits >> 8
    raw[:, 2:] = rng.integers(-128, 128, size=(blocks, 32)).astype(np.int8).view(np.uint8)
    return raw.reshape(-1)


def make_activations(rows, columns, rng, std=2.0):
    return oracle.bf16_bits(rng.normal(0.0, std, size=(rows, columns)).astype(np.float32))


def to_dev(a: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    if t.dtype == torch.uint16:
        t = t.view(torch.int16)
    return t.cuda()


def from_dev_u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def prepare(out, columns, rng):
    blocks = make_q8_blocks(out, columns, rng)
    q8_tiles = torch.zeros(K.Q8TilesBytes(out, columns), dtype=torch.uint8, device="cuda")
    K.Q8_0ToTiles(to_dev(blocks), out, columns, q8_tiles)
    dequant = torch.empty(out * columns, dtype=torch.int16, device="cuda")
    K.Q8TilesToBf16(q8_tiles, out, columns, dequant)
    bf16_tiles = torch.zeros(K.Bf16TilesBytes(out, columns) // 2, dtype=torch.int16, device="cuda")
    K.Bf16ToTiles(dequant, out, columns, bf16_tiles)
    return blocks, q8_tiles, dequant, bf16_tiles


@pytest.mark.parametrize("columns,out,row_counts", SHAPES)
def test_shape(cuda, columns, out, row_counts):
    rng = np.random.default_rng(1234 + columns * 7 + out)
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    torch.cuda.synchronize()

    # The repack writes exactly the oracle's tiles (bit for bit).
    assert np.array_equal(q8_tiles.cpu().numpy(), oracle.q8_0_to_tiles(blocks, out, columns))
    # Exact dequantization: bf16(scale * q) (products_test.cpp:175-185).
    values = oracle.q8_0_dequant(blocks, out, columns)
    host_dequant = from_dev_u16(dequant)
    assert np.array_equal(host_dequant, oracle.bf16_bits(values.astype(np.float32).reshape(-1)))
    # bf16 tiles round trip (products_test.cpp:186-190).
    unpacked = torch.empty_like(dequant)
    K.Bf16TilesToRows(bf16_tiles, out, columns, unpacked)
    assert torch.equal(unpacked, dequant)
    assert np.array_equal(bf16_tiles.cpu().view(torch.int16).numpy().view(np.uint16),
                          oracle.bf16_to_tiles(host_dequant, out, columns))

    worst = {}
    for rows in row_counts:
        x = make_activations(rows, columns, rng)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        x_dev = to_dev(x)
        exact_q8 = {a: oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out,
                                            before if a else None) for a in (False, True)}
        exact_bf16 = {a: oracle.product_exact(x, oracle.BF16_ROWS, host_dequant, rows, columns, out,
                                              before if a else None) for a in (False, True)}
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        for accumulate in (False, True):
            for target in (1, 0, 4096):
                plan = K.PlanWmma(rows, columns, out, target)
                assert plan.splits > 0
                for name, fn, weights, exact in (
                    ("q8", K.WmmaQ8, q8_tiles, exact_q8[accumulate]),
                    ("bf16 tiles", K.WmmaBf16, bf16_tiles, exact_bf16[accumulate]),
                ):
                    y.copy_(torch.from_numpy(before))
                    assert fn(x_dev, weights, y, rows, columns, out, accumulate, plan), name
                    torch.cuda.synchronize()
                    err = oracle.relative_error(y.cpu().numpy(), *exact)
                    key = (name, rows, plan.splits, accumulate)
                    worst[key] = err
                    assert err <= LIMIT, f"{name} rows {rows} splits {plan.splits}: {err:.3e}"
            # bf16 rows (SkinnyGemm) on the dequantized weights.
            y.copy_(torch.from_numpy(before))
            assert K.SkinnyGemm(x_dev, dequant, y, rows, columns, out, accumulate)
            torch.cuda.synchronize()
            err = oracle.relative_error(y.cpu().numpy(), *exact_bf16[accumulate])
            assert err <= LIMIT, f"skinny rows {rows}: {err:.3e}"
    assert K.DeviceError() == 0
    print(f"in {columns} out {out}: worst {max(worst.values()):.3e}")


def test_every_variant(cuda):
    """Each kernel shape on each format gives the same sums (config-0 shape)."""
    rng = np.random.default_rng(7)
    rows, columns, out = 22, 2048, 6144
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng)
    x_dev = to_dev(x)
    exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    exact_rows = oracle.product_exact(x, oracle.BF16_ROWS, from_dev_u16(dequant), rows, columns, out)
    y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    ran = {fmt: 0 for fmt in (_lib.WEIGHTS_Q8_TILES, _lib.WEIGHTS_BF16_TILES, _lib.WEIGHTS_BF16)}
    for variant in range(len(K.ProductVariants())):
        for splits in (1, 2, 3, 4, 8):
            bps = -(-columns // 32 // splits)
            if -(-(columns // 32) // bps) != splits:
                continue
            plan = _lib.WmmaPlan(splits, bps, 0, 0, variant)
            for fmt, w, ex in ((_lib.WEIGHTS_Q8_TILES, q8_tiles, exact),
                               (_lib.WEIGHTS_BF16_TILES, bf16_tiles, exact_rows),
                               (_lib.WEIGHTS_BF16, dequant, exact_rows)):
                y.zero_()
                if not K.Product(fmt, x_dev, w, y, rows, columns, out, False, plan):
                    continue  # this shape's shared memory exceeds the kernels' limit
                ran[fmt] += 1
                torch.cuda.synchronize()
                err = oracle.relative_error(y.cpu().numpy(), *ex)
                assert err <= LIMIT, f"variant {variant} splits {splits} format {fmt}: {err:.3e}"
    assert all(count >= 8 for count in ran.values()), ran


def test_bf16_output(cuda):
    """The bf16-output epilogue: bf16(fp32 sum)."""
    rng = np.random.default_rng(11)
    rows, columns, out = 22, 2048, 6144
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng, std=1.0)
    x_dev = to_dev(x)
    y32 = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    y16 = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
    assert K.Product(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y32, rows, columns, out)
    assert K.Product(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y16, rows, columns, out)
    torch.cuda.synchronize()
    # Same fp32 sums, rounded once to bf16 (RNE): bit-equal to rounding y32.
    expect = oracle.bf16_bits(y32.cpu().numpy())
    got = y16.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, expect)
    exact, mag = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    # One bf16 rounding (half an ulp: at most 2^-8 of the value) on top of
    # the fp32 sum's error.
    err = np.abs(y16.float().cpu().numpy() - exact)
    assert bool(np.all(err <= 2.0 ** -8 * np.abs(exact) + LIMIT * mag))


def test_fp32_transcription_agrees(cuda):
    """The device sums agree with the oracle's fp32 per-block transcription
    (wmma_products.hip:201-214) to float32 summation-order noise."""
    rng = np.random.default_rng(5)
    rows, columns, out = 22, 1024, 2560
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng)
    y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    assert K.WmmaQ8(to_dev(x), q8_tiles, y, rows, columns, out, False)
    torch.cuda.synchronize()
    ref = oracle.linear(x, oracle.Q8_0, blocks, rows, columns, out)
    exact, mag = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    assert float(np.max(np.abs(y.cpu().numpy() - ref) / mag)) <= 2e-6


@pytest.mark.parametrize("columns,out", [(1024, 2560), (4096, 1024)])
def test_linear(cuda, columns, out):
    """Bf16Gemm::Linear on Q8 and bf16 tiles, chunks of 32 rows up to and
    beyond 128 (products_test.cpp:256-313)."""
    rng = np.random.default_rng(99 + columns)
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    host_dequant = from_dev_u16(dequant)
    gemm = Bf16Gemm()
    for rows in (1, 22, 40, 130):
        x = make_activations(rows, columns, rng)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        x_dev = to_dev(x)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        for accumulate in (False, True):
            for fmt, w, ref_fmt, ref_w in (
                (_lib.WEIGHTS_Q8_TILES, q8_tiles, oracle.Q8_0, blocks),
                (_lib.WEIGHTS_BF16_TILES, bf16_tiles, oracle.BF16_ROWS, host_dequant),
                (_lib.WEIGHTS_BF16, dequant, oracle.BF16_ROWS, host_dequant),
            ):
                y.copy_(torch.from_numpy(before))
                gemm.Linear(x_dev, Matrix(fmt, w), y, rows, columns, out, accumulate)
                torch.cuda.synchronize()
                exact = oracle.product_exact(x, ref_fmt, ref_w, rows, columns, out,
                                             before if accumulate else None)
                err = oracle.relative_error(y.cpu().numpy(), *exact)
                assert err <= LIMIT, f"linear fmt {fmt} rows {rows}: {err:.3e}"
    gemm.close()


def test_unsupported_shapes(cuda):
    """Launchers return False (nothing launched) for shapes they do not take."""
    x = torch.zeros(64 * 48, dtype=torch.int16, device="cuda")
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    y = torch.zeros(64 * 64, dtype=torch.float32, device="cuda")
    assert not K.WmmaQ8(x, w, y, 129, 32, 16, False)     # more than 128 rows
    assert not K.SkinnyGemm(x, x, y, 33, 32, 16, False)   # SkinnyGemm: at most 32 rows
    assert not K.WmmaQ8(x, w, y, 1, 48, 16, False)       # in not a multiple of 32
    assert not K.WmmaQ8(x, w, y, 0, 32, 16, False)       # no rows
    assert not K.SkinnyGemm(x, x, y, 1, 16384, 2, False)  # in > 8192


def test_independent_launch_stream_plan(cuda):
    """Independent launches with no plan take the library's measured stream
    plan (config 0: one 384-row CTA per panel over the whole reduction) and
    give the same sums as the planner's dependent plan."""
    rng = np.random.default_rng(41)
    rows, columns, out = 22, 2048, 6144
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng)
    x_dev = to_dev(x)
    exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    y_stream = torch.empty(rows, out, dtype=torch.float32, device="cuda")
    y_chain = torch.empty_like(y_stream)
    assert K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y_stream, rows, columns, out,
                       _lib.PRODUCT_INDEPENDENT)
    assert K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y_chain, rows, columns, out, 0)
    torch.cuda.synchronize()
    for name, y in (("stream plan", y_stream), ("planner", y_chain)):
        err = oracle.relative_error(y.cpu().numpy(), *exact)
        assert err <= LIMIT, f"{name}: {err:.3e}"
    assert K.DeviceError() == 0


@pytest.mark.parametrize("rows,splits", [(1, 1), (5, 1), (22, 1), (22, 4), (32, 2)])
def test_half_tile_math_bit_equal(cuda, rows, splits):
    """Variant 14 (fp16 tile math over activations scaled by a power of two
    per row) gives variant 13's bf16 sums bit for bit, at row scales from
    1e-30 to 1e30 and with a zero row; and the oracle's sums within the
    limit. (Rows whose fp32 sums overflow may differ: an overflow inside
    one bf16 MMA can give NaN where the scaled sum overflows only when
    unscaled, to inf.)"""
    rng = np.random.default_rng(59 + rows)
    columns, out = 2048, 6144
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    base = rng.normal(0.0, 1.0, size=(rows, columns)).astype(np.float32)
    scales = np.array([1.0, 3e4, 1e-30, 0.0, 1e-3, 1e-20, 1.0, 1e30] * 4)[:rows]
    x = (base * scales[:, None]).astype(np.float32)
    x_bits = oracle.bf16_bits(x)
    x_dev = to_dev(x_bits)
    ys = {}
    for variant in (13, 14):
        # Split slices scale their own activations and unscale before the
        # cluster adds them up.
        plan = _lib.WmmaPlan(splits, columns // 32 // splits, 0, 0, variant)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        assert K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y, rows, columns, out, 0,
                           plan=plan)
        ys[variant] = y
    torch.cuda.synchronize()
    assert torch.equal(ys[13], ys[14])
    exact, mag = oracle.product_exact(x_bits, oracle.Q8_0, blocks, rows, columns, out)
    err = np.abs(ys[14].cpu().numpy() - exact) / np.maximum(mag, 1e-300)
    assert float(err.max()) <= LIMIT
    assert K.DeviceError() == 0


@pytest.mark.parametrize("columns,out", [(1024, 2560), (2048, 1024), (4096, 1024), (6144, 512)])
def test_wide_rows(cuda, columns, out):
    """33..128 activation rows in one launch (8 or 16 B tiles per warp) on
    every weight format, plain and accumulating, fp32 and bf16 output; for a
    long reduction (6144) no one-launch plan fits and the launcher runs
    32-row launches."""
    rng = np.random.default_rng(53 + columns)
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    host_dequant = from_dev_u16(dequant)
    for rows in (33, 48, 64, 65, 100, 128):
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        for accumulate in (False, True):
            for fmt, w, ref_fmt, ref_w in (
                (_lib.WEIGHTS_Q8_TILES, q8_tiles, oracle.Q8_0, blocks),
                (_lib.WEIGHTS_BF16_TILES, bf16_tiles, oracle.BF16_ROWS, host_dequant),
                (_lib.WEIGHTS_BF16, dequant, oracle.BF16_ROWS, host_dequant),
            ):
                y.copy_(torch.from_numpy(before))
                assert K.Product(fmt, x_dev, w, y, rows, columns, out, accumulate), (fmt, rows)
                torch.cuda.synchronize()
                exact = oracle.product_exact(x, ref_fmt, ref_w, rows, columns, out,
                                             before if accumulate else None)
                err = oracle.relative_error(y.cpu().numpy(), *exact)
                assert err <= LIMIT, f"fmt {fmt} rows {rows} acc {accumulate}: {err:.3e}"
        y16 = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
        assert K.Product(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y16, rows, columns, out)
        y32 = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        assert K.Product(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y32, rows, columns, out)
        torch.cuda.synchronize()
        assert np.array_equal(y16.cpu().view(torch.int16).numpy().view(np.uint16),
                              oracle.bf16_bits(y32.cpu().numpy()))
    assert K.DeviceError() == 0


# Row-split variants: (CTA groups, ways, groups per warp, stage, depth, row split).
ROW_SPLIT_VARIANTS = {25: (4, 2, 1, 4, 2, 2), 26: (4, 1, 1, 4, 4, 2), 27: (2, 2, 1, 4, 2, 2),
                      28: (4, 2, 1, 4, 2, 4), 29: (2, 2, 1, 4, 2, 4), 30: (8, 1, 1, 4, 2, 2),
                      31: (2, 1, 1, 4, 4, 4), 32: (1, 2, 1, 4, 2, 4), 33: (2, 4, 1, 4, 2, 2),
                      34: (2, 2, 1, 8, 2, 2), 35: (1, 4, 1, 4, 2, 4)}


def q8_footprint(shape, ntiles, blocks_per_split):
    """Shared memory of a Q8_0 launch (the launcher's FootprintOf)."""
    groups, ways, per_warp, stage, depth, split = shape
    align = lambda v: (v + 127) // 128 * 128
    row = blocks_per_split * 64
    x_stride = row if row % 128 == 64 else align(row) + 64
    warps = groups // per_warp * ways * split
    rings = warps * depth * per_warp * stage * 576
    reduction = ways * groups * ntiles * 32 * 16
    return align(ntiles * 8 * x_stride) + align(max(rings, reduction)) + (warps * depth + 1) * 8


def test_row_split_variants(cuda):
    """Variants whose warps split a group's activation tiles (two or four
    warps per group and way, 33..128 rows) against the double-precision
    oracle: every format, plain and accumulating, one and several splits
    (cluster reduction), a partial last panel (2560 outputs); at most 32
    rows they are refused."""
    variants = K.ProductVariants()
    for v, shape in ROW_SPLIT_VARIANTS.items():
        warps, groups, stage, depth = variants[v]
        assert (groups, stage, depth) == (shape[0], shape[3], shape[4])
        assert warps == shape[0] // shape[2] * shape[1] * shape[5]
    rng = np.random.default_rng(71)
    columns, out = 1024, 2560
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    host_dequant = from_dev_u16(dequant)
    ran = {v: 0 for v in ROW_SPLIT_VARIANTS}
    for rows in (33, 64, 65, 128):
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        before = rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        ntiles = 8 if rows <= 64 else 16
        for variant, shape in ROW_SPLIT_VARIANTS.items():
            for splits in (1, 4, 8):
                bps = -(-(columns // 32) // splits)
                if q8_footprint(shape, ntiles, bps) > 220 * 1024:
                    continue  # the launcher would run its own plan instead
                ran[variant] += 1
                plan = _lib.WmmaPlan(splits, bps, 0, 0, variant)
                for accumulate in (False, True):
                    for fmt, w, ref_fmt, ref_w in (
                        (_lib.WEIGHTS_Q8_TILES, q8_tiles, oracle.Q8_0, blocks),
                        (_lib.WEIGHTS_BF16_TILES, bf16_tiles, oracle.BF16_ROWS, host_dequant),
                        (_lib.WEIGHTS_BF16, dequant, oracle.BF16_ROWS, host_dequant),
                    ):
                        y.copy_(torch.from_numpy(before))
                        assert K.Product(fmt, x_dev, w, y, rows, columns, out, accumulate, plan), \
                            (variant, splits, fmt, rows)
                        torch.cuda.synchronize()
                        exact = oracle.product_exact(x, ref_fmt, ref_w, rows, columns, out,
                                                     before if accumulate else None)
                        err = oracle.relative_error(y.cpu().numpy(), *exact)
                        assert err <= LIMIT, \
                            f"variant {variant} splits {splits} fmt {fmt} rows {rows} acc {accumulate}: {err:.3e}"
    assert all(count >= 4 for count in ran.values()), ran
    x = to_dev(make_activations(32, columns, rng))
    y = torch.empty(32, out, dtype=torch.float32, device="cuda")
    for variant in ROW_SPLIT_VARIANTS:
        plan = _lib.WmmaPlan(8, 4, 0, 0, variant)
        assert not K.Product(_lib.WEIGHTS_Q8_TILES, x, q8_tiles, y, 32, columns, out, False, plan)
    assert K.DeviceError() == 0


@pytest.mark.parametrize("rows", [1, 22])
def test_half_tile_math_wide_rows(cuda, rows):
    """Variant 14 on rows whose values span far more than 2^31: every
    element N(0, 1) * 2^e with e uniform in [-60, 0]. Values more than about
    2^32 below their row's largest fall below fp16's subnormal step once the
    row is scaled and are rounded there (variant 13 forms them exactly), so
    the bits may differ from variant 13; the sums stay within the products'
    limit of the double-precision result, since each such rounding moves a
    product by less than 2^-40 of the row's largest one."""
    rng = np.random.default_rng(71 + rows)
    columns, out = 2048, 2560
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = (rng.normal(0.0, 1.0, size=(rows, columns)) *
         np.exp2(rng.uniform(-60.0, 0.0, size=(rows, columns)))).astype(np.float32)
    x_bits = oracle.bf16_bits(x)
    x_dev = to_dev(x_bits)
    exact, mag = oracle.product_exact(x_bits, oracle.Q8_0, blocks, rows, columns, out)
    ys = {}
    for variant in (13, 14):
        plan = _lib.WmmaPlan(1, columns // 32, 0, 0, variant)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        assert K.ProductEx(_lib.WEIGHTS_Q8_TILES, x_dev, q8_tiles, y, rows, columns, out, 0, plan=plan)
        ys[variant] = y
    torch.cuda.synchronize()
    for variant, y in ys.items():
        err = oracle.relative_error(y.cpu().numpy(), exact, mag)
        assert err <= LIMIT, f"variant {variant}: {err:.3e}"
    differ = int((ys[13] != ys[14]).sum())
    print(f"rows {rows}: {differ} of {rows * out} sums differ from variant 13's bits")
    assert K.DeviceError() == 0


def test_global_activation_variants(cuda):
    """The variants that read activation fragments from global memory
    (22-24) at every row count of their tile classes (rows past `m` read as
    zeros), accumulating and not, against the exact sums."""
    rng = np.random.default_rng(23)
    columns, out = 1024, 640
    blocks, q8_tiles, dequant, bf16_tiles = prepare(out, columns, rng)
    for rows in (1, 5, 8, 9, 17, 22, 32):
        x = make_activations(rows, columns, rng)
        x_dev = to_dev(x)
        before = rng.normal(0, 1, (rows, out)).astype(np.float32)
        for accumulate in (False, True):
            exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out,
                                         before if accumulate else None)
            exact_rows = oracle.product_exact(x, oracle.BF16_ROWS, from_dev_u16(dequant), rows, columns, out,
                                              before if accumulate else None)
            for variant in (22, 23, 24):
                for splits in (1, 2):
                    plan = _lib.WmmaPlan(splits, columns // 32 // splits, 0, 0, variant)
                    for fmt, w, ex in ((_lib.WEIGHTS_Q8_TILES, q8_tiles, exact),
                                       (_lib.WEIGHTS_BF16_TILES, bf16_tiles, exact_rows),
                                       (_lib.WEIGHTS_BF16, dequant, exact_rows)):
                        y = torch.from_numpy(before).cuda() if accumulate else \
                            torch.zeros(rows, out, dtype=torch.float32, device="cuda")
                        assert K.Product(fmt, x_dev, w, y, rows, columns, out, accumulate, plan)
                        torch.cuda.synchronize()
                        err = oracle.relative_error(y.cpu().numpy(), *ex)
                        assert err <= LIMIT, f"rows {rows} variant {variant} splits {splits} format {fmt}"
    assert K.DeviceError() == 0


def test_dependent_chain_of_products(cuda):
    """A chain where every product reads the previous one's bf16 output, on
    one stream without synchronizing (the generator's pattern): programmatic
    launch lets each product start before the previous ends, and the
    config-0 shape's early CTAs prefetch the later CTAs' weights into L2
    while it runs. Every link matches the exact sum of its own inputs."""
    rng = np.random.default_rng(31)
    rows = 22
    up_blocks, up_tiles, up_dequant, _ = prepare(6144, 2048, rng)        # 2048 -> 6144
    down_blocks, down_tiles, down_dequant, _ = prepare(2048, 6144, rng)  # 6144 -> 2048
    gemm = Bf16Gemm()
    for fmt, up_w, down_w, up_ref, down_ref, ref_fmt in (
            (_lib.WEIGHTS_Q8_TILES, up_tiles, down_tiles, up_blocks, down_blocks, oracle.Q8_0),
            (_lib.WEIGHTS_BF16, up_dequant, down_dequant, from_dev_u16(up_dequant), from_dev_u16(down_dequant),
             oracle.BF16_ROWS)):
        x = to_dev(make_activations(rows, 2048, rng, std=1.0)).view(torch.bfloat16)
        links = []
        current = x
        for i in range(6):
            up = i % 2 == 0
            out, columns = (6144, 2048) if up else (2048, 6144)
            y = torch.empty(rows, out, dtype=torch.bfloat16, device="cuda")
            gemm.LinearEx(current, Matrix(fmt, up_w if up else down_w), y, rows, columns, out)
            links.append((current, y, up))
            current = y
        torch.cuda.synchronize()
        for i, (xi, yi, up) in enumerate(links):
            out, columns = (6144, 2048) if up else (2048, 6144)
            x_bits = xi.view(torch.int16).cpu().numpy().view(np.uint16)
            exact, magnitude = oracle.product_exact(x_bits, ref_fmt, up_ref if up else down_ref, rows, columns, out)
            y_f = yi.float().cpu().numpy().reshape(-1)
            # One bf16 rounding of the output on top of the fp32 sum's error
            # (as test_bf16_output bounds it).
            err = np.abs(y_f - exact.reshape(-1))
            bound = 2.0 ** -8 * np.abs(exact.reshape(-1)) + LIMIT * magnitude.reshape(-1)
            assert bool(np.all(err <= bound)), f"format {fmt} link {i}"
    assert K.DeviceError() == 0
    gemm.close()
