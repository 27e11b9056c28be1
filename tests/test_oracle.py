"""The CPU oracle pinned against golden vectors and the reference's own test
oracle (no GPU needed).

Golden vectors (tests/golden/torch_numerics.json, made by make_golden.py)
hold torch's float32 results for the weight-free pieces the reference
restates from OpenBMB's PyTorch code. The products oracle is checked the way
tests/products_test.cpp checks the device: the float32 transcription against
the double-precision sum, limit 1e-5 of sum |x w|.
"""

import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = json.loads((Path(__file__).parent / "golden" / "torch_numerics.json").read_text())


def f32(hexes):
    return np.array([int(v, 16) for v in hexes], dtype=np.uint32).view(np.float32)


def u16(hexes):
    return np.array([int(v, 16) for v in hexes], dtype=np.uint16)


def ulps(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    return np.abs(ai - bi)


def test_bf16_rounding_matches_torch():
    """kernels/device_math.hpp:12-19 (RNE, quiet NaN) == torch's conversion."""
    x = f32(GOLDEN["bf16"]["x"])
    assert np.array_equal(oracle.bf16_bits(x), u16(GOLDEN["bf16"]["bits"]))


def test_bf16_nan_stays_quiet():
    nan = np.array([0x7F800001, 0xFF800001, 0x7FC00000], dtype=np.uint32).view(np.float32)
    bits = oracle.bf16_bits(nan)
    assert all((b & 0x7F80) == 0x7F80 and (b & 0x7F) != 0 and (b & 0x40) for b in bits)


def test_half_decode_matches_ieee():
    for b, v in zip(u16(GOLDEN["half"]["bits"]), f32(GOLDEN["half"]["value"])):
        assert np.float32(oracle.half_value(int(b))).view(np.uint32) == v.view(np.uint32)


def test_half_encode_round_to_nearest_even():
    rng = np.random.default_rng(0)
    values = np.concatenate([
        np.abs(rng.normal(0, 0.02, 20000) / 127),  # the weight-scale distribution
        rng.normal(0, 1, 2000), np.array([6.1e-5, 5.96e-8, 2.98e-8, 65504.0, 65519.0, 0.0]),
    ]).astype(np.float32)
    for v in values:
        assert oracle.half_bits(float(v)) == int(np.float16(v).view(np.uint16)), v


def test_linspace_matches_torch_within_one_ulp():
    """generator.cpp:21-37 restates torch.linspace with a separate multiply
    and add; torch's CPU kernel fuses them, so single values may differ by
    one unit in the last place."""
    for n, hexes in GOLDEN["linspace"].items():
        diff = ulps(oracle.linspace(1.0, 0.0, int(n)), f32(hexes))
        assert int(diff.max()) <= 1, n
    # Exactly equal at the sizes the sampler uses (10 steps -> 11 points).
    assert np.array_equal(oracle.linspace(1.0, 0.0, 11), f32(GOLDEN["linspace"]["11"]))


def test_euler_schedule():
    """generator.cpp:63-80: 10 steps, the first skipped (CFG-Zero*), times on
    the sway-sampled span."""
    t, dt, evaluate = oracle.euler_schedule(10)
    assert len(t) == 10
    assert list(evaluate) == [False] + [True] * 9
    span = f32(GOLDEN["sway_span"]["10"])
    assert int(ulps(t, span[:-1]).max()) <= 1
    np.testing.assert_allclose(t[:1] - dt[:1], span[1:2], rtol=0, atol=1e-7)
    assert abs(float(np.sum(dt)) - 1.0) < 1e-5
    expect = [1, .9564, .9090, .8540, .7878, .7071, .6090, .4910, .3511, .1877]
    np.testing.assert_allclose(t, expect, atol=6e-5)
    # max(1, int(0.04 * (n + 1))) steps skipped.
    for n, skipped in ((10, 1), (24, 1), (25, 1), (50, 2), (100, 4)):
        _, _, ev = oracle.euler_schedule(n)
        assert int((~ev).sum()) == skipped, n


def test_fsq_matches_torch():
    """kernels/generator_kernels.hip:291-297: round half to even like
    torch.round."""
    x = f32(GOLDEN["fsq"]["x"])
    out = np.empty(x.size, np.uint16)
    oracle.lib().vxo_quantize(x.ctypes.data, out.ctypes.data, x.size, 9.0)
    expect = u16(GOLDEN["fsq"]["bits"])
    # tanhf vs torch.tanh may differ by an ulp; a flipped rounding would move a
    # value by 1/9.
    vals = oracle.bf16_value(out)
    ref = oracle.bf16_value(expect)
    assert float(np.max(np.abs(vals - ref))) == 0.0


def test_sinusoid_matches_torch():
    for t, hexes in GOLDEN["sinusoid"].items():
        ours = oracle.sinusoid(float(t), 1024)
        ref = f32(hexes)
        # float32 angles up to 1000: sin/cos of the same float angle agree to
        # a few ulps of the angle's rounding.
        np.testing.assert_allclose(ours, ref, rtol=0, atol=2e-4)


def test_rope_table_matches_torch():
    g = GOLDEN["rope"]
    table = np.empty(g["positions"] * g["dim"], np.float32)
    factors = np.array(g["factors"], np.float64)
    oracle.lib().vxo_rope_table(g["theta"], g["dim"], factors.ctypes.data, 1.0, g["positions"],
                                table.ctypes.data)
    np.testing.assert_allclose(table, f32(g["table"]), rtol=0, atol=2e-6)


def make_q8(out, columns, rng):
    blocks = out * columns // 32
    raw = np.empty((blocks, 34), dtype=np.uint8)
    bits = rng.integers(0x1000, 0x1C01, size=blocks).astype(np.uint16)
    raw[:, 0] = bits & 0xFF
    raw[:, 1] = bits >> 8
    raw[:, 2:] = rng.integers(-128, 128, size=(blocks, 32)).astype(np.int8).view(np.uint8)
    return raw.reshape(-1)


@pytest.mark.parametrize("columns,out,rows", [(1024, 72, 22), (2048, 256, 5), (64, 128, 4)])
def test_fp32_product_within_reference_limit(columns, out, rows):
    """The float32 transcription of the products meets the reference test's
    limit against its double oracle (products_test.cpp:115-145, 1e-5)."""
    rng = np.random.default_rng(1234)
    blocks = make_q8(out, columns, rng)
    x = oracle.bf16_bits(rng.normal(0, 2, (rows, columns)).astype(np.float32))
    before = rng.normal(0, 1, (rows, out)).astype(np.float32)
    for accumulate in (False, True):
        y = before.copy() if accumulate else None
        y = oracle.linear(x, oracle.Q8_0, blocks, rows, columns, out, y=y, accumulate=accumulate)
        exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out,
                                     before if accumulate else None)
        assert oracle.relative_error(y, *exact) <= 1e-5
    w = oracle.bf16_bits(oracle.q8_0_dequant(blocks, out, columns).astype(np.float32))
    y = oracle.linear(x, oracle.BF16_ROWS, w, rows, columns, out)
    exact = oracle.product_exact(x, oracle.BF16_ROWS, w, rows, columns, out)
    assert oracle.relative_error(y, *exact) <= 1e-5


def test_error_metric_detects_a_planted_mistake():
    """A one-weight change in the oracle's product shows up in the metric."""
    rng = np.random.default_rng(9)
    rows, columns, out = 3, 256, 32
    blocks = make_q8(out, columns, rng)
    x = oracle.bf16_bits(rng.normal(0, 2, (rows, columns)).astype(np.float32))
    exact = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
    planted = blocks.copy()
    planted[2 + 5] ^= 0x10  # one int8 value of the first block
    y = oracle.linear(x, oracle.Q8_0, planted, rows, columns, out)
    assert oracle.relative_error(y, *exact) > 10 * 1e-5


def test_seeded_weights_reproduce():
    a = oracle.random_q8_0(7, 3, 48, 256)
    b = oracle.random_q8_0(7, 3, 48, 256)
    c = oracle.random_q8_0(8, 3, 48, 256)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    q = a.reshape(-1, 34)[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    scales = np.array([oracle.half_value(int(lo) | int(hi) << 8) for lo, hi in a.reshape(-1, 34)[:, :2]])
    # |N(0, 0.02)| / 127: mean 0.02 / 127 * sqrt(2 / pi)
    assert abs(scales.mean() / (0.02 / 127 * math.sqrt(2 / math.pi)) - 1) < 0.1
