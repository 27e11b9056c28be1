"""vx_product_host and vx_stage on a B200: products whose activations and
output live in page-locked host memory, and the SM-driven staging copies
they use instead of the copy engines.

The staged product must equal the device product bit for bit (same plan,
same sums; only where x and y travel differs), and through it the oracle's
double-precision sum within the products' limit, 1e-5 of sum |x w|
(products_test.cpp:229-237). Staging must move exactly the bytes asked, for
every piece width the kernel picks (16, 4 and 1 bytes), and nothing around
them.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K

from test_products import LIMIT, make_activations, prepare, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "nbytes,src_off,dst_off",
    [
        (270336, 0, 0),  # config 0's bf16 output: 16-byte pieces
        (90112, 0, 0),  # config 0's activations
        (4100, 4, 8),  # 4-byte pieces
        (1001, 1, 3),  # single bytes
        (16, 0, 0),
        (0, 0, 0),
    ],
)
def test_stage_round_trip(cuda, nbytes, src_off, dst_off):
    rng = np.random.default_rng(nbytes + 7 * src_off + dst_off)
    pad = 64
    host = torch.from_numpy(rng.integers(1, 256, size=nbytes + pad, dtype=np.uint8)).pin_memory()
    dev = torch.zeros(nbytes + pad, dtype=torch.uint8, device="cuda")
    back = torch.zeros(nbytes + pad, dtype=torch.uint8).pin_memory()
    K.Stage(dev[dst_off:], host[src_off:], nbytes)
    K.Stage(back[src_off:], dev[dst_off:], nbytes)
    torch.cuda.synchronize()
    got = dev.cpu()
    assert torch.equal(got[dst_off:dst_off + nbytes], host[src_off:src_off + nbytes])
    assert int(torch.count_nonzero(got[:dst_off])) == 0
    assert int(torch.count_nonzero(got[dst_off + nbytes:])) == 0
    assert torch.equal(back[src_off:src_off + nbytes], host[src_off:src_off + nbytes])
    assert int(torch.count_nonzero(back[:src_off])) == 0
    assert int(torch.count_nonzero(back[src_off + nbytes:])) == 0


def _host_case(rows, columns, out, dtype, accumulate, seed):
    rng = np.random.default_rng(seed)
    blocks, q8_tiles, _, _ = prepare(out, columns, rng)
    x = make_activations(rows, columns, rng, std=1.0)
    x_host = torch.from_numpy(x.view(np.int16)).pin_memory()
    start = torch.from_numpy(rng.normal(0.0, 1.0, size=(rows, out)).astype(np.float32)).to(dtype)
    y_ref = start.cuda() if accumulate else torch.zeros(rows, out, dtype=dtype, device="cuda")
    y_dev = y_ref.clone()
    return blocks, q8_tiles, x, x_host, start, y_ref, y_dev


@pytest.mark.parametrize(
    "rows,columns,out,dtype,accumulate",
    [
        (22, 2048, 6144, torch.bfloat16, False),  # config 0
        (22, 2048, 6144, torch.float32, False),
        (1, 1024, 2560, torch.float32, True),
        (5, 2048, 72, torch.float32, False),  # output rows not a multiple of 16
        (88, 1024, 8192, torch.bfloat16, False),  # wide tcgen05 plan
    ],
)
def test_product_host_equals_device_product(cuda, rows, columns, out, dtype, accumulate):
    blocks, q8_tiles, x, x_host, start, y_ref, y_dev = _host_case(
        rows, columns, out, dtype, accumulate, 500 + rows + out)
    x_dev = torch.zeros(rows, columns, dtype=torch.int16, device="cuda")
    y_host = torch.zeros(rows, out, dtype=dtype).pin_memory()
    flags = _lib.PRODUCT_ACCUMULATE if accumulate else 0
    assert K.ProductHost(_lib.WEIGHTS_Q8_TILES, x_host, x_dev, q8_tiles, y_dev, y_host,
                         rows, columns, out, flags)
    assert K.Product(_lib.WEIGHTS_Q8_TILES, to_dev(x), q8_tiles, y_ref, rows, columns, out,
                     accumulate=accumulate)
    torch.cuda.synchronize()
    assert torch.equal(x_dev.cpu(), x_host)
    assert torch.equal(y_dev.cpu(), y_ref.cpu())
    assert torch.equal(y_host, y_ref.cpu())
    if dtype == torch.float32:
        exact, mag = oracle.product_exact(x, oracle.Q8_0, blocks, rows, columns, out)
        if accumulate:
            exact = exact + start.numpy()
        err = np.abs(y_host.numpy() - exact) / np.maximum(mag, 1e-30)
        assert float(err.max()) <= LIMIT
    assert K.DeviceError() == 0


def test_product_host_in_graph(cuda):
    """The bench's end-to-end step: calls captured in a CUDA graph move
    fresh host activations in and the result out on every replay."""
    rows, columns, out = 22, 2048, 6144
    blocks, q8_tiles, x, x_host, _, y_ref, y_dev = _host_case(
        rows, columns, out, torch.bfloat16, False, 77)
    x_dev = torch.zeros(rows, columns, dtype=torch.int16, device="cuda")
    y_host = torch.zeros(rows, out, dtype=torch.bfloat16).pin_memory()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        assert K.ProductHost(_lib.WEIGHTS_Q8_TILES, x_host, x_dev, q8_tiles, y_dev, y_host,
                             rows, columns, out, stream=side)
        side.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            assert K.ProductHost(_lib.WEIGHTS_Q8_TILES, x_host, x_dev, q8_tiles, y_dev, y_host,
                                 rows, columns, out, stream=side)
    torch.cuda.synchronize()
    rng = np.random.default_rng(78)
    for _ in range(2):
        x2 = make_activations(rows, columns, rng, std=1.0)
        x_host.copy_(torch.from_numpy(x2.view(np.int16)))
        y_host.zero_()
        with torch.cuda.stream(side):
            graph.replay()
        side.synchronize()
        assert K.Product(_lib.WEIGHTS_Q8_TILES, to_dev(x2), q8_tiles, y_ref, rows, columns, out)
        torch.cuda.synchronize()
        assert torch.equal(y_host, y_ref.cpu())
    del graph


def test_product_host_rejects(cuda):
    rows, columns, out = 2, 1024, 1024
    _, q8_tiles, _, x_host, _, _, y_dev = _host_case(rows, columns, out, torch.float32, False, 3)
    x_dev = torch.zeros(rows, columns, dtype=torch.int16, device="cuda")
    y_host = torch.zeros(rows, out, dtype=torch.float32).pin_memory()
    # The product reads what the staging launch wrote: never independent.
    with pytest.raises(RuntimeError):
        K.ProductHost(_lib.WEIGHTS_Q8_TILES, x_host, x_dev, q8_tiles, y_dev, y_host,
                      rows, columns, out, _lib.PRODUCT_INDEPENDENT)
    # Host sides must be page-locked.
    with pytest.raises(ValueError):
        K.ProductHost(_lib.WEIGHTS_Q8_TILES, x_host.clone(), x_dev, q8_tiles, y_dev, y_host,
                      rows, columns, out)
    with pytest.raises(ValueError):
        K.Stage(torch.zeros(16, dtype=torch.uint8), x_host, 16)
    with pytest.raises(ValueError):
        K.Stage(x_dev, x_host, x_host.numel() * 2 + 2)
