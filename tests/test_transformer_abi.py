"""transformer.hpp through the C ABI (vx_kv_cache_*, vx_forward_stack,
vx_project): a caller-built two-layer stack of the released encoder shape
(1024 wide, 16 heads / 2 KV heads of 128, SwiGLU 4096, seeded Q8_0
weights) against the oracle's ForwardStack (transformer.cpp:55-100): a
five-row causal prefill, then one decode row at position 5 over the cache
the prefill filled. Tolerance: relative L2 1e-2 on the residual stream, the
final norm and the cache rows, as the stack tests use for fp32 states."""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from oracle.model import Cache, OracleGenerator
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K
from voxcpm_b200.generator import small_config
from voxcpm_b200.transformer import (AttentionLayoutC, KvCache, LayerWeightsC, ProjectionC, Project,
                                     StackScratchElements, StackWeightsC, ForwardStack, StackScratchC)

LIMIT = 1e-2


def rel_l2(got, ref):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def test_transformer_entries_reject_bad_arguments():
    """Argument checks before any launch (no device needed)."""
    lib = _lib.load()
    c = small_config().encoder
    bad = _lib.StackConfig(c.hidden, c.intermediate, c.layers, c.heads, c.kv_heads, 64, c.rms_eps, 1)
    assert not lib.vx_kv_cache_create(ctypes.byref(bad), 16, _lib.CACHE_F32)
    assert lib.vx_last_error()
    counts = (ctypes.c_size_t * 6)()
    assert lib.vx_stack_scratch_elements(ctypes.byref(bad), 4, counts) == _lib.VX_INVALID
    assert lib.vx_forward_stack(None, None, None, None, None, None, 1, None, None) == _lib.VX_INVALID
    assert lib.vx_project(None, None, None, 1, None) == _lib.VX_INVALID
    assert StackScratchElements(c, 3) == [3 * c.hidden, 3 * (c.heads + 2 * c.kv_heads) * 128,
                                          3 * c.heads * 128, 3 * c.heads * 128, 3 * 2 * c.intermediate,
                                          3 * c.intermediate]


class DeviceStack:
    """The oracle's seeded stack uploaded as Q8 tiles and bf16 norms."""

    def __init__(self, stack):
        self.keep = []
        cfg = stack.config
        self.config = _lib.StackConfig(cfg["hidden"], cfg["intermediate"], cfg["layers"], cfg["heads"],
                                       cfg["kv_heads"], cfg["head_dim"], cfg["rms_eps"], int(cfg["rope"]))
        layers = (LayerWeightsC * cfg["layers"])()
        for i, layer in enumerate(stack.layers):
            layers[i].input_norm = self.vector(layer["input_norm"])
            layers[i].post_norm = self.vector(layer["post_norm"])
            for name in ("qkv", "o", "gate_up", "down"):
                setattr(layers[i], name, self.projection(layer[name]))
        self.layers = layers
        self.weights = StackWeightsC(self.config, layers, self.vector(stack.norm))

    def vector(self, bits):
        t = torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16).copy()).cuda()
        self.keep.append(t)
        return t.data_ptr()

    def projection(self, p):
        assert p.format == oracle.Q8_0
        blocks = torch.from_numpy(np.asarray(p.weight, np.uint8)).cuda()
        tiles = torch.zeros(K.Q8TilesBytes(p.n_out, p.n_in), dtype=torch.uint8, device="cuda")
        K.Q8_0ToTiles(blocks, p.n_out, p.n_in, tiles)
        self.keep.append(tiles)
        bias = self.vector(p.bias) if p.bias is not None else None
        return ProjectionC(_lib.WEIGHTS_Q8_TILES, tiles.data_ptr(), bias, p.n_in, p.n_out)


@pytest.mark.gpu
@pytest.mark.parametrize("cache_type", [_lib.CACHE_F32, _lib.CACHE_BF16])
def test_forward_stack_prefill_then_decode(cuda, cache_type):
    c = small_config()
    ref = OracleGenerator(c, seed=3, bf16_cache=cache_type == _lib.CACHE_BF16)
    stack = ref.w.encoder
    dev = DeviceStack(stack)
    capacity = 16
    cache = KvCache(dev.config, capacity, cache_type)
    assert cache.capacity() == capacity and cache.keys(0) and not cache.keys(c.encoder.layers)
    ref_cache = Cache(stack.config, capacity, cache_type == _lib.CACHE_BF16)
    rope = torch.from_numpy(np.ascontiguousarray(ref.rope, np.float32)).cuda()
    width = c.encoder.hidden
    counts = StackScratchElements(dev.config, 5)
    buffers = [torch.zeros(n, dtype=torch.int16 if i in (0, 3, 5) else torch.float32, device="cuda")
               for i, n in enumerate(counts)]
    scratch = StackScratchC(*[b.data_ptr() for b in buffers])
    rng = np.random.default_rng(5)

    for rows, first, past in ((5, 0, 0), (1, 5, 5)):
        positions = np.arange(first, first + rows, dtype=np.int32)
        pos_dev = torch.from_numpy(positions).cuda()
        layout = AttentionLayoutC(pos_dev.data_ptr(), pos_dev.data_ptr(), rows, rows, past, 1)
        hidden = rng.normal(0, 1, (rows, width)).astype(np.float32)
        hidden_dev = torch.from_numpy(hidden.copy()).cuda()
        output_dev = torch.empty_like(hidden_dev)
        ForwardStack(dev.weights, rope, layout, cache, hidden_dev, output_dev, rows, scratch)
        torch.cuda.synchronize()
        ref_hidden = hidden.copy()
        ref_out = ref.forward_stack(stack, True, dict(positions=positions, cache_rows=positions,
                                                      rows_per_sequence=rows, keys_per_sequence=rows,
                                                      past=past, causal=True), ref_cache, ref_hidden)
        e_hidden = rel_l2(hidden_dev.cpu().numpy(), ref_hidden)
        e_out = rel_l2(output_dev.cpu().numpy(), ref_out)
        assert e_hidden < LIMIT and e_out < LIMIT, (rows, e_hidden, e_out)
    # The cache rows both calls wrote, layer 1 keys (bf16 caches hold bits).
    kv, d = c.encoder.kv_heads, 128
    elem = 4 if cache_type == _lib.CACHE_F32 else 2
    keys = torch.empty(kv * capacity * d * elem, dtype=torch.uint8, device="cuda")
    cudart = ctypes.CDLL("libcudart.so.12")
    assert cudart.cudaMemcpy(ctypes.c_void_p(keys.data_ptr()), ctypes.c_void_p(cache.keys(1)),
                             ctypes.c_size_t(keys.numel()), 3) == 0  # device to device
    raw = keys.cpu().numpy()
    got = (raw.view(np.float32) if elem == 4 else oracle.bf16_value(raw.view(np.uint16))).reshape(kv, capacity, d)
    assert rel_l2(got[:, :6], ref_cache.k[1][:, :6]) < LIMIT
    assert not np.any(got[:, 6:])  # untouched rows stay zero
    cache.close()


@pytest.mark.gpu
def test_project_adds_bias(cuda):
    """Project (transformer.cpp:47-53) on a biased Q8_0 projection of the
    released checkpoint (enc_to_lm, 1024 -> 2048)."""
    c = small_config()
    ref = OracleGenerator(c, seed=4)
    p = ref.w.enc_to_lm
    assert p.bias is not None
    dev = DeviceStack.__new__(DeviceStack)
    dev.keep = []
    proj = dev.projection(p)
    rng = np.random.default_rng(6)
    x = oracle.bf16_bits(rng.normal(0, 1, (3, p.n_in)).astype(np.float32))
    y = torch.empty(3, p.n_out, dtype=torch.float32, device="cuda")
    Project(proj, torch.from_numpy(x.view(np.int16)).cuda(), y, 3)
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), ref.project(p, x, 3)) < 1e-5
