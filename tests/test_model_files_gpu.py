"""A generator read from checkpoint files, on a B200 (tests/generator_test.cpp
reads the released files the same way; those weights are absent here, so the
files are written from the seeded checkpoint):
- a Q8_0 GGUF and a bf16 safetensors directory give the seeded generator's
  results bit for bit (same tiles, same kernels), with the configuration
  parsed from the files' config.json;
- F32 sources go through the device conversion and give the same bits;
- a file that mixes formats in the DiT (one layer bf16, the rest Q8_0) runs
  the per-kernel sequence and matches the oracle fed the same tensors;
- the load-time conversions (fp16 / fp32 / Q8_0 -> bf16) equal the oracle's
  rounding bit for bit, NaN, infinities, subnormals and unaligned pointers
  included.
"""

import numpy as np
import pytest
import torch

import oracle
from oracle.model import OracleGenerator
from voxcpm_b200 import _lib
from voxcpm_b200._lib import VxError, check, load
from voxcpm_b200.generator import Generator, small_config
from voxcpm_b200.model_files import ModelFiles, ParseConfig

from _checkpoints import (T, as_dtype, config_json, ggml_entry, seeded_values, tensor_list, write_directory,
                          write_gguf)
from _util import bits16, rel_l2, to_dev

pytestmark = pytest.mark.gpu

SEED = 21
LATENT_LIMIT = 2e-2
VELOCITY_LIMIT = 1e-2


def config():
    return small_config(layers=1, max_length=64, vocab=64)


def seeded(c, q8):
    return [(name, shape, *seeded_values(name, shape, kind, mean, std, SEED, q8))
            for name, shape, kind, mean, std in tensor_list(c)]


def gguf_from(c, path, tensors, abbreviate=()):
    model = {name: ggml_entry(kind, shape, values) for name, shape, kind, values in tensors}
    write_gguf(path, model, config_text=config_json(c), tokenizer_text='{"model": {}}', abbreviate=abbreviate)


def directory_from(c, root, tensors, dtype="BF16"):
    out = {}
    for name, shape, kind, values in tensors:
        assert kind == "BF16"
        out[name] = T(dtype, shape, as_dtype(kind, values, dtype))
    write_directory(root, out, config_json(c))


def prompt(c, seed=4, rows=6):
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, c.vocab, rows).astype(np.int32)
    audio = np.zeros(rows, np.int32)
    audio[-1] = 1
    feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
    feats[-1] = rng.normal(0, 1, (c.patch_size, c.feat_dim))
    return tokens, 1 - audio, audio, feats


def run(gen, c):
    """A velocity pair, a prefill and two patches: every output."""
    rng = np.random.default_rng(3)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    x = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    out = [gen.Velocity(mu, cond, x, 0.4)]
    gen.Prefill(*prompt(c))
    out.append(gen.State("lm_hidden", c.lm.hidden))
    for _ in range(2):
        latent, stop = gen.Step(rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32), 10, 2.0)
        out += [latent, stop]
    return out


def assert_same(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        assert np.array_equal(x, y), f"output {i} differs"


def test_gguf_q8_matches_seeded(cuda, tmp_path):
    c = config()
    path = tmp_path / "voxcpm2-q8_0.gguf"
    names = [n for n, *_ in tensor_list(c)]
    gguf_from(c, path, seeded(c, q8=True), abbreviate=names[::3])
    files = ModelFiles(path)
    assert files.gguf() and len(files.model_tensors()) == len(names)
    parsed = ParseConfig(files.config())
    gen = Generator.Create(parsed, files)
    files.close()
    ref = Generator(c, seed=SEED, checkpoint=_lib.CHECKPOINT_Q8)
    assert gen.weight_bytes() == ref.weight_bytes()
    assert gen.persistent() == ref.persistent()
    assert_same(run(gen, parsed), run(ref, c))
    gen.close()
    ref.close()


@pytest.mark.parametrize("dtype", ["BF16", "F32"])
def test_safetensors_bf16_matches_seeded(cuda, tmp_path, dtype):
    c = config()
    directory_from(c, tmp_path, seeded(c, q8=False), dtype)
    with ModelFiles(tmp_path) as files:
        parsed = ParseConfig(files.config())
        gen = Generator.Create(parsed, files, _lib.CACHE_BF16)
    ref = Generator(c, seed=SEED, checkpoint=_lib.CHECKPOINT_BF16, cache_type=_lib.CACHE_BF16)
    assert gen.weight_bytes() == ref.weight_bytes()
    assert_same(run(gen, parsed), run(ref, c))
    gen.close()
    ref.close()


def test_mixed_formats_against_oracle(cuda, tmp_path):
    """DiT layer 0 in bf16 (its Q8_0 values dequantized), stop_head in F32,
    everything else Q8_0: per-projection formats, the per-kernel DiT."""
    from voxcpm_b200.generator import released_config

    c = released_config()
    c.lm.layers = c.residual_lm.layers = c.encoder.layers = 1
    c.dit.layers = 2
    c.max_length, c.vocab = 64, 64
    tensors = []
    source = {}
    for name, shape, kind, values in seeded(c, q8=True):
        if kind == "Q8_0" and (name.startswith("feat_decoder.estimator.decoder.layers.0.")
                               or name == "stop_head.weight"):
            bits = oracle.bf16_bits(oracle.q8_0_dequant(values, shape[0], shape[1]).astype(np.float32))
            kind, values = "BF16", bits.reshape(-1)
        source[name] = (kind, values)
        if name == "stop_head.weight":
            kind, values = "F32", oracle.bf16_value(values)
        tensors.append((name, shape, kind, values))
    path = tmp_path / "mixed.gguf"
    gguf_from(c, path, tensors)
    with ModelFiles(path) as files:
        gen = Generator.Create(c, files)
    assert not gen.persistent(), "mixed DiT formats must run the per-kernel sequence"
    ref = OracleGenerator(c, source=source)
    rng = np.random.default_rng(5)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    x = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    v_err = rel_l2(gen.Velocity(mu, cond, x, 0.4), ref.velocity(mu, cond, x, 0.4))
    l_err = rel_l2(gen.DitPatch(mu, cond, x, 10, 2.0), ref.dit_patch(mu, cond, x, 10, 2.0))
    p = prompt(c)
    gen.Prefill(*p)
    ref.prefill(*p)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    latent, stop = gen.Step(noise, 10, 2.0)
    latent_r, stop_r = ref.step(noise, 10, 2.0)
    s_err = rel_l2(latent, latent_r)
    print(f"mixed: velocity {v_err:.3e} patch {l_err:.3e} step latent {s_err:.3e} "
          f"stop |d| {np.max(np.abs(stop - stop_r)):.3e}")
    assert v_err < VELOCITY_LIMIT and l_err < LATENT_LIMIT and s_err < LATENT_LIMIT
    assert np.max(np.abs(stop - stop_r)) < 5e-3
    gen.close()


def test_file_errors(cuda, tmp_path):
    c = config()
    tensors = seeded(c, q8=True)
    # A missing tensor, a wrong shape, an extra tensor.
    gguf_from(c, tmp_path / "a.gguf", tensors[1:])
    with ModelFiles(tmp_path / "a.gguf") as files, pytest.raises(VxError, match="lacks base_lm.embed_tokens"):
        Generator.Create(c, files)
    bad = [(n, (s[0] // 2, s[1]) if n == "stop_proj.weight" else s, k,
            v[: v.size // 2] if n == "stop_proj.weight" else v) for n, s, k, v in tensors]
    gguf_from(c, tmp_path / "b.gguf", bad)
    with ModelFiles(tmp_path / "b.gguf") as files, pytest.raises(VxError, match="unexpected shape"):
        Generator.Create(c, files)
    extra = tensors + [("extra.weight", (2,), "BF16", np.zeros(2, np.uint16))]
    gguf_from(c, tmp_path / "c.gguf", extra)
    with ModelFiles(tmp_path / "c.gguf") as files, pytest.raises(VxError, match="does not use"):
        Generator.Create(c, files)


# ------------------------------------------------------------ conversions

def special_floats(rng, n):
    """n floats led by NaNs, infinities, zeros, subnormals, the largest
    finite values and rounding ties (as many as fit)."""
    v = rng.normal(0, 3, max(n, 20)).astype(np.float32)
    v[:12] = [np.nan, -np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -3e-39, 3.4e38, -3.39e38, 1.0, 1.00390625]
    bits = v.view(np.uint32)
    bits[12:20] = [0x7F800001, 0xFFC00001, 0x3F808000, 0x3F818000, 0x3F807FFF, 0x00008000, 0x7F7FFFFF, 0x80018000]
    return v[:n].copy()


@pytest.mark.parametrize("count, offset", [(1, 0), (7, 1), (8, 0), (1000, 0), (1003, 3), (1 << 20, 0)])
def test_float_to_bf16(cuda, count, offset):
    rng = np.random.default_rng(count)
    v = special_floats(rng, count + offset)
    src = to_dev(v)
    out = torch.zeros(count + offset, dtype=torch.int16, device="cuda")
    check(load().vx_float_to_bf16(src.data_ptr() + 4 * offset, out.data_ptr() + 2 * offset, count, None))
    torch.cuda.synchronize()
    assert np.array_equal(bits16(out)[offset:], oracle.bf16_bits(v[offset:]))
    assert not bits16(out)[:offset].any()


@pytest.mark.parametrize("count, offset", [(1, 0), (9, 1), (4096, 0), (4099, 5)])
def test_half_to_bf16(cuda, count, offset):
    rng = np.random.default_rng(count)
    h = rng.integers(0, 1 << 16, max(count + offset, 6)).astype(np.uint16)
    h[:6] = [0x7C00, 0xFC00, 0x7E01, 0x0001, 0x8000, 0x03FF]
    h = h[: count + offset].copy()
    out = torch.zeros(count + offset, dtype=torch.int16, device="cuda")
    src = to_dev(h)
    check(load().vx_half_to_bf16(src.data_ptr() + 2 * offset, out.data_ptr() + 2 * offset, count, None))
    torch.cuda.synchronize()
    expect = oracle.bf16_bits(h.view(np.float16).astype(np.float32))
    assert np.array_equal(bits16(out)[offset:], expect[offset:])


@pytest.mark.parametrize("blocks, offset", [(1, 0), (5, 1), (4096, 0), (333, 4)])
def test_q8_0_to_bf16(cuda, blocks, offset):
    rng = np.random.default_rng(blocks)
    raw = rng.integers(0, 256, (blocks, 34)).astype(np.uint8)
    scales = rng.normal(0, 0.02, blocks).astype(np.float16)
    scales[:1] = np.float16(6e-8)  # subnormal scale
    scales[1:2] = np.array([0x7E55], np.uint16).view(np.float16)  # NaN scale with a payload
    raw[:, :2] = scales.view(np.uint8).reshape(blocks, 2)
    src = to_dev(raw.reshape(-1))
    out = torch.zeros(blocks * 32 + offset, dtype=torch.int16, device="cuda")
    check(load().vx_q8_0_to_bf16(src.data_ptr(), out.data_ptr() + 2 * offset, blocks * 32, None))
    torch.cuda.synchronize()
    q = raw[:, 2:].view(np.int8).astype(np.float32)
    wide = scales.astype(np.float32)[:, None]
    # IEEE: a NaN operand propagates (payload kept).
    products = np.where(np.isnan(wide), wide, wide * q)
    expect = oracle.bf16_bits(products.reshape(-1))
    assert np.array_equal(bits16(out)[offset:], expect)
    assert load().vx_q8_0_to_bf16(src.data_ptr(), out.data_ptr(), 33, None) == _lib.VX_INVALID
