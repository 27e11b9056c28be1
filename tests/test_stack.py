"""The stack and generation-step kernels against the CPU oracle, on a B200.

Each kernel of kernels/generator_kernels.hip is run through the C ABI on
seeded inputs at VoxCPM2's shapes (DiT 22 rows, encoder 5 rows, LM decode 1
row at context 512, prefill rows) and compared with the oracle's
restatement. Tolerances: bit-equal where the arithmetic is the same
sequence of float32 operations; otherwise bf16 outputs within one bf16 ulp
(>= 98% bit-equal) and float32 outputs within a few float32 ulps, because
the device fuses multiply-adds (a * c - b * s) and uses CUDA's expf / rsqrtf
where the oracle rounds each operation and uses glibc's.
"""

import numpy as np
import pytest
import torch

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K

from _util import assert_bf16_close, assert_f32_close, bits16, f32, to_dev

pytestmark = pytest.mark.gpu

HEADS, KV_HEADS, D = 16, 2, 128


def bf16_weights(rng, n, mean=0.0, std=0.05):
    return oracle.bf16_bits((mean + rng.normal(0, std, n)).astype(np.float32))


@pytest.mark.parametrize("rows,width", [(22, 1024), (5, 1024), (1, 2048), (40, 2048)])
def test_rms_norm(cuda, rows, width):
    rng = np.random.default_rng(rows * width)
    x = (rng.normal(0, 3, (rows, width))).astype(np.float32)
    w = bf16_weights(rng, width, 1.0, 0.05)
    out = torch.empty(rows, width, dtype=torch.int16, device="cuda")
    out32 = torch.empty(rows, width, dtype=torch.float32, device="cuda")
    K.RmsNorm(to_dev(x), to_dev(w), out, out32, rows, width, 1e-5)
    K.RmsNorm(to_dev(x), to_dev(w), out, None, rows, width, 1e-5)  # without the fp32 copy
    torch.cuda.synchronize()
    ref, ref32 = oracle.rms_norm(x, w, 1e-5, want_f32=True)
    assert_bf16_close(bits16(out), ref, what="rms bf16")
    # rsqrtf (device) vs 1 / sqrtf (oracle): a few float32 ulps.
    assert_f32_close(f32(out32), ref32, rtol=2e-6, atol=0, what="rms f32")


@pytest.mark.parametrize("cache_type", [_lib.CACHE_F32, _lib.CACHE_BF16])
@pytest.mark.parametrize("rope", [True, False])
def test_qkv_rope(cuda, cache_type, rope):
    rng = np.random.default_rng(3)
    rows, capacity = 22, 40
    width = (HEADS + 2 * KV_HEADS) * D
    qkv = rng.normal(0, 1, (rows, width)).astype(np.float32)
    table = oracle.rope_table(10000.0, D, 1.0 + rng.random(64), 1.0, 64)
    positions = (np.arange(rows) % 11).astype(np.int32)
    cache_rows = (np.arange(rows) + 7).astype(np.int32)
    k_ref = np.zeros((KV_HEADS, capacity, D), np.float32)
    v_ref = np.zeros((KV_HEADS, capacity, D), np.float32)
    q_ref = oracle.qkv_rope(qkv, table if rope else None, positions, cache_rows, k_ref, v_ref, HEADS,
                            KV_HEADS, D)
    dtype = torch.float32 if cache_type == _lib.CACHE_F32 else torch.int16
    k = torch.zeros(KV_HEADS, capacity, D, dtype=dtype, device="cuda")
    v = torch.zeros(KV_HEADS, capacity, D, dtype=dtype, device="cuda")
    q = torch.empty(rows, HEADS, D, dtype=torch.float32, device="cuda")
    K.QkvRope(to_dev(qkv), to_dev(table) if rope else None, to_dev(positions), to_dev(cache_rows), q, k, v,
              rows, HEADS, KV_HEADS, D, capacity, cache_type)
    torch.cuda.synchronize()
    assert_f32_close(f32(q), q_ref, rtol=1e-6, atol=1e-6, what="q")
    if cache_type == _lib.CACHE_F32:
        assert_f32_close(f32(k), k_ref, rtol=1e-6, atol=1e-6, what="k")
        assert np.array_equal(f32(v), v_ref)  # a plain copy
    else:
        assert_bf16_close(bits16(k), oracle.bf16_bits(k_ref), what="k bf16")
        assert np.array_equal(bits16(v), oracle.bf16_bits(v_ref))


ATTENTION_CASES = {
    # name: rows, rows_per_sequence, keys_per_sequence, past, causal, capacity
    "dit": (22, 11, 11, 0, False, 22),
    "encoder": (5, 5, 5, 0, False, 64),
    "lm_decode": (1, 1, 0, 512, True, 1024),
    "lm_decode_long": (1, 1, 0, 4000, True, 4096),
    "prefill": (40, 40, 0, 0, True, 64),
}


@pytest.mark.parametrize("cache_type", [_lib.CACHE_F32, _lib.CACHE_BF16])
@pytest.mark.parametrize("case", list(ATTENTION_CASES))
def test_attention(cuda, case, cache_type):
    rows, per_seq, keys_per_seq, past, causal, capacity = ATTENTION_CASES[case]
    rng = np.random.default_rng(len(case) + cache_type)
    q = rng.normal(0, 1, (rows, HEADS, D)).astype(np.float32)
    k = rng.normal(0, 1, (KV_HEADS, capacity, D)).astype(np.float32)
    v = rng.normal(0, 1, (KV_HEADS, capacity, D)).astype(np.float32)
    if cache_type == _lib.CACHE_BF16:
        # The oracle reads the same (bf16-rounded) cache values.
        k = oracle.bf16_value(oracle.bf16_bits(k)).reshape(k.shape)
        v = oracle.bf16_value(oracle.bf16_bits(v)).reshape(v.shape)
        k_dev, v_dev = to_dev(oracle.bf16_bits(k)), to_dev(oracle.bf16_bits(v))
    else:
        k_dev, v_dev = to_dev(k), to_dev(v)
    ref = oracle.attention(q, k, v, per_seq, keys_per_seq, past, causal, HEADS, KV_HEADS, D)
    out = torch.empty(rows, HEADS * D, dtype=torch.int16, device="cuda")
    K.Attention(to_dev(q), k_dev, v_dev, out, rows, per_seq, keys_per_seq, past, causal, HEADS, KV_HEADS,
                D, capacity, cache_type)
    torch.cuda.synchronize()
    assert_bf16_close(bits16(out), ref, what=f"attention {case}")
    if past > 0:
        # The same through a device-side position (graph replays).
        past_dev = torch.tensor([past], dtype=torch.int32, device="cuda")
        out2 = torch.empty_like(out)
        K.Attention(to_dev(q), k_dev, v_dev, out2, rows, per_seq, keys_per_seq, 0, causal, HEADS, KV_HEADS,
                    D, capacity, cache_type, past_device=past_dev, max_keys=capacity)
        torch.cuda.synchronize()
        assert_bf16_close(bits16(out2), ref, what=f"attention {case} (device position)")


def test_elementwise(cuda):
    rng = np.random.default_rng(17)
    rows, width = 22, 4096
    gate_up = rng.normal(0, 2, (rows, 2 * width)).astype(np.float32)
    out = torch.empty(rows, width, dtype=torch.int16, device="cuda")
    K.SwiGlu(to_dev(gate_up), out, rows, width)
    torch.cuda.synchronize()
    assert_bf16_close(bits16(out), oracle.swiglu(gate_up), what="swiglu")

    x = rng.normal(0, 2, (rows, 1024)).astype(np.float32)
    for silu in (False, True):
        o = torch.empty(rows, 1024, dtype=torch.int16, device="cuda")
        K.ToBf16(to_dev(x), o, x.size, silu)
        torch.cuda.synchronize()
        ref = oracle.to_bf16(x, silu)
        if silu:
            assert_bf16_close(bits16(o), ref, what="silu")
        else:
            assert np.array_equal(bits16(o), ref)

    bias = bf16_weights(rng, 1024, 0.0, 0.02)
    d = to_dev(x)
    K.AddBias(d, to_dev(bias), rows, 1024)
    torch.cuda.synchronize()
    assert np.array_equal(f32(d), oracle.add_bias(x, bias))

    a = rng.normal(0, 1, (3, 2048)).astype(np.float32)
    b = rng.normal(0, 1, (3, 2048)).astype(np.float32)
    sa = rng.random(3).astype(np.float32)
    o = torch.empty(3, 4096, dtype=torch.int16, device="cuda")
    K.ConcatRows(to_dev(a), to_dev(sa), 2048, to_dev(b), None, 2048, o, 3)
    torch.cuda.synchronize()
    assert np.array_equal(bits16(o), oracle.concat_rows(a, b, a_scale=sa))

    z = rng.normal(0, 1, 512).astype(np.float32)
    o = torch.empty(512, dtype=torch.int16, device="cuda")
    K.Quantize(to_dev(z), o, 512, 9.0)
    torch.cuda.synchronize()
    got = oracle.bf16_value(bits16(o))
    ref = oracle.bf16_value(oracle.quantize(z, 9.0))
    # tanhf may differ by an ulp: a level flips only at an exact tie.
    assert float(np.mean(got == ref)) >= 0.995 and float(np.max(np.abs(got - ref))) <= 1.0 / 9 + 1e-6


def test_row_plumbing(cuda):
    rng = np.random.default_rng(21)
    width, patch = 1024, 4
    mu = rng.normal(0, 1, (2, width)).astype(np.float32)
    time = rng.normal(0, 1, width).astype(np.float32)
    cond = rng.normal(0, 1, (patch, width)).astype(np.float32)
    x = rng.normal(0, 1, (patch, width)).astype(np.float32)
    out = torch.empty(22, width, dtype=torch.float32, device="cuda")
    K.AssembleDit(to_dev(mu), to_dev(time), to_dev(cond), to_dev(x), out, patch, width)
    torch.cuda.synchronize()
    assert np.array_equal(f32(out), oracle.assemble_dit(mu, time, cond, x, patch))

    special = bf16_weights(rng, width, 0.0, 1.0)
    rows_in = rng.normal(0, 1, (2 * patch, width)).astype(np.float32)
    o = torch.empty(2 * (patch + 1), width, dtype=torch.float32, device="cuda")
    K.PrependSpecial(to_dev(rows_in), to_dev(special), o, 2, patch, width)
    torch.cuda.synchronize()
    assert np.array_equal(f32(o), oracle.prepend_special(rows_in, special, 2, patch))

    src = rng.normal(0, 1, (22, width)).astype(np.float32)
    idx = np.array([7, 8, 9, 10, 18, 19, 20, 21], np.int32)
    g = torch.empty(8, width, dtype=torch.float32, device="cuda")
    K.GatherRows(to_dev(src), to_dev(idx), g, 8, width)
    s = torch.zeros(22, width, dtype=torch.float32, device="cuda")
    K.ScatterRows(g, to_dev(idx), s, 8, width)
    torch.cuda.synchronize()
    assert np.array_equal(f32(g), oracle.gather_rows(src, idx))
    expect = np.zeros_like(src)
    expect[idx] = src[idx]
    assert np.array_equal(f32(s), expect)

    mask = np.array([1, 0, 1], np.int32)
    qa = rng.normal(0, 1, (3, width)).astype(np.float32)
    pl = rng.normal(0, 1, (3, width)).astype(np.float32)
    o = torch.empty(3, width, dtype=torch.float32, device="cuda")
    K.SelectRows(to_dev(qa), to_dev(pl), to_dev(mask), o, 3, width)
    torch.cuda.synchronize()
    assert np.array_equal(f32(o), np.where(mask[:, None] != 0, qa, pl))

    table = bf16_weights(rng, 50 * 64, 0.0, 1.0).reshape(50, 64)
    ids = np.array([3, 49, 0, 7], np.int32)
    text = np.array([1, 1, 0, 1], np.int32)
    o = torch.empty(4, 64, dtype=torch.float32, device="cuda")
    K.Embed(to_dev(table), to_dev(ids), to_dev(text), o, 4, 64, 2.0)
    torch.cuda.synchronize()
    expect = oracle.bf16_value(table[ids]).reshape(4, 64) * 2.0 * text[:, None]
    assert np.array_equal(f32(o), expect.astype(np.float32))


def test_guided_euler(cuda):
    rng = np.random.default_rng(5)
    velocity = rng.normal(0, 1, (2, 256)).astype(np.float32)
    x = rng.normal(0, 1, 256).astype(np.float32)
    d = to_dev(x)
    K.GuidedEuler(to_dev(velocity), d, 256, 2.0, 0.0436)
    torch.cuda.synchronize()
    ref = oracle.guided_euler(velocity, x, 2.0, 0.0436)
    # The dot products sum in a different order: a few float32 ulps.
    assert_f32_close(f32(d), ref, rtol=1e-6, atol=1e-6, what="guided euler")
