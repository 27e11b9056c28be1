"""BASELINE config 3 at the benchmarked configuration, against the oracle, on
a B200: the released shapes at full depth (28-layer LM, 8-layer residual LM,
12-layer local encoder, 12-layer DiT; hidden 2048 / 1024, 16 query and 2 KV
heads of 128), seeded Q8_0 weights, the persistent DiT patch and one-row LM
stack kernels (the path bench.py times), bf16 and float32 KV caches.

- A prompt at full depth through Prefill and two steps, every state against
  the oracle's prefill and steps (generator.cpp:326-513,
  transformer.cpp:55-100).
- Steps at context 520 or more: the prompt of 520 rows runs on the device
  only (a full-depth prefill of that length takes the oracle minutes); the
  oracle then takes the generator's LM states and both LM caches after it,
  read back from the device, and both run the same three steps. Each of the
  LM stack kernel's 8 key chunks then holds 65 or more keys, so its
  per-chunk online softmax and the merge of the chunks run at the size the
  benchmark runs them.

Limits (relative L2 unless noted). At full depth the float32 summation
orders of the two sides differ in 28 + 8 layers, and a last-bit difference
before one of the many bf16 rounding points moves that value by a bf16 ulp,
so the LM states drift further than in the two-layer tests; FSQ then rounds
tanh*9 to levels, where such a drift can flip a level. The limits are the
reference's own full-depth ones (tests/generator_test.cpp:117-143): LM and
residual states after the prefill 1e-2, LM and residual states of a step
1e-1. Latents keep the tighter 2e-2 of its first step, for every step, and
stop logits an absolute 5e-3.
"""

import numpy as np
import pytest

from oracle.model import Cache, OracleGenerator
from voxcpm_b200 import _lib
from voxcpm_b200.generator import Generator, released_config
from voxcpm_b200.kernels import DeviceError

from _util import rel_l2

pytestmark = pytest.mark.gpu

LATENT_LIMIT = 2e-2
STOP_ATOL = 5e-3
PREFILL_LIMIT = 1e-2     # generator_test.cpp:117-119
STEP_STATE_LIMIT = 1e-1  # generator_test.cpp:141-143
SEED = 100


def config3(max_length: int):
    c = released_config()
    c.max_length = max_length
    c.vocab = 1024
    return c


def reset_oracle(ref: OracleGenerator, bf16: bool):
    """The oracle generator with fresh caches and state (the weights, which
    take seconds to regenerate, are kept)."""
    ref.bf16_cache = bf16
    ref.base_cache = Cache(ref.w.base_lm.config, ref.c.max_length, bf16)
    ref.residual_cache = Cache(ref.w.residual_lm.config, ref.c.max_length, bf16)
    ref.dit_cache = Cache(ref.w.dit.config, 2 * (3 + 2 * ref.patch), bf16)
    ref.position = 0


@pytest.fixture(scope="module")
def oracle_640():
    return OracleGenerator(config3(640), seed=SEED, q8=True)


def prompt(c, rows: int, audio_rows, seed: int):
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, c.vocab, rows).astype(np.int32)
    audio = np.zeros(rows, np.int32)
    audio[list(audio_rows)] = 1
    feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
    feats[list(audio_rows)] = rng.normal(0, 1, (len(audio_rows), c.patch_size, c.feat_dim))
    return tokens, 1 - audio, audio, feats


def compare_step(gen, ref, noise, what):
    hidden = gen.config.lm.hidden
    latent, stop = gen.Step(noise, 10, 2.0)
    latent_r, stop_r = ref.step(noise, 10, 2.0)
    errors = {
        "latent": rel_l2(latent, latent_r),
        "stop": float(np.max(np.abs(stop - stop_r))),
        "lm_output": rel_l2(gen.State("lm_output", hidden), ref.lm_output),
        "lm_hidden": rel_l2(gen.State("lm_hidden", hidden), ref.lm_hidden),
        "residual": rel_l2(gen.State("residual_hidden", hidden), ref.residual_hidden),
    }
    print(what, " ".join(f"{k} {v:.3e}" for k, v in errors.items()))
    assert errors["latent"] < LATENT_LIMIT, (what, errors)
    assert errors["stop"] < STOP_ATOL, (what, errors)
    for state in ("lm_output", "lm_hidden", "residual"):
        assert errors[state] < STEP_STATE_LIMIT, (what, errors)
    return errors


def test_config3_prefill_and_steps_full_depth(cuda, oracle_640):
    """A 24-row prompt (audio rows 9 and 23) through the full-depth prefill,
    then two steps, bf16 caches, against the oracle."""
    c = config3(640)
    ref = oracle_640
    reset_oracle(ref, bf16=True)
    gen = Generator(c, seed=SEED, checkpoint=_lib.CHECKPOINT_Q8, cache_type=_lib.CACHE_BF16)
    assert gen.persistent()
    p = prompt(c, 24, (9, 23), seed=31)
    gen.Prefill(*p)
    ref.prefill(*p)
    hidden = c.lm.hidden
    e_lm = rel_l2(gen.State("lm_output", hidden), ref.lm_output)
    e_hidden = rel_l2(gen.State("lm_hidden", hidden), ref.lm_hidden)
    e_res = rel_l2(gen.State("residual_hidden", hidden), ref.residual_hidden)
    print(f"prefill: lm_output {e_lm:.3e} lm_hidden {e_hidden:.3e} residual {e_res:.3e}")
    # lm_hidden is after FSQ (a step state's limit); the others before it.
    assert e_lm < PREFILL_LIMIT and e_res < PREFILL_LIMIT and e_hidden < STEP_STATE_LIMIT
    # The caches the prefill wrote (24 rows of every layer and KV head).
    for name, cache in (("base_cache_k", ref.base_cache.k), ("residual_cache_v", ref.residual_cache.v)):
        got = gen.State(name, cache.size).reshape(cache.shape)[:, :, :24]
        err = rel_l2(got, cache[:, :, :24])
        print(f"prefill {name}: rel L2 {err:.3e}")
        assert err < PREFILL_LIMIT, name
    rng = np.random.default_rng(32)
    for k in range(2):
        noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        compare_step(gen, ref, noise, f"step {k} (context {24 + k})")
    assert DeviceError() == 0
    gen.close()


@pytest.mark.parametrize("cache_type", [_lib.CACHE_BF16, _lib.CACHE_F32])
def test_config3_steps_at_context_520(cuda, oracle_640, cache_type):
    """Three steps from context 520 (the LM's persistent stack kernel over
    8 key chunks of 65+ keys each), the oracle started from the generator's
    states and caches after a device-only prefill of 520 rows."""
    c = config3(640)
    bf16 = cache_type == _lib.CACHE_BF16
    ref = oracle_640
    reset_oracle(ref, bf16=bf16)
    gen = Generator(c, seed=SEED, checkpoint=_lib.CHECKPOINT_Q8, cache_type=cache_type)
    assert gen.persistent()
    rows = 520
    gen.Prefill(*prompt(c, rows, (rows - 1,), seed=41))
    assert gen.position() == rows
    hidden = c.lm.hidden
    ref.lm_hidden = gen.State("lm_hidden", hidden)
    ref.residual_hidden = gen.State("residual_hidden", hidden)
    ref.prefix_cond = gen.State("prefix_cond", c.patch_size * c.feat_dim).reshape(c.patch_size, c.feat_dim)
    for name, array in (("base_cache_k", ref.base_cache.k), ("base_cache_v", ref.base_cache.v),
                        ("residual_cache_k", ref.residual_cache.k),
                        ("residual_cache_v", ref.residual_cache.v)):
        array[...] = gen.State(name, array.size).reshape(array.shape)
    ref.position = rows
    rng = np.random.default_rng(42)
    for k in range(3):
        noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        compare_step(gen, ref, noise, f"{'bf16' if bf16 else 'f32'} cache, step {k} (context {rows + k})")
    assert DeviceError() == 0
    gen.close()


def test_config3_sixteen_slots_at_context_128(cuda, oracle_640):
    """A GeneratorBatch of 16 slots at full depth (the bench's config 4
    batching), prompts of 128..143 rows, bf16 caches: two steps of all
    slots, then slot 8 takes a new request while the others continue, and a
    third step. Every slot against a single GPU generator fed the same
    request (the generator the other tests check against the oracle); slots
    0, 15 and the refilled slot 8 against the oracle itself, started from
    the slot's states and caches after its prefill."""
    import copy

    from voxcpm_b200.generator import GeneratorBatch

    c = config3(320)
    slots = 16
    hidden = c.lm.hidden
    batch = GeneratorBatch(c, slots, seed=SEED, checkpoint=_lib.CHECKPOINT_Q8, cache_type=_lib.CACHE_BF16)
    single = Generator(c, seed=SEED, checkpoint=_lib.CHECKPOINT_Q8, cache_type=_lib.CACHE_BF16)
    prompts = [prompt(c, 128 + s, (127 + s,), seed=200 + s) for s in range(slots)]
    for s in range(slots):
        batch.Prefill(s, *prompts[s])
    refill = prompt(c, 136, (100, 135), seed=300)
    rng = np.random.default_rng(7)
    noise = [rng.normal(0, 1, (slots, c.patch_size, c.feat_dim)).astype(np.float32) for _ in range(3)]

    def oracle_from_slot(s):
        ref = copy.copy(oracle_640)
        reset_oracle(ref, bf16=True)
        ref.c = c
        ref.base_cache = Cache(ref.w.base_lm.config, c.max_length, True)
        ref.residual_cache = Cache(ref.w.residual_lm.config, c.max_length, True)
        ref.lm_hidden = batch.State(s, "lm_hidden", hidden)
        ref.residual_hidden = batch.State(s, "residual_hidden", hidden)
        ref.prefix_cond = batch.State(s, "prefix_cond", c.patch_size * c.feat_dim).reshape(
            c.patch_size, c.feat_dim)
        for name, array in (("base_cache_k", ref.base_cache.k), ("base_cache_v", ref.base_cache.v),
                            ("residual_cache_k", ref.residual_cache.k),
                            ("residual_cache_v", ref.residual_cache.v)):
            array[...] = batch.State(s, name, array.size).reshape(array.shape)
        ref.position = batch.position(s)
        return ref

    refs = {s: oracle_from_slot(s) for s in (0, 15)}
    outs = []
    for k in range(2):
        latents, stop = batch.Step(noise[k])
        outs.append((latents, stop))
        for s, ref in refs.items():
            latent_r, stop_r = ref.step(noise[k][s], 10, 2.0)
            e = (rel_l2(latents[s], latent_r), float(np.max(np.abs(stop[s] - stop_r))),
                 rel_l2(batch.State(s, "residual_hidden", hidden), ref.residual_hidden))
            print(f"step {k} slot {s} vs oracle: latent {e[0]:.3e} stop {e[1]:.3e} residual {e[2]:.3e}")
            assert e[0] < LATENT_LIMIT and e[1] < STOP_ATOL and e[2] < STEP_STATE_LIMIT
    batch.Prefill(8, *refill)
    refs = {8: oracle_from_slot(8)}
    latents, stop = batch.Step(noise[2])
    outs.append((latents, stop))
    latent_r, stop_r = refs[8].step(noise[2][8], 10, 2.0)
    e = (rel_l2(latents[8], latent_r), float(np.max(np.abs(stop[8] - stop_r))))
    print(f"refilled slot 8 vs oracle: latent {e[0]:.3e} stop {e[1]:.3e}")
    assert e[0] < LATENT_LIMIT and e[1] < STOP_ATOL
    # Every slot against a single generator fed the same request.
    worst = 0.0
    for s in range(slots):
        single.Prefill(*prompts[s])
        for k in range(3):
            if k == 2 and s == 8:
                single.Prefill(*refill)
            latent, st = single.Step(noise[k][s])
            e_l = rel_l2(outs[k][0][s], latent)
            assert e_l < LATENT_LIMIT, (s, k, e_l)
            assert float(np.max(np.abs(outs[k][1][s] - st))) < STOP_ATOL, (s, k)
            worst = max(worst, e_l)
    print(f"16 slots vs single generators: worst latent rel L2 {worst:.3e}")
    assert batch.position(8) == 137 and batch.position(0) == 131
    assert DeviceError() == 0
    batch.close()
    single.close()
