"""Batched request slots (GeneratorBatch) on a B200:
- one active slot runs the same kernels as a single generator with the
  per-kernel DiT: identical bits;
- several active slots, each with its own prompt and noise, match the
  oracle's single-request generator (the limits of test_generator.py) and a
  single GPU generator per request;
- inactive slots keep their state; a slot takes a new request mid-run;
- graphs re-capture when a long prompt moves the shared work buffers.
"""

import numpy as np
import pytest

from oracle.model import OracleGenerator
from voxcpm_b200 import _lib
from voxcpm_b200._lib import VxError
from voxcpm_b200.generator import Generator, GeneratorBatch, small_config

from _util import rel_l2

pytestmark = pytest.mark.gpu

SEED = 13
LATENT_LIMIT = 2e-2
STATE_LIMIT = 2e-2
FSQ_STATE_LIMIT = 6e-2
STOP_ATOL = 5e-3


def config(max_length=160):
    return small_config(layers=1, max_length=max_length, vocab=64)


def prompt(c, seed, rows=7):
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, c.vocab, rows).astype(np.int32)
    audio = np.zeros(rows, np.int32)
    audio[-2:] = 1
    feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
    feats[-2:] = rng.normal(0, 1, (2, c.patch_size, c.feat_dim))
    return tokens, 1 - audio, audio, feats


def noises(c, slots, seed):
    return np.random.default_rng(seed).normal(0, 1, (slots, c.patch_size, c.feat_dim)).astype(np.float32)


def test_one_active_slot_is_the_single_generator(cuda):
    """The batch always runs the per-kernel DiT; the single generator does
    too with SetPersistent(False), which also turns off its persistent LM
    stacks. An LM FFN width the persistent LM kernel does not serve keeps
    both sides on the same LM kernels as well."""
    c = config()
    c.lm.intermediate = c.residual_lm.intermediate = 4096
    batch = GeneratorBatch(c, 3, seed=SEED)
    single = Generator(c, seed=SEED)
    single.SetPersistent(False)
    p = prompt(c, 1)
    batch.Prefill(0, *p)
    single.Prefill(*p)
    for k in range(3):
        n = noises(c, 3, 10 + k)
        latents, stop = batch.Step(n, active=[1, 0, 0])
        latent, stop1 = single.Step(n[0])
        assert np.array_equal(latents[0], latent) and np.array_equal(stop[0], stop1), f"step {k}"
        assert not latents[1:].any()
        for name in ("lm_hidden", "residual_hidden"):
            assert np.array_equal(batch.State(0, name, c.lm.hidden), single.State(name, c.lm.hidden))
    assert batch.position(0) == single.position() and batch.position(1) == 0
    batch.close()
    single.close()


def test_slots_match_oracle_and_single_generators(cuda):
    c = config()
    slots = 3
    batch = GeneratorBatch(c, slots, seed=SEED)
    refs = [OracleGenerator(c, seed=SEED) for _ in range(slots)]
    singles = [Generator(c, seed=SEED) for _ in range(slots)]
    for s in range(slots):
        p = prompt(c, 20 + s, rows=5 + 2 * s)
        batch.Prefill(s, *p)
        refs[s].prefill(*p)
        singles[s].Prefill(*p)
    hidden = c.lm.hidden
    for k in range(2):
        n = noises(c, slots, 30 + k)
        latents, stop = batch.Step(n)
        for s in range(slots):
            latent_r, stop_r = refs[s].step(n[s], 10, 2.0)
            latent_g, stop_g = singles[s].Step(n[s])
            errs = (rel_l2(latents[s], latent_r), float(np.max(np.abs(stop[s] - stop_r))),
                    rel_l2(batch.State(s, "lm_hidden", hidden), refs[s].lm_hidden),
                    rel_l2(batch.State(s, "residual_hidden", hidden), refs[s].residual_hidden),
                    rel_l2(latents[s], latent_g))
            print(f"step {k} slot {s}: latent {errs[0]:.3e} stop |d| {errs[1]:.3e} lm {errs[2]:.3e} "
                  f"residual {errs[3]:.3e} vs single GPU {errs[4]:.3e}")
            assert errs[0] < LATENT_LIMIT and errs[1] < STOP_ATOL
            assert errs[2] < FSQ_STATE_LIMIT and errs[3] < STATE_LIMIT and errs[4] < LATENT_LIMIT
            assert batch.position(s) == refs[s].position
    batch.close()
    for g in singles:
        g.close()


def test_inactive_slots_keep_state_and_refill(cuda):
    c = config()
    batch = GeneratorBatch(c, 3, seed=SEED)
    for s in range(3):
        batch.Prefill(s, *prompt(c, 40 + s))
    batch.Step(noises(c, 3, 1))
    held = batch.State(1, "lm_hidden", c.lm.hidden)
    position = batch.position(1)
    latents, stop = batch.Step(noises(c, 3, 2), active=[1, 0, 1])
    assert np.array_equal(batch.State(1, "lm_hidden", c.lm.hidden), held)
    assert batch.position(1) == position and not latents[1].any() and not stop[1].any()
    # A new request in slot 1 while 0 and 2 continue: slot 1 now matches a
    # fresh single generator fed the same request.
    fresh = Generator(c, seed=SEED)
    p = prompt(c, 50, rows=9)
    batch.Prefill(1, *p)
    fresh.Prefill(*p)
    for k in range(2):
        n = noises(c, 3, 60 + k)
        latents, _ = batch.Step(n)
        latent, _ = fresh.Step(n[1])
        err = rel_l2(latents[1], latent)
        print(f"refilled slot step {k}: vs single {err:.3e}")
        assert err < LATENT_LIMIT
    assert batch.position(1) == fresh.position()
    batch.close()
    fresh.close()


def test_graphs_recapture_after_long_prompt(cuda):
    """A long prompt reallocates the shared work buffers: the batch's graphs
    must follow (graph replay equals eager launches)."""
    c = config(max_length=200)
    graphed = GeneratorBatch(c, 2, seed=SEED)
    eager = GeneratorBatch(c, 2, seed=SEED)
    eager.SetGraphs(False)
    for b in (graphed, eager):
        b.Prefill(0, *prompt(c, 70))
        b.Prefill(1, *prompt(c, 71))
    n = noises(c, 2, 3)
    assert all(np.array_equal(x, y) for x, y in zip(graphed.Step(n), eager.Step(n)))
    long = prompt(c, 72, rows=150)
    for b in (graphed, eager):
        b.Prefill(0, *long)
    for k in range(2):
        n = noises(c, 2, 4 + k)
        a, b_ = graphed.Step(n), eager.Step(n)
        assert np.array_equal(a[0], b_[0]) and np.array_equal(a[1], b_[1]), f"step {k}"
    graphed.close()
    eager.close()


def test_batch_errors(cuda):
    c = config()
    batch = GeneratorBatch(c, 2, seed=SEED)
    batch.Prefill(0, *prompt(c, 1))
    with pytest.raises(VxError, match="slot 1 has no room"):
        batch.Step(noises(c, 2, 0))
    with pytest.raises(VxError, match="no such slot"):
        batch.Prefill(2, *prompt(c, 1))
    latents, _ = batch.Step(noises(c, 2, 0), active=[1, 0])
    assert latents[0].any()
    batch.close()
    with pytest.raises(VxError):
        GeneratorBatch(c, 0, seed=SEED)
