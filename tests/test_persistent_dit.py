"""The persistent DiT patch kernel on a B200.

One cooperative kernel runs the whole Euler/CFG loop of a patch (9 DiT
evaluations of the 12-layer DiT, dit_in/dit_out, the CFG-Zero* updates).
Checked against the oracle's restatement of the reference's arithmetic
(oracle/model.py) with the same limits as the per-kernel path, against that
per-kernel path itself, and for bit-for-bit repeatability (graph replay,
eager launch, a second generator). The kernel's split reductions sum in a
fixed order, so repeated runs must agree exactly.
"""

import numpy as np
import pytest

from oracle.model import OracleGenerator
from voxcpm_b200 import _lib
from voxcpm_b200.generator import Generator, released_config, small_config
from voxcpm_b200.kernels import DeviceError

from _util import rel_l2

pytestmark = pytest.mark.gpu

LATENT_LIMIT = 2e-2    # as in test_generator.py (the per-kernel path)
STOP_ATOL = 5e-3
STATE_LIMIT = 2e-2
# The persistent and per-kernel paths round to bf16 at the same points and
# differ only in float32 summation order; over 9 evaluations x 12 layers the
# latents stay within this relative L2 of each other.
PATHS_LIMIT = 1e-2


def dit_config():
    c = released_config()
    c.lm.layers = 1
    c.residual_lm.layers = 1
    c.max_length = 64
    return c


def inputs(config, seed):
    rng = np.random.default_rng(seed)
    p, f = config.patch_size, config.feat_dim
    mu = rng.normal(0, 1, 2 * config.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (p, f)).astype(np.float32)
    x = rng.normal(0, 1, (p, f)).astype(np.float32)
    return mu, cond, x


@pytest.mark.parametrize("checkpoint,cache_type", [
    (_lib.CHECKPOINT_Q8, _lib.CACHE_F32),
    (_lib.CHECKPOINT_BF16, _lib.CACHE_F32),
    (_lib.CHECKPOINT_Q8, _lib.CACHE_BF16),
])
def test_persistent_patch(cuda, checkpoint, cache_type):
    c = dit_config()
    q8 = checkpoint == _lib.CHECKPOINT_Q8
    gen = Generator(c, seed=7, checkpoint=checkpoint, cache_type=cache_type)
    assert gen.persistent()
    mu, cond, noise = inputs(c, 2)
    assert DeviceError() == 0
    latent = gen.DitPatch(mu, cond, noise, 10, 2.0)
    assert DeviceError() == 0, "a bounded wait of the persistent kernel expired"
    again = gen.DitPatch(mu, cond, noise, 10, 2.0)
    gen.SetGraphs(False)
    eager = gen.DitPatch(mu, cond, noise, 10, 2.0)
    assert np.array_equal(latent, again), "graph replays differ"
    assert np.array_equal(latent, eager), "graph replay differs from the eager launch"
    gen.SetPersistent(False)
    assert not gen.persistent()
    per_kernel = gen.DitPatch(mu, cond, noise, 10, 2.0)
    ref = OracleGenerator(c, seed=7, q8=q8, bf16_cache=cache_type == _lib.CACHE_BF16)
    latent_ref = ref.dit_patch(mu, cond, noise, 10, 2.0)
    e_ref = rel_l2(latent, latent_ref)
    e_paths = rel_l2(latent, per_kernel)
    print(f"persistent vs oracle {e_ref:.3e}, vs per-kernel {e_paths:.3e}, "
          f"per-kernel vs oracle {rel_l2(per_kernel, latent_ref):.3e}")
    assert e_ref < LATENT_LIMIT
    assert e_paths < PATHS_LIMIT
    gen.close()


def test_persistent_patch_other_schedules(cuda):
    """Other step counts and guidance scales (schedule re-upload), and a
    second generator with the same seed gives the same bits."""
    c = dit_config()
    gen = Generator(c, seed=5)
    twin = Generator(c, seed=5)
    ref = OracleGenerator(c, seed=5)
    mu, cond, noise = inputs(c, 4)
    for timesteps, cfg in [(4, 1.5), (10, 2.0), (2, 3.0)]:
        latent = gen.DitPatch(mu, cond, noise, timesteps, cfg)
        assert np.array_equal(latent, twin.DitPatch(mu, cond, noise, timesteps, cfg))
        err = rel_l2(latent, ref.dit_patch(mu, cond, noise, timesteps, cfg))
        print(f"timesteps {timesteps} cfg {cfg}: vs oracle {err:.3e}")
        assert err < LATENT_LIMIT
    assert DeviceError() == 0
    gen.close()
    twin.close()


def prompt(config, seed, rows=9, audio=(8,)):
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, config.vocab, rows).astype(np.int32)
    audio_mask = np.zeros(rows, np.int32)
    audio_mask[list(audio)] = 1
    text_mask = 1 - audio_mask
    feats = np.zeros((rows, config.patch_size, config.feat_dim), np.float32)
    feats[list(audio)] = rng.normal(0, 1, (len(audio), config.patch_size, config.feat_dim))
    return tokens, text_mask, audio_mask, feats


def test_persistent_steps(cuda):
    """Whole generation steps (one CUDA graph each, the persistent patch
    inside) against the oracle."""
    c = dit_config()
    c.vocab = 64
    hidden = c.lm.hidden
    gen = Generator(c, seed=11)
    assert gen.persistent()
    ref = OracleGenerator(c, seed=11)
    p = prompt(c, 5)
    gen.Prefill(*p)
    ref.prefill(*p)
    rng = np.random.default_rng(9)
    for k in range(2):
        noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        latent, stop = gen.Step(noise, 10, 2.0)
        latent_r, stop_r = ref.step(noise, 10, 2.0)
        e_lat = rel_l2(latent, latent_r)
        e_stop = float(np.max(np.abs(stop - stop_r)))
        e_res = rel_l2(gen.State("residual_hidden", hidden), ref.residual_hidden)
        print(f"step {k}: latent {e_lat:.3e} stop |d| {e_stop:.3e} residual {e_res:.3e}")
        assert e_lat < LATENT_LIMIT and e_stop < STOP_ATOL and e_res < STATE_LIMIT
    assert DeviceError() == 0
    gen.close()


def test_persistent_unsupported_shape(cuda):
    """A DiT of another shape keeps the per-kernel path."""
    c = small_config()
    c.dit.intermediate = 2048
    gen = Generator(c, seed=1)
    assert not gen.persistent()
    with pytest.raises(_lib.VxError):
        gen.SetPersistent(True)
    gen.SetPersistent(False)
    gen.close()


@pytest.mark.parametrize("cache_type", [_lib.CACHE_BF16, _lib.CACHE_F32])
def test_persistent_stacks_match_per_kernel_steps(cuda, cache_type):
    """Steps with the persistent DiT and one-row LM stacks against the same
    steps on the per-kernel path (the small configuration: released widths,
    two layers per stack), and against the oracle."""
    from voxcpm_b200.generator import small_config

    c = small_config()
    hidden = c.lm.hidden
    fast = Generator(c, seed=21, cache_type=cache_type)
    slow = Generator(c, seed=21, cache_type=cache_type)
    slow.SetPersistent(False)
    ref = OracleGenerator(c, seed=21, bf16_cache=cache_type == _lib.CACHE_BF16)
    p = prompt(c, 6, rows=12, audio=(5, 11))
    for g in (fast, slow):
        g.Prefill(*p)
    ref.prefill(*p)
    rng = np.random.default_rng(3)
    for k in range(3):
        noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        latent_f, stop_f = fast.Step(noise, 10, 2.0)
        latent_s, stop_s = slow.Step(noise, 10, 2.0)
        latent_r, stop_r = ref.step(noise, 10, 2.0)
        e_paths = rel_l2(latent_f, latent_s)
        e_lm = rel_l2(fast.State("lm_output", hidden), slow.State("lm_output", hidden))
        e_res = rel_l2(fast.State("residual_hidden", hidden), slow.State("residual_hidden", hidden))
        e_ref = rel_l2(latent_f, latent_r)
        e_lm_ref = rel_l2(fast.State("lm_output", hidden), ref.lm_output)
        print(f"step {k}: persistent vs per-kernel latent {e_paths:.3e} lm output {e_lm:.3e} "
              f"residual {e_res:.3e}; vs oracle latent {e_ref:.3e} lm output {e_lm_ref:.3e}")
        # States pass through FSQ, whose level flips (1/9 steps) feed the
        # residual LM: they get the state limit, the latent the tighter one.
        assert e_paths < PATHS_LIMIT and e_lm < STATE_LIMIT and e_res < STATE_LIMIT
        assert e_ref < LATENT_LIMIT and e_lm_ref < STATE_LIMIT
        assert float(np.max(np.abs(stop_f - stop_r))) < STOP_ATOL
    assert DeviceError() == 0
    fast.close()
    slow.close()


def test_aborted_patch_reports_device_timeout(cuda):
    """The regular DiT patch entry reports a launch whose bounded wait ran
    out (the stall test hook: one thread waits 20 ms for a word nothing
    sets, then aborts the launch) as VX_DEVICE_TIMEOUT; the error state is
    cleared and the next patch gives the same latent as before."""
    c = dit_config()
    gen = Generator(c, seed=11)
    gen.SetGraphs(False)  # the hook is read at launch, not baked into a graph
    rng = np.random.default_rng(8)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    before = gen.DitPatch(mu, cond, noise, 10, 2.0)
    lib = _lib.load()
    try:
        lib.vx_set_dit_stall_for_tests(20_000_000)
        with pytest.raises(_lib.VxError) as failure:
            gen.DitPatch(mu, cond, noise, 10, 2.0)
    finally:
        lib.vx_set_dit_stall_for_tests(0)
    assert failure.value.status == _lib.VX_DEVICE_TIMEOUT
    assert DeviceError() == 0
    after = gen.DitPatch(mu, cond, noise, 10, 2.0)
    assert np.array_equal(after, before)
    gen.close()


def test_persistent_kernels_at_fewer_ctas(cuda):
    """The persistent DiT and stack kernels split their work by the grid
    they get: capped at their minimum of 128 CTAs, a patch and steps match
    the oracle with the same limits and the uncapped kernels within the
    paths' limit."""
    lib = _lib.load()
    c = small_config()
    hidden = c.lm.hidden
    full = Generator(c, seed=31)
    lib.vx_set_persistent_max_ctas(128)
    try:
        capped = Generator(c, seed=31)
        ref = OracleGenerator(c, seed=31)
        mu, cond, noise = inputs(c, 9)
        latent_c = capped.DitPatch(mu, cond, noise, 10, 2.0)
        latent_f = full.DitPatch(mu, cond, noise, 10, 2.0)
        e_ref = rel_l2(latent_c, ref.dit_patch(mu, cond, noise, 10, 2.0))
        e_paths = rel_l2(latent_c, latent_f)
        print(f"patch at 128 CTAs: vs oracle {e_ref:.3e}, vs full grid {e_paths:.3e}")
        assert e_ref < LATENT_LIMIT and e_paths < PATHS_LIMIT
        p = prompt(c, 4, rows=10, audio=(9,))
        for g in (capped, full):
            g.Prefill(*p)
        ref.prefill(*p)
        rng = np.random.default_rng(8)
        for k in range(2):
            step_noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
            latent_c, stop_c = capped.Step(step_noise, 10, 2.0)
            latent_f, _ = full.Step(step_noise, 10, 2.0)
            latent_r, stop_r = ref.step(step_noise, 10, 2.0)
            e_lm = rel_l2(capped.State("lm_output", hidden), ref.lm_output)
            print(f"step {k} at 128 CTAs: latent vs oracle {rel_l2(latent_c, latent_r):.3e} "
                  f"vs full grid {rel_l2(latent_c, latent_f):.3e}, lm output vs oracle {e_lm:.3e}")
            assert rel_l2(latent_c, latent_r) < LATENT_LIMIT and rel_l2(latent_c, latent_f) < PATHS_LIMIT
            assert e_lm < STATE_LIMIT and float(np.max(np.abs(stop_c - stop_r))) < STOP_ATOL
        assert DeviceError() == 0
        capped.close()
    finally:
        lib.vx_set_persistent_max_ctas(0)
    full.close()


def test_persistent_kernels_without_the_cooperative_attribute(cuda):
    """Launched without the cooperative attribute (for profilers), the same
    grid on an idle GPU gives the same bits as the cooperative launch."""
    lib = _lib.load()
    c = small_config()
    mu, cond, noise = inputs(c, 12)
    coop = Generator(c, seed=41)
    p = prompt(c, 5, rows=10, audio=(9,))
    coop.Prefill(*p)
    step_noise = np.random.default_rng(2).normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    expected_patch = coop.DitPatch(mu, cond, noise, 10, 2.0)
    expected_step = coop.Step(step_noise, 10, 2.0)
    lib.vx_set_persistent_cooperative(0)
    try:
        plain = Generator(c, seed=41)
        plain.Prefill(*p)
        assert np.array_equal(plain.DitPatch(mu, cond, noise, 10, 2.0), expected_patch)
        latent, stop = plain.Step(step_noise, 10, 2.0)
        assert np.array_equal(latent, expected_step[0]) and np.array_equal(stop, expected_step[1])
        assert DeviceError() == 0
        plain.close()
    finally:
        lib.vx_set_persistent_cooperative(1)
    coop.close()
