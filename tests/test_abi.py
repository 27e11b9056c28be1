"""The C ABI without a GPU: the library loads, exports every function that
include/*.h declares, its ctypes table covers them, and its host-side parts
(planning, tile sizes, seeded weights) behave."""

import re
import subprocess
from pathlib import Path

import numpy as np

import oracle
from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^VX_API\s+[^(;]*?\b(vx_\w+)\s*\(", text, re.MULTILINE))
    return names


def exported_symbols() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIBRARY)], check=True,
                         capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.split()}


def test_library_exports_every_declared_function():
    declared = declared_functions()
    assert len(declared) > 20
    exported = exported_symbols()
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # Nothing else leaks: the C ABI is the whole interface.
    extra = {s for s in exported if s.startswith("vx_")} - declared
    assert not extra, f"exported but not declared: {sorted(extra)}"


def test_ctypes_table_covers_the_header():
    assert declared_functions() <= set(_lib.SIGNATURES)
    lib = _lib.load()
    for name in _lib.SIGNATURES:
        getattr(lib, name)


def test_host_queries():
    lib = _lib.load()
    assert lib.vx_version().startswith(b"voxcpm_b200")
    # kernels/wmma_products.hpp:29-38: rows padded to 16.
    assert K.Q8TilesBytes(6144, 2048) == 6144 // 16 * 64 * 544 == 13_369_344
    assert K.Q8TilesBytes(72, 1024) == 5 * 32 * 544
    assert K.Bf16TilesBytes(2, 2048) == 1 * 64 * 1024


def test_planner():
    # Every plan covers the reduction with nonempty splits of at most 2048
    # columns and at most 8 CTAs per cluster.
    for rows in (1, 2, 5, 8, 11, 22, 32):
        for columns, out in ((1024, 2560), (2048, 1024), (4096, 1024), (1024, 8192), (6144, 2048),
                             (2048, 6144), (8192, 512), (64, 1024), (2048, 2)):
            for target in (0, 1, 4096):
                plan = K.PlanWmma(rows, columns, out, target)
                kb = columns // 32
                assert 1 <= plan.splits <= 8
                assert plan.blocks_per_split * 32 <= 2048
                assert plan.splits * plan.blocks_per_split >= kb
                assert (plan.splits - 1) * plan.blocks_per_split < kb
                assert plan.partial_floats == 0 and plan.counters == 0
    assert K.PlanWmma(22, 2048, 6144, 1).splits == 2  # fewest allowed splits
    assert K.PlanWmma(22, 48, 16).splits == 0          # in not a multiple of 32


def test_planner_33_to_128_rows():
    """33..64 and 65..128 rows of VoxCPM2's Q8_0 shapes take the measured
    row-split plans (variants 25-35: warps that share a group's activation
    tiles), each within the reduction's limits; a row-split variant has
    more warps than its groups and ways alone would give (host only)."""
    variants = K.ProductVariants()
    expected = {(48, 1024, 2560): (33, 1), (64, 2048, 1024): (32, 4), (64, 4096, 1024): (34, 4),
                (100, 1024, 8192): (30, 2), (128, 2048, 1024): (29, 4), (128, 4096, 1024): (30, 8),
                (128, 2048, 12288): (30, 4)}
    for (rows, columns, out), (variant, splits) in expected.items():
        plan = K.PlanWmma(rows, columns, out, 0)
        assert (plan.variant, plan.splits) == (variant, splits), (rows, columns, out)
        kb = columns // 32
        assert plan.splits * plan.blocks_per_split >= kb
        assert (plan.splits - 1) * plan.blocks_per_split < kb
        warps, groups, _, _ = variants[plan.variant]
        assert warps > groups  # two or four warps per group and way


def test_spread_planner():
    """Spread plans (host only; without a device the SM count is B200's 148):
    one CTA per panel at least, at most one per SM, every run at most one
    panel's reduction, scratch for two ends of every CTA's run and one
    counter per 128-row panel."""
    for fmt in (_lib.WEIGHTS_BF16, _lib.WEIGHTS_BF16_TILES, _lib.WEIGHTS_Q8_TILES):
        for rows in (1, 5, 22, 32):
            for columns, out in ((1024, 2560), (2048, 1024), (4096, 1024), (1024, 8192), (6144, 2048),
                                 (2048, 6144), (2048, 12288), (64, 1024), (2048, 2), (1024, 72)):
                plan = K.PlanSpread(fmt, rows, columns, out)
                kb = columns // 32
                panels = -(-out // 128)
                assert plan.variant == _lib.SPREAD_VARIANT, (fmt, rows, columns, out)
                assert panels <= plan.splits <= 148
                assert plan.blocks_per_split == -(-(panels * kb) // plan.splits) <= kb
                assert plan.counters == panels
                assert plan.partial_floats == plan.splits * 2 * 8 * 32 * 16
    # Config 0: 48 panels x 64 blocks over 148 CTAs, runs of 21 units.
    plan = K.PlanSpread(_lib.WEIGHTS_Q8_TILES, 22, 2048, 6144)
    assert (plan.splits, plan.blocks_per_split) == (148, 21)
    assert K.PlanSpread(_lib.WEIGHTS_Q8_TILES, 33, 2048, 6144).splits == 0  # more than 32 rows
    assert K.PlanSpread(_lib.WEIGHTS_Q8_TILES, 22, 48, 16).splits == 0      # in not a multiple of 32
    assert K.PlanSpread(7, 22, 2048, 6144).splits == 0                      # unknown format


def test_library_weights_match_the_oracle_restatement():
    """vx_random_* (product) and the oracle's restatement give identical bytes."""
    for seed, tensor, rows, columns in ((0, 0, 48, 256), (123456789, 77, 16, 2048), (5, 3, 1, 32)):
        assert np.array_equal(K.RandomQ8_0(seed, tensor, rows, columns),
                              oracle.random_q8_0(seed, tensor, rows, columns))
    for mean, std in ((0.0, 0.02), (1.0, 0.05)):
        assert np.array_equal(K.RandomBf16(9, 4, 100_000, mean, std), oracle.random_bf16(9, 4, 100_000, mean, std))
    # Large enough to use the library's worker threads.
    assert np.array_equal(K.RandomQ8_0(1, 2, 512, 8192), oracle.random_q8_0(1, 2, 512, 8192))


def test_invalid_arguments_fail_without_a_gpu():
    lib = _lib.load()
    status = lib.vx_random_q8_0(0, 0, 4, 33, 0.01, None)
    assert status == _lib.VX_INVALID
    assert b"vx_random_q8_0" in lib.vx_last_error()


def test_host_math_matches_the_oracle():
    """The library's host-side schedule, time embedding and rotary table
    (generator.cpp:39-80, transformer.cpp:20-45) equal the oracle's bit for
    bit: both are float32 restatements run on the same host."""
    import ctypes

    lib = _lib.load()
    for n in (1, 4, 10, 16, 25, 50):
        t = np.empty(n, np.float32)
        dt = np.empty(n, np.float32)
        ev = np.empty(n, np.int32)
        assert lib.vx_euler_schedule(n, 1.0, t.ctypes.data, dt.ctypes.data, ev.ctypes.data, n) == n
        ot, odt, oev = oracle.euler_schedule(n)
        assert np.array_equal(t, ot) and np.array_equal(dt, odt) and np.array_equal(ev.astype(bool), oev)
    for t_value in (0.0, 0.63, 0.9564344, 1.0):
        ours = np.empty(1024, np.float32)
        assert lib.vx_sinusoid(t_value, 1024, ours.ctypes.data) == 0
        assert np.array_equal(ours, oracle.sinusoid(t_value, 1024))
    factors = (1.0 + np.random.default_rng(3).random(64) * 3.0).astype(np.float64)
    ours = np.empty(64 * 128, np.float32)
    ref = np.empty(64 * 128, np.float32)
    assert lib.vx_rope_table(10000.0, 128, factors.ctypes.data, 1.0, 64, ours.ctypes.data) == 0
    oracle.lib().vxo_rope_table(10000.0, 128, factors.ctypes.data, 1.0, 64, ref.ctypes.data)
    assert np.array_equal(ours, ref)
    del ctypes


def test_audio_vae_arguments_fail_without_a_gpu():
    """The AudioVAE's C ABI rejects bad configurations and null handles
    before any device work (vx_audio_vae_*)."""
    import ctypes

    from voxcpm_b200.vae import default_vae_config, vae_config

    lib = _lib.load()
    c = default_vae_config()
    assert (c.latent_dim, c.decoder_dim, c.decoder_rate_count, c.out_sample_rate) == (64, 2048, 6, 48000)
    assert list(c.decoder_rates[:6]) == [8, 6, 5, 2, 2, 2]
    assert list(c.sr_bin_boundaries[:3]) == [20000, 30000, 40000] and c.sr_bin_boundary_count == 3
    for bad in (vae_config(64, 2048, ()), vae_config(6, 64, (2,)), vae_config(64, 36, (2, 2))):
        assert not lib.vx_audio_vae_create(ctypes.byref(bad), 0)
        assert b"AudioVAE" in lib.vx_last_error()
    assert not lib.vx_audio_vae_create(None, 0)
    assert lib.vx_audio_vae_decode_hop(None) == 0
    assert lib.vx_audio_vae_reset(None) == _lib.VX_INVALID
    samples = ctypes.c_size_t(0)
    assert lib.vx_audio_vae_collect(None, None, 0, ctypes.byref(samples)) == _lib.VX_INVALID
    lib.vx_audio_vae_destroy(None)
