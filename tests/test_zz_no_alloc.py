"""The allocation-free DiT patch entry (vx_generator_dit_patch_static) on a
B200: through the C ABI, against the regular entry (vx_generator_dit_patch),
on two calls in a row, for Q8_0 and bf16 checkpoints. Both entries run the
same persistent kernel with the same summation order, so the latents must be
identical bit for bit; the second call must leave the device's free memory
unchanged (the first may load the library's module, which holds the fixed
array); and a launch whose bounded wait runs out must be reported as
VX_DEVICE_TIMEOUT, not as success. Collected last; also passes alone in a
fresh process.
"""

import ctypes

import numpy as np
import pytest

from voxcpm_b200 import _lib
from voxcpm_b200 import kernels as K
from voxcpm_b200.generator import Generator, released_config

pytestmark = pytest.mark.gpu


def _small_released(checkpoint, seed):
    c = released_config()
    c.lm.layers = 1
    c.residual_lm.layers = 1
    c.max_length = 64
    return c, Generator(c, seed=seed, checkpoint=checkpoint)


def _inputs(c, seed):
    rng = np.random.default_rng(seed)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    return mu, cond, noise


def _static(lib, gen, mu_d, cond_d, noise_d, latent_d):
    return lib.vx_generator_dit_patch_static(
        ctypes.c_void_p(gen._handle), mu_d.data_ptr(), cond_d.data_ptr(), noise_d.data_ptr(),
        10, ctypes.c_float(2.0), latent_d.data_ptr())


@pytest.mark.parametrize("checkpoint", [_lib.CHECKPOINT_Q8, _lib.CHECKPOINT_BF16])
def test_dit_patch_static_matches_regular_entry(cuda, checkpoint):
    import torch

    c, gen = _small_released(checkpoint, seed=7)
    assert gen.persistent()
    mu, cond, noise = _inputs(c, 2)
    # The regular entry (also prepares the 10-step schedule).
    regular = gen.DitPatch(mu, cond, noise, 10, 2.0)

    lib = _lib.load()
    mu_d = torch.from_numpy(mu).cuda()
    cond_d = torch.from_numpy(cond).cuda()
    noise_d = torch.from_numpy(noise).cuda()
    latent_d = torch.empty(c.patch_size * c.feat_dim, dtype=torch.float32, device="cuda")
    # The inputs are written on torch's stream; the entry copies them on the
    # generator's own stream, so they must be complete first.
    torch.cuda.synchronize()
    for call in range(2):
        latent_d.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        _lib.check(_static(lib, gen, mu_d, cond_d, noise_d, latent_d))
        free_after = torch.cuda.mem_get_info()[0]
        latent = latent_d.cpu().numpy().reshape(c.patch_size, c.feat_dim)
        assert np.array_equal(latent, regular), f"call {call}: differs from the regular entry"
        if call == 1:
            assert free_after == free_before, (
                f"the second call changed free device memory by {free_before - free_after} bytes")
    assert K.DeviceError() == 0
    gen.close()


def test_dit_patch_static_reports_device_timeout(cuda):
    """A launch whose bounded wait runs out (the stall test hook: a wait on a
    word nothing sets, 20 ms) returns VX_DEVICE_TIMEOUT and clears the error
    state; the next call succeeds with the regular entry's latent."""
    import torch

    c, gen = _small_released(_lib.CHECKPOINT_Q8, seed=3)
    mu, cond, noise = _inputs(c, 5)
    regular = gen.DitPatch(mu, cond, noise, 10, 2.0)
    lib = _lib.load()
    mu_d = torch.from_numpy(mu).cuda()
    cond_d = torch.from_numpy(cond).cuda()
    noise_d = torch.from_numpy(noise).cuda()
    latent_d = torch.empty(c.patch_size * c.feat_dim, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    try:
        lib.vx_set_dit_stall_for_tests(20_000_000)
        status = _static(lib, gen, mu_d, cond_d, noise_d, latent_d)
    finally:
        lib.vx_set_dit_stall_for_tests(0)
    assert status == _lib.VX_DEVICE_TIMEOUT, lib.vx_last_error().decode()
    assert b"aborted" in lib.vx_last_error()
    assert K.DeviceError() == 0  # the entry read and cleared the error bits
    _lib.check(_static(lib, gen, mu_d, cond_d, noise_d, latent_d))
    latent = latent_d.cpu().numpy().reshape(c.patch_size, c.feat_dim)
    assert np.array_equal(latent, regular)
    gen.close()


def test_dit_patch_static_needs_prepared_schedule(cuda):
    import torch

    c, gen = _small_released(_lib.CHECKPOINT_Q8, seed=1)
    lib = _lib.load()
    buf = torch.zeros(4096, dtype=torch.float32, device="cuda")
    status = lib.vx_generator_dit_patch_static(ctypes.c_void_p(gen._handle), buf.data_ptr(), buf.data_ptr(),
                                               buf.data_ptr(), 7, ctypes.c_float(2.0), buf.data_ptr())
    assert status == _lib.VX_INVALID
    gen.close()
