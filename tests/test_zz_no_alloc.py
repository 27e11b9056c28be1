"""The allocation-free DiT patch entry (vx_generator_dit_patch_static) on a
B200: through the C ABI, against the regular entry (vx_generator_dit_patch),
on two calls in a row. Collected last; also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest

from voxcpm_b200 import _lib
from voxcpm_b200.generator import Generator, released_config

from _util import rel_l2

pytestmark = pytest.mark.gpu

# Both entries run the same kernel with the same summation order; the limit
# is the per-kernel path's latent tolerance, far above what they differ by.
LIMIT = 1e-2


def test_dit_patch_static_matches_regular_entry(cuda):
    import torch

    c = released_config()
    c.lm.layers = 1
    c.residual_lm.layers = 1
    c.max_length = 64
    gen = Generator(c, seed=7)
    assert gen.persistent()
    rng = np.random.default_rng(2)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    # The regular entry (also prepares the 10-step schedule).
    regular = gen.DitPatch(mu, cond, noise, 10, 2.0)

    lib = _lib.load()
    mu_d = torch.from_numpy(mu).cuda()
    cond_d = torch.from_numpy(cond).cuda()
    noise_d = torch.from_numpy(noise).cuda()
    latent_d = torch.empty(c.patch_size * c.feat_dim, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for call in range(2):
        latent_d.fill_(float("nan"))
        torch.cuda.synchronize()
        _lib.check(lib.vx_generator_dit_patch_static(
            ctypes.c_void_p(gen._handle), mu_d.data_ptr(), cond_d.data_ptr(), noise_d.data_ptr(),
            10, ctypes.c_float(2.0), latent_d.data_ptr()))
        latent = latent_d.cpu().numpy().reshape(c.patch_size, c.feat_dim)
        err = rel_l2(latent, regular)
        print(f"call {call}: rel L2 vs the regular entry {err:.3e}, "
              f"bit-identical {np.array_equal(latent, regular)}")
        assert np.all(np.isfinite(latent))
        assert err < LIMIT
    gen.close()


def test_dit_patch_static_needs_prepared_schedule(cuda):
    import torch

    c = released_config()
    c.lm.layers = 1
    c.residual_lm.layers = 1
    c.max_length = 64
    gen = Generator(c, seed=1)
    lib = _lib.load()
    buf = torch.zeros(4096, dtype=torch.float32, device="cuda")
    status = lib.vx_generator_dit_patch_static(ctypes.c_void_p(gen._handle), buf.data_ptr(), buf.data_ptr(),
                                               buf.data_ptr(), 7, ctypes.c_float(2.0), buf.data_ptr())
    assert status == _lib.VX_INVALID
    gen.close()
