"""Pins the C restatement of the split-sum IBL ops (oracle.c, split-sum
IBL section; f_ops.cpp:2785-3415 with ibl_math.h) against the compiled
reference: EquirectSample and its banded map transpose (one and several
bands, background directions), IrradianceConv / PrefilterConv (rough 0,
mid, 1) forward and transpose, BrdfIntegrationLut and AvgPool2x2 with its
transpose, all BIT-EXACT (both call the host libm for the
transcendentals). Plus the identities the reference documents: a constant
environment L0 gives irradiance L0 and prefilter L0."""

import numpy as np
import pytest


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _env(seed, w=32, h=16, n=3):
    rng = np.random.default_rng(seed)
    return (rng.random((h, w, n)) * 3).astype(np.float32), rng


@pytest.mark.parametrize("dh,dw", [(12, 10), (64, 48)])
def test_equirect_sample_matches_reference(port, ref, dh, dw):
    env, rng = _env(dh)
    dirs = rng.standard_normal((dh, dw, 3)).astype(np.float32)
    dirs[0, 0] = 0.0          # background: no sample
    dirs[1, 1] = (0, 1, 0)    # pole
    dirs[2, 2] = (-1, 0, 0)   # atan2 seam
    gy = rng.standard_normal((dh, dw, 3)).astype(np.float32)
    out_r, g_r = ref.equirect_sample(env, dirs, gy)
    assert np.array_equal(bits(port.equirect_sample(env, dirs)), bits(out_r))
    assert np.array_equal(bits(port.equirect_sample_bwd(gy, dirs, 32, 16)),
                          bits(g_r))


def test_irradiance_conv_matches_reference(port, ref):
    env, rng = _env(3)
    gy = rng.standard_normal((8, 16, 3)).astype(np.float32)
    out_r, g_r = ref.irradiance_conv(env, 16, 8, gy)
    assert np.array_equal(bits(port.irradiance_conv(env, 16, 8)), bits(out_r))
    assert np.array_equal(bits(port.irradiance_conv_bwd(gy, 32, 16)),
                          bits(g_r))


@pytest.mark.parametrize("rough", [0.0, 0.3, 1.0])
def test_prefilter_conv_matches_reference(port, ref, rough):
    env, rng = _env(4)
    gy = rng.standard_normal((8, 16, 3)).astype(np.float32)
    out_r, g_r = ref.prefilter_conv(env, 16, 8, rough, gy)
    assert np.array_equal(bits(port.prefilter_conv(env, 16, 8, rough)),
                          bits(out_r))
    assert np.array_equal(bits(port.prefilter_conv_bwd(gy, 32, 16, rough)),
                          bits(g_r))


def test_brdf_lut_and_pool_match_reference(port, ref):
    assert np.array_equal(bits(port.brdf_lut(32, 16, 64)),
                          bits(ref.brdf_lut(32, 16, 64)))
    x, rng = _env(5, 16, 8, 2)
    gy = rng.standard_normal((4, 8, 2)).astype(np.float32)
    out_r, g_r = ref.avg_pool2x2(x, gy)
    assert np.array_equal(bits(port.avg_pool2x2(x)), bits(out_r))
    assert np.array_equal(bits(np.repeat(np.repeat(gy * np.float32(0.25), 2,
                                                   0), 2, 1)), bits(g_r))


def test_constant_environment_identities(port):
    env = np.full((16, 32, 3), 2.5, np.float32)
    np.testing.assert_allclose(port.irradiance_conv(env, 16, 8), 2.5,
                               rtol=2e-2)
    for rough in (0.1, 0.6, 1.0):
        np.testing.assert_allclose(port.prefilter_conv(env, 16, 8, rough),
                                   2.5, rtol=1e-5)
