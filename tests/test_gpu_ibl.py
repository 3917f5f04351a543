"""GPU parity of the split-sum IBL ops (csrc/ibl.cu) against the C
restatement (pinned bit-exact to the reference in test_oracle_ibl.py).
The reference's transcendentals are the host libm's and CUDA's differ by a
few ulps (as the reference's own GLSL twins do), and the convolutions and
transposes sum in another order: outputs and gradients within 1e-4 abs +
1e-3 rel; AvgPool2x2 and its transpose BIT-EXACT."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = dict(atol=1e-4, rtol=1e-3)


def T(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)


def npy(t):
    return t.detach().cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _env(seed, w=64, h=32, n=3):
    rng = np.random.default_rng(seed)
    return (rng.random((h, w, n)) * 3).astype(np.float32), rng


@pytest.mark.parametrize("n", [1, 3, 4])
def test_equirect_sample_and_grad(cuda, port, n):
    from opendressi_b200 import ops

    env, rng = _env(n, n=n)
    dirs = rng.standard_normal((96, 80, 3)).astype(np.float32)
    dirs[0, :8] = 0.0
    gy = rng.standard_normal((96, 80, n)).astype(np.float32)
    out = ops.equirect_sample(T(env, cuda), T(dirs, cuda))
    np.testing.assert_allclose(npy(out), port.equirect_sample(env, dirs),
                               **TOL)
    g = ops.equirect_sample_grad(T(gy, cuda), T(dirs, cuda), 64, 32)
    np.testing.assert_allclose(npy(g), port.equirect_sample_bwd(gy, dirs, 64,
                                                                32), **TOL)


def test_irradiance_conv_and_grad(cuda, port):
    from opendressi_b200 import ops

    env, rng = _env(7)
    gy = rng.standard_normal((16, 32, 3)).astype(np.float32)
    np.testing.assert_allclose(npy(ops.irradiance_conv(T(env, cuda), 32,
                                                       16)),
                               port.irradiance_conv(env, 32, 16), **TOL)
    np.testing.assert_allclose(npy(ops.irradiance_conv_grad(T(gy, cuda), 64,
                                                            32)),
                               port.irradiance_conv_bwd(gy, 64, 32), **TOL)


@pytest.mark.parametrize("rough", [0.0, 0.25, 0.6, 1.0])
def test_prefilter_conv_and_grad(cuda, port, rough):
    from opendressi_b200 import ops

    env, rng = _env(8)
    gy = rng.standard_normal((16, 32, 3)).astype(np.float32)
    np.testing.assert_allclose(npy(ops.prefilter_conv(T(env, cuda), 32, 16,
                                                      rough)),
                               port.prefilter_conv(env, 32, 16, rough), **TOL)
    np.testing.assert_allclose(npy(ops.prefilter_conv_grad(T(gy, cuda), 64,
                                                           32, rough)),
                               port.prefilter_conv_bwd(gy, 64, 32, rough),
                               **TOL)


def test_brdf_lut(cuda, port):
    from opendressi_b200 import ops

    np.testing.assert_allclose(npy(ops.brdf_lut(64, 32, 128, cuda)),
                               port.brdf_lut(64, 32, 128), **TOL)


def test_avg_pool_bitexact(cuda, port):
    from opendressi_b200 import ops

    x, rng = _env(9, 128, 64, 3)
    assert np.array_equal(bits(npy(ops.avg_pool2x2(T(x, cuda)))),
                          bits(port.avg_pool2x2(x)))
    gy = rng.standard_normal((32, 64, 3)).astype(np.float32)
    assert np.array_equal(
        bits(npy(ops.avg_pool2x2_grad(T(gy, cuda)))),
        bits(np.repeat(np.repeat(gy * np.float32(0.25), 2, 0), 2, 1)))
