"""Pins the C restatement of the PBR shading graph (oracle.c, PBR shading
section: examples/common/pbr_graph.cpp:47-138 without normal mapping, the
differentiable split-sum IBL of ibl.cpp:22-60) against the compiled
reference driving BuildPbrShade itself: per-pixel G-buffer leaves of a
sphere, w x h material textures read at the pixel centres, the IBL maps of
a random environment, Mean L1 / L2 loss. The render is BIT-EXACT; the loss
and the gradients (albedo, metallic-roughness, and the environment through
EquirectSample / IrradianceConv / PrefilterConv / pooling) agree within
1e-4 abs + 1e-3 rel -- the hand-written backward follows the reference
autodiff's op rules, only its sums run in another order."""

import numpy as np
import pytest

from opendressi_b200 import scene


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _inputs(seed, w=32, h=32):
    gn, gp, mask, frame = scene.sphere_gbuffer(w, h, seed=seed)
    rng = np.random.default_rng(seed)
    alb = rng.random((h, w, 3)).astype(np.float32)
    mr = np.stack([rng.random((h, w)), rng.uniform(0.02, 1.05, (h, w)),
                   rng.random((h, w))], -1).astype(np.float32)
    ao = rng.uniform(0.5, 1, (h, w, 3)).astype(np.float32)
    em = (rng.random((h, w, 3)) * 0.05).astype(np.float32)
    env = scene.ibl_environment(64, 32, seed=seed)
    tgt = (rng.random((h, w, 3)) * 0.8).astype(np.float32)
    return gn, gp, mask, frame, alb, mr, ao, em, env, tgt


@pytest.mark.parametrize("seed,levels,loss_kind", [(0, 6, 1), (1, 5, 2),
                                                   (2, 2, 1)])
def test_pbr_shade_matches_reference(port, ref, seed, levels, loss_kind):
    gn, gp, mask, frame, alb, mr, ao, em, env, tgt = _inputs(seed)
    r = ref.pbr_shade_grad(gn, gp, mask, alb, mr, ao, em, frame, env, levels,
                           32, 32, 64, tgt, loss_kind)
    lut = port.brdf_lut(32, 32, 64)
    p = port.pbr_shade_grad(gn, gp, mask, alb, mr, ao, em, frame, env, levels,
                            lut, tgt, loss_kind)
    assert np.array_equal(bits(p[0]), bits(r[0]))
    assert p[1] == pytest.approx(r[1], rel=1e-5)
    for a, b in zip(p[2:], r[2:]):
        np.testing.assert_allclose(a, b, atol=1e-4, rtol=1e-3)
    # the gradients are not trivially small
    assert np.abs(r[2]).max() > 1e-5 and np.abs(r[4]).max() > 1e-5


def test_pbr_shade_gradient_matches_finite_differences(port):
    """The restatement's own backward against central differences of its
    loss (L2; a few albedo / metallic / env entries with the largest
    gradients). Roughness is left to the reference pin: it also selects the
    BRDF-LUT texel, through which the reference's TextureBilinear passes no
    gradient, so differences include a term the gradient by design has
    not."""
    gn, gp, mask, frame, alb, mr, ao, em, env, tgt = _inputs(3, 16, 16)
    lut = port.brdf_lut(32, 32, 64)
    args = lambda a, m, e: (gn, gp, mask, a, m, ao, em, frame, e, 5, lut,
                            tgt, 2)
    _, _, ga, gm, ge = port.pbr_shade_grad(*args(alb, mr, env))
    eps = 2e-3
    gm_metal = np.zeros_like(gm)
    gm_metal[..., 2] = gm[..., 2]
    for arr, grad, which in ((alb, ga, 0), (mr, gm_metal, 1), (env, ge, 2)):
        for i in np.argsort(-np.abs(grad.ravel()))[:3]:
            hi = [alb.copy(), mr.copy(), env.copy()]
            lo = [alb.copy(), mr.copy(), env.copy()]
            hi[which].flat[i] += eps
            lo[which].flat[i] -= eps
            lp = port.pbr_shade_grad(*args(*hi))[1]
            lm = port.pbr_shade_grad(*args(*lo))[1]
            num = (lp - lm) / (2 * eps)
            assert abs(grad.flat[i] - num) <= 1e-6 + 2e-2 * abs(num), (which, i)
