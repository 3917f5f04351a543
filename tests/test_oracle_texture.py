"""Pins the C restatement of the texture path (oracle.c, texturing section):
bilinear sampling and GatherByInverseUVBilinear against golden outputs of
the reference and the compiled reference itself (bit-exact); nearest
sampling / GatherByInverseUV by their GLSL definition (no reference CPU
kernel); the first-principles C2 mip path by adjoint and finite-difference
checks (no reference implementation exists)."""

import os

import numpy as np
import pytest

from conftest import GOLDEN

from opendressi_b200 import scene


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _gbuffer(port, sc, view, res):
    clip = port.transform_clip(sc.pos, sc.mvps[view])
    attr = np.concatenate([sc.uv, np.ones((sc.n_verts, 1), np.float32)], 1)
    return clip, port.rasterize_hard(clip, attr, sc.faces_f, res, res)


def test_golden_tex_small(port):
    g = np.load(os.path.join(GOLDEN, "tex_small.npz"))
    sc = scene.texture_scene(level=3, n_views=1, res=64, tex_size=64,
                             levels=6, seed=2)
    clip, gbuf = _gbuffer(port, sc, 0, 64)
    assert np.array_equal(bits(gbuf), bits(g["gbuf"]))
    inv_uv = port.rasterize_hard(port.uv_as_clip(sc.uv),
                                 port.screen_attr(clip, 64, 64), sc.faces_f,
                                 64, 64)
    assert np.array_equal(bits(inv_uv), bits(g["inv_uv"]))
    uv = np.ascontiguousarray(gbuf[..., :2])
    assert np.array_equal(bits(port.texture_bilinear(g["tex"], uv)),
                          bits(g["out"]))
    assert np.array_equal(bits(port.gather_inv_uv_bilinear(g["gy"], inv_uv,
                                                            uv)),
                          bits(g["gtex"]))


def test_nearest_texture_and_gather_definition(port):
    """Nearest = texel (floor(u W), floor(v H)) clamped; the gather hands a
    texel the gradient of a screen pixel that samples it."""
    rng = np.random.default_rng(5)
    tex = rng.random((8, 16, 2)).astype(np.float32)
    uv = rng.uniform(-0.2, 1.2, (40, 2)).astype(np.float32)
    out = port.texture_nearest(tex, uv)
    x = np.clip(np.floor(uv[:, 0] * 16).astype(int), 0, 15)
    y = np.clip(np.floor(uv[:, 1] * 8).astype(int), 0, 7)
    assert np.array_equal(out, tex[y, x])
    # inverse-UV table pointing every texel at the screen pixel that
    # samples it (identity mapping of a 16x8 screen)
    sh, sw = 8, 16
    ys, xs = np.mgrid[0:sh, 0:sw]
    uv_s = np.stack([(xs + 0.5) / sw, (ys + 0.5) / sh], -1).astype(np.float32)
    inv = np.stack([xs + 0.5, ys + 0.5, np.ones_like(xs), np.zeros_like(xs)],
                   -1).astype(np.float32)
    gy = rng.standard_normal((sh, sw, 2)).astype(np.float32)
    assert np.array_equal(port.gather_inv_uv(gy, inv, uv_s), gy)


def test_mip_fold_is_the_adjoint_of_mip_build(port):
    rng = np.random.default_rng(1)
    w, levels = 32, 6
    x = rng.standard_normal((w, w, 3)).astype(np.float32)
    y = rng.standard_normal(port.mip_floats(w, 3, levels)).astype(np.float32)
    lhs = float(np.dot(port.mip_build(x, levels).astype(np.float64),
                       y.astype(np.float64)))
    rhs = float(np.dot(x.ravel().astype(np.float64),
                       port.mip_fold(y, w, 3, levels)[:w * w * 3]
                       .astype(np.float64)))
    assert abs(lhs - rhs) <= 1e-4 * max(1.0, abs(lhs))


def test_trilinear_grad_is_the_adjoint(port):
    rng = np.random.default_rng(2)
    w, levels, npx = 32, 5, 300
    pyr = rng.standard_normal(port.mip_floats(w, 3, levels)).astype(np.float32)
    uv = rng.uniform(-0.1, 1.1, (npx, 2)).astype(np.float32)
    lod = rng.uniform(0.0, levels - 1.0, (npx,)).astype(np.float32)
    lod[:20] = 0.0
    g = rng.standard_normal((npx, 3)).astype(np.float32)
    lhs = float(np.dot(port.texture_trilinear(pyr, w, 3, levels, uv, lod)
                       .ravel().astype(np.float64), g.ravel()))
    rhs = float(np.dot(pyr.astype(np.float64),
                       port.texture_trilinear_grad(g, w, 3, levels, uv, lod)
                       .astype(np.float64)))
    assert abs(lhs - rhs) <= 1e-3 * max(1.0, abs(lhs))


def test_c2_grad_matches_finite_differences(port):
    sc = scene.texture_scene(level=2, n_views=2, res=32, tex_size=16,
                             levels=4, seed=4)
    rng = np.random.default_rng(6)
    targets = rng.random((2, 32, 32, 3)).astype(np.float32)
    tex = rng.random((16, 16, 3)).astype(np.float32)
    _, grad, _ = port.c2_loss_grad(tex, 4, sc.pos, sc.uv, sc.faces_f, sc.mvps,
                                   targets, 32)
    idx = np.argsort(-np.abs(grad.ravel()))[:12]
    h = 1e-2
    for i in idx:
        p, m = tex.copy(), tex.copy()
        p.flat[i] += h
        m.flat[i] -= h
        lp, _, _ = port.c2_loss_grad(p, 4, sc.pos, sc.uv, sc.faces_f, sc.mvps,
                                     targets, 32)
        lm, _, _ = port.c2_loss_grad(m, 4, sc.pos, sc.uv, sc.faces_f, sc.mvps,
                                     targets, 32)
        num = (lp - lm) / (2 * h)
        assert abs(grad.flat[i] - num) <= 1e-5 + 1e-2 * abs(num), i


def test_c2_run_decreases_loss(port):
    sc = scene.texture_scene(level=3, n_views=2, res=48, tex_size=32,
                             levels=5, seed=7)
    gt = scene.checker_texture(3, 32, 8)
    # the renders of the target texture are the targets
    _, _, targets = port.c2_loss_grad(gt, 5, sc.pos, sc.uv, sc.faces_f,
                                      sc.mvps,
                                      np.zeros((2, 48, 48, 3), np.float32),
                                      48, want_pred=True)
    trace, tex = port.c2_run(np.full((32, 32, 3), 0.5, np.float32), 5, sc.pos,
                             sc.uv, sc.faces_f, sc.mvps, targets, 48, 5e-2,
                             15)
    assert trace[-1] < 0.5 * trace[0]


@pytest.mark.parametrize("seed", [31, 32])
def test_port_matches_reference_texture_bilinear(port, ref, seed):
    rng = np.random.default_rng(seed)
    sc = scene.texture_scene(level=3, n_views=1, res=40, tex_size=32,
                             levels=5, seed=seed)
    clip, gbuf = _gbuffer(port, sc, 0, 40)
    uv = np.ascontiguousarray(gbuf[..., :2])
    inv_uv = ref.rasterize_hard(port.uv_as_clip(sc.uv),
                                port.screen_attr(clip, 40, 40), sc.faces_f,
                                32, 32)
    n = int(rng.integers(1, 5))
    tex = rng.random((32, 32, n)).astype(np.float32)
    gy = rng.standard_normal((40, 40, n)).astype(np.float32)
    out_r, g_r = ref.texture_bilinear(tex, uv, inv_uv, gy)
    assert np.array_equal(bits(port.texture_bilinear(tex, uv)), bits(out_r))
    assert np.array_equal(bits(port.gather_inv_uv_bilinear(gy, inv_uv, uv)),
                          bits(g_r))
