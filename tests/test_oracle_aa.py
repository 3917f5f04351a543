"""Pins the C restatement of the screen-space anti-aliasing path
(oracle.c: orc_antialias*, orc_aa_*) before it is trusted: the reference's
own AntiAlias tests re-expressed (tests/test_antialias.cpp:153-273 of the
reference), golden fixtures written by the reference itself
(tests/golden/make_golden.py: aa_small, aa_sphere_64), and the compiled
reference on fresh seeded inputs where it is built."""

import os

import numpy as np
import pytest

from conftest import GOLDEN
import scenes as S

from opendressi_b200 import scene

K_SCREEN = 16


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def clip16(sx, sy, z, w=1.0):
    """Clip() of the reference's AA tests, evaluated in float32."""
    f = np.float32
    s = f(K_SCREEN)
    return [(f(sx) / s * f(2) - f(1)) * f(w), (f(sy) / s * f(2) - f(1)) * f(w),
            f(z) * f(w), f(w)]


def fixed_buffers(port, verts, faces, attr=None):
    """FixedBufferAa: img / tri rasterized once from the unperturbed clip."""
    clip = np.asarray(verts, np.float32)
    faces = np.asarray(faces, np.float32)
    if attr is None:
        attr = np.ones(clip.shape[0], np.float32)
    img = port.rasterize_hard(clip, np.asarray(attr, np.float32), faces,
                              K_SCREEN, K_SCREEN)[..., 0]
    tri = port.rasterize_face_id(clip, faces, K_SCREEN, K_SCREEN)
    vft = port.vertex_faces_tex(faces, clip.shape[0])
    return clip, faces, img, tri, vft


TRI = [clip16(4.3, 3.8, 0.5), clip16(12.4, 5.2, 0.5), clip16(5.1, 12.6, 0.5)]


def test_aa_forward_interior_boundary_background(port):
    clip, faces, mask, tri, _ = fixed_buffers(port, TRI, [[0, 1, 2]])
    out = port.antialias(mask, tri, clip, faces)
    n_in = n_bd = n_bg = 0
    for y in range(1, K_SCREEN - 1):
        for x in range(1, K_SCREEN - 1):
            m = mask[y, x]
            uniform = bool(np.all(mask[y - 1:y + 2, x - 1:x + 2] == m))
            v = out[y, x]
            if uniform:
                assert abs(v - m) <= 1e-6
                if m > 0.5:
                    n_in += 1
                else:
                    n_bg += 1
            else:
                assert 0.0 <= v <= 1.0
                if 1e-6 < v < 1 - 1e-6:
                    n_bd += 1
    assert n_in > 0 and n_bd > 0 and n_bg > 0


def _mean_sq_loss(aa, target):
    d = target - aa
    return float(np.mean(d.astype(np.float64) ** 2))


def test_aa_grad_img_matches_finite_differences(port):
    clip, faces, img, tri, _ = fixed_buffers(port, TRI, [[0, 1, 2]])
    target = (0.1 + 0.6 * (np.arange(K_SCREEN * K_SCREEN) % 7) / 6.0).astype(
        np.float32).reshape(K_SCREEN, K_SCREEN)
    aa = port.antialias(img, tri, clip, faces)
    gy = (-2.0 * (target - aa) / aa.size).astype(np.float32)
    analytic = port.antialias_bwd_img(gy, tri, clip, faces)
    h = 1e-3
    for i in range(0, img.size, 7):
        p, m = img.copy(), img.copy()
        p.flat[i] += h
        m.flat[i] -= h
        num = (_mean_sq_loss(port.antialias(p, tri, clip, faces), target) -
               _mean_sq_loss(port.antialias(m, tri, clip, faces), target)) / (2 * h)
        assert abs(analytic.flat[i] - num) <= 1e-5 + 1e-3 * abs(num)


def test_aa_grad_vtx_matches_finite_differences(port):
    verts = [clip16(4.3, 3.8, 0.5), clip16(12.4, 5.2, 0.5, 1.3),
             clip16(5.1, 12.6, 0.5)]
    clip, faces, img, tri, vft = fixed_buffers(port, verts, [[0, 1, 2]])
    target = np.full((K_SCREEN, K_SCREEN), 0.35, np.float32)
    aa = port.antialias(img, tri, clip, faces)
    gy = (-2.0 * (target - aa) / aa.size).astype(np.float32)
    analytic = port.antialias_bwd_vtx(gy, img, tri, clip, faces, vft, 0.0, 0)
    h = 1e-3
    for i in range(clip.size):
        p, m = clip.copy(), clip.copy()
        p.flat[i] += h
        m.flat[i] -= h
        num = (_mean_sq_loss(port.antialias(img, tri, p, faces), target) -
               _mean_sq_loss(port.antialias(img, tri, m, faces), target)) / (2 * h)
        assert abs(analytic.flat[i] - num) <= 2e-3 + 2e-2 * abs(num), i
        if i % 4 == 2:
            assert analytic.flat[i] == 0.0


def test_aa_occlusion_front_edge_owns_gradient(port):
    verts = [clip16(-40, -40, 0.8), clip16(100, -40, 0.8), clip16(-40, 100, 0.8),
             clip16(5.2, 4.7, 0.2), clip16(11.6, 6.3, 0.2), clip16(6.4, 11.8, 0.2)]
    clip, faces, img, tri, vft = fixed_buffers(
        port, verts, [[0, 1, 2], [3, 4, 5]], [0.2, 0.2, 0.2, 0.9, 0.9, 0.9])
    gy = np.full(img.shape, 1.0 / img.size, np.float32)  # d Mean / d aa
    g = port.antialias_bwd_vtx(gy, img, tri, clip, faces, vft, 0.0, 0)
    assert float(np.abs(g[:3]).sum()) == 0.0
    assert float(np.abs(g[3:]).sum()) > 1e-4


def test_hash_to_unit_range_and_spread(port):
    u = np.array([port.hash_to_unit(f, s, 3, 2) for f in range(64)
                  for s in range(8)])
    assert u.min() >= 0.0 and u.max() < 1.0
    assert 0.4 < u.mean() < 0.6


# ---------------------------------------------------------------- goldens

def _aa_small_inputs(port):
    w, h = 48, 40
    clip, faces = S.random_triangles(11, 40, max(w, h), spread=1.1,
                                     w_range=(0.3, 2.5))
    clip[:2, 3] = -clip[:2, 3]
    nv = clip.shape[0]
    rng = np.random.default_rng(12)
    attr = rng.random((nv, 3)).astype(np.float32)
    vft = port.vertex_faces_tex(faces, nv)
    return clip, faces, attr, vft, w, h


def test_golden_aa_small(port):
    g = golden("aa_small")
    clip, faces, attr, vft, w, h = _aa_small_inputs(port)
    img = port.rasterize_hard(clip, attr, faces, w, h)
    tri = port.rasterize_face_id(clip, faces, w, h)
    assert np.array_equal(bits(img), bits(g["img"]))
    assert np.array_equal(bits(tri), bits(g["tri"]))
    assert np.array_equal(bits(port.antialias(img, tri, clip, faces)),
                          bits(g["aa"]))
    assert np.array_equal(bits(port.antialias_bwd_img(g["gy"], tri, clip,
                                                      faces)), bits(g["gimg"]))
    assert np.array_equal(
        bits(port.antialias_bwd_vtx(g["gy"], img, tri, clip, faces, vft, 0.0,
                                    0)), bits(g["gclip0"]))
    assert np.array_equal(
        bits(port.antialias_bwd_vtx(g["gy"], img, tri, clip, faces, vft, 3.0,
                                    8)), bits(g["gclip8"]))


def test_golden_aa_sphere_64(port):
    g = golden("aa_sphere_64")
    sc = scene.silhouette_scene(level=3, n_views=2, res=64, seed=1)
    vft = port.vertex_faces_tex(sc.faces_f, sc.n_verts)
    targets = port.aa_targets(sc.target_pos, sc.faces_f, sc.mvps, 64)
    assert np.array_equal(bits(targets), bits(g["targets"]))
    _, grad0, _ = port.aa_silhouette_loss_grad(sc.pos0, sc.faces_f, vft,
                                               sc.mvps, targets, 64,
                                               int(g["n_samples"]), 0.0)
    assert np.array_equal(bits(grad0), bits(g["grad0"]))
    trace, pos = port.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                        targets, 64, int(g["n_samples"]),
                                        float(g["lr"]), len(g["trace"]))
    assert np.array_equal(bits(trace), bits(g["trace"]))
    assert np.array_equal(bits(pos), bits(g["pos"]))


# ---------------------------------------- compiled reference (if built)

@pytest.mark.parametrize("seed,n_samples", [(21, 0), (22, 8), (23, 3)])
def test_port_matches_reference_aa_random(port, ref, seed, n_samples):
    rng = np.random.default_rng(seed)
    w, h = int(rng.integers(17, 60)), int(rng.integers(17, 60))
    clip, faces = S.random_triangles(seed, 50, max(w, h), spread=1.2,
                                     w_range=(0.2, 3.0))
    clip[:3, 3] = -clip[:3, 3]
    faces[5] = faces[6]
    faces[7, 1] = faces[7, 0]
    nv = clip.shape[0]
    nc = int(rng.integers(1, 5))
    attr = rng.random((nv, nc)).astype(np.float32)
    img = port.rasterize_hard(clip, attr, faces, w, h)
    if nc == 1:
        img = img[..., 0]
    tri = port.rasterize_face_id(clip, faces, w, h)
    vft = ref.vertex_faces_tex(faces, nv)
    gy = rng.standard_normal(img.shape).astype(np.float32)
    sd = float(rng.integers(0, 100))
    aa_r, gi_r, gc_r = ref.antialias(img, tri, clip, faces, vft, sd,
                                     n_samples, gy)
    assert np.array_equal(bits(port.antialias(img, tri, clip, faces)),
                          bits(aa_r))
    assert np.array_equal(bits(port.antialias_bwd_img(gy, tri, clip, faces)),
                          bits(gi_r))
    assert np.array_equal(
        bits(port.antialias_bwd_vtx(gy, img, tri, clip, faces, vft, sd,
                                    n_samples)), bits(gc_r))


def test_port_matches_reference_aa_run(port, ref):
    sc = scene.silhouette_scene(level=2, n_views=3, res=40, seed=7)
    vft = ref.vertex_faces_tex(sc.faces_f, sc.n_verts)
    targets = port.aa_targets(sc.target_pos, sc.faces_f, sc.mvps, 40)
    t1, p1, _, _ = ref.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                         targets, 40, 8, 1e-2, 4, threads=1)
    t3, p3, _, _ = ref.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                         targets, 40, 8, 1e-2, 4, threads=3)
    tp, pp = port.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                    targets, 40, 8, 1e-2, 4, threads=2)
    np.testing.assert_allclose(t3, t1, rtol=1e-5)
    np.testing.assert_allclose(tp, t1, rtol=1e-5)
    np.testing.assert_allclose(pp, p1, atol=1e-5)
