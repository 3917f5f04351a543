"""GPU parity of the screen-space AA ops (dressi_antialias /
dressi_antialias_grad) against the reference's golden outputs and the C
restatement: the forward and the image transpose BIT-EXACT, the vertex
gradient (float atomics) within 1e-4 abs + 1e-3 rel."""

import os

import numpy as np
import pytest

from conftest import GOLDEN
import scenes as S

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def T(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)


def npy(t):
    return t.detach().cpu().numpy()


def assert_bitexact(gpu, cpu, what):
    g, c = bits(gpu), bits(cpu)
    if not np.array_equal(g, c):
        bad = np.argwhere(g != c)
        i = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatching words, first at "
                             f"{i}: gpu={np.asarray(gpu)[i]!r} "
                             f"cpu={np.asarray(cpu)[i]!r}")


def test_golden_aa_small(cuda, port):
    from opendressi_b200 import ops

    g = np.load(os.path.join(GOLDEN, "aa_small.npz"))
    w, h = 48, 40
    clip, faces = S.random_triangles(11, 40, max(w, h), spread=1.1,
                                     w_range=(0.3, 2.5))
    clip[:2, 3] = -clip[:2, 3]
    vft = port.vertex_faces_tex(faces, clip.shape[0])
    img, tri = T(g["img"], cuda), T(g["tri"], cuda)
    c, f = T(clip, cuda), T(faces, cuda)
    assert_bitexact(npy(ops.antialias(img, tri, c, f)), g["aa"], "AntiAlias")
    gi, gc0 = ops.antialias_grad(T(g["gy"], cuda), img, tri, c, f)
    assert_bitexact(npy(gi), g["gimg"], "AntiAliasBwdImg")
    np.testing.assert_allclose(npy(gc0), g["gclip0"], atol=1e-4, rtol=1e-3)
    _, gc8 = ops.antialias_grad(T(g["gy"], cuda), img, tri, c, f,
                                vft=T(vft, cuda), seed=3.0, n_samples=8,
                                want_img=False)
    np.testing.assert_allclose(npy(gc8), g["gclip8"], atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("seed,w,h,nc,n_samples", [
    (31, 16, 16, 1, 0), (32, 33, 17, 3, 8), (33, 64, 48, 4, 5),
    (34, 1, 1, 1, 0), (35, 130, 70, 2, 8)])
def test_antialias_random_matches_port(cuda, port, seed, w, h, nc, n_samples):
    from opendressi_b200 import ops

    rng = np.random.default_rng(seed)
    clip, faces = S.random_triangles(seed, 60, max(w, h), spread=1.2,
                                     w_range=(0.2, 3.0))
    clip[:3, 3] = -clip[:3, 3]      # behind the camera
    faces[5] = faces[6]             # duplicate face
    faces[7, 1] = faces[7, 0]       # repeated vertex
    nv = clip.shape[0]
    attr = rng.random((nv, nc)).astype(np.float32)
    img = port.rasterize_hard(clip, attr, faces, w, h)
    if nc == 1:
        img = img[..., 0]
    tri = port.rasterize_face_id(clip, faces, w, h)
    vft = port.vertex_faces_tex(faces, nv)
    gy = rng.standard_normal(img.shape).astype(np.float32)
    sd = float(rng.integers(0, 50))
    c, f = T(clip, cuda), T(faces, cuda)
    assert_bitexact(npy(ops.antialias(T(img, cuda), T(tri, cuda), c, f)),
                    port.antialias(img, tri, clip, faces), "AntiAlias")
    gi, gc = ops.antialias_grad(T(gy, cuda), T(img, cuda), T(tri, cuda), c, f,
                                vft=T(vft, cuda), seed=sd,
                                n_samples=n_samples)
    assert_bitexact(npy(gi), port.antialias_bwd_img(gy, tri, clip, faces),
                    "AntiAliasBwdImg")
    np.testing.assert_allclose(
        npy(gc), port.antialias_bwd_vtx(gy, img, tri, clip, faces, vft, sd,
                                        n_samples), atol=1e-4, rtol=1e-3)


def test_antialias_views_batched(cuda, port):
    from opendressi_b200 import ops

    w, h = 40, 36
    _, faces = S.random_triangles(40, 50, 40)
    imgs, tris, clips, gys = [], [], [], []
    rng = np.random.default_rng(4)
    for v in range(3):
        c = S.random_triangles(41 + v, 50, 40)[0]
        clips.append(c)
        imgs.append(port.rasterize_hard(c, np.ones(c.shape[0], np.float32),
                                        faces, w, h)[..., 0])
        tris.append(port.rasterize_face_id(c, faces, w, h))
        gys.append(rng.standard_normal((h, w)).astype(np.float32))
    out = ops.antialias(T(np.stack(imgs), cuda), T(np.stack(tris), cuda),
                        T(np.stack(clips), cuda), T(faces, cuda))
    _, gc = ops.antialias_grad(T(np.stack(gys), cuda), T(np.stack(imgs), cuda),
                               T(np.stack(tris), cuda),
                               T(np.stack(clips), cuda), T(faces, cuda),
                               want_img=False)
    for v in range(3):
        assert_bitexact(npy(out[v]), port.antialias(imgs[v], tris[v],
                                                    clips[v], faces),
                        f"view {v}")
        np.testing.assert_allclose(
            npy(gc[v]), port.antialias_bwd_vtx(gys[v], imgs[v], tris[v],
                                               clips[v], faces,
                                               np.zeros((1, clips[v].shape[0]),
                                                        np.float32), 0.0, 0),
            atol=1e-4, rtol=1e-3)


def test_antialias_index_error(cuda):
    import torch
    from opendressi_b200 import ops
    from opendressi_b200._native import DressiError

    clip, faces = S.random_triangles(5, 4, 16)
    bad = faces.copy()
    bad[2, 1] = 1e6
    tri = torch.zeros((16, 16), device=cuda)
    with pytest.raises(DressiError):
        ops.antialias(torch.zeros((16, 16), device=cuda), tri,
                      T(clip, cuda), T(bad, cuda))
        ops.check_status()


@pytest.mark.parametrize("wild", [False, True])
def test_antialias_mask_matches_port(cuda, port, wild):
    """0/1 masks take the equal-value shortcut; a view with a face whose
    screen coordinates are huge turns it off. Bit-exact either way."""
    from opendressi_b200 import ops

    w, h = 70, 50
    clip, faces = S.random_triangles(77, 80, max(w, h), spread=1.0,
                                     w_range=(0.5, 2.0))
    if wild:
        clip[0, 0] = 1e30 * clip[0, 3]
    nv = clip.shape[0]
    mask = port.rasterize_hard(clip, np.ones(nv, np.float32), faces, w,
                               h)[..., 0]
    tri = port.rasterize_face_id(clip, faces, w, h)
    out = ops.antialias(T(mask, cuda), T(tri, cuda), T(clip, cuda),
                        T(faces, cuda))
    assert_bitexact(npy(out), port.antialias(mask, tri, clip, faces),
                    "AntiAlias mask")
