"""GPU parity of the indexed-access ops (csrc/faces.cu) against the C
restatement (pinned bit-exact to the reference in test_oracle_faces.py):
ScreenCoord, LookupFaces and its transpose, FaceFetch and both backwards,
all BIT-EXACT (one thread per output, the reference's loop order);
out-of-range ids reported through the status word."""

import numpy as np
import pytest

from opendressi_b200 import scene

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def T(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)


def npy(t):
    return t.detach().cpu().numpy()


def test_screen_coord(cuda, port):
    from opendressi_b200 import _native as N
    from opendressi_b200 import ops

    for w, h in [(1, 2), (7, 5), (1024, 768)]:
        assert np.array_equal(bits(npy(ops.screen_coord(w, h, cuda))),
                              bits(port.screen_coord(w, h)))
    with pytest.raises(N.DressiError, match="non-uniform"):
        ops.screen_coord(1, 1, cuda)


@pytest.mark.parametrize("level", [2, 5])
def test_lookup_faces_bitexact(cuda, port, level):
    from opendressi_b200 import ops

    sc = scene.silhouette_scene(level=level, n_views=1, res=16, seed=level)
    vf = port.vertex_faces_tex(sc.faces_f, sc.n_verts)
    rng = np.random.default_rng(level)
    for n in (1, 2, 4):
        attr = rng.standard_normal((sc.n_verts, n)).astype(np.float32)
        for k in range(3):
            out = npy(ops.lookup_faces(T(attr, cuda), T(sc.faces_f, cuda), k))
            assert np.array_equal(bits(out),
                                  bits(port.lookup_faces(attr, sc.faces_f,
                                                         k)))
            gy = rng.standard_normal(out.shape).astype(np.float32)
            g = npy(ops.lookup_faces_grad(T(gy, cuda), T(sc.faces_f, cuda),
                                          T(vf, cuda), k))
            assert np.array_equal(bits(g), bits(port.lookup_faces_bwd(
                gy, sc.faces_f, vf, k)))


@pytest.mark.parametrize("res,n_samples,radius,seed",
                         [(64, 0, 0.0, 0.0), (64, 4, 1.5, 3.0),
                          (257, 9, 3.0, 11.0), (1024, 0, 0.0, 0.0),
                          (1024, 8, 2.0, 5.0)])
def test_face_fetch_bitexact(cuda, port, res, n_samples, radius, seed):
    from opendressi_b200 import ops

    sc = scene.silhouette_scene(level=4, n_views=1, res=res, seed=3)
    clip = port.transform_clip(sc.pos0, sc.mvps[0])
    prj = [port.lookup_faces(clip, sc.faces_f, k) for k in range(3)]
    idx = port.rasterize_face_id(clip, sc.faces_f, res, res)
    rng = np.random.default_rng(res + n_samples)
    n = 3
    attr = rng.standard_normal((sc.n_faces, n)).astype(np.float32)
    gy = rng.standard_normal((res, res, n)).astype(np.float32)
    out = npy(ops.face_fetch(T(attr, cuda), T(idx, cuda)))
    assert np.array_equal(bits(out), bits(port.face_fetch(attr, idx)))
    g = npy(ops.face_fetch_grad(T(gy, cuda), T(idx, cuda),
                                *[T(p, cuda) for p in prj], seed, radius,
                                n_samples))
    assert np.array_equal(bits(g), bits(port.face_fetch_bwd(
        gy, idx, *prj, seed, radius, n_samples)))
    assert np.count_nonzero(g) > 0


def test_index_out_of_range_reports_status(cuda, port):
    from opendressi_b200 import _native as N
    from opendressi_b200 import ops

    sc = scene.silhouette_scene(level=2, n_views=1, res=16, seed=1)
    faces = sc.faces_f.copy()
    faces[3, 1] = float(sc.n_verts + 5)
    attr = np.ones((sc.n_verts, 2), np.float32)
    with pytest.raises(N.DressiError, match="out of range"):
        ops.lookup_faces(T(attr, cuda), T(faces, cuda), 1)
        ops.check_status()
    vf = port.vertex_faces_tex(sc.faces_f, sc.n_verts)
    vf[0, 0] = float(sc.n_faces + 2)
    with pytest.raises(N.DressiError, match="out of range"):
        ops.lookup_faces_grad(T(np.ones((sc.n_faces, 2), np.float32), cuda),
                              T(sc.faces_f, cuda), T(vf, cuda), 0)
        ops.check_status()
