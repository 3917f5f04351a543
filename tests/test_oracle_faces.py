"""Pins the C restatement of the paper's indexed-access ops (oracle.c,
indexed-access section; f_ops.cpp:1490-1799) against the compiled
reference: ScreenCoord, LookupFaces and its exact transpose (icospheres and
non-manifold soups with repeated corners), FaceFetch and both of its
backwards (the exact bbox scan and the hashed edge samples, several seeds,
radii and sample counts) BIT-EXACT; plus the reference's own known-answer
and finite-difference tests (tests/test_softras.cpp:155-207)."""

import numpy as np
import pytest

from opendressi_b200 import scene


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _soup(seed):
    rng = np.random.default_rng(seed)
    nv = int(rng.integers(6, 120))
    f = rng.integers(0, nv, (int(rng.integers(3, 300)), 3))
    f = f[(f[:, 0] != f[:, 1]) & (f[:, 1] != f[:, 2]) & (f[:, 0] != f[:, 2])]
    f = np.concatenate([f, f[:2]])   # duplicated faces
    return nv, f.astype(np.float32), rng


def test_screen_coord(port, ref):
    # ({1, 1} is a uniform size, which the reference rejects)
    for w, h in [(1, 2), (5, 3), (64, 17)]:
        out = port.screen_coord(w, h)
        assert np.array_equal(bits(out), bits(ref.screen_coord(w, h)))
        assert out[h - 1, w - 1, 0] == w - 0.5 and out[0, 0, 1] == 0.5


@pytest.mark.parametrize("case", ["ico2", "ico4", "soup0", "soup1"])
def test_lookup_faces_matches_reference(port, ref, case):
    if case.startswith("ico"):
        sc = scene.silhouette_scene(level=int(case[3]), n_views=1, res=16,
                                    seed=1)
        nv, faces = sc.n_verts, sc.faces_f
        rng = np.random.default_rng(3)
    else:
        nv, faces, rng = _soup(int(case[4]))
    vf = ref.vertex_faces_tex(faces, nv)
    for n in (1, 3, 4):
        attr = rng.standard_normal((nv, n)).astype(np.float32)
        for k in range(3):
            o_p = port.lookup_faces(attr, faces, k)
            gy = rng.standard_normal(o_p.shape).astype(np.float32)
            o_r, g_r = ref.lookup_faces(attr, faces, vf, k, gy=gy)
            assert np.array_equal(bits(o_p), bits(o_r))
            assert np.array_equal(bits(port.lookup_faces_bwd(gy, faces, vf,
                                                             k)), bits(g_r))


def _id_scene(level, res, seed):
    from oracle import pyoracle  # noqa: F401  (port fixture builds it)

    sc = scene.silhouette_scene(level=level, n_views=1, res=res, seed=seed)
    return sc


@pytest.mark.parametrize("n_samples,radius,seed", [(0, 0.0, 0.0),
                                                   (4, 1.5, 3.0),
                                                   (9, 3.0, 17.0),
                                                   (1, 0.5, 123456.0)])
def test_face_fetch_matches_reference(port, ref, n_samples, radius, seed):
    sc = _id_scene(3, 48, 2)
    clip = port.transform_clip(sc.pos0, sc.mvps[0])
    prj = [port.lookup_faces(clip, sc.faces_f, k) for k in range(3)]
    idx = port.rasterize_face_id(clip, sc.faces_f, 48, 48)
    rng = np.random.default_rng(n_samples)
    for n in (1, 2, 3):
        attr = rng.standard_normal((sc.n_faces, n)).astype(np.float32)
        gy = rng.standard_normal((48, 48, n)).astype(np.float32)
        o_r, g_r = ref.face_fetch(attr, idx, *prj, seed, radius, n_samples,
                                  gy=gy)
        assert np.array_equal(bits(port.face_fetch(attr, idx)), bits(o_r))
        g_p = port.face_fetch_bwd(gy, idx, *prj, seed, radius, n_samples)
        assert np.array_equal(bits(g_p), bits(g_r))
        if n_samples:
            assert np.count_nonzero(g_p) > 0


def test_face_fetch_edge_cases_match_reference(port, ref):
    """Ids past the table, a face behind the camera (w <= 1e-6) and a
    degenerate (zero-length edge) face."""
    rng = np.random.default_rng(5)
    nf, w, h = 4, 9, 7
    idx = rng.integers(0, nf + 3, (h, w)).astype(np.float32)
    attr = rng.standard_normal((nf, 2)).astype(np.float32)
    prj = [np.zeros((nf, 4), np.float32) for _ in range(3)]
    for k in range(3):
        prj[k][:, :2] = rng.uniform(-1, 1, (nf, 2))
        prj[k][:, 3] = 1.0
    prj[0][1, 3] = 0.0                      # behind the camera
    prj[1][2] = prj[0][2]                   # degenerate edge
    gy = rng.standard_normal((h, w, 2)).astype(np.float32)
    for ns, rad in [(0, 0.0), (6, 2.0)]:
        o_r, g_r = ref.face_fetch(attr, idx, *prj, 1.0, rad, ns, gy=gy)
        assert np.array_equal(bits(port.face_fetch(attr, idx)), bits(o_r))
        assert np.array_equal(bits(port.face_fetch_bwd(gy, idx, *prj, 1.0,
                                                       rad, ns)), bits(g_r))


def test_face_fetch_forward_known_answer(port):
    """tests/test_softras.cpp:174-202 (FaceFetchForward)."""
    attr = np.array([[1, 2], [3, 4]], np.float32)
    idx = np.array([0, 1, 1, 2, 2, 0, 1, 0, 0, 2, 2, 1],
                   np.float32).reshape(3, 4)
    out = port.face_fetch(attr, idx)
    for p, i in enumerate(idx.ravel()):
        f = int(i + 0.5) - 1
        exp = attr[f] if f >= 0 else np.zeros(2, np.float32)
        assert np.array_equal(out.reshape(-1, 2)[p], exp)


def test_face_fetch_exact_backward_is_the_adjoint(port):
    """n_samples = 0: <gy, FaceFetch(a)> = <FaceFetchBwd(gy), a>."""
    sc = _id_scene(3, 64, 4)
    clip = port.transform_clip(sc.pos0, sc.mvps[0])
    prj = [port.lookup_faces(clip, sc.faces_f, k) for k in range(3)]
    idx = port.rasterize_face_id(clip, sc.faces_f, 64, 64)
    rng = np.random.default_rng(1)
    a = rng.standard_normal((sc.n_faces, 3)).astype(np.float32)
    gy = rng.standard_normal((64, 64, 3)).astype(np.float32)
    lhs = np.sum(gy.astype(np.float64) * port.face_fetch(a, idx))
    rhs = np.sum(port.face_fetch_bwd(gy, idx, *prj, 0.0, 0.0, 0)
                 .astype(np.float64) * a)
    assert lhs == pytest.approx(rhs, rel=1e-5)


def test_lookup_faces_grad_matches_finite_differences(port, ref):
    """tests/test_softras.cpp:155-172: loss = sum_k Mean(Sigmoid(
    LookupFaces(clip, k) * (0.7 + 0.3 k))) over two faces; the exact
    transpose against central differences (step 1e-3, rel 2e-2, abs
    2e-3)."""
    clip = np.array([[4.3, 3.8, 0.5, 1.0], [12.4, 5.2, 0.5, 1.3],
                     [5.1, 12.6, 0.5, 1.0], [11.2, 12.1, 0.5, 1.0]],
                    np.float32)
    clip[:, :2] = clip[:, :2] / 8.0 - 1.0   # pixel positions -> NDC at 16^2
    faces = np.array([[0, 1, 2], [1, 3, 2]], np.float32)
    vf = ref.vertex_faces_tex(faces, 4)

    def loss(c):
        s = 0.0
        for k in range(3):
            t = port.lookup_faces(c, faces, k).astype(np.float64)
            s += np.mean(1.0 / (1.0 + np.exp(-t * (0.7 + 0.3 * k))))
        return s

    g = np.zeros((4, 4), np.float32)
    for k in range(3):
        t = port.lookup_faces(clip, faces, k).astype(np.float64)
        a = 0.7 + 0.3 * k
        sg = 1.0 / (1.0 + np.exp(-t * a))
        gy = (sg * (1.0 - sg) * a / t.size).astype(np.float32)
        g += port.lookup_faces_bwd(gy, faces, vf, k)
    eps = 1e-3
    for v in range(4):
        for c in range(4):
            cp, cm = clip.copy(), clip.copy()
            cp[v, c] += eps
            cm[v, c] -= eps
            fd = (loss(cp) - loss(cm)) / (2 * eps)
            assert abs(g[v, c] - fd) <= 2e-3 + 2e-2 * abs(fd), (v, c)
