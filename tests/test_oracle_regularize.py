"""Pins the C restatement of the silhouette optimizer's regulariser
(oracle.c, regularisers section; examples/silhouette_optimization/
run.cpp:407-420 over f_ops.cpp:1983-2181 and SumAll f_ops.cpp:1119-1149)
against the compiled reference: mesh tables and regularised gradients
BIT-EXACT on icospheres and on non-manifold triangle soups (isolated
vertices, degenerate faces, edges shared by more than two faces); the full
regularised silhouette runs (HardSoftRas and AA) within the run tolerance."""

import numpy as np
import pytest

from opendressi_b200 import scene


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _soup(seed):
    rng = np.random.default_rng(seed)
    nv = int(rng.integers(8, 300))
    f = rng.integers(0, nv, (int(rng.integers(4, 600)), 3))
    f = f[(f[:, 0] != f[:, 1]) & (f[:, 1] != f[:, 2]) & (f[:, 0] != f[:, 2])]
    pos = rng.standard_normal((nv, 3)).astype(np.float32)
    pos[1] = pos[0]   # zero-area faces through vertices 0 and 1
    return pos, f.astype(np.float32), rng


@pytest.mark.parametrize("level", [1, 3])
def test_mesh_tables_match_reference(port, ref, level):
    sc = scene.silhouette_scene(level=level, n_views=1, res=16, seed=level)
    vn_r, fa_r = ref.mesh_tables(sc.faces_f, sc.n_verts)
    assert np.array_equal(port.vertex_neighbors_tex(sc.faces_f, sc.n_verts),
                          vn_r)
    assert np.array_equal(port.face_neighbors_tex(sc.faces_f), fa_r)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_mesh_tables_match_reference_soup(port, ref, seed):
    pos, f, _ = _soup(seed)
    vn_r, fa_r = ref.mesh_tables(f, pos.shape[0])
    assert np.array_equal(port.vertex_neighbors_tex(f, pos.shape[0]), vn_r)
    assert np.array_equal(port.face_neighbors_tex(f), fa_r)


@pytest.mark.parametrize("level,lap,nrm", [(2, 0.15, 0.4), (3, 0.5, 0.5),
                                           (5, 0.15, 0.4), (3, 0.0, 0.0)])
def test_regularized_grad_matches_reference(port, ref, level, lap, nrm):
    sc = scene.silhouette_scene(level=level, n_views=1, res=16, seed=level)
    rng = np.random.default_rng(level)
    pos = (sc.pos0 + 0.01 * rng.standard_normal(sc.pos0.shape)).astype(
        np.float32)
    g = (1e-3 * rng.standard_normal(pos.shape)).astype(np.float32)
    assert np.array_equal(bits(port.regularized_grad(pos, sc.faces_f, g, lap,
                                                     nrm)),
                          bits(ref.regularized_grad(pos, sc.faces_f, g, lap,
                                                    nrm)))


@pytest.mark.parametrize("seed", [3, 4, 5])
def test_regularized_grad_matches_reference_soup(port, ref, seed):
    pos, f, rng = _soup(seed)
    g = rng.standard_normal(pos.shape).astype(np.float32)
    assert np.array_equal(bits(port.regularized_grad(pos, f, g, 0.3, 0.7)),
                          bits(ref.regularized_grad(pos, f, g, 0.3, 0.7)))


def test_regularizer_terms_definition(port):
    """Laplacian weight alone: the added term is pos minus the mean of the
    vertex's neighbours, scaled from its own RMS to the data RMS."""
    sc = scene.silhouette_scene(level=2, n_views=1, res=16, seed=1)
    rng = np.random.default_rng(9)
    g = rng.standard_normal(sc.pos0.shape).astype(np.float32)
    out = port.regularized_grad(sc.pos0, sc.faces_f, g, 1.0, 0.0)
    vn = port.vertex_neighbors_tex(sc.faces_f, sc.n_verts)
    mean = np.stack([sc.pos0[vn[:, v][vn[:, v] >= 0].astype(int)].mean(0)
                     for v in range(sc.n_verts)])
    lap = sc.pos0 - mean
    rms = lambda x: np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-24)
    np.testing.assert_allclose(out - g, lap * (rms(g) / rms(lap)), rtol=1e-4,
                               atol=1e-5)


def test_port_matches_reference_regularized_runs(port, ref):
    sc = scene.silhouette_scene(level=2, n_views=3, res=40, seed=11)
    vft = ref.vertex_faces_tex(sc.faces_f, sc.n_verts)
    targets = np.stack([(port.rasterize_face_id(
        port.transform_clip(sc.target_pos, m), sc.faces_f, 40, 40)
        > 0).astype(np.float32) for m in sc.mvps])
    kw = dict(laplacian=0.15, normal=0.4)
    t1, p1, _, _ = ref.silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                      targets, 40, sc.radius_px, sc.sigma,
                                      1e-2, 4, threads=1, **kw)
    t3, p3, _, _ = ref.silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                      targets, 40, sc.radius_px, sc.sigma,
                                      1e-2, 4, threads=3, **kw)
    tp, pp = port.silhouette_run(sc.pos0, sc.faces_f, sc.mvps, targets, 40,
                                 sc.radius_px, sc.sigma, 1e-2, 4, threads=2,
                                 **kw)
    _, p0, _, _ = ref.silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                     targets, 40, sc.radius_px, sc.sigma,
                                     1e-2, 4, threads=1)
    np.testing.assert_allclose(t3, t1, rtol=1e-5)
    np.testing.assert_allclose(p3, p1, atol=1e-5)
    np.testing.assert_allclose(tp, t1, rtol=1e-5)
    np.testing.assert_allclose(pp, p1, atol=1e-5)
    assert np.abs(p1 - p0).max() > 1e-3   # the regulariser acted

    aa_t = port.aa_targets(sc.target_pos, sc.faces_f, sc.mvps, 40)
    kw = dict(laplacian=0.5, normal=0.5)
    a1, q1, _, _ = ref.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps,
                                         aa_t, 40, 8, 1e-2, 4, threads=1, **kw)
    ap, qp = port.aa_silhouette_run(sc.pos0, sc.faces_f, vft, sc.mvps, aa_t,
                                    40, 8, 1e-2, 4, threads=2, **kw)
    np.testing.assert_allclose(ap, a1, rtol=1e-5)
    np.testing.assert_allclose(qp, q1, atol=1e-5)


@pytest.mark.parametrize("n_px,nc", [(1, 1), (200, 3), (256, 4), (257, 1),
                                     (1000, 2), (30726, 3)])
def test_sum_all_matches_reference(port, ref, n_px, nc):
    rng = np.random.default_rng(n_px + nc)
    x = (rng.standard_normal((n_px, nc)) *
         np.exp(rng.uniform(-8, 8, (n_px, 1)))).astype(np.float32)
    assert bits(port.sum_all(x)) == bits(ref.sum_all(x))


def test_regularizer_ops_compose(port):
    """The composite equals its parts (VertexNeighborMean, the two NC
    stages, SumAll) assembled as run.cpp:407-420 does."""
    sc = scene.silhouette_scene(level=3, n_views=1, res=16, seed=4)
    rng = np.random.default_rng(4)
    pos = (sc.pos0 + 0.02 * rng.standard_normal(sc.pos0.shape)).astype(
        np.float32)
    g = (1e-2 * rng.standard_normal(pos.shape)).astype(np.float32)
    f, nv = sc.faces_f, sc.n_verts
    glap = pos - port.vertex_neighbor_mean(
        pos, port.vertex_neighbors_tex(f, nv))
    gnrm = port.nc_vertex_grad(
        port.nc_face_term(pos, f, port.face_neighbors_tex(f)), pos, f,
        port.vertex_faces_tex(f, nv))
    inv = np.float32(1.0) / np.float32(nv * 3)

    def rms(x):
        return np.sqrt(port.sum_all(x * x) * inv + np.float32(1e-24))

    s_lap = rms(g) / rms(glap) * np.float32(0.15)
    s_nrm = rms(g) / rms(gnrm) * np.float32(0.4)
    exp = (g + glap * s_lap) + gnrm * s_nrm
    assert np.array_equal(bits(port.regularized_grad(pos, f, g, 0.15, 0.4)),
                          bits(exp))
