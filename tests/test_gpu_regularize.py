"""GPU parity of the optimizer-side regulariser (VertexNeighborMean,
NormalConsistencyFaceTerm / VertexGrad, SumAll and the regularised gradient
of examples/silhouette_optimization/run.cpp:407-420) against the C
restatement, itself pinned bit-exact to the reference: every op BIT-EXACT;
inside the silhouette plans, the first regularised Adam step bit-exact from
the plan's own data gradient, and regularised runs within the run tolerance
(loss traces 1e-3 rel)."""

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


def _cases():
    out = []
    for lvl in (3, 5):
        sc = scene.silhouette_scene(level=lvl, n_views=1, res=16, seed=lvl)
        rng = np.random.default_rng(lvl)
        pos = (sc.pos0 + 0.02 * rng.standard_normal(sc.pos0.shape)).astype(
            np.float32)
        out.append((pos, sc.faces_f, rng))
    rng = np.random.default_rng(7)
    nv = 250
    f = rng.integers(0, nv, (500, 3))
    f = f[(f[:, 0] != f[:, 1]) & (f[:, 1] != f[:, 2]) & (f[:, 0] != f[:, 2])]
    pos = rng.standard_normal((nv, 3)).astype(np.float32)
    pos[1] = pos[0]   # degenerate faces
    out.append((pos, f.astype(np.float32), rng))
    return out


@pytest.mark.parametrize("case", [0, 1, 2])
def test_ops_bitexact(cuda, port, case):
    from opendressi_b200 import ops

    pos, f, rng = _cases()[case]
    nv = pos.shape[0]
    vn = ops.vertex_neighbors_tex(f, nv)
    fa = ops.face_neighbors_tex(f)
    vf = ops.vertex_faces_tex(f, nv)
    mean = ops.vertex_neighbor_mean(T(pos, cuda), T(vn, cuda))
    assert np.array_equal(bits(npy(mean)),
                          bits(port.vertex_neighbor_mean(pos, vn)))
    term = ops.normal_consistency_face_term(T(pos, cuda), T(f, cuda),
                                            T(fa, cuda))
    term_cpu = port.nc_face_term(pos, f, fa)
    assert np.array_equal(bits(npy(term)), bits(term_cpu))
    vg = ops.normal_consistency_vertex_grad(T(term_cpu, cuda), T(pos, cuda),
                                            T(f, cuda), T(vf, cuda))
    assert np.array_equal(bits(npy(vg)),
                          bits(port.nc_vertex_grad(term_cpu, pos, f, vf)))
    g = (1e-3 * rng.standard_normal(pos.shape)).astype(np.float32)
    for lap, nrm in [(0.15, 0.4), (0.5, 0.5), (0.0, 1.0)]:
        out = ops.regularized_grad(T(pos, cuda), T(f, cuda), T(g, cuda), lap,
                                   nrm)
        assert np.array_equal(bits(npy(out)),
                              bits(port.regularized_grad(pos, f, g, lap,
                                                         nrm))), (lap, nrm)


@pytest.mark.parametrize("n_px,nc", [(1, 1), (256, 4), (257, 3), (5000, 2),
                                     (122_883, 3)])
def test_sum_all_bitexact(cuda, port, n_px, nc):
    from opendressi_b200 import ops

    rng = np.random.default_rng(n_px)
    x = (rng.standard_normal((n_px, nc)) *
         np.exp(rng.uniform(-8, 8, (n_px, 1)))).astype(np.float32)
    assert bits(npy(ops.sum_all(T(x, cuda)))[0]) == bits(port.sum_all(x))


def test_table_index_out_of_range_reports_status(cuda):
    from opendressi_b200 import _native as N
    from opendressi_b200 import ops

    pos, f, _ = _cases()[0]
    vn = ops.vertex_neighbors_tex(f, pos.shape[0])
    vn[0, 5] = float(pos.shape[0] + 10)   # read would be out of range
    with pytest.raises(N.DressiError, match="out of range"):
        ops.vertex_neighbor_mean(T(pos, cuda), T(vn, cuda))
        ops.check_status()
    fa = ops.face_neighbors_tex(f)
    fa[3, 0] = 1e7
    with pytest.raises(N.DressiError, match="out of range"):
        ops.normal_consistency_face_term(T(pos, cuda), T(f, cuda),
                                         T(fa, cuda))
        ops.check_status()


def _targets(port, sc):
    return np.stack([(port.rasterize_face_id(
        port.transform_clip(sc.target_pos, m), sc.faces_f, sc.res, sc.res)
        > 0).astype(np.float32) for m in sc.mvps])


def _first_step_bitexact(plan, port, sc, lap, nrm, lr):
    """Positions after one plan step equal the C restatement's regulariser
    + in-graph Adam applied to the plan's own data gradient."""
    from opendressi_b200 import _native as N

    plan.step(1)
    g = plan.download(N.SLOT_GRAD).reshape(-1, 3)
    greg = port.regularized_grad(sc.pos0, sc.faces_f, g, lap, nrm)
    p = np.ascontiguousarray(sc.pos0, np.float32).copy()
    m, v = np.zeros_like(p), np.zeros_like(p)
    port.adam(p, m, v, 0.0, greg, lr)
    assert np.array_equal(bits(plan.download(N.SLOT_PARAM).reshape(-1, 3)),
                          bits(p))


def test_silhouette_plan_regularized(cuda, port):
    """Icosphere-4, 4 views at 256^2 with the example's HardSoftRas weights
    (0.15 / 0.4): first step bit-exact, 20-iteration trace vs the port."""
    from opendressi_b200 import _native as N
    from opendressi_b200.plans import SilhouettePlan

    sc = scene.silhouette_scene(level=4, n_views=4, res=256, seed=1)
    targets = _targets(port, sc)
    plan = SilhouettePlan.from_scene(sc, lr=1e-3, laplacian=0.15, normal=0.4)
    plan.upload(N.SLOT_PARAM, sc.pos0)
    plan.upload(N.SLOT_TARGET, targets)
    _first_step_bitexact(plan, port, sc, 0.15, 0.4, 1e-3)
    n = 20
    plan.step(n - 1)
    trace_cpu, pos_cpu = port.silhouette_run(
        sc.pos0, sc.faces_f, sc.mvps, targets, 256, sc.radius_px, sc.sigma,
        1e-3, n, threads=4, laplacian=0.15, normal=0.4)
    np.testing.assert_allclose(plan.loss_history(n), trace_cpu, rtol=1e-3)
    pos = plan.download(N.SLOT_PARAM).reshape(-1, 3)
    close = np.isclose(pos, pos_cpu, atol=1e-4, rtol=1e-3)
    assert close.mean() > 0.995
    assert np.abs(pos - pos_cpu).max() <= 4.0 * 1e-3 * n
    # the regulariser acted: an unregularised plan ends elsewhere
    plain = SilhouettePlan.from_scene(sc, lr=1e-3)
    plain.upload(N.SLOT_PARAM, sc.pos0)
    plain.upload(N.SLOT_TARGET, targets)
    plain.step(n)
    assert np.abs(plain.download(N.SLOT_PARAM).reshape(-1, 3) - pos).max() \
        > 1e-4
    assert plan.status() == 0


def test_aa_plan_regularized(cuda, port):
    """AA plan, icosphere-4, 3 views at 256^2, the example's AA weights
    (0.5 / 0.5), stochastic vertex gradients."""
    from opendressi_b200 import _native as N
    from opendressi_b200.plans import AaSilhouettePlan

    sc = scene.silhouette_scene(level=4, n_views=3, res=256, seed=2)
    plan = AaSilhouettePlan.from_scene(sc, lr=1e-2, n_samples=8,
                                       laplacian=0.5, normal=0.5)
    plan.render_targets(sc.target_pos)
    targets = plan.download(N.SLOT_TARGET).reshape(3, 256, 256)
    plan.upload(N.SLOT_PARAM, sc.pos0)
    _first_step_bitexact(plan, port, sc, 0.5, 0.5, 1e-2)
    plan.step(9)
    vft = port.vertex_faces_tex(sc.faces_f, sc.n_verts)
    trace_cpu, pos_cpu = port.aa_silhouette_run(
        sc.pos0, sc.faces_f, vft, sc.mvps, targets, 256, 8, 1e-2, 10,
        threads=3, laplacian=0.5, normal=0.5)
    np.testing.assert_allclose(plan.loss_history(10), trace_cpu, rtol=1e-3)
    pos = plan.download(N.SLOT_PARAM).reshape(-1, 3)
    close = np.isclose(pos, pos_cpu, atol=1e-4, rtol=1e-3)
    assert close.mean() > 0.995
    assert np.abs(pos - pos_cpu).max() <= 4.0 * 1e-2 * 10


@pytest.mark.parametrize("aa", [False, True])
def test_sharded_phases_with_regularizer_match_fused(cuda, port, aa):
    """Phase 0 (forward/backward + the pos-only regulariser terms), the
    gradient sum, then phase 1 (scales from the summed gradient + Adam)
    reproduce the fused regularised iteration."""
    from opendressi_b200 import _native as N
    from opendressi_b200.plans import AaSilhouettePlan, SilhouettePlan

    sc = scene.silhouette_scene(level=3, n_views=4, res=96, seed=5)
    kw = dict(lr=1e-2, laplacian=0.5, normal=0.5)

    def make(views=None):
        if aa:
            p = AaSilhouettePlan.from_scene(sc, views=views, **kw)
            p.render_targets(sc.target_pos)
        else:
            p = SilhouettePlan.from_scene(sc, views=views, **kw)
            t = _targets(port, sc)
            p.upload(N.SLOT_TARGET, t if views is None else t[views])
        p.upload(N.SLOT_PARAM, sc.pos0)
        return p

    full = make()
    shards = [make([0, 1]), make([2, 3])]
    for _ in range(3):
        full.step(1)
        for sp in shards:
            sp.forward_backward()
        g = sum(sp.grad_tensor().clone() for sp in shards)
        for sp in shards:
            sp.grad_tensor().copy_(g)
            sp.apply_update()
    p_full = full.download(N.SLOT_PARAM)
    for sp in shards:
        np.testing.assert_allclose(sp.download(N.SLOT_PARAM), p_full,
                                   atol=1e-5, rtol=1e-4)
