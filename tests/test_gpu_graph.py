"""GPU parity of the generic graph path (DressiAD: BuildBackward, the fusion
planner's pixel programs, the quad-tree Sum, the rendering kernels, Adam in
the optimizer graph, reactive pruning) against the compiled reference's own
F:: graphs, BuildBackward and CpuEvaluator (oracle/ref_driver.cpp
ref_graph_eval) and against the C restatement's training loops.

Tolerances: values and gradients 1e-4 abs (scaled by the value's magnitude
for long chains) + 1e-3 rel -- CUDA's sin/exp/log/pow differ from the host
libm by a few ulps, + - * / and sqrt are IEEE in both; losses after N Adam
steps 1e-3 rel."""

import numpy as np
import pytest

import graph_programs as gp
from opendressi_b200 import examples as gm
from opendressi_b200 import graph as G
from opendressi_b200 import scene

pytestmark = pytest.mark.gpu

f = G.f
VT = G.VType


def _close(got, exp, rtol=1e-3, atol=1e-4, what=""):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    assert got.shape == exp.shape, what
    scale = max(1.0, float(np.nanmax(np.abs(exp))) if exp.size else 1.0)
    np.testing.assert_allclose(got, exp, rtol=rtol, atol=atol * scale,
                               equal_nan=True, err_msg=what)


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("w,h", [(7, 5), (64, 33), (300, 1)])
def test_random_pixel_programs_match_reference(cuda, ref, seed, w, h):
    """Random elementwise graphs over every pixel-wise op (vectors,
    broadcasting {1,1} values, compose / extract): forward values and the
    gradients of every leaf (BuildBackward through the fused programs, the
    quad-tree Sum for the {1,1} leaf) against the reference."""
    rec, leaves = gp.random_program(seed, w, h)
    exp = gp.ref_eval(ref, rec, grads_of=leaves)
    got, ad = gp.ours_eval(rec, grads_of=leaves)
    names = ["total", "loss"] + [f"grad{i}" for i in range(len(leaves))]
    for g, e, n in zip(got, exp, names):
        _close(g, e, what=f"seed {seed} {n}")
    st = ad.stats()
    # the planner fused the chain: far fewer kernels than ops
    assert st["n_programs"] >= 1
    assert st["kernels_per_iter"] < st["n_exec_funcs"]
    assert ad.status() == 0


@pytest.mark.parametrize("w,h", [(256, 256), (97, 61), (1, 300), (5000, 1)])
def test_sum_and_mean_follow_the_reference_tree(cuda, ref, w, h):
    """Sum / Mean of images (the reference's 2x2 quad tree, odd extents
    included): bit-exact, the same float additions in the same order."""
    rng = np.random.default_rng(w * 7 + h)
    rec = gp.Recorder()
    x = rec.leaf(VT.VEC3, w, h, rng.standard_normal(w * h * 3), True)
    s = rec.op("Sum", x)
    m = rec.op("Mean", x)
    loss = rec.op("Mul", m, m)
    rec.set_loss(loss)
    rec.eval(s)
    rec.eval(m)
    exp = gp.ref_eval(ref, rec)
    got, _ = gp.ours_eval(rec)
    for g, e in zip(got, exp):
        assert np.array_equal(g.view(np.uint32), e.view(np.uint32)), (g, e)


def test_image_fit_graph_matches_plan_and_restatement(cuda, port):
    """Config C1 written with F:: ops and the in-graph Adam: the 12-step
    golden trace of the reference and the 500-step run of the restatement
    (final loss 1e-3 rel); the planner lowers the iteration to a handful of
    kernels."""
    import os

    from conftest import GOLDEN

    g = np.load(os.path.join(GOLDEN, "image_fit_32.npz"))
    p0, t0 = scene.image_fit_scene(0, 32, 32)
    ad = G.DressiAD(0)
    p, tg, loss = gm.image_fit(ad, 32, 32, lr=1e-2)
    ad.mark_output(loss)
    ad.send_img(p, p0)
    ad.send_img(tg, t0)
    n = len(g["trace"])
    trace = []
    for _ in range(n):
        ad.exec_step()
        trace.append(float(ad.recv_img(loss).reshape(-1)[0]))
    np.testing.assert_allclose(trace, g["trace"], rtol=1e-5)
    np.testing.assert_allclose(ad.recv_img(p).reshape(32, 32, 4), g["param"],
                               atol=1e-5)
    st = ad.stats()
    assert st["kernels_per_iter"] <= 8, st
    # full size: 256^2 x 4, 500 iterations
    p0, t0 = scene.image_fit_scene(0, 256, 256)
    trace_cpu, _ = port.image_fit_run(p0, t0, 1e-2, 500)
    ad = G.DressiAD(0)
    p, tg, loss = gm.image_fit(ad, 256, 256, lr=1e-2)
    ad.mark_output(loss)
    ad.send_img(p, p0)
    ad.send_img(tg, t0)
    for _ in range(499):
        ad.exec_step()
    ad.exec_step()
    last = float(ad.recv_img(loss).reshape(-1)[0])
    assert last == pytest.approx(trace_cpu[-1], rel=1e-3)
    assert ad.status() == 0


def test_reactive_pruning_keeps_results(cuda):
    """A static branch (a {1,1} weight computed from a leaf that is never
    sent again) is pruned from the replayed graph once the dirty pattern is
    stable; sending the leaf again re-includes it (the reactive cache of
    src/dressi_ad.cpp:287-308)."""
    rng = np.random.default_rng(3)
    x = G.Variable(VT.FLOAT, 64, 64)
    a = G.Variable(VT.FLOAT, 64, 64)
    wt = f.mean(f.exp(a) * f.sin(a))      # depends on `a` only: static
    y = x * wt
    loss = f.mean(y * y)
    x.set_requires_grad_recursively(True)
    ad = G.DressiAD(0)
    ad.set_loss_var(loss)
    ad.mark_output(loss)
    ad.set_rebuild_counts(2, 0)
    xa = rng.standard_normal((64, 64)).astype(np.float32)
    aa = rng.standard_normal((64, 64)).astype(np.float32)
    ad.send_img(x, xa)
    ad.send_img(a, aa)
    losses, execd = [], []
    for it in range(5):
        ad.send_img(x, xa * (1 + 0.1 * it))   # x changes every iteration
        ad.exec_step()
        losses.append(float(ad.recv_img(loss).reshape(-1)[0]))
        execd.append(ad.stats()["n_exec_funcs"])
    assert execd[-1] < execd[0], execd
    assert ad.stats()["pruning_active"] == 1
    w_ref = np.mean(np.exp(aa.astype(np.float64)) * np.sin(aa))
    for it, l in enumerate(losses):
        y_ref = xa.astype(np.float64) * (1 + 0.1 * it) * w_ref
        assert l == pytest.approx(np.mean(y_ref * y_ref), rel=1e-4)
    # `a` changes: the branch is re-included and the value follows
    aa2 = aa * 0.5
    ad.send_img(a, aa2)
    ad.exec_step()
    ad.exec_step()
    w2 = np.mean(np.exp(aa2.astype(np.float64)) * np.sin(aa2))
    y2 = xa.astype(np.float64) * 1.4 * w2
    assert float(ad.recv_img(loss).reshape(-1)[0]) == pytest.approx(
        np.mean(y2 * y2), rel=1e-4)


@pytest.mark.parametrize("reg", [False, True])
def test_silhouette_graph_matches_restatement(cuda, port, reg):
    """Config C3 written with F:: ops (SoftClip, RasterizeSoft, the
    elementwise silhouette loss, SumPixelWise over views, the example's
    regulariser, in-graph Adam), icosphere-3, 3 views at 96^2: the
    per-iteration loss and the positions after 6 steps against the C
    restatement's run (the same arithmetic as the fused SilhouettePlan)."""
    sc = scene.silhouette_scene(level=3, n_views=3, res=96, seed=2)
    targets = np.stack([(port.rasterize_face_id(
        port.transform_clip(sc.target_pos, m), sc.faces_f, 96, 96)
        > 0).astype(np.float32) for m in sc.mvps])
    lap, nrm = (0.15, 0.4) if reg else (0.0, 0.0)
    ad = G.DressiAD(0)
    sg = gm.SilhouetteGraph(ad, sc.faces_f, sc.n_verts, sc.mvps, 96,
                            sc.radius_px, sc.sigma, 1e-2, lap, nrm)
    sg.send_static(targets)
    ad.send_img(sg.pos, sc.pos0)
    n = 6
    trace = []
    for _ in range(n):
        ad.exec_step()
        trace.append(sg.loss_value())
    trace_cpu, pos_cpu = port.silhouette_run(
        sc.pos0, sc.faces_f, sc.mvps, targets, 96, sc.radius_px, sc.sigma,
        1e-2, n, laplacian=lap, normal=nrm)
    np.testing.assert_allclose(trace, trace_cpu, rtol=1e-3)
    pos = ad.recv_img(sg.pos).reshape(-1, 3)
    close = np.isclose(pos, pos_cpu, atol=1e-4, rtol=1e-3)
    assert close.mean() > 0.99
    assert ad.status() == 0
