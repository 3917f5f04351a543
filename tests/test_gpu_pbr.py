"""GPU parity of the C5 plan (split-sum PBR material + environment
optimisation, csrc/pbr.cu) against the C restatement (pinned to the
reference's BuildPbrShade + BuildBackward in test_oracle_pbr.py), on the
same G-buffers (the hard raster is bit-exact with the reference): targets
and renders within 1e-4 abs + 1e-3 rel (CUDA's transcendentals differ from
the host libm by a few ulps, and the shading is compiled with FMA contraction
and the <= 2 ulp division, as shader compilers do), the first gradient of
[albedo | mr | env]
within 1e-4 abs + 1e-3 rel, loss traces within 1e-3 rel; the sharded
phases reproduce the fused iteration."""

import numpy as np
import pytest

from opendressi_b200 import scene

pytestmark = pytest.mark.gpu

TOL = dict(atol=1e-4, rtol=1e-3)


def _scene(n_views=2, res=64, seed=3):
    return scene.pbr_scene(level=3, n_views=n_views, res=res, tex_size=64,
                           env_w=64, env_h=32, levels=5, seed=seed)


def _plan(sc, **kw):
    from opendressi_b200.plans import PbrPlan

    kw.setdefault("lut_size", 32)
    kw.setdefault("lut_samples", 64)
    return PbrPlan.from_scene(sc, **kw)


def _gbuffers(port, sc):
    out = []
    ones = np.ones((sc.n_verts, 1), np.float32)
    uvh = np.concatenate([sc.uv, ones, 0 * ones], 1)
    for v in range(sc.n_views):
        clip = port.transform_clip(sc.pos, sc.mvps[v])
        g_uvh = port.rasterize_hard(clip, uvh, sc.faces_f, sc.res, sc.res)
        g = port.rasterize_hard(clip, sc.pos, sc.faces_f, sc.res, sc.res)
        frame = np.concatenate([sc.frames[v], sc.light]).astype(np.float32)
        out.append((g, g, np.ascontiguousarray(g_uvh[..., 2]),
                    np.ascontiguousarray(g_uvh[..., :2]), frame))
    return out


def _port_step(port, sc, gbufs, alb, mr, env, targets, lut, loss_kind=1):
    ga = np.zeros_like(alb)
    gm = np.zeros_like(mr)
    ge = np.zeros_like(env)
    maps, loss = [], 0.0
    for v, (g_n, g_p, mask, uv, frame) in enumerate(gbufs):
        t = (targets[v] if targets is not None
             else np.zeros((sc.res, sc.res, 3), np.float32))
        m, l = port.pbr_view_grad(g_n, g_p, mask, uv, alb, mr, frame, env,
                                  sc.levels, lut, t, loss_kind, ga, gm, ge)
        maps.append(m)
        loss += l
    return np.stack(maps), loss, ga, gm, ge


def test_pbr_plan_matches_port(cuda, port):
    from opendressi_b200 import _native as N

    sc = _scene()
    plan = _plan(sc)
    plan.render_targets(sc.albedo_gt, sc.mr_gt, sc.env_gt)
    targets = plan.download(N.SLOT_TARGET).reshape(sc.n_views, sc.res,
                                                   sc.res, 3)
    gb = _gbuffers(port, sc)
    lut = port.brdf_lut(32, 32, 64)
    t_cpu = _port_step(port, sc, gb, sc.albedo_gt, sc.mr_gt, sc.env_gt,
                       None, lut)[0]
    np.testing.assert_allclose(targets, t_cpu, **TOL)
    assert targets.std() > 0.05   # a real image
    # the initial parameters: render, then one step's gradient
    plan.upload(N.SLOT_PARAM, plan.pack(sc.albedo0, sc.mr0, sc.env0))
    mapped, loss, ga, gm, ge = _port_step(port, sc, gb, sc.albedo0, sc.mr0,
                                          sc.env0, targets, lut)
    np.testing.assert_allclose(plan.render().cpu().numpy(), mapped, **TOL)
    plan.step(1)
    assert plan.loss() == pytest.approx(loss, rel=1e-3)
    g = plan.unpack(plan.download(N.SLOT_GRAD))
    for got, exp in zip(g, (ga, gm, ge)):
        np.testing.assert_allclose(got, exp, **TOL)
    assert np.abs(ga).max() > 1e-6 and np.abs(ge).max() > 1e-6
    assert plan.status() == 0


def test_pbr_plan_trace(cuda, port):
    """8 Adam iterations (with the maps' [0, 1] and the env's >= 0 clamps)
    against the port's; the loss falls."""
    from opendressi_b200 import _native as N

    sc = _scene(seed=4)
    plan = _plan(sc, lr=5e-2)
    plan.render_targets(sc.albedo_gt, sc.mr_gt, sc.env_gt)
    targets = plan.download(N.SLOT_TARGET).reshape(sc.n_views, sc.res,
                                                   sc.res, 3)
    plan.upload(N.SLOT_PARAM, plan.pack(sc.albedo0, sc.mr0, sc.env0))
    n = 8
    plan.step(n)
    gb = _gbuffers(port, sc)
    lut = port.brdf_lut(32, 32, 64)
    p = plan.pack(sc.albedo0, sc.mr0, sc.env0)
    m, v = np.zeros_like(p), np.zeros_like(p)
    t = 0.0
    trace = []
    t2 = sc.tex_size * sc.tex_size * 3
    for _ in range(n):
        _, loss, ga, gm, ge = _port_step(port, sc, gb, *plan.unpack(p),
                                         targets, lut)
        trace.append(loss)
        g = plan.pack(ga, gm, ge)
        t = port.adam(p, m, v, t, g, 5e-2)
        p[:2 * t2] = np.clip(p[:2 * t2], 0.0, 1.0)
        p[2 * t2:] = np.maximum(p[2 * t2:], 0.0)
    hist = plan.loss_history(n)
    np.testing.assert_allclose(hist, trace, rtol=1e-3)
    assert hist[-1] < hist[0]
    close = np.isclose(plan.download(N.SLOT_PARAM), p, atol=1e-4, rtol=1e-3)
    assert close.mean() > 0.995


def test_pbr_sharded_phases_match_fused(cuda):
    from opendressi_b200 import _native as N

    sc = _scene(n_views=4, seed=5)
    full = _plan(sc)
    shards = [_plan(sc, views=[0, 1]), _plan(sc, views=[2, 3])]
    p0 = full.pack(sc.albedo0, sc.mr0, sc.env0)
    for pl in [full] + shards:
        pl.render_targets(sc.albedo_gt, sc.mr_gt, sc.env_gt)
        pl.upload(N.SLOT_PARAM, p0)
    for _ in range(3):
        full.step(1)
        for sp in shards:
            sp.forward_backward()
        g = sum(sp.grad_tensor().clone() for sp in shards)
        for sp in shards:
            sp.grad_tensor().copy_(g)
            sp.apply_update()
    pf = full.download(N.SLOT_PARAM)
    for sp in shards:
        close = np.isclose(sp.download(N.SLOT_PARAM), pf, atol=1e-5,
                           rtol=1e-4)
        assert close.mean() > 0.995
