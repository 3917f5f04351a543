"""GPU parity of the texture ops (dressi_texture / dressi_texture_grad) and
of the C2 texture-optimisation plan. Sampling, inverse-UV gathers, targets
and renders are BIT-EXACT with the reference's golden outputs / the C
restatement; the scattered texture gradient (float atomics) within 1e-4
abs + 1e-3 rel; loss traces within 1e-3 rel."""

import os

import numpy as np
import pytest

from conftest import GOLDEN

from opendressi_b200 import scene

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def T(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)


def npy(t):
    return t.detach().cpu().numpy()


def test_golden_tex_small(cuda):
    from opendressi_b200 import ops

    g = np.load(os.path.join(GOLDEN, "tex_small.npz"))
    uv = np.ascontiguousarray(g["gbuf"][..., :2])
    out = ops.texture(T(g["tex"], cuda), T(uv, cuda), "linear")
    assert np.array_equal(bits(npy(out)), bits(g["out"]))
    gt = ops.texture_grad(T(g["gy"], cuda), T(g["inv_uv"], cuda),
                          T(uv, cuda), "linear")
    assert np.array_equal(bits(npy(gt)), bits(g["gtex"]))


@pytest.mark.parametrize("n", [1, 3, 4])
def test_nearest_texture_and_gather_match_port(cuda, port, n):
    from opendressi_b200 import ops

    sc = scene.texture_scene(level=3, n_views=1, res=48, tex_size=32,
                             levels=5, seed=n)
    clip = port.transform_clip(sc.pos, sc.mvps[0])
    attr = np.concatenate([sc.uv, np.ones((sc.n_verts, 1), np.float32)], 1)
    uv = np.ascontiguousarray(port.rasterize_hard(clip, attr, sc.faces_f, 48,
                                                  48)[..., :2])
    inv_uv = port.rasterize_hard(port.uv_as_clip(sc.uv),
                                 port.screen_attr(clip, 48, 48), sc.faces_f,
                                 32, 32)
    rng = np.random.default_rng(n)
    tex = rng.random((32, 32, n)).astype(np.float32)
    gy = rng.standard_normal((48, 48, n)).astype(np.float32)
    for mode, fs, fg in [("nearest", port.texture_nearest, port.gather_inv_uv),
                         ("linear", port.texture_bilinear,
                          port.gather_inv_uv_bilinear)]:
        out = ops.texture(T(tex, cuda), T(uv, cuda), mode)
        assert np.array_equal(bits(npy(out)), bits(fs(tex, uv))), mode
        g = ops.texture_grad(T(gy, cuda), T(inv_uv, cuda), T(uv, cuda), mode)
        assert np.array_equal(bits(npy(g)), bits(fg(gy, inv_uv, uv))), mode


def _plan(sc, **kw):
    from opendressi_b200.plans import TexturePlan

    plan = TexturePlan.from_scene(sc, **kw)
    plan.render_targets(sc.gt_tex)
    return plan


def test_texture_plan_matches_port(cuda, port):
    from opendressi_b200 import _native as N

    sc = scene.texture_scene(level=3, n_views=2, res=96, tex_size=64,
                             levels=7, seed=5)
    plan = _plan(sc, lr=1e-2)
    targets = plan.download(N.SLOT_TARGET).reshape(2, 96, 96, 3)
    zeros = np.zeros((2, 96, 96, 3), np.float32)
    _, _, t_cpu = port.c2_loss_grad(sc.gt_tex, 7, sc.pos, sc.uv, sc.faces_f,
                                    sc.mvps, zeros, 96, want_pred=True)
    assert np.array_equal(bits(targets), bits(t_cpu))
    plan.upload(N.SLOT_PARAM, sc.tex0)
    _, g_cpu, p_cpu = port.c2_loss_grad(sc.tex0, 7, sc.pos, sc.uv, sc.faces_f,
                                        sc.mvps, targets, 96, want_pred=True)
    assert np.array_equal(bits(plan.render().cpu().numpy()), bits(p_cpu))
    plan.step(1)
    np.testing.assert_allclose(plan.download(N.SLOT_GRAD).reshape(64, 64, 3),
                               g_cpu, atol=1e-4, rtol=1e-3)
    plan.step(5)
    trace, tex = port.c2_run(sc.tex0, 7, sc.pos, sc.uv, sc.faces_f, sc.mvps,
                             targets, 96, 1e-2, 6)
    np.testing.assert_allclose(plan.loss_history(6), trace, rtol=1e-3)
    close = np.isclose(plan.download(N.SLOT_PARAM).reshape(64, 64, 3), tex,
                       atol=1e-4, rtol=1e-3)
    assert close.mean() > 0.995
    assert plan.status() == 0


def test_texture_sharded_phases_match_fused(cuda):
    from opendressi_b200 import _native as N

    sc = scene.texture_scene(level=3, n_views=4, res=64, tex_size=32,
                             levels=6, seed=6)
    full = _plan(sc, lr=1e-2)
    shards = [_plan(sc, lr=1e-2, views=[0, 1]), _plan(sc, lr=1e-2, views=[2, 3])]
    for p in [full] + shards:
        p.upload(N.SLOT_PARAM, sc.tex0)
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
        close = np.isclose(sp.download(N.SLOT_PARAM), p_full, atol=1e-5,
                           rtol=1e-4)
        assert close.mean() > 0.995
