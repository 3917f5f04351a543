"""GPU parity of the nvdiffrast-style facade (opendressi_b200.torch_api,
mirroring the reference's dressi.torch ops) against the C restatement:
rasterize / interpolate / texture / antialias / rasterize_soft forwards
BIT-EXACT; deterministic backwards (image transposes, gathers) bit-exact,
scattered vertex gradients within 1e-4 abs + 1e-3 rel."""

import numpy as np
import pytest

from oracle import pyoracle
from opendressi_b200 import scene

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def npy(t):
    return t.detach().cpu().numpy()


def _mesh_pos(seed, level=3, res=64):
    """GL clip positions [V, 4] of a displaced icosphere and tri [F, 3]."""
    sc = scene.silhouette_scene(level=level, n_views=2, res=res, seed=seed)
    port = pyoracle.Port()
    clip = port.transform_clip(sc.target_pos, sc.mvps[0])
    # the silhouette scene's matrices give Vulkan depth; make a GL-style
    # clip z in [-w, w] so the facade's conversion is exercised
    gl = clip.copy()
    gl[:, 2] = 2.0 * clip[:, 2] - clip[:, 3]
    return gl.astype(np.float32), sc.faces.astype(np.int64), sc


def _clip_vk(pos):
    out = pos.copy()
    out[:, 2] = np.float32(0.5) * (pos[:, 2] + pos[:, 3])
    return out


def _rast_ref(port, pos, tri, h, w):
    clip_vk = _clip_vk(pos)
    flat = tri.ravel()
    clip3 = np.ascontiguousarray(clip_vk[flat])
    corner = np.tile(np.array([[1, 0], [0, 1], [0, 0]], np.float32),
                     (tri.shape[0], 1))
    attr4 = np.concatenate([corner, pos[flat][:, 2:4]], 1)
    fseq = np.arange(tri.size, dtype=np.float32).reshape(-1, 3)
    g = port.rasterize_hard(clip3, attr4, fseq, w, h)
    tid = port.rasterize_face_id(clip3, fseq, w, h)
    mask = (tid > np.float32(0.5)).astype(np.float32)
    zw = g[..., 2] / (g[..., 3] + (np.float32(1.0) - mask))
    return np.stack([g[..., 0], g[..., 1], zw, tid], -1)


def test_rasterize_and_interpolate(cuda, port):
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(1)
    h, w = 60, 72
    ctx = dr.RasterizeContext()
    rast, db = dr.rasterize(ctx, torch.tensor(pos, device=cuda),
                            torch.tensor(tri, device=cuda), (h, w))
    ref = _rast_ref(port, pos, tri, h, w)
    assert np.array_equal(bits(npy(rast[0])), bits(ref))
    assert float(db.abs().sum()) == 0.0
    rng = np.random.default_rng(2)
    attr = rng.standard_normal((pos.shape[0], 3)).astype(np.float32)
    at = torch.tensor(attr, device=cuda, requires_grad=True)
    out, _ = dr.interpolate(at, rast, torch.tensor(tri, device=cuda))
    f = np.rint(ref[..., 3]).astype(np.int64) - 1
    cov = f >= 0
    fi = np.where(cov, f, 0)
    a = [np.where(cov[..., None], attr[tri[fi, k]], np.float32(0.0))
         for k in range(3)]
    u, v = ref[..., 0:1], ref[..., 1:2]
    exp = (u * a[0] + v * a[1]) + ((np.float32(1.0) - u) - v) * a[2]
    assert np.array_equal(bits(npy(out[0])), bits(exp))
    gy = rng.standard_normal(out.shape).astype(np.float32)
    out.backward(torch.tensor(gy, device=cuda))
    g_ref = np.zeros_like(attr, dtype=np.float64)
    wk = [u[..., 0], v[..., 0], (np.float32(1.0) - u[..., 0]) - v[..., 0]]
    for k in range(3):
        np.add.at(g_ref, tri[fi[cov], k],
                  (gy[0][cov] * wk[k][cov][:, None]).astype(np.float64))
    np.testing.assert_allclose(npy(at.grad), g_ref, atol=1e-4, rtol=1e-3)


def test_texture_through_uv_provenance(cuda, port):
    import torch
    from opendressi_b200 import torch_api as dr

    sc = scene.texture_scene(level=3, n_views=1, res=48, tex_size=32,
                             levels=5, seed=3)
    pos = port.transform_clip(sc.pos, sc.mvps[0])
    pos[:, 2] = 2.0 * pos[:, 2] - pos[:, 3]   # GL depth
    tri = sc.faces.astype(np.int64)
    ctx = dr.RasterizeContext()
    pt, tt = torch.tensor(pos, device=cuda), torch.tensor(tri, device=cuda)
    rast, _ = dr.rasterize(ctx, pt, tt, (48, 48))
    uv, _ = dr.interpolate(torch.tensor(sc.uv, device=cuda), rast, tt)
    rng = np.random.default_rng(4)
    tex = rng.random((32, 32, 3)).astype(np.float32)
    for mode, fs, fg in [("nearest", port.texture_nearest, port.gather_inv_uv),
                         ("linear", port.texture_bilinear,
                          port.gather_inv_uv_bilinear)]:
        tx = torch.tensor(tex, device=cuda, requires_grad=True)
        out = dr.texture(tx, uv, filter_mode=mode)
        uv_np = npy(uv[0])
        assert np.array_equal(bits(npy(out[0])), bits(fs(tex, uv_np))), mode
        gy = rng.standard_normal(out.shape).astype(np.float32)
        out.backward(torch.tensor(gy, device=cuda))
        inv_uv = port.rasterize_hard(port.uv_as_clip(sc.uv),
                                     port.screen_attr(_clip_vk(pos), 48, 48),
                                     sc.faces_f, 32, 32)
        assert np.array_equal(bits(npy(tx.grad)),
                              bits(fg(gy[0], inv_uv, uv_np))), mode


@pytest.mark.parametrize("n_samples", [0, 8])
def test_antialias(cuda, port, n_samples):
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(5)
    h, w = 64, 64
    ctx = dr.RasterizeContext()
    pt = torch.tensor(pos, device=cuda, requires_grad=True)
    tt = torch.tensor(tri, device=cuda)
    rast, _ = dr.rasterize(ctx, pt, tt, (h, w))
    rng = np.random.default_rng(6)
    color = rng.random((1, h, w, 3)).astype(np.float32)
    ct = torch.tensor(color, device=cuda, requires_grad=True)
    out = dr.antialias(ct, rast, pt, tt, n_samples=n_samples)
    tid = npy(rast[0, ..., 3])
    clip_vk = _clip_vk(pos)
    faces_f = tri.astype(np.float32)
    assert np.array_equal(bits(npy(out[0])),
                          bits(port.antialias(color[0], tid, clip_vk, faces_f)))
    gy = rng.standard_normal(out.shape).astype(np.float32)
    out.backward(torch.tensor(gy, device=cuda))
    assert np.array_equal(bits(npy(ct.grad[0])),
                          bits(port.antialias_bwd_img(gy[0], tid, clip_vk,
                                                      faces_f)))
    vft = port.vertex_faces_tex(faces_f, pos.shape[0])
    gc = port.antialias_bwd_vtx(gy[0], color[0], tid, clip_vk, faces_f, vft,
                                1.0, n_samples)   # first backward: seed 1
    gp = gc.copy()
    gp[:, 2] = np.float32(0.5) * gc[:, 2]
    gp[:, 3] = gc[:, 3] + np.float32(0.5) * gc[:, 2]
    np.testing.assert_allclose(npy(pt.grad), gp, atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("peels", [1, 2])
def test_rasterize_soft(cuda, port, peels):
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(7)
    h, w, r = 56, 64, 3.0
    ctx = dr.RasterizeContext()
    pt = torch.tensor(pos, device=cuda, requires_grad=True)
    out = dr.rasterize_soft(ctx, pt, torch.tensor(tri, device=cuda), (h, w),
                            radius_px=r, peels=peels)
    clip_vk = _clip_vk(pos)
    faces_f = tri.astype(np.float32)
    soft = port.soft_clip(clip_vk, faces_f, w, h, r)
    fid, fs = pyoracle.soft_inputs(tri.shape[0])
    prev = None
    layers = []
    for k in range(peels):
        rs = port.rasterize_soft(soft, fid, fs, clip_vk, faces_f, w, h, r,
                                 prev)
        layers.append(rs)
        dist, cov = rs[..., 0], rs[..., 3]
        ge = (dist >= 0).astype(np.float32)
        one = np.float32(1.0)
        half = np.float32(0.5)
        prev = cov * (ge * (np.clip(rs[..., 2], 0, 1) * half) +
                      (one - ge) * (np.clip(dist * np.float32(-1.0 / r), 0, 1)
                                    * half + half))
        prev = prev.astype(np.float32)
    for k in range(peels):
        assert np.array_equal(bits(npy(out[0, k])), bits(layers[k])), k
    rng = np.random.default_rng(8)
    gy = rng.standard_normal(out.shape).astype(np.float32)
    out.backward(torch.tensor(gy, device=cuda))
    gc = sum(port.dist_grad(gy[0, k, ..., 0], layers[k], clip_vk, faces_f, w,
                            h) for k in range(peels))
    gp = gc.copy()
    gp[:, 2] = np.float32(0.5) * gc[:, 2]
    gp[:, 3] = gc[:, 3] + np.float32(0.5) * gc[:, 2]
    np.testing.assert_allclose(npy(pt.grad), gp, atol=1e-4, rtol=1e-3)


def test_antialias_silhouette_optimisation_runs(cuda):
    """A short nvdiffrast-style loop: rasterize + interpolate + antialias,
    L2 to a target silhouette; the loss decreases."""
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(9, level=3, res=96)
    tgt_pos = pos.copy()
    tgt_pos[:, :2] *= 1.15
    ctx = dr.RasterizeContext()
    tt = torch.tensor(tri, device=cuda)

    def render(p):
        rast, _ = dr.rasterize(ctx, p, tt, (96, 96))
        ones = torch.ones((p.shape[-2], 1), device=cuda)
        mask, _ = dr.interpolate(ones, rast, tt)
        return dr.antialias(mask, rast, p, tt, n_samples=8)

    with torch.no_grad():
        target = render(torch.tensor(tgt_pos, device=cuda))
    p = torch.tensor(pos, device=cuda, requires_grad=True)
    opt = torch.optim.Adam([p], lr=1e-2)
    losses = []
    for _ in range(30):
        opt.zero_grad()
        loss = ((render(p) - target) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < 0.7 * losses[0]


def test_ops_under_torch_compile_and_no_sync(cuda):
    """The ops are torch.library custom ops with fake implementations: a
    function using them compiles with torch.compile (graph breaks allowed
    around the mesh-table lookups) and gives the eager results, forward and
    backward. No op reads the device status back: check_status() is the one
    synchronisation."""
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(11, level=3, res=64)
    ctx = dr.RasterizeContext()
    tt = torch.tensor(tri, device=cuda)
    target = torch.rand((1, 64, 64, 1), device=cuda)

    def loss_fn(p):
        rast, _ = dr.rasterize(ctx, p, tt, (64, 64))
        ones = torch.ones((p.shape[-2], 1), device=cuda)
        mask, _ = dr.interpolate(ones, rast, tt)
        aa = dr.antialias(mask, rast, p, tt, n_samples=0)
        soft = dr.rasterize_soft(ctx, p, tt, (64, 64), radius_px=2.0)
        return ((aa - target) ** 2).mean() + 1e-3 * soft[..., 0].mean()

    p1 = torch.tensor(pos, device=cuda, requires_grad=True)
    l1 = loss_fn(p1)
    l1.backward()
    compiled = torch.compile(loss_fn, fullgraph=False)
    p2 = torch.tensor(pos, device=cuda, requires_grad=True)
    l2 = compiled(p2)
    l2.backward()
    # the compiled graph fuses the loss arithmetic around the custom ops
    # (its own reduction order), so the results agree to rounding
    torch.testing.assert_close(l2.detach(), l1.detach(), atol=0, rtol=1e-5)
    torch.testing.assert_close(p2.grad, p1.grad, atol=1e-5, rtol=1e-4)
    assert dr.check_status() == 0
    # the ops are registered custom ops with fake kernels
    assert hasattr(torch.ops.dressi_b200, "rasterize")
    assert hasattr(torch.ops.dressi_b200, "antialias_grad")


def test_mesh_cache_pins_tri(cuda, port):
    """A tri tensor freed and replaced by another of the same shape must not
    hit the cached tables of the first (the cache keeps the first alive)."""
    import torch
    from opendressi_b200 import torch_api as dr

    pos, tri, _ = _mesh_pos(13)
    ctx = dr.RasterizeContext()
    pt = torch.tensor(pos, device=cuda)
    t1 = torch.tensor(tri, device=cuda)
    r1, _ = dr.rasterize(ctx, pt, t1, (48, 48))
    ptr1 = t1.data_ptr()
    del t1
    tri2 = tri[:, [0, 2, 1]].copy()            # same shape, other faces
    tri2[: tri.shape[0] // 2] = tri2[: tri.shape[0] // 2][::-1]
    t2 = torch.tensor(tri2, device=cuda)
    r2, _ = dr.rasterize(ctx, pt, t2, (48, 48))
    assert t2.data_ptr() != ptr1
    ref2 = _rast_ref(port, pos, tri2, 48, 48)
    assert np.array_equal(bits(npy(r2[0])), bits(ref2))
    ctx.clear_cache()


def test_ops_run_on_the_inputs_device():
    """Inputs on a device other than the current one: the ops run there (on
    that device's current stream), with no peer access involved."""
    import torch
    from opendressi_b200 import torch_api as dr

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    from opendressi_b200 import _native

    _native.load()
    pos, tri, _ = _mesh_pos(15)
    ctx = dr.RasterizeContext()
    outs = []
    for dev in ("cuda:0", "cuda:1"):
        torch.cuda.set_device(0)
        p = torch.tensor(pos, device=dev, requires_grad=True)
        t = torch.tensor(tri, device=dev)
        rast, _ = dr.rasterize(ctx, p, t, (40, 40))
        mask, _ = dr.interpolate(torch.ones((pos.shape[0], 1), device=dev),
                                 rast, t)
        out = dr.antialias(mask, rast, p, t, n_samples=0)
        out.sum().backward()
        assert out.device == torch.device(dev) and p.grad.device == out.device
        outs.append((npy(out), npy(p.grad)))
    assert np.array_equal(outs[0][0], outs[1][0])
    np.testing.assert_allclose(outs[0][1], outs[1][1], atol=1e-5)
    assert dr.check_status("cuda:1") == 0
