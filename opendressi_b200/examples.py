"""The benchmark workloads written as graphs with the graph API
(opendressi_b200.graph), composed as the reference's examples compose them
(examples/silhouette_optimization/run.cpp:228-437, examples/image_fitting of
unclearness/opendressi): the F:: forward, BuildBackward inside
DressiAD.exec_step, and the in-graph Adam of the optimizer callback with
its state kept on the device through add_update. The fused plans
(opendressi_b200.plans) compute the same iterations with hand-fused
kernels."""

from __future__ import annotations

import numpy as np

from . import graph as G

f = G.f
VT = G.VType


def adam_optimizer(ad: G.DressiAD, lr: float, b1=0.9, b2=0.999, eps=1e-8,
                   reg=None):
    """DressiAD.set_optimizer callback of the in-graph Adam
    (run.cpp:421-436); reg(x, g) -> g rewrites the gradient first (the
    example's regulariser). Returns the list its state leaves go into."""
    state = []

    def opt(xs, gxs):
        outs = []
        for x, g in zip(xs, gxs):
            if reg is not None:
                g = reg(x, g)
            m = G.Variable(x.vtype, x.width, x.height)
            v = G.Variable(x.vtype, x.width, x.height)
            t = G.Variable(VT.FLOAT, 1, 1)
            t_new = t + 1.0
            m_new = m * b1 + g * (1.0 - b1)
            v_new = v * b2 + g * g * (1.0 - b2)
            bc1 = 1.0 - f.pow(f.constant(b1), t_new)
            bc2 = 1.0 - f.pow(f.constant(b2), t_new)
            step = (m_new / bc1) / (f.sqrt(v_new / bc2) + eps) * lr
            ad.add_update(m, m_new)
            ad.add_update(v, v_new)
            ad.add_update(t, t_new)
            state.append((m, v, t))
            outs.append(x - step)
        return outs

    ad.set_optimizer(opt)
    return state


def image_fit(ad: G.DressiAD, w: int, h: int, lr: float = 1e-2):
    """Config C1: Mean((p - target)^2) over a VEC4 image, Adam on p."""
    p = G.Variable(VT.VEC4, w, h)
    tg = G.Variable(VT.VEC4, w, h)
    diff = p - f.stop_gradient(tg)
    loss = f.mean(diff * diff)
    p.set_requires_grad_recursively(True)
    ad.set_loss_var(loss)
    adam_optimizer(ad, lr)
    return p, tg, loss


def clip_of(pos: G.Variable, m: np.ndarray) -> G.Variable:
    """MVP (pos, 1) with column constants (geometry_utils.cpp:391-402):
    row r = x m[r] + y m[4+r] + z m[8+r] + m[12+r]."""
    x, y, z = f.get_x(pos), f.get_y(pos), f.get_z(pos)
    m = [float(v) for v in np.asarray(m, np.float32).reshape(16)]

    def row(r):
        return x * m[r] + y * m[4 + r] + z * m[8 + r] + m[12 + r]

    return f.vec4v(row(0), row(1), row(2), row(3))


class SilhouetteGraph:
    """Config C3 as a graph: per view RasterizeSoft of SoftClip(clip), pred =
    max(cov step(0, d), cov sigmoid(d |d| k)), loss = SumPixelWise over views
    of (target - pred)^2 / R^2, the example's regulariser and Adam."""

    def __init__(self, ad: G.DressiAD, faces_f, n_verts, mvps, res, radius,
                 sigma, lr, laplacian=0.0, normal=0.0):
        faces_f = np.ascontiguousarray(faces_f, np.float32)
        nf = faces_f.shape[0]
        self.ad = ad
        self.n_verts, self.res = n_verts, res
        self.pos = G.Variable(VT.VEC3, n_verts, 1)
        self.faces = G.Variable(VT.VEC3, nf, 1)
        vft_np = G.vertex_faces_tex(faces_f, n_verts)
        self.vft = G.Variable(VT.FLOAT, n_verts, vft_np.shape[0])
        self.face_id = G.Variable(VT.FLOAT, nf * 3, 1)
        self.faces_soft = G.Variable(VT.IVEC3, nf, 1)
        self.targets = [G.Variable(VT.FLOAT, res, res) for _ in mvps]
        k = float(np.float32(2.0 / res) * np.float32(2.0 / res)
                  / np.float32(sigma))
        c = float(np.float32(1.0) / np.float32(res * res))
        losses = []
        for m, tg in zip(mvps, self.targets):
            clip = clip_of(self.pos, m)
            soft = f.soft_clip(clip, self.faces, res, res, radius)
            rs = f.rasterize_soft(soft, self.face_id, self.faces_soft, clip,
                                  self.faces, self.vft, res, res, radius)
            dist, cov = f.get_x(rs), f.get_w(rs)
            hard = cov * f.step(f.constant(0.0), dist)
            sft = cov * f.sigmoid(dist * f.abs(dist) * k)
            pred = f.max(hard, sft)
            diff = f.stop_gradient(tg) - pred
            losses.append(diff * diff * c)
        self.loss = f.sum_pixel_wise(losses)
        self.pos.set_requires_grad_recursively(True)
        ad.set_loss_var(self.loss)
        ad.mark_output(self.loss)
        reg = None
        if laplacian or normal:
            vn = G.vertex_neighbors_tex(faces_f, n_verts)
            fa = G.face_neighbors_tex(faces_f)
            self.vnb = G.Variable(VT.FLOAT, n_verts, vn.shape[0])
            self.vfa = G.Variable(VT.VEC3, nf, 1)
            self._reg_data = [(self.vnb, vn), (self.vfa, fa)]
            inv_cnt = float(np.float32(1.0) / np.float32(n_verts * 3))

            def rms(x):
                return f.sqrt(f.sum_all(x * x) * inv_cnt + 1e-24)

            def reg(x, g):
                data_rms = rms(g)
                g_lap = x - f.vertex_neighbor_mean(x, self.vnb)
                g_nrm = f.normal_consistency_vertex_grad(
                    f.normal_consistency_face_term(x, self.faces, self.vfa),
                    x, self.faces, self.vft)
                return (g + g_lap * (data_rms / rms(g_lap) * laplacian)
                        + g_nrm * (data_rms / rms(g_nrm) * normal))
        else:
            self._reg_data = []
        self.state = adam_optimizer(ad, lr, reg=reg)
        fid = np.repeat(np.arange(nf, dtype=np.float32), 3)
        self._static = [(self.faces, faces_f), (self.vft, vft_np),
                        (self.face_id, fid),
                        (self.faces_soft,
                         np.arange(nf * 3, dtype=np.float32))]

    def send_static(self, targets):
        for v, d in self._static + self._reg_data:
            self.ad.send_img(v, d)
        for v, t in zip(self.targets, targets):
            self.ad.send_img(v, t)

    def loss_value(self) -> float:
        return float(self.ad.recv_img(self.loss).astype(np.float64).sum())
