"""The paper's HardSoftRas silhouette path, composed from this package's
CUDA ops with torch autograd, as the reference's silhouette example
composes it from `F::` ops (examples/silhouette_optimization/
run.cpp:229-436):

    clip      = MVP (pos, 1)                              per view
    layers    = RasterizeSoft(SoftClip(clip), ...)       K peels, no gradient
    tri_k     = LookupFaces(clip, faces, vertex_faces, k) exact transpose
    per layer: idx = (face_id + 1) * cov; the pixel's face corners fetched
               with FaceFetch (backward: the face's edge samples, jitter =
               the Adam counter); D = mask * sigmoid(signed edge distance *
               7 / r)
    pred      = max(cov_0 * step(0, dist_0), 1 - prod_k (1 - D_k))   (Eq. 6)
    loss      = sum over views and pixels of (target - pred)^2 / R^2

then the example's regulariser (relative to the data-gradient RMS) and
Adam. The indexed ops, the raster and the regulariser are the CUDA kernels
of this package (`ops`); the per-pixel elementwise chain runs as torch
operations in the reference's operation order, with the reference
autodiff's tie rules where torch's differ (Min / Max ties go to the first
operand). Every scalar constant is rounded to float32 the way the
reference computes it (e.g. 1 / r in float)."""

from __future__ import annotations

import numpy as np
import torch

from . import ops


def _f(x) -> float:
    """A float32 constant as the reference computes it."""
    return float(np.float32(x))


def _min_ref(x0, x1):
    # F::Min: the minimum; ties (and NaN) take x0, whose gradient it gets
    return torch.where(x1 < x0, x1, x0)


def _max_ref(x0, x1):
    return torch.where(x0 < x1, x1, x0)


def _step(x):
    # F::Step(0, x) = x < 0 ? 0 : 1 (no gradient)
    return (x >= 0).to(torch.float32)


def _dot2(a, b):
    return a[..., 0] * b[..., 0] + a[..., 1] * b[..., 1]


class _LookupFaces(torch.autograd.Function):
    @staticmethod
    def forward(fctx, attr, faces, vertex_faces, corner):
        fctx.save_for_backward(faces, vertex_faces)
        fctx.corner = corner
        return ops.lookup_faces(attr, faces, corner)

    @staticmethod
    def backward(fctx, gy):
        faces, vf = fctx.saved_tensors
        g = ops.lookup_faces_grad(gy.contiguous(), faces, vf, fctx.corner)
        return g, None, None, None


class _FaceFetch(torch.autograd.Function):
    @staticmethod
    def forward(fctx, tri, idx, prj0, prj1, prj2, seed, radius_px,
                n_samples):
        fctx.save_for_backward(idx, prj0, prj1, prj2)
        fctx.cfg = (float(seed), float(radius_px), int(n_samples))
        return ops.face_fetch(tri, idx)

    @staticmethod
    def backward(fctx, gy):
        idx, p0, p1, p2 = fctx.saved_tensors
        seed, radius, n = fctx.cfg
        g = ops.face_fetch_grad(gy.contiguous(), idx, p0, p1, p2, seed,
                                radius, n)
        return g, None, None, None, None, None, None, None


def clip_of(pos: torch.Tensor, mvp) -> torch.Tensor:
    """MVP (pos, 1) per vertex, row r = ((x m[r] + y m[4+r]) + z m[8+r]) +
    m[12+r] (column-major m; examples/common/geometry_utils.cpp:391-402)."""
    m = torch.as_tensor(np.ascontiguousarray(mvp, np.float32).reshape(16),
                        device=pos.device)
    x, y, z = pos[:, 0], pos[:, 1], pos[:, 2]
    rows = [x * m[r] + y * m[4 + r] + z * m[8 + r] + m[12 + r]
            for r in range(4)]
    return torch.stack(rows, 1)


class PaperHsr:
    """Static tables of one mesh and screen for the paper path: faces
    [F, 3] (float ids), VertexFacesTex [max_deg, V], the soft geometry
    tables of SoftClip's 3F corner vertices, and the pixel centres."""

    def __init__(self, faces, n_verts: int, res: int, radius_px: float,
                 n_samples: int = 8, peels: int = 1, device=None):
        dev = torch.device("cuda", torch.cuda.current_device()) \
            if device is None else torch.device(device)
        f = np.ascontiguousarray(faces, np.float32).reshape(-1, 3)
        nf = f.shape[0]
        self.n_faces, self.n_verts, self.res = nf, int(n_verts), int(res)
        self.radius = float(radius_px)
        self.n_samples, self.peels = int(n_samples), max(1, int(peels))
        self.faces = torch.as_tensor(f, device=dev)
        self.vertex_faces = torch.as_tensor(
            ops.vertex_faces_tex(f, n_verts), device=dev).contiguous()
        self.face_id = torch.as_tensor(
            np.repeat(np.arange(nf, dtype=np.float32), 3), device=dev)
        self.faces_soft = torch.as_tensor(
            np.arange(3 * nf, dtype=np.float32).reshape(nf, 3), device=dev)
        self.pc = ops.screen_coord(res, res, dev)
        self.inv_r = _f(np.float32(1.0) / np.float32(radius_px))
        self.sigma_scale = _f(np.float32(7.0) / np.float32(radius_px))
        self.inv_n = _f(np.float32(1.0) / np.float32(res * res))

    def layers(self, clip: torch.Tensor) -> list[torch.Tensor]:
        """The K soft layers [R, R, 4] of one view (no gradient)."""
        r, R = self.radius, self.res
        with torch.no_grad():
            c = clip.detach().contiguous()
            soft = ops.soft_clip(c, self.faces, R, R, r)
            out, prev = [], None
            for _ in range(self.peels):
                rs = ops.rasterize_soft(soft, self.face_id, self.faces_soft,
                                        c, self.faces, R, R, r,
                                        prev_depth=prev)
                out.append(rs)
                dist, z, cov = rs[..., 0], rs[..., 2], rs[..., 3]
                ge = _step(dist)
                prev = (cov * (ge * (z.clamp(0.0, 1.0) * 0.5) + (1.0 - ge) *
                               ((-dist * self.inv_r).clamp(0.0, 1.0) * 0.5 +
                                0.5))).contiguous()
        return out

    def _soft_prob(self, idx, tris, seed):
        R = float(self.res)
        mask = (idx > 0.5).to(torch.float32)
        prj = [t.detach() for t in tris]

        def screen_of(tri):
            c = _FaceFetch.apply(tri, idx, prj[0], prj[1], prj[2], seed,
                                 self.radius, self.n_samples)
            w = c[..., 3] + (1.0 - mask)
            sx = (c[..., 0] / w * 0.5 + 0.5) * R
            sy = (c[..., 1] / w * 0.5 + 0.5) * R
            return torch.stack([sx, sy], -1)

        s = [screen_of(t) for t in tris]
        pc = self.pc

        def edge_dist(a, b):
            e = b - a
            t = (_dot2(pc - a, e) / (_dot2(e, e) + 1e-12)).clamp(0.0, 1.0)
            dd = pc - (a + t.unsqueeze(-1) * e)
            return torch.sqrt(_dot2(dd, dd) + 1e-12)

        def edge_cross(a, b):
            e = b - a
            return (e[..., 0] * (pc[..., 1] - a[..., 1]) -
                    e[..., 1] * (pc[..., 0] - a[..., 0]))

        dmin = _min_ref(_min_ref(edge_dist(s[0], s[1]), edge_dist(s[1], s[2])),
                        edge_dist(s[2], s[0]))
        cr = [edge_cross(s[0], s[1]), edge_cross(s[1], s[2]),
              edge_cross(s[2], s[0])]
        inside = _min_ref(_step(cr[0]) * _step(cr[1]) * _step(cr[2]) +
                          _step(-cr[0]) * _step(-cr[1]) * _step(-cr[2]),
                          torch.ones_like(dmin))
        dist = (inside * 2.0 - 1.0) * dmin
        return mask * torch.sigmoid(dist * self.sigma_scale)

    def predict(self, clip: torch.Tensor, seed: float) -> torch.Tensor:
        """pred [R, R] of one view; differentiable w.r.t. clip."""
        tris = [_LookupFaces.apply(clip, self.faces, self.vertex_faces, k)
                for k in range(3)]
        one_minus, hard = None, None
        for k, rs in enumerate(self.layers(clip)):
            dist, fid, cov = rs[..., 0], rs[..., 1], rs[..., 3]
            idx = ((fid + 1.0) * cov).contiguous()
            d = self._soft_prob(idx, tris, seed)
            one_minus = (1.0 - d) if one_minus is None \
                else one_minus * (1.0 - d)
            if k == 0:
                hard = cov * _step(dist)
        return _max_ref(hard, 1.0 - one_minus)

    def loss(self, pos: torch.Tensor, mvps, targets: torch.Tensor,
             seed: float) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """Sum over views and pixels of (target - pred)^2 / R^2."""
        total, preds = None, []
        for v in range(len(mvps)):
            pred = self.predict(clip_of(pos, mvps[v]), seed)
            preds.append(pred)
            diff = targets[v] - pred
            term = (diff * diff * self.inv_n).sum()
            total = term if total is None else total + term
        return total, preds


class PaperSilhouetteOptimizer:
    """The example's optimisation loop on the paper path: data gradient by
    autograd, the regulariser (ops.regularized_grad) and Adam
    (run.cpp:407-436); FaceFetch's jitter is the Adam counter."""

    def __init__(self, hsr: PaperHsr, pos0, mvps, targets, lr: float = 0.01,
                 laplacian: float = 0.15, normal: float = 0.4):
        dev = hsr.faces.device
        self.hsr = hsr
        self.pos = torch.as_tensor(np.ascontiguousarray(pos0, np.float32),
                                   device=dev).clone()
        self.mvps = [np.ascontiguousarray(m, np.float32) for m in mvps]
        self.targets = torch.as_tensor(np.ascontiguousarray(targets,
                                                            np.float32),
                                       device=dev)
        self.m = torch.zeros_like(self.pos)
        self.v = torch.zeros_like(self.pos)
        self.t = 0.0
        self.lr, self.laplacian, self.normal = lr, laplacian, normal

    def step(self) -> float:
        p = self.pos.clone().requires_grad_(True)
        loss, _ = self.hsr.loss(p, self.mvps, self.targets, self.t)
        (g,) = torch.autograd.grad(loss, p)
        if self.laplacian != 0.0 or self.normal != 0.0:
            g = ops.regularized_grad(self.pos, self.hsr.faces, g.contiguous(),
                                     self.laplacian, self.normal)
        b1, b2, eps = _f(0.9), _f(0.999), _f(1e-8)
        t_new = self.t + 1.0
        self.m = self.m * b1 + g * _f(1.0 - np.float32(b1))
        self.v = self.v * b2 + g * g * _f(1.0 - np.float32(b2))
        bc1 = _f(np.float32(1.0) - np.float32(b1) ** np.float32(t_new))
        bc2 = _f(np.float32(1.0) - np.float32(b2) ** np.float32(t_new))
        step = (self.m / bc1) / (torch.sqrt(self.v / bc2) + eps) * self.lr
        self.pos = self.pos - step
        self.t = t_new
        return float(loss.detach())
