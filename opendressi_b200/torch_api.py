"""nvdiffrast-style ops on CUDA tensors, mirroring the reference's
``dressi.torch`` (python/dressi/torch/ops.py): ``rasterize``,
``interpolate``, ``texture``, ``antialias`` and ``rasterize_soft`` with the
same arguments, defaults and outputs, differentiable through
torch.autograd.

The reference evaluates each call on its Vulkan engine after copying the
tensors to the host (ops.py:1-14); here every op runs on the tensors' own
device and stream through the C ABI (include/dressi_b200.h), with no host
round trip. As in the reference:

- ``rasterize`` returns (rast, rast_db): rast[..., :] = (u, v, z/w,
  triangle_id + 1), 0 = background, not differentiable w.r.t. pos (the
  geometry gradients come from ``antialias`` / ``rasterize_soft``);
  rast_db is zeros.
- ``interpolate`` is differentiable w.r.t. attr (the exact VJP).
- ``texture`` samples nearest (the reference's v1) or, as an extension,
  bilinear ("linear"); differentiable w.r.t. tex through the inverse-UV
  table built from the uv's provenance (uv must come from ``interpolate``
  of a vertex attribute over a ``rasterize`` output).
- ``antialias`` is differentiable w.r.t. color and pos; n_samples = 0 is
  the exact vertex backward, > 0 the stochastic edge samples, whose seed
  advances per backward call as in the reference (ops.py:520-524).
- ``rasterize_soft`` returns [N, K, H, W, 4] RasterizeSoft layers (K depth
  peels) and is differentiable w.r.t. pos through the dist channel.

Clip positions are OpenGL-style (z in [-w, w]); they are converted to the
Vulkan depth range (z_vk = 0.5 (z + w)) before rasterization, and gradients
back (convert.py:93-109).
"""

from __future__ import annotations

import threading
import weakref

import numpy as np
import torch

from . import _native as N

__all__ = ["RasterizeContext", "RasterizeVulkanContext", "rasterize",
           "interpolate", "texture", "antialias", "rasterize_soft"]


# ---------------------------------------------------------------- context

class _Mesh:
    def __init__(self, tri: torch.Tensor, device):
        if tri.dim() != 2 or tri.shape[1] != 3:
            raise ValueError(f"tri must be [F, 3] int, got {tuple(tri.shape)}")
        if tri.dtype not in (torch.int32, torch.int64):
            raise TypeError(f"tri must be int32/int64, got {tri.dtype}")
        self.faces_f = tri.to(device=device, dtype=torch.float32).contiguous()
        self.n_faces = tri.shape[0]
        t = tri.detach().cpu().numpy().astype(np.int64)
        self.n_verts = int(t.max()) + 1 if t.size else 0
        # VertexFacesTex (mesh_utils.cpp:53-69): {V, max_deg}, -1 padding
        deg = np.bincount(t.ravel(), minlength=self.n_verts) if t.size else \
            np.zeros(0, np.int64)
        max_deg = max(1, int(deg.max()) if deg.size else 1)
        vft = np.full((max_deg, self.n_verts), -1.0, np.float32)
        fill = np.zeros(self.n_verts, np.int64)
        for f in range(t.shape[0]):
            for k in range(3):
                v = t[f, k]
                vft[fill[v], v] = float(f)
                fill[v] += 1
        self.vft = torch.from_numpy(vft).to(device)
        self.max_deg = max_deg
        self.faces_seq = torch.arange(self.n_faces * 3, dtype=torch.float32,
                                      device=device).reshape(-1, 3)
        self.corner_face_id = torch.arange(
            self.n_faces, dtype=torch.float32,
            device=device).repeat_interleave(3).contiguous()


class RasterizeContext:
    """Holds per-mesh tables (float faces, the vertex -> face table) and
    the stochastic-backward seed counters; the counterpart of the
    reference's RasterizeVulkanContext, minus the graphics context."""

    def __init__(self, device=None, output_db: bool = False):
        del output_db
        self.device = torch.device(device) if device is not None else None
        self._meshes: dict = {}
        self._seeds: dict = {}
        self.lock = threading.Lock()

    def mesh(self, tri: torch.Tensor) -> _Mesh:
        device = self.device or (tri.device if tri.is_cuda else
                                 torch.device("cuda"))
        key = (tri.data_ptr(), tuple(tri.shape), str(tri.dtype),
               tri._version, str(device))
        with self.lock:
            md = self._meshes.get(key)
            if md is None:
                md = _Mesh(tri, device)
                self._meshes[key] = md
            return md

    def next_seed(self, key) -> int:
        with self.lock:
            s = self._seeds.get(key, 0) + 1
            self._seeds[key] = s
            return s


RasterizeVulkanContext = RasterizeContext  # the reference's class name


# ------------------------------------------------------------- provenance

_prov: dict = {}


def _attach(t: torch.Tensor, info) -> None:
    k = id(t)
    _prov[k] = info
    weakref.finalize(t, _prov.pop, k, None)


def _lookup(t: torch.Tensor, what: str):
    info = _prov.get(id(t))
    if info is None:
        raise RuntimeError(f"dressi.torch: tensor is not the output of "
                           f"{what}()")
    return info


class _RastInfo:
    def __init__(self, ctx, pos, tri, resolution):
        self.ctx, self.pos, self.tri, self.resolution = ctx, pos, tri, resolution


class _InterpInfo:
    def __init__(self, attr, rast_info):
        self.attr, self.rast_info = attr, rast_info


# ---------------------------------------------------------------- helpers

def _stream():
    return torch.cuda.current_stream().cuda_stream


def _f32(t, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be a CUDA tensor")
    return t.detach().to(torch.float32).contiguous()


def _status(device):
    return torch.zeros(1, dtype=torch.int32, device=device)


def _check(st):
    if int(st.item()) & N.STATUS_INDEX_RANGE:
        raise N.DressiError(N.ERR_DEVICE, "index out of range (face or "
                                          "vertex id)")


def _batch(pos: torch.Tensor) -> torch.Tensor:
    """[V, 4] or [N, V, 4] -> [N, V, 4]."""
    if pos.dim() == 2:
        return pos.unsqueeze(0)
    if pos.dim() == 3:
        return pos
    raise ValueError(f"pos must be [V, 4] or [N, V, 4], got {tuple(pos.shape)}")


def _clip_gl_to_vk(pos: torch.Tensor) -> torch.Tensor:
    out = pos.clone()
    out[..., 2] = 0.5 * (pos[..., 2] + pos[..., 3])
    return out


def _clip_grad_vk_to_gl(g: torch.Tensor) -> torch.Tensor:
    out = g.clone()
    out[..., 2] = 0.5 * g[..., 2]
    out[..., 3] = g[..., 3] + 0.5 * g[..., 2]
    return out


def _resolution(resolution):
    h, w = int(resolution[0]), int(resolution[1])
    if h <= 0 or w <= 0:
        raise ValueError(f"resolution must be positive [H, W], got "
                         f"{resolution}")
    return h, w


def _needs_grad(*ts):
    return torch.is_grad_enabled() and any(
        isinstance(t, torch.Tensor) and t.requires_grad for t in ts)


# -------------------------------------------------------------- rasterize

def rasterize(ctx: RasterizeContext, pos, tri, resolution, ranges=None,
              grad_db: bool = False):
    """(rast, rast_db): rast = (u, v, z/w, triangle_id + 1) [N, H, W, 4]."""
    if ranges is not None:
        raise NotImplementedError("dressi.torch: range mode is not supported")
    del grad_db
    h, w = _resolution(resolution)
    pos_b = _batch(_f32(pos, "pos"))
    if pos_b.shape[2] != 4:
        raise ValueError(f"pos must have 4 components, got {pos_b.shape[2]}")
    md = ctx.mesh(tri)
    n = pos_b.shape[0]
    clip_vk = _clip_gl_to_vk(pos_b).contiguous()
    rast = torch.empty((n, h, w, 4), dtype=torch.float32, device=pos_b.device)
    st = _status(pos_b.device)
    N.call("dressi_rasterize_uvzw", clip_vk.data_ptr(), pos_b.data_ptr(),
           pos_b.shape[1], md.faces_f.data_ptr(), md.n_faces, n, w, h,
           rast.data_ptr(), st.data_ptr(), _stream())
    _check(st)
    _attach(rast, _RastInfo(ctx, pos_b, tri, (h, w)))
    return rast, torch.zeros_like(rast)


# ------------------------------------------------------------ interpolate

class _InterpolateFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, attr, rast, md):
        a = _f32(attr, "attr")
        shared = a.dim() == 2
        a_b = a.unsqueeze(0) if shared else a
        r = _f32(rast, "rast")
        n, h, w = r.shape[0], r.shape[1], r.shape[2]
        c = a_b.shape[-1]
        out = torch.empty((n, h, w, c), dtype=torch.float32, device=a.device)
        st = _status(a.device)
        N.call("dressi_interpolate", a_b.data_ptr(), c, a_b.shape[1],
               a_b.shape[0], r.data_ptr(), md.faces_f.data_ptr(), md.n_faces,
               n, w, h, out.data_ptr(), st.data_ptr(), _stream())
        _check(st)
        fctx.md = md
        fctx.shape = (shared, a_b.shape[0], a_b.shape[1], c, n, h, w)
        fctx.save_for_backward(rast)
        return out

    @staticmethod
    def backward(fctx, grad_out):
        (rast,) = fctx.saved_tensors
        shared, av, nv, c, n, h, w = fctx.shape
        g = _f32(grad_out, "grad_out")
        r = _f32(rast, "rast")
        ga = torch.zeros((av, nv, c), dtype=torch.float32, device=g.device)
        st = _status(g.device)
        N.call("dressi_interpolate_grad", g.data_ptr(), c, nv, av,
               r.data_ptr(), fctx.md.faces_f.data_ptr(), fctx.md.n_faces, n,
               w, h, ga.data_ptr(), st.data_ptr(), _stream())
        return (ga[0] if shared else ga), None, None


def interpolate(attr, rast, tri, rast_db=None, diff_attrs=None):
    """(pixel_attr, None): u a0 + v a1 + (1 - u - v) a2 per pixel;
    differentiable w.r.t. attr ([V, C] shared or [N, V, C])."""
    if rast_db is not None or diff_attrs is not None:
        raise NotImplementedError(
            "dressi.torch.interpolate: rast_db/diff_attrs are not supported")
    rinfo = _lookup(rast, "rasterize")
    md = rinfo.ctx.mesh(tri)
    out = _InterpolateFn.apply(attr, rast, md)
    _attach(out, _InterpInfo(attr, rinfo))
    return out, None


# ---------------------------------------------------------------- texture

_FILTER = {"auto": 0, "nearest": 0, "linear": 1}


class _TextureFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, tex, uv, iinfo, filt):
        t = _f32(tex, "tex")
        if t.dim() == 4:
            if t.shape[0] != 1:
                raise NotImplementedError(
                    "dressi.torch.texture: per-item texture batches are not "
                    "supported (pass [H, W, C] or [1, H, W, C])")
            t = t[0]
        u = _f32(uv, "uv")
        th, tw, c = t.shape
        out = torch.empty(u.shape[:-1] + (c,), dtype=torch.float32,
                          device=t.device)
        N.call("dressi_texture", t.data_ptr(), tw, th, c, u.data_ptr(),
               u.numel() // 2, filt, out.data_ptr(), _stream())
        fctx.iinfo, fctx.filt = iinfo, filt
        fctx.tex_shape = tex.shape
        fctx.save_for_backward(uv)
        return out

    @staticmethod
    def backward(fctx, grad_out):
        (uv,) = fctx.saved_tensors
        iinfo = fctx.iinfo
        if iinfo is None:
            raise RuntimeError(
                "dressi.torch.texture: the texture gradient needs `uv` from "
                "dressi.torch.interpolate (inverse-UV table)")
        rinfo = iinfo.rast_info
        md = rinfo.ctx.mesh(rinfo.tri)
        h, w = rinfo.resolution
        th, tw, c = fctx.tex_shape[-3:]
        vtx_uv = _f32(iinfo.attr, "uv attr")
        g = _f32(grad_out, "grad_out")
        u = _f32(uv, "uv")
        n = u.shape[0]
        gt = torch.zeros((th, tw, c), dtype=torch.float32, device=g.device)
        clip_vk = _clip_gl_to_vk(rinfo.pos)
        one = torch.ones((), device=g.device)
        for i in range(n):
            a = vtx_uv[i if vtx_uv.dim() == 3 and vtx_uv.shape[0] > 1 else 0] \
                if vtx_uv.dim() == 3 else vtx_uv
            # UvAsClip / ScreenAttr (mesh_utils.cpp:180-203)
            uv_clip = torch.stack([a[:, 0] * 2.0 - 1.0, a[:, 1] * 2.0 - 1.0,
                                   torch.full_like(a[:, 0], 0.5),
                                   one.expand_as(a[:, 0])], 1).contiguous()
            cv = clip_vk[i if clip_vk.shape[0] > 1 else 0]
            wv = cv[:, 3]
            sattr = torch.stack([(cv[:, 0] / wv * 0.5 + 0.5) * float(w),
                                 (cv[:, 1] / wv * 0.5 + 0.5) * float(h),
                                 one.expand_as(wv),
                                 torch.zeros_like(wv)], 1).contiguous()
            inv_uv = torch.empty((th, tw, 4), dtype=torch.float32,
                                 device=g.device)
            st = _status(g.device)
            N.call("dressi_rasterize", uv_clip.data_ptr(), uv_clip.shape[0],
                   sattr.data_ptr(), 4, md.faces_f.data_ptr(), md.n_faces, 1,
                   tw, th, inv_uv.data_ptr(), st.data_ptr(), _stream())
            gi = torch.empty((th, tw, c), dtype=torch.float32, device=g.device)
            N.call("dressi_texture_grad", g[i].contiguous().data_ptr(), w, h,
                   c, inv_uv.data_ptr(), tw, th, u[i].contiguous().data_ptr(),
                   fctx.filt, gi.data_ptr(), _stream())
            gt += gi
        if len(fctx.tex_shape) == 4:
            gt = gt.unsqueeze(0)
        return gt, None, None, None


def texture(tex, uv, uv_da=None, mip_level_bias=None, mip=None,
            filter_mode="auto", boundary_mode="wrap", max_mip_level=None):
    """Samples tex [H, W, C] at uv [N, H, W, 2] -> [N, H, W, C]; nearest
    ("auto" / "nearest", the reference's v1) or bilinear ("linear")."""
    if uv_da is not None or mip_level_bias is not None or mip is not None:
        raise NotImplementedError("dressi.torch.texture: mipmaps unsupported "
                                  "(the C2 TexturePlan has a mip pipeline)")
    if filter_mode not in _FILTER:
        raise NotImplementedError(
            f"dressi.torch.texture: filter_mode='{filter_mode}' unsupported")
    del boundary_mode, max_mip_level
    iinfo = _prov.get(id(uv))
    if uv.dim() == 3:
        uv = uv.unsqueeze(0)
    return _TextureFn.apply(tex, uv, iinfo, _FILTER[filter_mode])


# -------------------------------------------------------------- antialias

class _AntiAliasFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, color, rast, pos, ctx, md, n_samples, boost):
        col = _f32(color, "color")
        col_b = col.unsqueeze(0) if col.dim() == 3 else col
        r = _f32(rast, "rast")
        pos_b = _batch(_f32(pos, "pos"))
        n, h, w, c = col_b.shape
        if c > 4:
            raise ValueError("dressi.torch.antialias: color must have 1..4 "
                             "channels")
        tid = r[..., 3].contiguous()
        clip_vk = _clip_gl_to_vk(pos_b)
        if clip_vk.shape[0] != n:
            clip_vk = clip_vk.expand(n, -1, -1)
        clip_vk = clip_vk.contiguous()
        out = torch.empty_like(col_b)
        st = _status(col.device)
        N.call("dressi_antialias", col_b.data_ptr(), c, tid.data_ptr(),
               clip_vk.data_ptr(), clip_vk.shape[1], md.faces_f.data_ptr(),
               md.n_faces, n, w, h, out.data_ptr(), st.data_ptr(), _stream())
        _check(st)
        fctx.md, fctx.ctx = md, ctx
        fctx.n_samples, fctx.boost = n_samples, boost
        fctx.shapes = (color.dim(), pos.dim())
        fctx.save_for_backward(col_b, tid, clip_vk)
        return out if color.dim() == 4 else out[0]

    @staticmethod
    def backward(fctx, grad_out):
        col_b, tid, clip_vk = fctx.saved_tensors
        md = fctx.md
        n, h, w, c = col_b.shape
        g = _f32(grad_out, "grad_out")
        g_b = g.unsqueeze(0) if g.dim() == 3 else g
        want_img, want_pos = fctx.needs_input_grad[0], fctx.needs_input_grad[2]
        gi = torch.empty_like(col_b) if want_img else None
        gc = (torch.zeros((n, clip_vk.shape[1], 4), dtype=torch.float32,
                          device=g.device) if want_pos else None)
        if want_img or want_pos:
            key = ("antialias", h, w, md.n_faces, md.n_verts, c, n)
            it = fctx.ctx.next_seed(key)
            st = _status(g.device)
            for i in range(n):
                # the reference seeds item i of backward call k with k n + i
                seed = float(it * n + i)
                N.call("dressi_antialias_grad",
                       g_b[i].contiguous().data_ptr(),
                       col_b[i].contiguous().data_ptr(), c,
                       tid[i].contiguous().data_ptr(),
                       clip_vk[i].contiguous().data_ptr(), clip_vk.shape[1],
                       md.faces_f.data_ptr(), md.n_faces, md.vft.data_ptr(),
                       md.max_deg, seed, fctx.n_samples, 1, w, h,
                       gi[i].data_ptr() if want_img else None,
                       gc[i].data_ptr() if want_pos else None,
                       st.data_ptr(), _stream())
        out_gc = None
        if gi is not None:
            out_gc = gi if fctx.shapes[0] == 4 else gi[0]
        out_gp = None
        if gc is not None:
            gp = _clip_grad_vk_to_gl(gc) * fctx.boost
            out_gp = gp.sum(0) if fctx.shapes[1] == 2 else gp
        return out_gc, None, out_gp, None, None, None, None


def antialias(color, rast, pos, tri, topology_hash=None,
              pos_gradient_boost=1.0, n_samples=8):
    """Dr.Hair screen-space AA of color [N, H, W, C] given rast and pos;
    differentiable w.r.t. color and pos."""
    del topology_hash
    rinfo = _lookup(rast, "rasterize")
    md = rinfo.ctx.mesh(tri)
    return _AntiAliasFn.apply(color, rast, pos, rinfo.ctx, md, int(n_samples),
                              float(pos_gradient_boost))


# --------------------------------------------------------- rasterize_soft

class _RasterizeSoftFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, pos, md, resolution, radius_px, peels):
        h, w = resolution
        pos_b = _batch(_f32(pos, "pos"))
        n, nv = pos_b.shape[0], pos_b.shape[1]
        clip_vk = _clip_gl_to_vk(pos_b).contiguous()
        st = _status(pos_b.device)
        soft = torch.empty((n, md.n_faces * 3, 4), dtype=torch.float32,
                           device=pos_b.device)
        N.call("dressi_soft_clip", clip_vk.data_ptr(), nv,
               md.faces_f.data_ptr(), md.n_faces, n, w, h, float(radius_px),
               soft.data_ptr(), st.data_ptr(), _stream())
        fid = md.corner_face_id.expand(n, -1).contiguous()
        out = torch.empty((n, peels, h, w, 4), dtype=torch.float32,
                          device=pos_b.device)
        prev = None
        for k in range(peels):
            layer = torch.empty((n, h, w, 4), dtype=torch.float32,
                                device=pos_b.device)
            N.call("dressi_rasterize_soft", soft.data_ptr(), md.n_faces * 3,
                   fid.data_ptr(), md.faces_seq.data_ptr(), md.n_faces,
                   clip_vk.data_ptr(), nv, md.faces_f.data_ptr(), n, w, h,
                   float(radius_px),
                   None if prev is None else prev.data_ptr(),
                   layer.data_ptr(), st.data_ptr(), _stream())
            out[:, k] = layer
            if k + 1 < peels:
                # the next peel's threshold: this layer's Eq.3 shifted depth
                # rebuilt from its channels (ops.py:628-636)
                dist_c, cov = layer[..., 0], layer[..., 3]
                ge = (dist_c >= 0).to(torch.float32)
                prev = (cov * (ge * (layer[..., 2].clamp(0.0, 1.0) * 0.5) +
                               (1.0 - ge) * ((dist_c * (-1.0 / radius_px))
                                             .clamp(0.0, 1.0) * 0.5 + 0.5))
                        ).contiguous()
        _check(st)
        fctx.md = md
        fctx.dims = (n, nv, h, w, peels, pos.dim())
        fctx.save_for_backward(out, clip_vk)
        return out

    @staticmethod
    def backward(fctx, grad_out):
        out, clip_vk = fctx.saved_tensors
        n, nv, h, w, peels, pdim = fctx.dims
        md = fctx.md
        g = _f32(grad_out, "grad_out")
        gc = torch.zeros((n, nv, 4), dtype=torch.float32, device=g.device)
        st = _status(g.device)
        for k in range(peels):
            gy = g[:, k, :, :, 0].contiguous()   # the dist channel
            rs = out[:, k].contiguous()
            N.call("dressi_rasterize_soft_grad", gy.data_ptr(), rs.data_ptr(),
                   clip_vk.data_ptr(), nv, md.faces_f.data_ptr(), md.n_faces,
                   n, w, h, gc.data_ptr(), st.data_ptr(), _stream())
        gp = _clip_grad_vk_to_gl(gc)
        return (gp.sum(0) if pdim == 2 else gp), None, None, None, None


def rasterize_soft(ctx: RasterizeContext, pos, tri, resolution,
                   radius_px: float = 3.0, peels: int = 1):
    """HardSoftRas layers [N, K, H, W, 4] = (dist_px, face_id, hard_z,
    coverage) per peel; differentiable w.r.t. pos through dist."""
    h, w = _resolution(resolution)
    md = ctx.mesh(tri)
    return _RasterizeSoftFn.apply(pos, md, (h, w), float(radius_px),
                                  max(1, int(peels)))
