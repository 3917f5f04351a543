"""nvdiffrast-style ops on CUDA tensors, mirroring the reference's
``dressi.torch`` (python/dressi/torch/ops.py): ``rasterize``,
``interpolate``, ``texture``, ``antialias`` and ``rasterize_soft`` with the
same arguments, defaults and outputs.

Each op is a ``torch.library`` custom op (namespace ``dressi_b200``) with a
fake (meta) implementation for shape propagation and a registered autograd
formula, so the ops trace under ``torch.compile`` and run inside CUDA graphs.
They run on the input tensors' own device and its current stream through the
C ABI (include/dressi_b200.h), with no host round trip and no
synchronisation: the reference's index errors set bits of a per-device
status word that ``check_status()`` reads (one synchronisation for any
number of ops).

As in the reference:

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
  the exact vertex backward, > 0 the stochastic edge samples. The seeds
  follow the reference's schedule (ops.py:520-524: item i of call k gets
  k n + i); the call counter advances when the forward runs.
- ``rasterize_soft`` returns [N, K, H, W, 4] RasterizeSoft layers (K depth
  peels) and is differentiable w.r.t. pos through the dist channel.

Clip positions are OpenGL-style (z in [-w, w]); they are converted to the
Vulkan depth range (z_vk = 0.5 (z + w)) before rasterization and the
gradients flow back through that conversion (convert.py:93-109).
"""

from __future__ import annotations

import threading
import weakref

import numpy as np
import torch
from torch.library import custom_op

from . import _native as N
from .ops import check_status, status_word

__all__ = ["RasterizeContext", "RasterizeVulkanContext", "rasterize",
           "interpolate", "texture", "antialias", "rasterize_soft",
           "check_status"]

Tensor = torch.Tensor


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# ---------------------------------------------------------------- context

class _Mesh:
    """Device tables of one triangle tensor: float faces, the vertex -> face
    table (VertexFacesTex, mesh_utils.cpp:53-69), the sequential soft faces
    and corner face ids. Holds `tri` so its memory cannot be reused by
    another tensor while the tables are cached (the reference's MeshData
    pins its source for the same reason, meshdata.py:19-22)."""

    def __init__(self, tri: Tensor, device):
        if tri.dim() != 2 or tri.shape[1] != 3:
            raise ValueError(f"tri must be [F, 3] int, got {tuple(tri.shape)}")
        if tri.dtype not in (torch.int32, torch.int64):
            raise TypeError(f"tri must be int32/int64, got {tri.dtype}")
        self.src = tri
        self.faces_f = tri.to(device=device, dtype=torch.float32).contiguous()
        self.n_faces = tri.shape[0]
        t = tri.detach().cpu().numpy().astype(np.int64)
        self.n_verts = int(t.max()) + 1 if t.size else 0
        deg = np.bincount(t.reshape(-1), minlength=self.n_verts) if t.size \
            else np.zeros(0, np.int64)
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
    """Holds per-mesh tables and the stochastic-backward seed counters; the
    counterpart of the reference's RasterizeVulkanContext, minus the
    graphics context."""

    def __init__(self, device=None, output_db: bool = False):
        del output_db
        self.device = torch.device(device) if device is not None else None
        self._meshes: dict = {}
        self._seeds: dict = {}
        self.lock = threading.Lock()

    @torch.compiler.disable
    def mesh(self, tri: Tensor, device=None) -> _Mesh:
        device = torch.device(device) if device is not None else (
            self.device or (tri.device if tri.is_cuda else
                            torch.device("cuda", torch.cuda.current_device())))
        if tri.is_cuda and tri.device != device:
            raise ValueError(f"tri is on {tri.device}, the op runs on "
                             f"{device}")
        key = (tri.data_ptr(), tuple(tri.shape), str(tri.dtype),
               tri._version, str(device))
        with self.lock:
            md = self._meshes.get(key)
            if md is None or md.src is not tri:
                md = _Mesh(tri, device)
                self._meshes[key] = md
            return md

    def clear_cache(self) -> None:
        """Drops every cached mesh table (and the pinned tri tensors)."""
        with self.lock:
            self._meshes.clear()

    @torch.compiler.disable
    def next_seed(self, key) -> int:
        with self.lock:
            s = self._seeds.get(key, 0) + 1
            self._seeds[key] = s
            return s


RasterizeVulkanContext = RasterizeContext  # the reference's class name


# ------------------------------------------------------------- provenance

_prov: dict = {}


@torch.compiler.disable
def _attach(t: Tensor, info) -> None:
    k = id(t)
    _prov[k] = info
    weakref.finalize(t, _prov.pop, k, None)


@torch.compiler.disable
def _lookup(t: Tensor, what: str):
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

def _f32(t, name):
    if not isinstance(t, Tensor) or not t.is_cuda:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be a CUDA tensor")
    return t.to(torch.float32).contiguous()


def _batch(pos: Tensor) -> Tensor:
    """[V, 4] or [N, V, 4] -> [N, V, 4]."""
    if pos.dim() == 2:
        return pos.unsqueeze(0)
    if pos.dim() == 3:
        return pos
    raise ValueError(f"pos must be [V, 4] or [N, V, 4], got {tuple(pos.shape)}")


def _clip_gl_to_vk(pos: Tensor) -> Tensor:
    # z_vk = 0.5 (z + w); differentiable, so the gradient flows back through
    # the reference's transpose (clip_grad_vk_to_gl, convert.py:100-109)
    z = 0.5 * (pos[..., 2:3] + pos[..., 3:4])
    return torch.cat([pos[..., 0:2], z, pos[..., 3:4]], -1).contiguous()


def _resolution(resolution):
    h, w = int(resolution[0]), int(resolution[1])
    if h <= 0 or w <= 0:
        raise ValueError(f"resolution must be positive [H, W], got "
                         f"{resolution}")
    return h, w


def _same_device(*ts):
    devs = {t.device for t in ts if isinstance(t, Tensor) and t.is_cuda}
    if len(devs) > 1:
        raise ValueError(f"dressi.torch: inputs on several devices {devs}")


# ------------------------------------------------------- custom ops: raster

@custom_op("dressi_b200::rasterize", mutates_args=())
def _rasterize_op(clip_vk: Tensor, pos_gl: Tensor, faces_f: Tensor, h: int,
                  w: int) -> Tensor:
    n = clip_vk.shape[0]
    with torch.cuda.device(clip_vk.device):
        rast = torch.empty((n, h, w, 4), dtype=torch.float32,
                           device=clip_vk.device)
        N.call("dressi_rasterize_uvzw", clip_vk.data_ptr(), pos_gl.data_ptr(),
               clip_vk.shape[1], faces_f.data_ptr(), faces_f.shape[0], n, w,
               h, rast.data_ptr(), status_word(clip_vk.device).data_ptr(),
               _stream(clip_vk))
    return rast


@_rasterize_op.register_fake
def _(clip_vk, pos_gl, faces_f, h, w):
    return clip_vk.new_empty((clip_vk.shape[0], h, w, 4))


def rasterize(ctx: RasterizeContext, pos, tri, resolution, ranges=None,
              grad_db: bool = False):
    """(rast, rast_db): rast = (u, v, z/w, triangle_id + 1) [N, H, W, 4]."""
    if ranges is not None:
        raise NotImplementedError("dressi.torch: range mode is not supported")
    del grad_db
    h, w = _resolution(resolution)
    _same_device(pos, tri)
    pos_b = _batch(_f32(pos, "pos")).detach()
    if pos_b.shape[2] != 4:
        raise ValueError(f"pos must have 4 components, got {pos_b.shape[2]}")
    md = ctx.mesh(tri, pos_b.device)
    rast = _rasterize_op(_clip_gl_to_vk(pos_b), pos_b, md.faces_f, h, w)
    _attach(rast, _RastInfo(ctx, pos_b, tri, (h, w)))
    return rast, torch.zeros_like(rast)


# --------------------------------------------------- custom ops: interpolate

@custom_op("dressi_b200::interpolate", mutates_args=())
def _interpolate_op(attr_b: Tensor, rast: Tensor, faces_f: Tensor) -> Tensor:
    n, h, w = rast.shape[0], rast.shape[1], rast.shape[2]
    c = attr_b.shape[-1]
    with torch.cuda.device(attr_b.device):
        out = torch.empty((n, h, w, c), dtype=torch.float32,
                          device=attr_b.device)
        N.call("dressi_interpolate", attr_b.data_ptr(), c, attr_b.shape[1],
               attr_b.shape[0], rast.data_ptr(), faces_f.data_ptr(),
               faces_f.shape[0], n, w, h, out.data_ptr(),
               status_word(attr_b.device).data_ptr(), _stream(attr_b))
    return out


@_interpolate_op.register_fake
def _(attr_b, rast, faces_f):
    return attr_b.new_empty((rast.shape[0], rast.shape[1], rast.shape[2],
                             attr_b.shape[-1]))


@custom_op("dressi_b200::interpolate_grad", mutates_args=())
def _interpolate_grad_op(gy: Tensor, rast: Tensor, faces_f: Tensor,
                         attr_views: int, n_verts: int) -> Tensor:
    n, h, w, c = gy.shape
    with torch.cuda.device(gy.device):
        ga = torch.zeros((attr_views, n_verts, c), dtype=torch.float32,
                         device=gy.device)
        N.call("dressi_interpolate_grad", gy.data_ptr(), c, n_verts,
               attr_views, rast.data_ptr(), faces_f.data_ptr(),
               faces_f.shape[0], n, w, h, ga.data_ptr(),
               status_word(gy.device).data_ptr(), _stream(gy))
    return ga


@_interpolate_grad_op.register_fake
def _(gy, rast, faces_f, attr_views, n_verts):
    return gy.new_empty((attr_views, n_verts, gy.shape[-1]))


def _interp_setup(ctx, inputs, output):
    attr_b, rast, faces_f = inputs
    ctx.save_for_backward(rast, faces_f)
    ctx.dims = (attr_b.shape[0], attr_b.shape[1])


def _interp_backward(ctx, g):
    rast, faces_f = ctx.saved_tensors
    av, nv = ctx.dims
    return _interpolate_grad_op(g.contiguous(), rast, faces_f, av, nv), \
        None, None


_interpolate_op.register_autograd(_interp_backward, setup_context=_interp_setup)


def interpolate(attr, rast, tri, rast_db=None, diff_attrs=None):
    """(pixel_attr, None): u a0 + v a1 + (1 - u - v) a2 per pixel;
    differentiable w.r.t. attr ([V, C] shared or [N, V, C])."""
    if rast_db is not None or diff_attrs is not None:
        raise NotImplementedError(
            "dressi.torch.interpolate: rast_db/diff_attrs are not supported")
    _same_device(attr, rast, tri)
    rinfo = _lookup(rast, "rasterize")
    md = rinfo.ctx.mesh(tri, rast.device)
    a = _f32(attr, "attr")
    a_b = a.unsqueeze(0) if a.dim() == 2 else a
    out = _interpolate_op(a_b, _f32(rast, "rast").detach(), md.faces_f)
    _attach(out, _InterpInfo(attr, rinfo))
    return out, None


# ------------------------------------------------------ custom ops: texture

_FILTER = {"auto": 0, "nearest": 0, "linear": 1}


@custom_op("dressi_b200::texture", mutates_args=())
def _texture_op(tex: Tensor, uv: Tensor, vtx_uv: Tensor, clip_vk: Tensor,
                faces_f: Tensor, sh: int, sw: int, filt: int) -> Tensor:
    th, tw, c = tex.shape
    with torch.cuda.device(tex.device):
        out = torch.empty(uv.shape[:-1] + (c,), dtype=torch.float32,
                          device=tex.device)
        N.call("dressi_texture", tex.data_ptr(), tw, th, c, uv.data_ptr(),
               uv.numel() // 2, filt, out.data_ptr(), _stream(tex))
    return out


@_texture_op.register_fake
def _(tex, uv, vtx_uv, clip_vk, faces_f, sh, sw, filt):
    return tex.new_empty(tuple(uv.shape[:-1]) + (tex.shape[-1],))


@custom_op("dressi_b200::texture_grad", mutates_args=())
def _texture_grad_op(gy: Tensor, uv: Tensor, vtx_uv: Tensor, clip_vk: Tensor,
                     faces_f: Tensor, th: int, tw: int, filt: int) -> Tensor:
    n, h, w, c = gy.shape
    dev = gy.device
    with torch.cuda.device(dev):
        gt = torch.zeros((th, tw, c), dtype=torch.float32, device=dev)
        one = torch.ones((), device=dev)
        st = status_word(dev)
        for i in range(n):
            a = vtx_uv[i if vtx_uv.shape[0] > 1 else 0]
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
            inv_uv = torch.empty((th, tw, 4), dtype=torch.float32, device=dev)
            N.call("dressi_rasterize", uv_clip.data_ptr(), uv_clip.shape[0],
                   sattr.data_ptr(), 4, faces_f.data_ptr(), faces_f.shape[0],
                   1, tw, th, inv_uv.data_ptr(), st.data_ptr(), _stream(gy))
            gi = torch.empty((th, tw, c), dtype=torch.float32, device=dev)
            N.call("dressi_texture_grad", gy[i].contiguous().data_ptr(), w, h,
                   c, inv_uv.data_ptr(), tw, th, uv[i].contiguous().data_ptr(),
                   filt, gi.data_ptr(), _stream(gy))
            gt += gi
    return gt


@_texture_grad_op.register_fake
def _(gy, uv, vtx_uv, clip_vk, faces_f, th, tw, filt):
    return gy.new_empty((th, tw, gy.shape[-1]))


def _tex_setup(ctx, inputs, output):
    tex, uv, vtx_uv, clip_vk, faces_f, sh, sw, filt = inputs
    ctx.save_for_backward(uv, vtx_uv, clip_vk, faces_f)
    ctx.meta = (tex.shape[0], tex.shape[1], filt)


def _tex_backward(ctx, g):
    uv, vtx_uv, clip_vk, faces_f = ctx.saved_tensors
    th, tw, filt = ctx.meta
    if vtx_uv.numel() == 0:
        raise RuntimeError(
            "dressi.torch.texture: the texture gradient needs `uv` from "
            "dressi.torch.interpolate (inverse-UV table)")
    gt = _texture_grad_op(g.contiguous(), uv, vtx_uv, clip_vk, faces_f, th,
                          tw, filt)
    return gt, None, None, None, None, None, None, None


_texture_op.register_autograd(_tex_backward, setup_context=_tex_setup)


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
    _same_device(tex, uv)
    iinfo = _prov.get(id(uv))
    t = _f32(tex, "tex")
    batched = t.dim() == 4
    if batched:
        if t.shape[0] != 1:
            raise NotImplementedError(
                "dressi.torch.texture: per-item texture batches are not "
                "supported (pass [H, W, C] or [1, H, W, C])")
        t = t[0]
    u = _f32(uv, "uv")
    if u.dim() == 3:
        u = u.unsqueeze(0)
    if iinfo is not None:
        rinfo = iinfo.rast_info
        md = rinfo.ctx.mesh(rinfo.tri, u.device)
        vtx_uv = _f32(iinfo.attr, "uv attr").detach()
        if vtx_uv.dim() == 2:
            vtx_uv = vtx_uv.unsqueeze(0)
        clip_vk = _clip_gl_to_vk(rinfo.pos.detach())
        sh, sw = rinfo.resolution
        faces_f = md.faces_f
    else:
        vtx_uv = clip_vk = faces_f = u.new_empty((0,))
        sh = sw = 0
    out = _texture_op(t, u.detach(), vtx_uv, clip_vk, faces_f, sh, sw,
                      _FILTER[filter_mode])
    return out


# ---------------------------------------------------- custom ops: antialias

@custom_op("dressi_b200::antialias", mutates_args=())
def _antialias_op(color: Tensor, tid: Tensor, clip_vk: Tensor,
                  faces_f: Tensor, vft: Tensor, seed_base: int,
                  n_samples: int, boost: float) -> Tensor:
    n, h, w, c = color.shape
    with torch.cuda.device(color.device):
        out = torch.empty_like(color)
        N.call("dressi_antialias", color.data_ptr(), c, tid.data_ptr(),
               clip_vk.data_ptr(), clip_vk.shape[1], faces_f.data_ptr(),
               faces_f.shape[0], n, w, h, out.data_ptr(),
               status_word(color.device).data_ptr(), _stream(color))
    return out


@_antialias_op.register_fake
def _(color, tid, clip_vk, faces_f, vft, seed_base, n_samples, boost):
    return torch.empty_like(color)


@custom_op("dressi_b200::antialias_grad", mutates_args=())
def _antialias_grad_op(gy: Tensor, color: Tensor, tid: Tensor,
                       clip_vk: Tensor, faces_f: Tensor, vft: Tensor,
                       seed_base: int, n_samples: int, boost: float,
                       want_img: bool, want_pos: bool
                       ) -> tuple[Tensor, Tensor]:
    n, h, w, c = color.shape
    dev = gy.device
    with torch.cuda.device(dev):
        gi = torch.empty_like(color) if want_img else color.new_empty((0,))
        gc = (torch.zeros((n, clip_vk.shape[1], 4), dtype=torch.float32,
                          device=dev) if want_pos else color.new_empty((0,)))
        st = status_word(dev)
        for i in range(n):
            # item i of backward call k is seeded k n + i (ops.py:520-524)
            seed = float(seed_base * n + i)
            N.call("dressi_antialias_grad", gy[i].contiguous().data_ptr(),
                   color[i].contiguous().data_ptr(), c,
                   tid[i].contiguous().data_ptr(),
                   clip_vk[i].contiguous().data_ptr(), clip_vk.shape[1],
                   faces_f.data_ptr(), faces_f.shape[0], vft.data_ptr(),
                   vft.shape[0], seed, n_samples, 1, w, h,
                   gi[i].data_ptr() if want_img else None,
                   gc[i].data_ptr() if want_pos else None,
                   st.data_ptr(), _stream(gy))
        if want_pos and boost != 1.0:
            gc = gc * boost
    return gi, gc


@_antialias_grad_op.register_fake
def _(gy, color, tid, clip_vk, faces_f, vft, seed_base, n_samples, boost,
      want_img, want_pos):
    gi = torch.empty_like(color) if want_img else color.new_empty((0,))
    gc = (color.new_empty((color.shape[0], clip_vk.shape[1], 4)) if want_pos
          else color.new_empty((0,)))
    return gi, gc


def _aa_setup(ctx, inputs, output):
    color, tid, clip_vk, faces_f, vft, seed_base, n_samples, boost = inputs
    ctx.save_for_backward(color, tid, clip_vk, faces_f, vft)
    ctx.meta = (seed_base, n_samples, boost)


def _aa_backward(ctx, g):
    color, tid, clip_vk, faces_f, vft = ctx.saved_tensors
    seed_base, n_samples, boost = ctx.meta
    want_img, want_pos = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
    if not (want_img or want_pos):
        return (None,) * 8
    gi, gc = _antialias_grad_op(g.contiguous(), color, tid, clip_vk, faces_f,
                                vft, seed_base, n_samples, boost, want_img,
                                want_pos)
    return (gi if want_img else None, None, gc if want_pos else None, None,
            None, None, None, None)


_antialias_op.register_autograd(_aa_backward, setup_context=_aa_setup)


def antialias(color, rast, pos, tri, topology_hash=None,
              pos_gradient_boost=1.0, n_samples=8):
    """Dr.Hair screen-space AA of color [N, H, W, C] given rast and pos;
    differentiable w.r.t. color and pos."""
    del topology_hash
    _same_device(color, rast, pos, tri)
    rinfo = _lookup(rast, "rasterize")
    col = _f32(color, "color")
    col_b = col.unsqueeze(0) if col.dim() == 3 else col
    n, h, w, c = col_b.shape
    if c > 4:
        raise ValueError("dressi.torch.antialias: color must have 1..4 "
                         "channels")
    md = rinfo.ctx.mesh(tri, col_b.device)
    tid = _f32(rast, "rast")[..., 3].detach().contiguous()
    clip_vk = _clip_gl_to_vk(_batch(_f32(pos, "pos")))
    if clip_vk.shape[0] != n:
        clip_vk = clip_vk.expand(n, -1, -1)
    seed = rinfo.ctx.next_seed(("antialias", h, w, md.n_faces, md.n_verts, c,
                                n))
    out = _antialias_op(col_b, tid, clip_vk.contiguous(), md.faces_f, md.vft,
                        int(seed), int(n_samples), float(pos_gradient_boost))
    return out if col.dim() == 4 else out[0]


# ----------------------------------------------- custom ops: rasterize_soft

@custom_op("dressi_b200::rasterize_soft", mutates_args=())
def _rasterize_soft_op(clip_vk: Tensor, faces_f: Tensor, faces_seq: Tensor,
                       corner_face_id: Tensor, h: int, w: int,
                       radius_px: float, peels: int) -> Tensor:
    n, nv = clip_vk.shape[0], clip_vk.shape[1]
    nf = faces_f.shape[0]
    dev = clip_vk.device
    with torch.cuda.device(dev):
        st = status_word(dev)
        s = _stream(clip_vk)
        soft = torch.empty((n, nf * 3, 4), dtype=torch.float32, device=dev)
        N.call("dressi_soft_clip", clip_vk.data_ptr(), nv, faces_f.data_ptr(),
               nf, n, w, h, float(radius_px), soft.data_ptr(), st.data_ptr(),
               s)
        fid = corner_face_id.expand(n, -1).contiguous()
        out = torch.empty((n, peels, h, w, 4), dtype=torch.float32,
                          device=dev)
        prev = None
        for k in range(peels):
            layer = torch.empty((n, h, w, 4), dtype=torch.float32, device=dev)
            N.call("dressi_rasterize_soft", soft.data_ptr(), nf * 3,
                   fid.data_ptr(), faces_seq.data_ptr(), nf,
                   clip_vk.data_ptr(), nv, faces_f.data_ptr(), n, w, h,
                   float(radius_px),
                   None if prev is None else prev.data_ptr(),
                   layer.data_ptr(), st.data_ptr(), s)
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
    return out


@_rasterize_soft_op.register_fake
def _(clip_vk, faces_f, faces_seq, corner_face_id, h, w, radius_px, peels):
    return clip_vk.new_empty((clip_vk.shape[0], peels, h, w, 4))


@custom_op("dressi_b200::rasterize_soft_grad", mutates_args=())
def _rasterize_soft_grad_op(gy: Tensor, out: Tensor, clip_vk: Tensor,
                            faces_f: Tensor) -> Tensor:
    n, peels, h, w, _ = out.shape
    nv = clip_vk.shape[1]
    dev = gy.device
    with torch.cuda.device(dev):
        gc = torch.zeros((n, nv, 4), dtype=torch.float32, device=dev)
        st = status_word(dev)
        for k in range(peels):
            gk = gy[:, k, :, :, 0].contiguous()   # the dist channel
            rs = out[:, k].contiguous()
            N.call("dressi_rasterize_soft_grad", gk.data_ptr(), rs.data_ptr(),
                   clip_vk.data_ptr(), nv, faces_f.data_ptr(),
                   faces_f.shape[0], n, w, h, gc.data_ptr(), st.data_ptr(),
                   _stream(gy))
    return gc


@_rasterize_soft_grad_op.register_fake
def _(gy, out, clip_vk, faces_f):
    return clip_vk.new_empty((out.shape[0], clip_vk.shape[1], 4))


def _rs_setup(ctx, inputs, output):
    clip_vk, faces_f = inputs[0], inputs[1]
    ctx.save_for_backward(output, clip_vk, faces_f)


def _rs_backward(ctx, g):
    out, clip_vk, faces_f = ctx.saved_tensors
    gc = _rasterize_soft_grad_op(g.contiguous(), out, clip_vk, faces_f)
    return gc, None, None, None, None, None, None, None


_rasterize_soft_op.register_autograd(_rs_backward, setup_context=_rs_setup)


def rasterize_soft(ctx: RasterizeContext, pos, tri, resolution,
                   radius_px: float = 3.0, peels: int = 1):
    """HardSoftRas layers [N, K, H, W, 4] = (dist_px, face_id, hard_z,
    coverage) per peel; differentiable w.r.t. pos through dist."""
    h, w = _resolution(resolution)
    _same_device(pos, tri)
    pos_b = _batch(_f32(pos, "pos"))
    md = ctx.mesh(tri, pos_b.device)
    return _rasterize_soft_op(_clip_gl_to_vk(pos_b), md.faces_f, md.faces_seq,
                              md.corner_face_id, h, w, float(radius_px),
                              max(1, int(peels)))
