"""Op-level entry points on torch CUDA tensors (zero-copy; current stream).

Each function mirrors one reference op (src/core/f_ops.cpp) and calls the
C ABI with raw device pointers. Inputs are float32 CUDA tensors in the
reference layouts; views are stacked along a leading dimension.

Errors the reference raises as DressiError (bad shapes, and -- through the
device status word -- out-of-range indices) raise DressiError here.
"""

from __future__ import annotations

import torch

from . import _native as N

__all__ = [
    "soft_clip",
    "rasterize_soft",
    "rasterize_soft_grad",
    "rasterize_face_id",
    "rasterize",
    "antialias",
    "antialias_grad",
    "texture",
    "texture_grad",
    "vertex_faces_tex",
    "vertex_neighbors_tex",
    "face_neighbors_tex",
    "vertex_neighbor_mean",
    "normal_consistency_face_term",
    "normal_consistency_vertex_grad",
    "sum_all",
    "regularized_grad",
    "equirect_sample",
    "equirect_sample_grad",
    "irradiance_conv",
    "irradiance_conv_grad",
    "prefilter_conv",
    "prefilter_conv_grad",
    "brdf_lut",
    "avg_pool2x2",
    "avg_pool2x2_grad",
    "check_status",
]


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dev(t: torch.Tensor, name: str, ndim: int | None = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be float32")
    if ndim is not None and t.dim() != ndim:
        raise N.DressiError(N.ERR_INVALID,
                            f"{name} must have {ndim} dims, got {t.dim()}")
    return t.contiguous()


def _ptr(t):
    return None if t is None else t.data_ptr()


# Index errors the reference throws from inside its CPU kernels are bits of
# a device status word here. Every op ORs into one persistent word per
# device instead of reading its own back, so an op never waits for the GPU;
# check_status() synchronises once and raises for every op since the last
# check. set_eager_checks(True) restores a check after every op.
_words: dict = {}
_eager = False


def set_eager_checks(on: bool) -> None:
    """Check the status word (synchronising) after every op when on."""
    global _eager
    _eager = bool(on)


def status_word(device=None) -> torch.Tensor:
    """The device's accumulated status word (an int32 CUDA tensor)."""
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{key}")
        _words[key] = w
    return w


def _new_status(device):
    return status_word(device)


def check_status(device=None, reset: bool = True) -> int:
    """Synchronises with `device` (a device, a tensor on it, or None for
    the current device) and raises DressiError if a kernel reported an
    index error since the last check; reset clears the word."""
    if isinstance(device, torch.Tensor):
        device = device.device
    w = status_word(device)
    word = int(w.item()) & 0xFFFFFFFF
    if reset and word:
        w.zero_()
    if word & N.STATUS_INDEX_RANGE:
        raise N.DressiError(N.ERR_DEVICE,
                            "index out of range (face or vertex id)")
    return word


def _after(status: torch.Tensor) -> None:
    if _eager:
        check_status(status.device)


def _views(t: torch.Tensor, base_dims: int) -> tuple[torch.Tensor, int]:
    """Adds a leading view dimension when absent."""
    if t.dim() == base_dims:
        return t.unsqueeze(0), 1
    return t, t.shape[0]


def _match_views(t: torch.Tensor, views: int, name: str) -> torch.Tensor:
    """Broadcasts a single-view input over `views`; rejects other counts."""
    if t.shape[0] == views:
        return t
    if t.shape[0] == 1:
        return t.expand(views, *t.shape[1:]).contiguous()
    raise N.DressiError(N.ERR_INVALID, f"{name}: {t.shape[0]} views, "
                        f"expected {views}")


def soft_clip(clip, faces, width: int, height: int, radius_px: float,
              check: bool = True):
    """F::SoftClip: clip [(views,) V, 4], faces [F, 3] -> [(views,) 3F, 4]."""
    squeeze = clip.dim() == 2
    clip = _dev(clip, "clip")
    faces = _dev(faces, "faces", 2)
    clip, views = _views(clip, 2)
    n_faces = faces.shape[0]
    out = torch.empty((views, 3 * n_faces, 4), dtype=torch.float32,
                      device=clip.device)
    st = _new_status(clip.device)
    N.call("dressi_soft_clip", clip.data_ptr(), clip.shape[1],
           faces.data_ptr(), n_faces, views, width, height, float(radius_px),
           out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out[0] if squeeze else out


def rasterize_soft(soft_clip, face_id, faces_soft, hard_clip, faces_tex,
                   width: int, height: int, radius_px: float,
                   prev_depth=None, check: bool = True):
    """F::RasterizeSoft -> [(views,) H, W, 4] (dist, face_id, hard_z, cov).

    soft_clip [(views,) 3F, 4], face_id [(views,) 3F], faces_soft [F, 3],
    hard_clip [(views,) V, 4], faces_tex [F, 3], prev_depth [(views,) H, W]
    (depth-peeling variant) or None."""
    squeeze = soft_clip.dim() == 2
    soft_clip = _dev(soft_clip, "soft_clip")
    face_id = _dev(face_id, "face_id")
    hard_clip = _dev(hard_clip, "hard_clip")
    faces_soft = _dev(faces_soft, "faces_soft", 2)
    faces_tex = _dev(faces_tex, "faces_tex", 2)
    soft_clip, views = _views(soft_clip, 2)
    face_id, _ = _views(face_id, 1)
    hard_clip, _ = _views(hard_clip, 2)
    if prev_depth is not None:
        prev_depth = _dev(prev_depth, "prev_depth")
        prev_depth, _ = _views(prev_depth, 2)
    n_faces = faces_soft.shape[0]
    face_id = _match_views(face_id, views, "face_id")
    hard_clip = _match_views(hard_clip, views, "hard_clip")
    if prev_depth is not None:
        prev_depth = _match_views(prev_depth, views, "prev_depth")
    out = torch.empty((views, height, width, 4), dtype=torch.float32,
                      device=soft_clip.device)
    st = _new_status(soft_clip.device)
    N.call("dressi_rasterize_soft", soft_clip.data_ptr(), soft_clip.shape[1],
           face_id.data_ptr(), faces_soft.data_ptr(), n_faces,
           hard_clip.data_ptr(), hard_clip.shape[1], faces_tex.data_ptr(),
           views, width, height, float(radius_px), _ptr(prev_depth),
           out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out[0] if squeeze else out


def rasterize_soft_grad(gy, rs, clip, faces, check: bool = True):
    """ColSum(GatherDistGrad): d(sum gy*dist)/d clip -> [(views,) V, 4]."""
    squeeze = clip.dim() == 2
    gy = _dev(gy, "gy")
    rs = _dev(rs, "rs")
    clip = _dev(clip, "clip")
    faces = _dev(faces, "faces", 2)
    gy, views = _views(gy, 2)
    rs, _ = _views(rs, 3)
    clip, _ = _views(clip, 2)
    rs = _match_views(rs, views, "rs")
    clip = _match_views(clip, views, "clip")
    h, w = gy.shape[1], gy.shape[2]
    grad = torch.zeros((views, clip.shape[1], 4), dtype=torch.float32,
                       device=clip.device)
    st = _new_status(clip.device)
    N.call("dressi_rasterize_soft_grad", gy.data_ptr(), rs.data_ptr(),
           clip.data_ptr(), clip.shape[1], faces.data_ptr(), faces.shape[0],
           views, w, h, grad.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return grad[0] if squeeze else grad


def rasterize_face_id(clip, faces, width: int, height: int,
                      with_depth: bool = False, check: bool = True):
    """F::RasterizeFaceId -> [(views,) H, W] float(face)+1, 0 background."""
    squeeze = clip.dim() == 2
    clip = _dev(clip, "clip")
    faces = _dev(faces, "faces", 2)
    clip, views = _views(clip, 2)
    out = torch.empty((views, height, width), dtype=torch.float32,
                      device=clip.device)
    depth = torch.empty_like(out) if with_depth else None
    st = _new_status(clip.device)
    N.call("dressi_rasterize_face_id", clip.data_ptr(), clip.shape[1],
           faces.data_ptr(), faces.shape[0], views, width, height,
           out.data_ptr(), _ptr(depth), st.data_ptr(), _stream())
    if check:
        _after(st)
    if squeeze:
        out = out[0]
        depth = depth[0] if depth is not None else None
    return (out, depth) if with_depth else out


def rasterize(clip, attr, faces, width: int, height: int, check: bool = True):
    """F::Rasterize -> [(views,) H, W, C] perspective-correct attribute."""
    squeeze = clip.dim() == 2
    clip = _dev(clip, "clip")
    attr = _dev(attr, "attr")
    faces = _dev(faces, "faces", 2)
    clip, views = _views(clip, 2)
    if attr.dim() == 1:
        attr = attr.unsqueeze(-1)
    attr, _ = _views(attr, 2)
    attr = _match_views(attr, views, "attr")
    n_comp = attr.shape[-1]
    out = torch.empty((views, height, width, n_comp), dtype=torch.float32,
                      device=clip.device)
    st = _new_status(clip.device)
    N.call("dressi_rasterize", clip.data_ptr(), clip.shape[1],
           attr.data_ptr(), n_comp, faces.data_ptr(), faces.shape[0], views,
           width, height, out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out[0] if squeeze else out


def _aa_inputs(img_like, tri, clip, faces, name):
    """Normalises AntiAlias inputs: img_like [(views,) H, W(, C)], tri
    [(views,) H, W], clip [(views,) V, 4], faces [F, 3]."""
    tri = _dev(tri, "tri")
    squeeze = tri.dim() == 2
    tri, views = _views(tri, 2)
    h, w = tri.shape[1], tri.shape[2]
    x = _dev(img_like, name)
    if x.dim() == (2 if squeeze else 3):
        x = x.unsqueeze(-1)
    x, _ = _views(x, 3)
    x = _match_views(x, views, name)
    if x.shape[1] != h or x.shape[2] != w:
        raise N.DressiError(N.ERR_INVALID, f"{name} must match tri's size")
    clip = _dev(clip, "clip")
    clip, _ = _views(clip, 2)
    clip = _match_views(clip, views, "clip")
    faces = _dev(faces, "faces", 2)
    return x, tri, clip, faces, views, h, w, squeeze


def antialias(img, tri, clip, faces, check: bool = True):
    """F::AntiAlias (Dr.Hair screen-space AA): img [(views,) H, W(, C)],
    tri [(views,) H, W] = float(face)+1, clip [(views,) V, 4], faces [F, 3]
    -> an image shaped like img."""
    shape = img.shape
    x, tri, clip, faces, views, h, w, _ = _aa_inputs(img, tri, clip, faces,
                                                      "img")
    out = torch.empty_like(x)
    st = _new_status(x.device)
    N.call("dressi_antialias", x.data_ptr(), x.shape[-1], tri.data_ptr(),
           clip.data_ptr(), clip.shape[1], faces.data_ptr(), faces.shape[0],
           views, w, h, out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out.reshape(shape)


def antialias_grad(gy, img, tri, clip, faces, vft=None, seed: float = 0.0,
                   n_samples: int = 0, want_img: bool = True,
                   want_clip: bool = True, check: bool = True):
    """AntiAlias backward: (d img, d clip) of sum(gy * AntiAlias(img)).
    n_samples == 0 gives the exact vertex gradient; > 0 the reference's
    stochastic edge samples seeded by `seed` over vft [max_deg, V]
    (VertexFacesTex). Returns (grad_img or None, grad_clip or None)."""
    shape = gy.shape
    x = None
    if want_clip:
        x = _aa_inputs(img, tri, clip, faces, "img")[0]
    g, tri, clip, faces, views, h, w, squeeze = _aa_inputs(gy, tri, clip,
                                                            faces, "gy")
    vft_t = None
    max_deg = 0
    if want_clip and n_samples > 0:
        if vft is None:
            raise N.DressiError(N.ERR_INVALID,
                                "stochastic samples need vft (VertexFacesTex)")
        vft_t = _dev(vft, "vft", 2)
        max_deg = vft_t.shape[0]
    gi = torch.empty_like(g) if want_img else None
    gc = (torch.zeros((views, clip.shape[1], 4), dtype=torch.float32,
                      device=g.device) if want_clip else None)
    st = _new_status(g.device)
    N.call("dressi_antialias_grad", g.data_ptr(), _ptr(x), g.shape[-1],
           tri.data_ptr(), clip.data_ptr(), clip.shape[1], faces.data_ptr(),
           faces.shape[0], _ptr(vft_t), max_deg, float(seed), int(n_samples),
           views, w, h, _ptr(gi), _ptr(gc), st.data_ptr(), _stream())
    if check:
        _after(st)
    if gi is not None:
        gi = gi.reshape(shape)
    if gc is not None and squeeze:
        gc = gc[0]
    return gi, gc


_FILTERS = {"nearest": 0, "linear": 1, "bilinear": 1}


def texture(tex, uv, filter_mode: str = "nearest"):
    """F::Texture (nearest) / F::TextureBilinear ("linear"): tex [H, W, C]
    (C 1..4) sampled at uv [..., 2] -> [..., C]."""
    tex = _dev(tex, "tex", 3)
    uv = _dev(uv, "uv")
    if uv.shape[-1] != 2:
        raise N.DressiError(N.ERR_INVALID, "uv must end with 2 components")
    n = tex.shape[2]
    out = torch.empty(uv.shape[:-1] + (n,), dtype=torch.float32,
                      device=tex.device)
    N.call("dressi_texture", tex.data_ptr(), tex.shape[1], tex.shape[0], n,
           uv.data_ptr(), uv.numel() // 2, _FILTERS[filter_mode],
           out.data_ptr(), _stream())
    return out


def texture_grad(gy, inv_uv, uv_screen, filter_mode: str = "nearest"):
    """The texture gradient of `texture` through the inverse-UV table
    (GatherByInverseUV / GatherByInverseUVBilinear): gy [H, W, C], inv_uv
    [TH, TW, 4], uv_screen [H, W, 2] -> [TH, TW, C]."""
    gy = _dev(gy, "gy", 3)
    inv_uv = _dev(inv_uv, "inv_uv", 3)
    uv_screen = _dev(uv_screen, "uv_screen", 3)
    n = gy.shape[2]
    out = torch.empty((inv_uv.shape[0], inv_uv.shape[1], n),
                      dtype=torch.float32, device=gy.device)
    N.call("dressi_texture_grad", gy.data_ptr(), gy.shape[1], gy.shape[0], n,
           inv_uv.data_ptr(), inv_uv.shape[1], inv_uv.shape[0],
           uv_screen.data_ptr(), _FILTERS[filter_mode], out.data_ptr(),
           _stream())
    return out


# ---- optimizer-side regulariser (examples/silhouette_optimization/
# run.cpp:407-420) and its mesh tables (mesh_utils.cpp:53-101)

def _host_faces(faces):
    import numpy as np

    if isinstance(faces, torch.Tensor):
        faces = faces.detach().cpu().numpy()
    return np.ascontiguousarray(faces, np.float32).reshape(-1, 3)


def _deg_table(fn, faces, n_verts: int, cap: int):
    import ctypes as C

    import numpy as np

    f = _host_faces(faces)
    out = np.zeros(cap * n_verts, np.float32)
    deg = C.c_uint32(0)
    N.call(fn, f.ctypes.data, f.shape[0], n_verts, cap, out.ctypes.data,
           C.byref(deg))
    return out[: deg.value * n_verts].reshape(deg.value, n_verts)


def vertex_faces_tex(faces, n_verts: int, cap: int = 64):
    """VertexFacesTex: host float table {V, max_deg} as [max_deg, V]
    (incident faces in face order, -1 padding)."""
    return _deg_table("dressi_vertex_faces_tex", faces, n_verts, cap)


def vertex_neighbors_tex(faces, n_verts: int, cap: int = 64):
    """VertexNeighborsTex: host float table [max_deg, V] (sorted
    neighbours, -1 padding)."""
    return _deg_table("dressi_vertex_neighbors_tex", faces, n_verts, cap)


def face_neighbors_tex(faces):
    """FaceNeighborsTex: host float table [F, 3] (-1 padding)."""
    import numpy as np

    f = _host_faces(faces)
    out = np.zeros((f.shape[0], 3), np.float32)
    N.call("dressi_face_neighbors_tex", f.ctypes.data, f.shape[0],
           out.ctypes.data)
    return out


def vertex_neighbor_mean(pos, nbrs, check: bool = True):
    """F::VertexNeighborMean: pos [V, 3], nbrs [deg, V] -> [V, 3]."""
    pos = _dev(pos, "pos", 2)
    nbrs = _dev(nbrs, "nbrs", 2)
    out = torch.empty_like(pos)
    st = _new_status(pos.device)
    N.call("dressi_vertex_neighbor_mean", pos.data_ptr(), pos.shape[0],
           nbrs.data_ptr(), nbrs.shape[0], out.data_ptr(), st.data_ptr(),
           _stream())
    if check:
        _after(st)
    return out


def normal_consistency_face_term(pos, faces, face_adj, check: bool = True):
    """F::NormalConsistencyFaceTerm: pos [V, 3], faces [F, 3], face_adj
    [F, 3] -> [F, 3]."""
    pos = _dev(pos, "pos", 2)
    faces = _dev(faces, "faces", 2)
    face_adj = _dev(face_adj, "face_adj", 2)
    out = torch.empty_like(faces)
    st = _new_status(pos.device)
    N.call("dressi_normal_consistency_face_term", pos.data_ptr(),
           pos.shape[0], faces.data_ptr(), faces.shape[0],
           face_adj.data_ptr(), out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out


def normal_consistency_vertex_grad(term, pos, faces, vtx_faces,
                                   check: bool = True):
    """F::NormalConsistencyVertexGrad: term [F, 3], pos [V, 3], faces
    [F, 3], vtx_faces [deg, V] -> [V, 3]."""
    term = _dev(term, "term", 2)
    pos = _dev(pos, "pos", 2)
    faces = _dev(faces, "faces", 2)
    vtx_faces = _dev(vtx_faces, "vtx_faces", 2)
    out = torch.empty_like(pos)
    st = _new_status(pos.device)
    N.call("dressi_normal_consistency_vertex_grad", term.data_ptr(),
           pos.data_ptr(), pos.shape[0], faces.data_ptr(), faces.shape[0],
           vtx_faces.data_ptr(), vtx_faces.shape[0], out.data_ptr(),
           st.data_ptr(), _stream())
    if check:
        _after(st)
    return out


def sum_all(x):
    """F::SumAll of x [N, C] (C 1..4) or [N] -> a 1-element tensor, with
    the reference's summation order."""
    x = _dev(x, "x")
    nc = 1 if x.dim() == 1 else x.shape[-1]
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    N.call("dressi_sum_all", x.data_ptr(), x.numel() // nc, nc,
           out.data_ptr(), _stream())
    return out


def regularized_grad(pos, faces, g, laplacian: float, normal: float,
                     nbrs=None, face_adj=None, vtx_faces=None,
                     check: bool = True):
    """The silhouette optimizer's regularised gradient: g + g_lap (rms(g) /
    rms(g_lap) laplacian) + g_nrm (rms(g) / rms(g_nrm) normal). The mesh
    tables are built from faces when not given."""
    pos = _dev(pos, "pos", 2)
    faces = _dev(faces, "faces", 2)
    g = _dev(g, "g", 2)
    dev = pos.device
    nv = pos.shape[0]
    if nbrs is None:
        nbrs = torch.as_tensor(vertex_neighbors_tex(faces, nv), device=dev)
    if face_adj is None:
        face_adj = torch.as_tensor(face_neighbors_tex(faces), device=dev)
    if vtx_faces is None:
        vtx_faces = torch.as_tensor(vertex_faces_tex(faces, nv), device=dev)
    nbrs = _dev(nbrs, "nbrs", 2)
    face_adj = _dev(face_adj, "face_adj", 2)
    vtx_faces = _dev(vtx_faces, "vtx_faces", 2)
    out = torch.empty_like(g)
    st = _new_status(dev)
    N.call("dressi_regularized_grad", pos.data_ptr(), nv, faces.data_ptr(),
           faces.shape[0], nbrs.data_ptr(), nbrs.shape[0],
           face_adj.data_ptr(), vtx_faces.data_ptr(), vtx_faces.shape[0],
           g.data_ptr(), float(laplacian), float(normal), out.data_ptr(),
           st.data_ptr(), _stream())
    if check:
        _after(st)
    return out


# ---- split-sum IBL (config C5; f_ops.cpp:2785-3415)

def _img3(t, name):
    t = _dev(t, name)
    if t.dim() == 2:
        t = t.unsqueeze(-1)
    if t.dim() != 3 or not 1 <= t.shape[2] <= 4:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be [H, W, C<=4]")
    return t.contiguous()


def equirect_sample(env, dirs):
    """F::EquirectSample: env [H, W, C] sampled along dirs [..., 3]."""
    env = _img3(env, "env")
    dirs = _dev(dirs, "dirs")
    n = env.shape[2]
    out = torch.empty(dirs.shape[:-1] + (n,), dtype=torch.float32,
                      device=env.device)
    N.call("dressi_equirect_sample", env.data_ptr(), env.shape[1],
           env.shape[0], n, dirs.data_ptr(), dirs.numel() // 3,
           out.data_ptr(), _stream())
    return out


def equirect_sample_grad(gy, dirs, width: int, height: int):
    """The map gradient of equirect_sample: gy [..., C] -> [H, W, C]."""
    gy = _dev(gy, "gy")
    dirs = _dev(dirs, "dirs")
    n = gy.shape[-1]
    out = torch.empty((height, width, n), dtype=torch.float32,
                      device=gy.device)
    N.call("dressi_equirect_sample_grad", gy.data_ptr(), dirs.data_ptr(),
           dirs.numel() // 3, width, height, n, out.data_ptr(), _stream())
    return out


def irradiance_conv(env, width: int, height: int):
    """F::IrradianceConv: env [H, W, C] -> [height, width, C]."""
    env = _img3(env, "env")
    n = env.shape[2]
    out = torch.empty((height, width, n), dtype=torch.float32,
                      device=env.device)
    N.call("dressi_irradiance_conv", env.data_ptr(), env.shape[1],
           env.shape[0], n, width, height, out.data_ptr(), _stream())
    return out


def irradiance_conv_grad(gy, width: int, height: int):
    """The env gradient of irradiance_conv: gy [h, w, C] -> [height,
    width, C]."""
    gy = _img3(gy, "gy")
    n = gy.shape[2]
    out = torch.empty((height, width, n), dtype=torch.float32,
                      device=gy.device)
    N.call("dressi_irradiance_conv_grad", gy.data_ptr(), gy.shape[1],
           gy.shape[0], n, width, height, out.data_ptr(), _stream())
    return out


def prefilter_conv(env, width: int, height: int, roughness: float):
    """F::PrefilterConv: env [H, W, C] -> [height, width, C]."""
    env = _img3(env, "env")
    n = env.shape[2]
    out = torch.empty((height, width, n), dtype=torch.float32,
                      device=env.device)
    N.call("dressi_prefilter_conv", env.data_ptr(), env.shape[1],
           env.shape[0], n, width, height, float(roughness), out.data_ptr(),
           _stream())
    return out


def prefilter_conv_grad(gy, width: int, height: int, roughness: float):
    """The env gradient of prefilter_conv: gy [h, w, C] -> [height, width,
    C]."""
    gy = _img3(gy, "gy")
    n = gy.shape[2]
    out = torch.empty((height, width, n), dtype=torch.float32,
                      device=gy.device)
    N.call("dressi_prefilter_conv_grad", gy.data_ptr(), gy.shape[1],
           gy.shape[0], n, width, height, float(roughness), out.data_ptr(),
           _stream())
    return out


def brdf_lut(width: int = 256, height: int = 256, n_samples: int = 512,
             device=None):
    """F::BrdfIntegrationLut: [height, width, 2] (A, B)."""
    dev = device if device is not None else torch.device("cuda")
    out = torch.empty((height, width, 2), dtype=torch.float32, device=dev)
    N.call("dressi_brdf_lut", width, height, n_samples, out.data_ptr(),
           _stream())
    return out


def avg_pool2x2(x):
    """F::AvgPool2x2: [H, W, C] -> [H/2, W/2, C] (even sizes)."""
    x = _img3(x, "x")
    h, w, n = x.shape
    out = torch.empty((h // 2, w // 2, n), dtype=torch.float32,
                      device=x.device)
    N.call("dressi_avg_pool2x2", x.data_ptr(), w, h, n, out.data_ptr(),
           _stream())
    return out


def avg_pool2x2_grad(gy):
    """The transpose of avg_pool2x2: [h, w, C] -> [2h, 2w, C]."""
    gy = _img3(gy, "gy")
    h, w, n = gy.shape
    out = torch.empty((2 * h, 2 * w, n), dtype=torch.float32,
                      device=gy.device)
    N.call("dressi_avg_pool2x2_grad", gy.data_ptr(), 2 * w, 2 * h, n,
           out.data_ptr(), _stream())
    return out


# ------------------------------------------------- indexed access (HSR)

def _comp2(t: torch.Tensor, name: str) -> torch.Tensor:
    """[N] or [N, n] (n 1..4) as a contiguous [N, n] float32 CUDA tensor."""
    t = _dev(t, name)
    if t.dim() == 1:
        t = t.unsqueeze(1)
    if t.dim() != 2 or not 1 <= t.shape[1] <= 4:
        raise N.DressiError(N.ERR_INVALID, f"{name} must be [N, 1..4]")
    return t.contiguous()


def screen_coord(w: int, h: int, device=None) -> torch.Tensor:
    """F::ScreenCoord: [h, w, 2] pixel centres (x + 0.5, y + 0.5)."""
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if device is None else torch.device(device)
    out = torch.empty((h, w, 2), dtype=torch.float32, device=dev)
    N.call("dressi_screen_coord", w, h, out.data_ptr(), _stream())
    return out


def lookup_faces(attr, faces, corner: int, check: bool = True):
    """F::LookupFaces: attr [V, n], faces [F, 3] (float ids) -> [F, n] =
    attr[faces[:, corner]]."""
    attr = _comp2(attr, "attr")
    faces = _dev(faces, "faces", 2)
    nf = faces.shape[0]
    out = torch.empty((nf, attr.shape[1]), dtype=torch.float32,
                      device=attr.device)
    st = _new_status(attr.device)
    N.call("dressi_lookup_faces", attr.data_ptr(), attr.shape[0],
           attr.shape[1], faces.data_ptr(), nf, corner, out.data_ptr(),
           st.data_ptr(), _stream())
    if check:
        _after(st)
    return out


def lookup_faces_grad(gy, faces, vertex_faces, corner: int,
                      check: bool = True):
    """LookupFacesBwd: gy [F, n], vertex_faces [max_deg, V] (VertexFacesTex)
    -> [V, n]."""
    gy = _comp2(gy, "gy")
    faces = _dev(faces, "faces", 2)
    vf = _dev(vertex_faces, "vertex_faces", 2)
    md, nv = vf.shape
    out = torch.empty((nv, gy.shape[1]), dtype=torch.float32,
                      device=gy.device)
    st = _new_status(gy.device)
    N.call("dressi_lookup_faces_grad", gy.data_ptr(), gy.shape[1],
           faces.data_ptr(), faces.shape[0], vf.data_ptr(), nv, md, corner,
           out.data_ptr(), st.data_ptr(), _stream())
    if check:
        _after(st)
    return out


def face_fetch(attr, idx):
    """F::FaceFetch forward: attr [F, n], idx [H, W] float face ids (0 =
    background) -> [H, W, n]."""
    attr = _comp2(attr, "attr")
    idx = _dev(idx, "idx", 2)
    h, w = idx.shape
    out = torch.empty((h, w, attr.shape[1]), dtype=torch.float32,
                      device=attr.device)
    N.call("dressi_face_fetch", attr.data_ptr(), attr.shape[0],
           attr.shape[1], idx.data_ptr(), w, h, out.data_ptr(), _stream())
    return out


def face_fetch_grad(gy, idx, prj0, prj1, prj2, seed: float = 0.0,
                    radius_px: float = 1.0, n_samples: int = 4):
    """FaceFetchBwd: gy [H, W, n], idx [H, W], prj* [F, 4] corner clip
    positions -> [F, n]. n_samples 0: the exact VJP."""
    gy = _dev(gy, "gy", 3)
    idx = _dev(idx, "idx", 2)
    prj = [_dev(p, f"prj{k}", 2) for k, p in enumerate((prj0, prj1, prj2))]
    h, w, n = gy.shape
    nf = prj[0].shape[0]
    out = torch.empty((nf, n), dtype=torch.float32, device=gy.device)
    N.call("dressi_face_fetch_grad", gy.data_ptr(), n, idx.data_ptr(), w, h,
           prj[0].data_ptr(), prj[1].data_ptr(), prj[2].data_ptr(), nf,
           float(seed), float(radius_px), n_samples, out.data_ptr(),
           _stream())
    return out
