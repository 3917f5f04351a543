"""Fused fwd + bwd + Adam iterations resident on one device (CUDA graphs).

``SilhouettePlan`` is the HardSoftRas silhouette optimisation (config C3),
``AaSilhouettePlan`` the screen-space-AA one (C4), ``ImageFitPlan`` the 2-D
image fit (C1). All hold every buffer of
the iteration on the device; ``step(n)`` replays the captured iteration n
times with no host traffic, like the reference's DressiAD::execStep replaying
one recorded command buffer (src/dressi_ad.cpp:461-480).

State access mirrors DressiAD::sendImg / recvImg (include/dressi/
dressi_ad.h:114-131): ``upload(slot, array)`` / ``download(slot)`` take host
numpy arrays or CUDA tensors.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N

__all__ = ["Plan", "SilhouettePlan", "AaSilhouettePlan", "TexturePlan",
           "ImageFitPlan"]


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Plan:
    """Owns a dressi_plan handle."""

    def __init__(self, handle, device: int):
        self._h = handle
        self.device = device

    # -- lifetime -----------------------------------------------------------
    def close(self):
        if self._h:
            N.call("dressi_plan_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- slots --------------------------------------------------------------
    def slot_bytes(self, slot: int) -> int:
        n = C.c_size_t(0)
        N.call("dressi_plan_slot_bytes", self._h, slot, C.byref(n))
        return n.value

    def slot_tensor(self, slot: int, shape=None) -> torch.Tensor:
        """Zero-copy CUDA tensor view of a resident slot (float32)."""
        ptr = C.c_void_p(0)
        N.call("dressi_plan_slot_ptr", self._h, slot, C.byref(ptr))
        n = self.slot_bytes(slot) // 4
        shape = tuple(shape) if shape is not None else (n,)

        class _Iface:
            __cuda_array_interface__ = {
                "shape": shape, "typestr": "<f4",
                "data": (ptr.value, False), "version": 3, "strides": None,
            }

        with torch.cuda.device(self.device):
            return torch.as_tensor(_Iface(), device=f"cuda:{self.device}")

    def upload(self, slot: int, data, stream=None):
        if isinstance(data, torch.Tensor) and data.is_cuda:
            t = data.detach().to(torch.float32).contiguous()
            N.call("dressi_plan_upload", self._h, slot, t.data_ptr(),
                   t.numel() * 4, 1, _stream_ptr(stream))
            return
        a = np.ascontiguousarray(
            data.cpu().numpy() if isinstance(data, torch.Tensor) else data,
            dtype=np.float32)
        N.call("dressi_plan_upload", self._h, slot, a.ctypes.data, a.nbytes,
               0, _stream_ptr(stream))
        torch.cuda.current_stream().synchronize() if stream is None else \
            stream.synchronize()

    def download(self, slot: int, out=None, stream=None):
        n = self.slot_bytes(slot)
        if isinstance(out, torch.Tensor) and out.is_cuda:
            N.call("dressi_plan_download", self._h, slot, out.data_ptr(), n,
                   1, _stream_ptr(stream))
            return out
        a = out if out is not None else np.empty(n // 4, np.float32)
        N.call("dressi_plan_download", self._h, slot, a.ctypes.data, n, 0,
               _stream_ptr(stream))
        (stream or torch.cuda.current_stream()).synchronize()
        return a

    # -- execution ----------------------------------------------------------
    def step(self, n_iters: int = 1, stream=None):
        N.call("dressi_plan_exec", self._h, int(n_iters), _stream_ptr(stream))

    def record_phase(self, phase: int, stream=None):
        """Launches phase 0 (forward + backward into GRAD) or 1 (the update)
        directly on the stream, so that a CUDA-graph capture running there
        records it (dressi_plan_record_phase)."""
        N.call("dressi_plan_record_phase", self._h, int(phase),
               _stream_ptr(stream))

    def status(self, stream=None) -> int:
        w = C.c_uint32(0)
        N.call("dressi_plan_status", self._h, C.byref(w), _stream_ptr(stream))
        return w.value

    def launches_per_iter(self) -> int:
        n = C.c_uint32(0)
        N.call("dressi_plan_launches_per_iter", self._h, C.byref(n))
        return n.value

    def profile(self, n_iters: int = 5, stream=None) -> list[dict]:
        """Per-kernel CUDA-event timing of n_iters un-graphed iterations:
        [{"name", "total_ms", "launches", "avg_ms"}] in launch order."""
        cap = 64
        names = (C.c_char_p * cap)()
        ms = (C.c_float * cap)()
        cnt = (C.c_uint32 * cap)()
        n = C.c_uint32(0)
        N.call("dressi_plan_profile", self._h, int(n_iters),
               _stream_ptr(stream), cap, names, ms, cnt, C.byref(n))
        out = []
        for i in range(min(n.value, cap)):
            out.append({"name": names[i].decode(), "total_ms": float(ms[i]),
                        "launches": int(cnt[i]),
                        "avg_ms": float(ms[i]) / max(1, int(cnt[i]))})
        return out

    def loss(self) -> float:
        return float(self.download(N.SLOT_LOSS)[0])

    def loss_history(self, n: int) -> np.ndarray:
        """Losses of the first n iterations (ring of 4096 by default)."""
        return self.download(N.SLOT_LOSS_HISTORY)[:n].copy()


class SilhouettePlan(Plan):
    """C3/C4 silhouette optimisation of vertex positions (HardSoftRas).
    laplacian / normal: the optimizer-side regulariser weights of the
    reference example (run.cpp:407-420; its defaults 0.15 / 0.4 here,
    0.5 / 0.5 for the AA plan); 0 / 0 = none."""

    def __init__(self, faces, mvps, n_verts: int, res: int, radius_px: float,
                 sigma: float = 1e-4, lr: float = 1e-3, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, device: int = 0,
                 loss_history: int = 4096, laplacian: float = 0.0,
                 normal: float = 0.0, _paper=None):
        faces = np.ascontiguousarray(faces, np.float32).reshape(-1, 3)
        mvps = np.ascontiguousarray(mvps, np.float32).reshape(-1, 16)
        self.n_verts, self.n_faces = int(n_verts), faces.shape[0]
        self.n_views, self.res = mvps.shape[0], int(res)
        d = N.SilhouetteDesc()
        d.struct_size = C.sizeof(N.SilhouetteDesc)
        d.n_verts, d.n_faces = self.n_verts, self.n_faces
        d.n_views, d.res = self.n_views, self.res
        d.radius_px, d.sigma, d.lr = radius_px, sigma, lr
        d.beta1, d.beta2, d.eps = beta1, beta2, eps
        d.faces = faces.ctypes.data_as(C.POINTER(C.c_float))
        d.mvps = mvps.ctypes.data_as(C.POINTER(C.c_float))
        d.loss_history = loss_history
        d.device = device
        d.laplacian, d.normal = laplacian, normal
        h = C.c_void_p(0)
        if _paper is None:
            N.call("dressi_silhouette_plan_create", C.byref(d), C.byref(h))
        else:
            N.call("dressi_paper_silhouette_plan_create", C.byref(d),
                   int(_paper[0]), int(_paper[1]), C.byref(h))
        super().__init__(h, device)

    @classmethod
    def from_scene(cls, scene, device: int = 0, views=None, **kw):
        mvps = scene.mvps if views is None else scene.mvps[views]
        kw.setdefault("lr", scene.lr)
        kw.setdefault("sigma", scene.sigma)
        radius = kw.pop("radius_px", scene.radius_px)
        return cls(scene.faces_f, mvps, scene.n_verts, scene.res, radius,
                   device=device, **kw)

    def render_targets(self, target_pos, stream=None):
        tp = np.ascontiguousarray(target_pos, np.float32)
        N.call("dressi_plan_render_targets", self._h,
               tp.ctypes.data_as(C.POINTER(C.c_float)), _stream_ptr(stream))

    def render(self, stream=None) -> torch.Tensor:
        """RasterizeSoft images of the current positions [views, R, R, 4]."""
        N.call("dressi_plan_render", self._h, _stream_ptr(stream))
        return self.slot_tensor(N.SLOT_RASTER,
                                (self.n_views, self.res, self.res, 4)).clone()

    def forward_backward(self, stream=None):
        """Phase 0 of a sharded iteration: local gradient into GRAD."""
        N.call("dressi_plan_exec_phase", self._h, 0, _stream_ptr(stream))

    def apply_update(self, stream=None):
        """Phase 1: Adam from the (all-reduced) GRAD slot."""
        N.call("dressi_plan_exec_phase", self._h, 1, _stream_ptr(stream))

    def grad_tensor(self) -> torch.Tensor:
        return self.slot_tensor(N.SLOT_GRAD, (self.n_verts, 3))

    def set_deterministic(self, on: bool = True):
        """Deterministic gradient mode: per-face then per-vertex gathers in
        a fixed order instead of float atomics (bit-identical reruns)."""
        N.call("dressi_plan_set_deterministic", self._h, int(bool(on)))

    def loss_tensor(self) -> torch.Tensor:
        return self.slot_tensor(N.SLOT_LOSS, (1,))


class PaperSilhouettePlan(SilhouettePlan):
    """The silhouette example's own HardSoftRas technique (the paper path,
    run.cpp:229-396) as one fused plan: `peels` (1..4) soft layers, the
    per-pixel edge distance from FaceFetch of the LookupFaces corners, Eq. 6
    union, FaceFetch's backward with n_samples hashed edge samples per face
    (0: exact) jittered by the Adam counter. radius_px sets the sigmoid
    scale (7 / radius_px); sigma is unused."""

    def __init__(self, faces, mvps, n_verts: int, res: int, radius_px: float,
                 peels: int = 1, n_samples: int = 8, **kw):
        kw.setdefault("sigma", 1.0)
        super().__init__(faces, mvps, n_verts, res, radius_px,
                         _paper=(peels, n_samples), **kw)


class AaSilhouettePlan(SilhouettePlan):
    """C4 silhouette optimisation with screen-space AA (Dr.Hair): hard
    raster + AntiAlias, vertex gradient from n_samples stochastic edge
    samples per face (0: the exact scan)."""

    def __init__(self, faces, mvps, n_verts: int, res: int,
                 n_samples: int = 8, lr: float = 1e-3, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, device: int = 0,
                 loss_history: int = 4096, laplacian: float = 0.0,
                 normal: float = 0.0):
        faces = np.ascontiguousarray(faces, np.float32).reshape(-1, 3)
        mvps = np.ascontiguousarray(mvps, np.float32).reshape(-1, 16)
        self.n_verts, self.n_faces = int(n_verts), faces.shape[0]
        self.n_views, self.res = mvps.shape[0], int(res)
        self.n_samples = int(n_samples)
        d = N.AaSilhouetteDesc()
        d.struct_size = C.sizeof(N.AaSilhouetteDesc)
        d.n_verts, d.n_faces = self.n_verts, self.n_faces
        d.n_views, d.res = self.n_views, self.res
        d.n_samples = self.n_samples
        d.lr, d.beta1, d.beta2, d.eps = lr, beta1, beta2, eps
        d.faces = faces.ctypes.data_as(C.POINTER(C.c_float))
        d.mvps = mvps.ctypes.data_as(C.POINTER(C.c_float))
        d.loss_history = loss_history
        d.device = device
        d.laplacian, d.normal = laplacian, normal
        h = C.c_void_p(0)
        N.call("dressi_aa_silhouette_plan_create", C.byref(d), C.byref(h))
        Plan.__init__(self, h, device)

    @classmethod
    def from_scene(cls, scene, device: int = 0, views=None, n_samples=8,
                   **kw):
        mvps = scene.mvps if views is None else scene.mvps[views]
        kw.setdefault("lr", scene.lr)
        return cls(scene.faces_f, mvps, scene.n_verts, scene.res,
                   n_samples=n_samples, device=device, **kw)

    def render(self, stream=None) -> torch.Tensor:
        """Anti-aliased predictions of the current positions [views, R, R]."""
        N.call("dressi_plan_render", self._h, _stream_ptr(stream))
        return self.slot_tensor(N.SLOT_RASTER,
                                (self.n_views, self.res, self.res)).clone()


class TexturePlan(Plan):
    """C2 texture optimisation: trilinear sampling of a box-filtered mip
    pyramid of the optimised texture on a fixed UV-mapped mesh, per-view
    Mean L2 loss, Adam on the texture."""

    def __init__(self, pos, uv, faces, mvps, res: int, tex_size: int,
                 levels: int, lr: float = 1e-2, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, device: int = 0,
                 loss_history: int = 4096):
        pos = np.ascontiguousarray(pos, np.float32).reshape(-1, 3)
        uv = np.ascontiguousarray(uv, np.float32).reshape(-1, 2)
        faces = np.ascontiguousarray(faces, np.float32).reshape(-1, 3)
        mvps = np.ascontiguousarray(mvps, np.float32).reshape(-1, 16)
        self.n_views, self.res = mvps.shape[0], int(res)
        self.tex_size, self.levels = int(tex_size), int(levels)
        d = N.TextureDesc()
        d.struct_size = C.sizeof(N.TextureDesc)
        d.n_verts, d.n_faces = pos.shape[0], faces.shape[0]
        d.n_views, d.res = self.n_views, self.res
        d.tex_size, d.levels = self.tex_size, self.levels
        d.lr, d.beta1, d.beta2, d.eps = lr, beta1, beta2, eps
        fp = C.POINTER(C.c_float)
        d.pos = pos.ctypes.data_as(fp)
        d.uv = uv.ctypes.data_as(fp)
        d.faces = faces.ctypes.data_as(fp)
        d.mvps = mvps.ctypes.data_as(fp)
        d.loss_history = loss_history
        d.device = device
        h = C.c_void_p(0)
        N.call("dressi_texture_plan_create", C.byref(d), C.byref(h))
        super().__init__(h, device)

    @classmethod
    def from_scene(cls, scene, device: int = 0, views=None, **kw):
        mvps = scene.mvps if views is None else scene.mvps[views]
        kw.setdefault("lr", scene.lr)
        return cls(scene.pos, scene.uv, scene.faces_f, mvps, scene.res,
                   scene.tex_size, scene.levels, device=device, **kw)

    def render_targets(self, target_tex, stream=None):
        """Targets = the renders of `target_tex` [T, T, 3] (host)."""
        tt = np.ascontiguousarray(target_tex, np.float32)
        N.call("dressi_plan_render_targets", self._h,
               tt.ctypes.data_as(C.POINTER(C.c_float)), _stream_ptr(stream))

    def render(self, stream=None) -> torch.Tensor:
        """Renders of the current texture [views, R, R, 3]."""
        N.call("dressi_plan_render", self._h, _stream_ptr(stream))
        return self.slot_tensor(N.SLOT_RASTER,
                                (self.n_views, self.res, self.res, 3)).clone()

    def forward_backward(self, stream=None):
        N.call("dressi_plan_exec_phase", self._h, 0, _stream_ptr(stream))

    def apply_update(self, stream=None):
        N.call("dressi_plan_exec_phase", self._h, 1, _stream_ptr(stream))

    def grad_tensor(self) -> torch.Tensor:
        return self.slot_tensor(N.SLOT_GRAD,
                                (self.tex_size, self.tex_size, 3))

    def loss_tensor(self) -> torch.Tensor:
        return self.slot_tensor(N.SLOT_LOSS, (1,))


class ImageFitPlan(Plan):
    """C1 image fitting: Mean((param - target)^2) + Adam, one fused pass."""

    def __init__(self, width: int, height: int, lr: float = 1e-2,
                 device: int = 0):
        h = C.c_void_p(0)
        N.call("dressi_image_fit_plan_create", width, height, float(lr),
               device, C.byref(h))
        self.width, self.height = width, height
        super().__init__(h, device)


class PbrPlan(Plan):
    """C5: split-sum PBR material + environment optimisation on a fixed UV
    mesh. PARAM = [albedo | metallic-roughness | env] (flat), optimised by
    Adam with the maps clamped to [0, 1] and the env to >= 0."""

    def __init__(self, pos, normal, uv, faces, mvps, frames, light, res: int,
                 tex_size: int, env_w: int, env_h: int, levels: int = 6,
                 lut_size: int = 256, lut_samples: int = 512,
                 loss_kind: int = 1, lr: float = 1e-2, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, device: int = 0,
                 loss_history: int = 4096):
        arrs = [np.ascontiguousarray(a, np.float32) for a in
                (pos, normal, uv, faces, mvps, frames, light)]
        self._keep = arrs
        pos, normal, uv, faces, mvps, frames, light = arrs
        self.n_views, self.res = mvps.reshape(-1, 16).shape[0], int(res)
        self.tex_size, self.env_w, self.env_h = tex_size, env_w, env_h
        d = N.PbrDesc()
        d.struct_size = C.sizeof(N.PbrDesc)
        d.n_verts = pos.reshape(-1, 3).shape[0]
        d.n_faces = faces.reshape(-1, 3).shape[0]
        d.n_views, d.res = self.n_views, self.res
        d.tex_size, d.env_w, d.env_h = tex_size, env_w, env_h
        d.levels, d.lut_size, d.lut_samples = levels, lut_size, lut_samples
        d.loss_kind = loss_kind
        d.lr, d.beta1, d.beta2, d.eps = lr, beta1, beta2, eps
        fp = C.POINTER(C.c_float)
        d.pos, d.normal = pos.ctypes.data_as(fp), normal.ctypes.data_as(fp)
        d.uv, d.faces = uv.ctypes.data_as(fp), faces.ctypes.data_as(fp)
        d.mvps, d.frames = mvps.ctypes.data_as(fp), frames.ctypes.data_as(fp)
        d.light = light.ctypes.data_as(fp)
        d.loss_history = loss_history
        d.device = device
        h = C.c_void_p(0)
        N.call("dressi_pbr_plan_create", C.byref(d), C.byref(h))
        super().__init__(h, device)

    @classmethod
    def from_scene(cls, scene, device: int = 0, views=None, **kw):
        sel = slice(None) if views is None else views
        kw.setdefault("lr", scene.lr)
        kw.setdefault("levels", scene.levels)
        return cls(scene.pos, scene.pos, scene.uv, scene.faces_f,
                   scene.mvps[sel], scene.frames[sel], scene.light,
                   scene.res, scene.tex_size, scene.env_gt.shape[1],
                   scene.env_gt.shape[0], device=device, **kw)

    @staticmethod
    def pack(albedo, mr, env) -> np.ndarray:
        return np.concatenate([np.ascontiguousarray(a, np.float32).ravel()
                               for a in (albedo, mr, env)])

    def unpack(self, flat):
        t2 = self.tex_size * self.tex_size * 3
        a = flat[:t2].reshape(self.tex_size, self.tex_size, 3)
        m = flat[t2:2 * t2].reshape(self.tex_size, self.tex_size, 3)
        e = flat[2 * t2:].reshape(self.env_h, self.env_w, 3)
        return a, m, e

    def render_targets(self, albedo, mr, env, stream=None):
        flat = self.pack(albedo, mr, env)
        N.call("dressi_plan_render_targets", self._h,
               flat.ctypes.data_as(C.POINTER(C.c_float)), _stream_ptr(stream))

    def render(self, stream=None) -> torch.Tensor:
        """Tone-mapped renders of the current parameters [views, R, R, 3]."""
        N.call("dressi_plan_render", self._h, _stream_ptr(stream))
        return self.slot_tensor(N.SLOT_RASTER,
                                (self.n_views, self.res, self.res, 3)).clone()

    def forward_backward(self, stream=None):
        N.call("dressi_plan_exec_phase", self._h, 0, _stream_ptr(stream))

    def apply_update(self, stream=None):
        N.call("dressi_plan_exec_phase", self._h, 1, _stream_ptr(stream))

    def grad_tensor(self) -> torch.Tensor:
        n = self.slot_bytes(N.SLOT_GRAD) // 4
        return self.slot_tensor(N.SLOT_GRAD, (n,))

    def loss_tensor(self) -> torch.Tensor:
        return self.slot_tensor(N.SLOT_LOSS, (1,))
