"""TEST INFRASTRUCTURE ONLY: ctypes bindings of the CPU checkers.

``Port`` wraps liboracle.so (this repository's C restatement, oracle.c);
``Ref`` wraps _ref/libdressi_ref.so (the unmodified reference CPU code built
in place by oracle/Makefile plus ref_driver.cpp). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arm import
this module.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdressi_ref.so")

_f32p = C.POINTER(C.c_float)
_u32 = C.c_uint32


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def build_port() -> str:
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    return PORT_SO


def build_ref(ref_dir: str | None = None) -> str | None:
    """Builds _ref/libdressi_ref.so from the reference checkout named by
    `ref_dir` or, when that is None, by the DRESSI_REF_DIR environment
    variable. Without a checkout (the GPU box has none) it returns the
    prebuilt library if there is one, else None."""
    if ref_dir is None:
        ref_dir = os.environ.get("DRESSI_REF_DIR")
    if not ref_dir or not os.path.isdir(os.path.join(ref_dir, "src",
                                                     "core")):
        return REF_SO if os.path.exists(REF_SO) else None
    subprocess.run(["make", "-s", "-j8", "-C", HERE, "ref",
                    f"REF_DIR={ref_dir}"], check=True)
    return REF_SO


def ref_available() -> bool:
    return os.path.exists(REF_SO)


class _Lib:
    prefix = ""

    def __init__(self, path):
        self.lib = C.CDLL(path)
        p = self.prefix
        L = self.lib
        getattr(L, p + "last_error").restype = C.c_char_p

    def _err(self, rc, what):
        if rc != 0:
            msg = getattr(self.lib, self.prefix + "last_error")().decode()
            raise RuntimeError(f"{what}: {msg}")


class Port(_Lib):
    """liboracle.so -- the C restatement."""

    prefix = "orc_"

    def __init__(self, path=None):
        if path is None:
            path = PORT_SO
            if not os.path.exists(path):
                build_port()
        super().__init__(path)

    def soft_clip(self, clip, faces, w, h, radius):
        clip, faces = _f32(clip), _f32(faces)
        out = np.zeros((faces.shape[0] * 3, 4), np.float32)
        self._err(self.lib.orc_soft_clip(_fp(clip), _u32(clip.shape[0]),
                                         _fp(faces), _u32(faces.shape[0]),
                                         _u32(w), _u32(h), C.c_float(radius),
                                         _fp(out)), "soft_clip")
        return out

    def rasterize_soft(self, soft_clip, face_id, faces_soft, hard_clip,
                       faces_tex, w, h, radius, prev_depth=None):
        soft_clip, face_id, faces_soft = map(_f32, (soft_clip, face_id,
                                                    faces_soft))
        hard_clip, faces_tex = _f32(hard_clip), _f32(faces_tex)
        pd = None if prev_depth is None else _f32(prev_depth)
        out = np.zeros((h, w, 4), np.float32)
        self._err(self.lib.orc_rasterize_soft(
            _fp(soft_clip), _u32(soft_clip.shape[0]), _fp(face_id),
            _fp(faces_soft), _u32(faces_soft.shape[0]), _fp(hard_clip),
            _u32(hard_clip.shape[0]), _fp(faces_tex), _u32(w), _u32(h),
            C.c_float(radius), _fp(pd), _fp(out)), "rasterize_soft")
        return out

    def rasterize_face_id(self, clip, faces, w, h):
        clip, faces = _f32(clip), _f32(faces)
        out = np.zeros((h, w), np.float32)
        self._err(self.lib.orc_rasterize_face_id(
            _fp(clip), _u32(clip.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _u32(w), _u32(h), _fp(out)), "rasterize_face_id")
        return out

    def rasterize_hard(self, clip, attr, faces, w, h):
        clip, faces = _f32(clip), _f32(faces)
        attr = _f32(attr)
        nc = 1 if attr.ndim == 1 else attr.shape[1]
        out = np.zeros((h, w, nc), np.float32)
        self._err(self.lib.orc_rasterize_hard(
            _fp(clip), _u32(clip.shape[0]), _fp(attr), _u32(nc), _fp(faces),
            _u32(faces.shape[0]), _u32(w), _u32(h), _fp(out)),
            "rasterize_hard")
        return out

    def dist_grad(self, gy, rs, clip, faces, w, h):
        gy, rs, clip, faces = map(_f32, (gy, rs, clip, faces))
        out = np.zeros((clip.shape[0], 4), np.float32)
        self._err(self.lib.orc_dist_grad(
            _fp(gy), _fp(rs), _fp(clip), _u32(clip.shape[0]), _fp(faces),
            _u32(faces.shape[0]), _u32(w), _u32(h), _fp(out)), "dist_grad")
        return out

    def transform_clip(self, pos, mvp):
        pos, mvp = _f32(pos), _f32(mvp)
        out = np.zeros((pos.shape[0], 4), np.float32)
        self.lib.orc_transform_clip(_fp(pos), _u32(pos.shape[0]), _fp(mvp),
                                    _fp(out))
        return out

    def silhouette_loss_grad(self, pos, faces, mvps, targets, res, radius,
                             sigma, want_rs=False, threads=1):
        pos, faces, mvps, targets = map(_f32, (pos, faces, mvps, targets))
        nv = mvps.shape[0]
        grad = np.zeros_like(pos)
        loss = C.c_double(0.0)
        rs = np.zeros((nv, res, res, 4), np.float32) if want_rs else None
        self._err(self.lib.orc_silhouette_loss_grad_mt(
            _fp(pos), _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _u32(nv), _u32(res), C.c_float(radius), C.c_float(sigma),
            _fp(mvps), _fp(targets), C.byref(loss), _fp(grad), _fp(rs),
            _u32(max(1, int(threads)))), "silhouette_loss_grad")
        return loss.value, grad, rs

    def silhouette_run(self, pos, faces, mvps, targets, res, radius, sigma,
                       lr, n_iters, threads=1, laplacian=0.0, normal=0.0):
        pos = _f32(pos).copy()
        faces, mvps, targets = map(_f32, (faces, mvps, targets))
        trace = np.zeros(n_iters, np.float32)
        self._err(self.lib.orc_silhouette_run(
            _fp(pos), _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _u32(mvps.shape[0]), _u32(res), C.c_float(radius),
            C.c_float(sigma), C.c_float(lr), _fp(mvps), _fp(targets),
            _u32(n_iters), _u32(threads), C.c_float(laplacian),
            C.c_float(normal), _fp(trace)), "silhouette_run")
        return trace, pos

    def adam(self, param, m, v, t, grad, lr, b1=0.9, b2=0.999, eps=1e-8):
        """One in-graph Adam step in place (orc_adam); returns the new t."""
        for a in (param, m, v, grad):
            assert a.dtype == np.float32 and a.flags.c_contiguous
        tt = C.c_float(t)
        self.lib.orc_adam(_fp(param), _fp(m), _fp(v), C.byref(tt), _fp(grad),
                          _u32(param.size), C.c_float(lr), C.c_float(b1),
                          C.c_float(b2), C.c_float(eps))
        return tt.value

    def image_fit_run(self, param, target, lr, n_iters):
        param = _f32(param).copy()
        target = _f32(target)
        h, w = param.shape[:2]
        trace = np.zeros(n_iters, np.float32)
        self._err(self.lib.orc_image_fit_run(
            _fp(param), _fp(target), _u32(w), _u32(h), C.c_float(lr),
            _u32(n_iters), _fp(trace)), "image_fit_run")
        return trace, param

    def antialias(self, img, tri, clip, faces):
        img, tri, clip, faces = map(_f32, (img, tri, clip, faces))
        h, w = tri.shape
        nc = 1 if img.ndim == 2 else img.shape[2]
        out = np.zeros_like(img)
        self._err(self.lib.orc_antialias(
            _fp(img), _u32(nc), _fp(tri), _fp(clip), _u32(clip.shape[0]),
            _fp(faces), _u32(faces.shape[0]), _u32(w), _u32(h), _fp(out)),
            "antialias")
        return out

    def antialias_bwd_img(self, gy, tri, clip, faces):
        gy, tri, clip, faces = map(_f32, (gy, tri, clip, faces))
        h, w = tri.shape
        nc = 1 if gy.ndim == 2 else gy.shape[2]
        out = np.zeros_like(gy)
        self._err(self.lib.orc_antialias_bwd_img(
            _fp(gy), _u32(nc), _fp(tri), _fp(clip), _u32(clip.shape[0]),
            _fp(faces), _u32(faces.shape[0]), _u32(w), _u32(h), _fp(out)),
            "antialias_bwd_img")
        return out

    def antialias_bwd_vtx(self, gy, img, tri, clip, faces, vft, seed,
                          n_samples):
        gy, img, tri, clip, faces, vft = map(_f32, (gy, img, tri, clip,
                                                    faces, vft))
        h, w = tri.shape
        nc = 1 if gy.ndim == 2 else gy.shape[2]
        out = np.zeros((clip.shape[0], 4), np.float32)
        self._err(self.lib.orc_antialias_bwd_vtx(
            _fp(gy), _fp(img), _u32(nc), _fp(tri), _fp(clip),
            _u32(clip.shape[0]), _fp(faces), _u32(faces.shape[0]), _fp(vft),
            _u32(vft.shape[0]), C.c_float(seed), _u32(n_samples), _u32(w),
            _u32(h), _fp(out)), "antialias_bwd_vtx")
        return out

    def hash_to_unit(self, f, s, seed, salt):
        self.lib.orc_hash_to_unit.restype = C.c_float
        return float(self.lib.orc_hash_to_unit(_u32(f), _u32(s), _u32(seed),
                                               _u32(salt)))

    def aa_targets(self, target_pos, faces, mvps, res):
        target_pos, faces, mvps = map(_f32, (target_pos, faces, mvps))
        out = np.zeros((mvps.shape[0], res, res), np.float32)
        self._err(self.lib.orc_aa_targets(
            _fp(target_pos), _u32(target_pos.shape[0]), _fp(faces),
            _u32(faces.shape[0]), _u32(mvps.shape[0]), _u32(res), _fp(mvps),
            _fp(out)), "aa_targets")
        return out

    def aa_silhouette_loss_grad(self, pos, faces, vft, mvps, targets, res,
                                n_samples, seed, threads=1, want_pred=False):
        pos, faces, vft, mvps, targets = map(_f32, (pos, faces, vft, mvps,
                                                    targets))
        nv = mvps.shape[0]
        grad = np.zeros_like(pos)
        loss = C.c_double(0.0)
        pred = np.zeros((nv, res, res), np.float32) if want_pred else None
        self._err(self.lib.orc_aa_silhouette_loss_grad(
            _fp(pos), _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _fp(vft), _u32(vft.shape[0]), _u32(nv), _u32(res),
            _u32(n_samples), C.c_float(seed), _fp(mvps), _fp(targets),
            _u32(threads), C.byref(loss), _fp(grad), _fp(pred)),
            "aa_silhouette_loss_grad")
        return loss.value, grad, pred

    def aa_silhouette_run(self, pos, faces, vft, mvps, targets, res,
                          n_samples, lr, n_iters, threads=1, laplacian=0.0,
                          normal=0.0):
        pos = _f32(pos).copy()
        faces, vft, mvps, targets = map(_f32, (faces, vft, mvps, targets))
        trace = np.zeros(n_iters, np.float32)
        self._err(self.lib.orc_aa_silhouette_run(
            _fp(pos), _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _fp(vft), _u32(vft.shape[0]), _u32(mvps.shape[0]), _u32(res),
            _u32(n_samples), C.c_float(lr), _fp(mvps), _fp(targets),
            _u32(n_iters), _u32(threads), C.c_float(laplacian),
            C.c_float(normal), _fp(trace)), "aa_silhouette_run")
        return trace, pos

    # ---- texturing
    def texture_bilinear(self, tex, uv):
        tex, uv = _f32(tex), _f32(uv)
        th, tw = tex.shape[:2]
        n = 1 if tex.ndim == 2 else tex.shape[2]
        out = np.zeros(uv.shape[:-1] + ((n,) if tex.ndim == 3 else ()),
                       np.float32)
        self._err(self.lib.orc_texture_bilinear(
            _fp(tex), _u32(tw), _u32(th), _u32(n), _fp(uv),
            _u32(uv.size // 2), _fp(out)), "texture_bilinear")
        return out

    def texture_nearest(self, tex, uv):
        tex, uv = _f32(tex), _f32(uv)
        th, tw = tex.shape[:2]
        n = 1 if tex.ndim == 2 else tex.shape[2]
        out = np.zeros(uv.shape[:-1] + ((n,) if tex.ndim == 3 else ()),
                       np.float32)
        self._err(self.lib.orc_texture_nearest(
            _fp(tex), _u32(tw), _u32(th), _u32(n), _fp(uv),
            _u32(uv.size // 2), _fp(out)), "texture_nearest")
        return out

    def _gather(self, fn, gy, inv_uv, uv_screen):
        gy, inv_uv, uv_screen = map(_f32, (gy, inv_uv, uv_screen))
        sh, sw = uv_screen.shape[:2]
        th, tw = inv_uv.shape[:2]
        n = 1 if gy.ndim == 2 else gy.shape[2]
        out = np.zeros((th, tw) + ((n,) if gy.ndim == 3 else ()), np.float32)
        self._err(getattr(self.lib, fn)(
            _fp(gy), _u32(sw), _u32(sh), _u32(n), _fp(inv_uv), _u32(tw),
            _u32(th), _fp(uv_screen), _fp(out)), fn)
        return out

    def gather_inv_uv_bilinear(self, gy, inv_uv, uv_screen):
        return self._gather("orc_gather_inv_uv_bilinear", gy, inv_uv,
                            uv_screen)

    def gather_inv_uv(self, gy, inv_uv, uv_screen):
        return self._gather("orc_gather_inv_uv", gy, inv_uv, uv_screen)

    def uv_as_clip(self, uv):
        uv = _f32(uv)
        out = np.zeros((uv.shape[0], 4), np.float32)
        self.lib.orc_uv_as_clip(_fp(uv), _u32(uv.shape[0]), _fp(out))
        return out

    def screen_attr(self, clip, sw, sh):
        clip = _f32(clip)
        out = np.zeros((clip.shape[0], 4), np.float32)
        self.lib.orc_screen_attr(_fp(clip), _u32(clip.shape[0]), _u32(sw),
                                 _u32(sh), _fp(out))
        return out

    def mip_floats(self, w, n, levels):
        self.lib.orc_mip_floats.restype = C.c_size_t
        return int(self.lib.orc_mip_floats(_u32(w), _u32(n), _u32(levels)))

    def mip_build(self, tex0, levels):
        tex0 = _f32(tex0)
        w, n = tex0.shape[0], tex0.shape[2]
        pyr = np.zeros(self.mip_floats(w, n, levels), np.float32)
        self._err(self.lib.orc_mip_build(_fp(tex0), _u32(w), _u32(n),
                                         _u32(levels), _fp(pyr)), "mip_build")
        return pyr

    def texture_lod(self, uv, mask, w_tex, levels):
        uv, mask = _f32(uv), _f32(mask)
        h, w = mask.shape
        lod = np.zeros((h, w), np.float32)
        self.lib.orc_texture_lod(_fp(uv), _fp(mask), _u32(w), _u32(h),
                                 _u32(w_tex), _u32(levels), _fp(lod))
        return lod

    def texture_trilinear(self, pyr, w, n, levels, uv, lod):
        pyr, uv, lod = map(_f32, (pyr, uv, lod))
        out = np.zeros(lod.shape + (n,), np.float32)
        self._err(self.lib.orc_texture_trilinear(
            _fp(pyr), _u32(w), _u32(n), _u32(levels), _fp(uv), _fp(lod),
            _u32(lod.size), _fp(out)), "texture_trilinear")
        return out

    def texture_trilinear_grad(self, g, w, n, levels, uv, lod):
        g, uv, lod = map(_f32, (g, uv, lod))
        gpyr = np.zeros(self.mip_floats(w, n, levels), np.float32)
        self._err(self.lib.orc_texture_trilinear_grad(
            _fp(g), _u32(w), _u32(n), _u32(levels), _fp(uv), _fp(lod),
            _u32(lod.size), _fp(gpyr)), "texture_trilinear_grad")
        return gpyr

    def mip_fold(self, gpyr, w, n, levels):
        gpyr = _f32(gpyr).copy()
        self.lib.orc_mip_fold(_fp(gpyr), _u32(w), _u32(n), _u32(levels))
        return gpyr

    def c2_loss_grad(self, tex, levels, pos, uv_v, faces, mvps, targets, res,
                     want_pred=False):
        tex, pos, uv_v, faces, mvps, targets = map(
            _f32, (tex, pos, uv_v, faces, mvps, targets))
        w = tex.shape[0]
        grad = np.zeros_like(tex)
        loss = C.c_double(0.0)
        pred = (np.zeros((mvps.shape[0], res, res, 3), np.float32)
                if want_pred else None)
        self._err(self.lib.orc_c2_loss_grad(
            _fp(tex), _u32(w), _u32(levels), _fp(pos), _fp(uv_v),
            _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]), _fp(mvps),
            _u32(mvps.shape[0]), _u32(res), _fp(targets), C.byref(loss),
            _fp(grad), _fp(pred)), "c2_loss_grad")
        return loss.value, grad, pred

    def c2_run(self, tex, levels, pos, uv_v, faces, mvps, targets, res, lr,
               n_iters):
        tex = _f32(tex).copy()
        pos, uv_v, faces, mvps, targets = map(_f32, (pos, uv_v, faces, mvps,
                                                     targets))
        trace = np.zeros(n_iters, np.float32)
        self._err(self.lib.orc_c2_run(
            _fp(tex), _u32(tex.shape[0]), _u32(levels), _fp(pos), _fp(uv_v),
            _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]), _fp(mvps),
            _u32(mvps.shape[0]), _u32(res), _fp(targets), C.c_float(lr),
            _u32(n_iters), _fp(trace)), "c2_run")
        return trace, tex

    def vertex_faces_tex(self, faces, n_verts, cap=64):
        faces = _f32(faces)
        out = np.zeros(n_verts * cap, np.float32)
        md = _u32(0)
        self._err(self.lib.orc_vertex_faces_tex(
            _fp(faces), _u32(faces.shape[0]), _u32(n_verts), _u32(cap),
            _fp(out), C.byref(md)), "vertex_faces_tex")
        return out[: n_verts * md.value].reshape(md.value, n_verts)

    # ---- split-sum IBL (C5)
    def equirect_sample(self, env, dirs):
        env, dirs = _f32(env), _f32(dirs)
        mh, mw = env.shape[:2]
        n = 1 if env.ndim == 2 else env.shape[2]
        out = np.zeros(dirs.shape[:-1] + ((n,) if env.ndim == 3 else ()),
                       np.float32)
        self.lib.orc_equirect_sample(_fp(env), _u32(mw), _u32(mh), _u32(n),
                                     _fp(dirs), C.c_size_t(dirs.size // 3),
                                     _fp(out))
        return out

    def equirect_sample_bwd(self, gy, dirs, mw, mh):
        gy, dirs = _f32(gy), _f32(dirs)
        dh, dw = dirs.shape[:2]
        n = 1 if gy.ndim == 2 else gy.shape[2]
        out = np.zeros((mh, mw) + ((n,) if gy.ndim == 3 else ()), np.float32)
        self._err(self.lib.orc_equirect_sample_bwd(
            _fp(gy), _fp(dirs), _u32(dw), _u32(dh), _u32(mw), _u32(mh),
            _u32(n), _fp(out)), "equirect_sample_bwd")
        return out

    def irradiance_conv(self, env, ow, oh):
        env = _f32(env)
        sh, sw, n = env.shape
        out = np.zeros((oh, ow, n), np.float32)
        self.lib.orc_irradiance_conv(_fp(env), _u32(sw), _u32(sh), _u32(n),
                                     _u32(ow), _u32(oh), _fp(out))
        return out

    def irradiance_conv_bwd(self, gy, sw, sh):
        gy = _f32(gy)
        oh, ow, n = gy.shape
        out = np.zeros((sh, sw, n), np.float32)
        self.lib.orc_irradiance_conv_bwd(_fp(gy), _u32(ow), _u32(oh), _u32(n),
                                         _u32(sw), _u32(sh), _fp(out))
        return out

    def prefilter_alpha(self, rough):
        self.lib.orc_prefilter_alpha.restype = C.c_float
        return np.float32(self.lib.orc_prefilter_alpha(C.c_float(rough)))

    def prefilter_conv_norm(self, ow, oh, sw, sh, alpha):
        out = np.zeros((oh, ow), np.float32)
        self.lib.orc_prefilter_conv_norm(_u32(ow), _u32(oh), _u32(sw),
                                         _u32(sh), C.c_float(alpha), _fp(out))
        return out

    def prefilter_conv(self, env, ow, oh, rough, norm=None):
        env = _f32(env)
        sh, sw, n = env.shape
        alpha = self.prefilter_alpha(rough)
        if norm is None:
            norm = self.prefilter_conv_norm(ow, oh, sw, sh, alpha)
        out = np.zeros((oh, ow, n), np.float32)
        self.lib.orc_prefilter_conv(_fp(env), _u32(sw), _u32(sh), _u32(n),
                                    _fp(_f32(norm)), _u32(ow), _u32(oh),
                                    C.c_float(alpha), _fp(out))
        return out

    def prefilter_conv_bwd(self, gy, sw, sh, rough, norm=None):
        gy = _f32(gy)
        oh, ow, n = gy.shape
        alpha = self.prefilter_alpha(rough)
        if norm is None:
            norm = self.prefilter_conv_norm(ow, oh, sw, sh, alpha)
        out = np.zeros((sh, sw, n), np.float32)
        self.lib.orc_prefilter_conv_bwd(_fp(gy), _fp(_f32(norm)), _u32(ow),
                                        _u32(oh), _u32(n), _u32(sw), _u32(sh),
                                        C.c_float(alpha), _fp(out))
        return out

    def brdf_lut(self, w, h, n_samples):
        out = np.zeros((h, w, 2), np.float32)
        self.lib.orc_brdf_lut(_u32(w), _u32(h), _u32(n_samples), _fp(out))
        return out

    def avg_pool2x2(self, x):
        x = _f32(x)
        h, w = x.shape[:2]
        n = 1 if x.ndim == 2 else x.shape[2]
        out = np.zeros((h // 2, w // 2) + x.shape[2:], np.float32)
        self.lib.orc_avg_pool2x2(_fp(x), _u32(w), _u32(h), _u32(n), _fp(out))
        return out

    def pbr_shade_grad(self, g_n, g_p, mask, albedo, mr, ao, emissive, frame,
                       env, levels, lut, target, loss_kind=1):
        h, w = mask.shape
        eh, ew = env.shape[:2]
        lh, lw = lut.shape[:2]
        args = [_f32(a) for a in (g_n, g_p, mask, albedo, mr, ao, emissive,
                                   frame, env, lut, target)]
        mapped = np.zeros((h, w, 3), np.float32)
        ga = np.zeros((h, w, 3), np.float32)
        gm = np.zeros((h, w, 3), np.float32)
        ge = np.zeros((eh, ew, 3), np.float32)
        loss = C.c_double(0.0)
        self._err(self.lib.orc_pbr_shade_grad(
            _u32(w), _u32(h), _fp(args[0]), _fp(args[1]), _fp(args[2]),
            _fp(args[3]), _fp(args[4]), _fp(args[5]), _fp(args[6]),
            _fp(args[7]), _fp(args[8]), _u32(ew), _u32(eh), _u32(levels),
            _fp(args[9]), _u32(lw), _u32(lh), _fp(args[10]),
            C.c_int(loss_kind), _fp(mapped), C.byref(loss), _fp(ga),
            _fp(gm), _fp(ge)), "pbr_shade_grad")
        return mapped, loss.value, ga, gm, ge

    def pbr_view_grad(self, g_n, g_p, mask, uv, albedo, mr, frame, env,
                      levels, lut, target, loss_kind, g_albedo, g_mr, g_env):
        """One textured view of the C5 shading (ao = 1, emissive = 0):
        returns (mapped, loss) and ADDS the gradients into g_*."""
        h, w = mask.shape
        th, tw = albedo.shape[:2]
        eh, ew = env.shape[:2]
        lh, lw = lut.shape[:2]
        ao = np.ones((1, 1, 3), np.float32)
        em = np.zeros((1, 1, 3), np.float32)
        args = [_f32(a) for a in (g_n, g_p, mask, uv, albedo, mr, frame, env,
                                   lut, target)]
        mapped = np.zeros((h, w, 3), np.float32)
        loss = C.c_double(0.0)
        for a in (g_albedo, g_mr, g_env):
            assert a.dtype == np.float32 and a.flags.c_contiguous
        self._err(self.lib.orc_pbr_shade_grad_uv(
            _u32(w), _u32(h), _fp(args[0]), _fp(args[1]), _fp(args[2]),
            _fp(args[3]), _u32(tw), _u32(th), _fp(args[4]), _fp(args[5]),
            _fp(ao), _fp(em), _fp(args[6]), _fp(args[7]), _u32(ew), _u32(eh),
            _u32(levels), _fp(args[8]), _u32(lw), _u32(lh), _fp(args[9]),
            C.c_int(loss_kind), _fp(mapped), C.byref(loss), _fp(g_albedo),
            _fp(g_mr), _fp(g_env)), "pbr_view_grad")
        return mapped, loss.value

    def vertex_neighbors_tex(self, faces, n_verts, cap=64):
        faces = _f32(faces)
        out = np.zeros(n_verts * cap, np.float32)
        md = _u32(0)
        self._err(self.lib.orc_vertex_neighbors_tex(
            _fp(faces), _u32(faces.shape[0]), _u32(n_verts), _u32(cap),
            _fp(out), C.byref(md)), "vertex_neighbors_tex")
        return out[: n_verts * md.value].reshape(md.value, n_verts)

    def face_neighbors_tex(self, faces):
        faces = _f32(faces)
        out = np.zeros((faces.shape[0], 3), np.float32)
        self._err(self.lib.orc_face_neighbors_tex(
            _fp(faces), _u32(faces.shape[0]), _fp(out)), "face_neighbors_tex")
        return out

    def vertex_neighbor_mean(self, pos, vnbrs):
        pos, vnbrs = _f32(pos), _f32(vnbrs)
        out = np.zeros_like(pos)
        self.lib.orc_vertex_neighbor_mean(_fp(pos), _u32(pos.shape[0]),
                                          _fp(vnbrs), _u32(vnbrs.shape[0]),
                                          _fp(out))
        return out

    def nc_face_term(self, pos, faces, fadj):
        pos, faces, fadj = map(_f32, (pos, faces, fadj))
        out = np.zeros((faces.shape[0], 3), np.float32)
        self.lib.orc_nc_face_term(_fp(pos), _fp(faces), _u32(faces.shape[0]),
                                  _fp(fadj), _fp(out))
        return out

    def nc_vertex_grad(self, term, pos, faces, vft):
        term, pos, faces, vft = map(_f32, (term, pos, faces, vft))
        out = np.zeros_like(pos)
        self.lib.orc_nc_vertex_grad(_fp(term), _fp(pos), _u32(pos.shape[0]),
                                    _fp(faces), _fp(vft), _u32(vft.shape[0]),
                                    _fp(out))
        return out

    # indexed access of the paper's HardSoftRas (f_ops.cpp:1490-1799)
    def screen_coord(self, w, h):
        out = np.zeros((h, w, 2), np.float32)
        self.lib.orc_screen_coord(_u32(w), _u32(h), _fp(out))
        return out

    def lookup_faces(self, attr, faces, corner):
        attr, faces = _f32(attr), _f32(faces)
        nv = attr.shape[0]
        n = 1 if attr.ndim == 1 else attr.shape[1]
        out = np.zeros((faces.shape[0], n), np.float32)
        self._err(self.lib.orc_lookup_faces(
            _fp(attr), _u32(nv), _u32(n), _fp(faces), _u32(faces.shape[0]),
            _u32(corner), _fp(out)), "lookup_faces")
        return out

    def lookup_faces_bwd(self, gy, faces, vf, corner):
        """vf: [max_deg, V] (VertexFacesTex)."""
        gy, faces, vf = _f32(gy), _f32(faces), _f32(vf)
        n = 1 if gy.ndim == 1 else gy.shape[1]
        md, nv = vf.shape
        out = np.zeros((nv, n), np.float32)
        self._err(self.lib.orc_lookup_faces_bwd(
            _fp(gy), _u32(n), _fp(faces), _u32(faces.shape[0]), _fp(vf),
            _u32(nv), _u32(md), _u32(corner), _fp(out)), "lookup_faces_bwd")
        return out

    def face_fetch(self, attr, idx):
        attr, idx = _f32(attr), _f32(idx)
        n = 1 if attr.ndim == 1 else attr.shape[1]
        out = np.zeros(idx.shape + (n,), np.float32)
        self.lib.orc_face_fetch(_fp(attr), _u32(attr.shape[0]), _u32(n),
                                _fp(idx), C.c_size_t(idx.size), _fp(out))
        return out

    def face_fetch_bwd(self, gy, idx, prj0, prj1, prj2, seed, radius_px,
                       n_samples):
        gy, idx = _f32(gy), _f32(idx)
        prj = [_f32(p) for p in (prj0, prj1, prj2)]
        h, w = idx.shape
        n = gy.shape[-1]
        nf = prj[0].shape[0]
        out = np.zeros((nf, n), np.float32)
        self.lib.orc_face_fetch_bwd(
            _fp(gy), _u32(n), _fp(idx), _u32(w), _u32(h), _fp(prj[0]),
            _fp(prj[1]), _fp(prj[2]), _u32(nf), C.c_float(seed),
            C.c_float(radius_px), _u32(n_samples), _fp(out))
        return out

    def sum_all(self, x):
        x = _f32(x)
        nc = 1 if x.ndim == 1 else x.shape[-1]
        self.lib.orc_sum_all.restype = C.c_float
        return np.float32(self.lib.orc_sum_all(_fp(x), C.c_size_t(x.size // nc),
                                               _u32(nc)))

    def regularized_grad(self, pos, faces, g, laplacian, normal, vnbrs=None,
                         fadj=None, vft=None):
        pos, faces, g = _f32(pos), _f32(faces), _f32(g)
        nv = pos.shape[0]
        vnbrs = self.vertex_neighbors_tex(faces, nv) if vnbrs is None else vnbrs
        fadj = self.face_neighbors_tex(faces) if fadj is None else fadj
        vft = self.vertex_faces_tex(faces, nv) if vft is None else vft
        out = np.zeros_like(pos)
        self._err(self.lib.orc_regularized_grad(
            _fp(pos), _u32(nv), _fp(faces), _u32(faces.shape[0]),
            _fp(_f32(vnbrs)), _u32(vnbrs.shape[0]), _fp(_f32(fadj)),
            _fp(_f32(vft)), _u32(vft.shape[0]), _fp(g), C.c_float(laplacian),
            C.c_float(normal), _fp(out)), "regularized_grad")
        return out


class Ref(_Lib):
    """_ref/libdressi_ref.so -- the reference CPU implementation."""

    prefix = "ref_"

    def __init__(self, path=None):
        super().__init__(path or REF_SO)

    def soft_clip(self, clip, faces, w, h, radius):
        clip, faces = _f32(clip), _f32(faces)
        out = np.zeros((faces.shape[0] * 3, 4), np.float32)
        self._err(self.lib.ref_soft_clip(_fp(clip), _u32(clip.shape[0]),
                                         _fp(faces), _u32(faces.shape[0]),
                                         _u32(w), _u32(h), C.c_float(radius),
                                         _fp(out)), "soft_clip")
        return out

    def rasterize_soft(self, soft_clip, face_id, faces_soft, hard_clip,
                       faces_tex, vft, w, h, radius, prev_depth=None):
        soft_clip, face_id, faces_soft = map(_f32, (soft_clip, face_id,
                                                    faces_soft))
        hard_clip, faces_tex, vft = map(_f32, (hard_clip, faces_tex, vft))
        pd = None if prev_depth is None else _f32(prev_depth)
        out = np.zeros((h, w, 4), np.float32)
        self._err(self.lib.ref_rasterize_soft(
            _fp(soft_clip), _fp(face_id), _fp(faces_soft),
            _u32(faces_soft.shape[0]), _fp(hard_clip), _u32(hard_clip.shape[0]),
            _fp(faces_tex), _fp(vft), _u32(vft.shape[0]), _u32(w), _u32(h),
            C.c_float(radius), _fp(pd), _fp(out)), "rasterize_soft")
        return out

    def rasterize_face_id(self, clip, faces, w, h):
        clip, faces = _f32(clip), _f32(faces)
        out = np.zeros((h, w), np.float32)
        self._err(self.lib.ref_rasterize_face_id(
            _fp(clip), _u32(clip.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _u32(w), _u32(h), _fp(out)), "rasterize_face_id")
        return out

    def rasterize_hard(self, clip, attr, faces, w, h):
        clip, faces, attr = _f32(clip), _f32(faces), _f32(attr)
        nc = 1 if attr.ndim == 1 else attr.shape[1]
        out = np.zeros((h, w, nc), np.float32)
        self._err(self.lib.ref_rasterize_hard(
            _fp(clip), _u32(clip.shape[0]), _fp(attr), _u32(nc), _fp(faces),
            _u32(faces.shape[0]), _u32(w), _u32(h), _fp(out)),
            "rasterize_hard")
        return out

    def dist_grad(self, soft_clip, face_id, faces_soft, hard_clip, faces_tex,
                  vft, w, h, radius, gy):
        args = list(map(_f32, (soft_clip, face_id, faces_soft, hard_clip,
                               faces_tex, vft, gy)))
        soft_clip, face_id, faces_soft, hard_clip, faces_tex, vft, gy = args
        grad = np.zeros((hard_clip.shape[0], 4), np.float32)
        rs = np.zeros((h, w, 4), np.float32)
        self._err(self.lib.ref_dist_grad(
            _fp(soft_clip), _fp(face_id), _fp(faces_soft),
            _u32(faces_soft.shape[0]), _fp(hard_clip), _u32(hard_clip.shape[0]),
            _fp(faces_tex), _fp(vft), _u32(vft.shape[0]), _u32(w), _u32(h),
            C.c_float(radius), _fp(gy), _fp(grad), _fp(rs)), "dist_grad")
        return grad, rs

    def silhouette_run(self, pos, faces, vft, mvps, targets, res, radius,
                       sigma, lr, n_iters, threads=1, want_grad0=False,
                       laplacian=0.0, normal=0.0):
        pos, faces, vft, mvps, targets = map(_f32, (pos, faces, vft, mvps,
                                                    targets))
        trace = np.zeros(n_iters, np.float32)
        pos_out = np.zeros_like(pos)
        grad0 = np.zeros_like(pos) if want_grad0 else None
        secs = C.c_double(0.0)
        self._err(self.lib.ref_silhouette_run(
            _u32(pos.shape[0]), _u32(faces.shape[0]), _u32(mvps.shape[0]),
            _u32(res), C.c_float(radius), C.c_float(sigma), C.c_float(lr),
            _fp(pos), _fp(faces), _fp(vft), _u32(vft.shape[0]), _fp(mvps),
            _fp(targets), _u32(n_iters), _u32(threads), C.c_float(laplacian),
            C.c_float(normal), _fp(trace), _fp(pos_out), _fp(grad0),
            C.byref(secs)), "silhouette_run")
        return trace, pos_out, grad0, secs.value

    def antialias(self, img, tri, clip, faces, vft, seed=0.0, n_samples=0,
                  gy=None):
        """AntiAlias forward; with gy also (image grad, clip grad)."""
        img, tri, clip, faces, vft = map(_f32, (img, tri, clip, faces, vft))
        h, w = tri.shape
        nc = 1 if img.ndim == 2 else img.shape[2]
        out = np.zeros_like(img)
        gi = gc = None
        if gy is not None:
            gy = _f32(gy)
            gi = np.zeros_like(img)
            gc = np.zeros((clip.shape[0], 4), np.float32)
        self._err(self.lib.ref_antialias(
            _fp(img), _u32(nc), _fp(tri), _fp(clip), _u32(clip.shape[0]),
            _fp(faces), _u32(faces.shape[0]), _fp(vft), _u32(vft.shape[0]),
            C.c_float(seed), _u32(n_samples), _u32(w), _u32(h), _fp(gy),
            _fp(out), _fp(gi), _fp(gc)), "antialias")
        return out if gy is None else (out, gi, gc)

    def texture_bilinear(self, tex, uv, inv_uv, gy=None):
        """TextureBilinear forward; with gy also its texture gradient."""
        tex, uv, inv_uv = map(_f32, (tex, uv, inv_uv))
        th, tw = tex.shape[:2]
        sh, sw = uv.shape[:2]
        n = 1 if tex.ndim == 2 else tex.shape[2]
        out = np.zeros((sh, sw) + ((n,) if tex.ndim == 3 else ()), np.float32)
        g = None
        if gy is not None:
            gy = _f32(gy)
            g = np.zeros_like(tex)
        self._err(self.lib.ref_texture_bilinear(
            _fp(tex), _u32(tw), _u32(th), _u32(n), _fp(uv), _u32(sw),
            _u32(sh), _fp(inv_uv), _fp(gy), _fp(out), _fp(g)),
            "texture_bilinear")
        return out if gy is None else (out, g)

    def aa_silhouette_run(self, pos, faces, vft, mvps, targets, res,
                          n_samples, lr, n_iters, threads=1,
                          want_grad0=False, laplacian=0.0, normal=0.0):
        pos, faces, vft, mvps, targets = map(_f32, (pos, faces, vft, mvps,
                                                    targets))
        trace = np.zeros(n_iters, np.float32)
        pos_out = np.zeros_like(pos)
        grad0 = np.zeros_like(pos) if want_grad0 else None
        secs = C.c_double(0.0)
        self._err(self.lib.ref_aa_silhouette_run(
            _u32(pos.shape[0]), _u32(faces.shape[0]), _u32(mvps.shape[0]),
            _u32(res), _u32(n_samples), C.c_float(lr), _fp(pos), _fp(faces),
            _fp(vft), _u32(vft.shape[0]), _fp(mvps), _fp(targets),
            _u32(n_iters), _u32(threads), C.c_float(laplacian),
            C.c_float(normal), _fp(trace), _fp(pos_out), _fp(grad0),
            C.byref(secs)), "aa_silhouette_run")
        return trace, pos_out, grad0, secs.value

    def image_fit_run(self, param, target, lr, n_iters):
        param, target = _f32(param), _f32(target)
        h, w = param.shape[:2]
        trace = np.zeros(n_iters, np.float32)
        out = np.zeros_like(param)
        secs = C.c_double(0.0)
        self._err(self.lib.ref_image_fit_run(
            _u32(w), _u32(h), _fp(param), _fp(target), C.c_float(lr),
            _u32(n_iters), _fp(trace), _fp(out), C.byref(secs)),
            "image_fit_run")
        return trace, out, secs.value

    def vertex_faces_tex(self, faces, n_verts, cap=64):
        faces = _f32(faces)
        out = np.zeros(n_verts * cap, np.float32)
        md = _u32(0)
        self._err(self.lib.ref_vertex_faces_tex(
            _fp(faces), _u32(faces.shape[0]), _u32(n_verts), _u32(cap),
            _fp(out), C.byref(md)), "vertex_faces_tex")
        return out[: n_verts * md.value].reshape(md.value, n_verts)

    # ---- split-sum IBL (C5): (out, grad of the input image for gy)
    def _img(self, x):
        x = _f32(x)
        h, w = x.shape[:2]
        return x, w, h, 1 if x.ndim == 2 else x.shape[2]

    def equirect_sample(self, env, dirs, gy=None):
        env, mw, mh, n = self._img(env)
        dirs = _f32(dirs)
        dh, dw = dirs.shape[:2]
        out = np.zeros((dh, dw) + env.shape[2:], np.float32)
        g = np.zeros_like(env) if gy is not None else None
        self._err(self.lib.ref_equirect_sample(
            _fp(env), _u32(mw), _u32(mh), _u32(n), _fp(dirs), _u32(dw),
            _u32(dh), _fp(None if gy is None else _f32(gy)), _fp(out),
            _fp(g)), "equirect_sample")
        return out if gy is None else (out, g)

    def irradiance_conv(self, env, ow, oh, gy=None):
        env, sw, sh, n = self._img(env)
        out = np.zeros((oh, ow) + env.shape[2:], np.float32)
        g = np.zeros_like(env) if gy is not None else None
        self._err(self.lib.ref_irradiance_conv(
            _fp(env), _u32(sw), _u32(sh), _u32(n), _u32(ow), _u32(oh),
            _fp(None if gy is None else _f32(gy)), _fp(out), _fp(g)),
            "irradiance_conv")
        return out if gy is None else (out, g)

    def prefilter_conv(self, env, ow, oh, rough, gy=None):
        env, sw, sh, n = self._img(env)
        out = np.zeros((oh, ow) + env.shape[2:], np.float32)
        g = np.zeros_like(env) if gy is not None else None
        self._err(self.lib.ref_prefilter_conv(
            _fp(env), _u32(sw), _u32(sh), _u32(n), _u32(ow), _u32(oh),
            C.c_float(rough), _fp(None if gy is None else _f32(gy)),
            _fp(out), _fp(g)), "prefilter_conv")
        return out if gy is None else (out, g)

    def avg_pool2x2(self, x, gy=None):
        x, w, h, n = self._img(x)
        out = np.zeros((h // 2, w // 2) + x.shape[2:], np.float32)
        g = np.zeros_like(x) if gy is not None else None
        self._err(self.lib.ref_avg_pool2x2(
            _fp(x), _u32(w), _u32(h), _u32(n),
            _fp(None if gy is None else _f32(gy)), _fp(out), _fp(g)),
            "avg_pool2x2")
        return out if gy is None else (out, g)

    def brdf_lut(self, w, h, n_samples):
        out = np.zeros((h, w, 2), np.float32)
        self._err(self.lib.ref_brdf_lut(_u32(w), _u32(h), _u32(n_samples),
                                        _fp(out)), "brdf_lut")
        return out

    def pbr_shade_grad(self, g_n, g_p, mask, albedo, mr, ao, emissive, frame,
                       env, levels, lut_w, lut_h, lut_samples, target,
                       loss_kind=1):
        h, w = mask.shape
        eh, ew = env.shape[:2]
        args = [_f32(a) for a in (g_n, g_p, mask, albedo, mr, ao, emissive,
                                   frame, env, target)]
        mapped = np.zeros((h, w, 3), np.float32)
        ga = np.zeros((h, w, 3), np.float32)
        gm = np.zeros((h, w, 3), np.float32)
        ge = np.zeros((eh, ew, 3), np.float32)
        loss = C.c_float(0.0)
        self._err(self.lib.ref_pbr_shade_grad(
            _u32(w), _u32(h), _fp(args[0]), _fp(args[1]), _fp(args[2]),
            _fp(args[3]), _fp(args[4]), _fp(args[5]), _fp(args[6]),
            _fp(args[7]), _fp(args[8]), _u32(ew), _u32(eh), _u32(levels),
            _u32(lut_w), _u32(lut_h), _u32(lut_samples), _fp(args[9]),
            C.c_int(loss_kind), _fp(mapped), C.byref(loss), _fp(ga),
            _fp(gm), _fp(ge)), "pbr_shade_grad")
        return mapped, loss.value, ga, gm, ge

    def mesh_tables(self, faces, n_verts, cap=64):
        """(vertex neighbours {max_deg, V}, face neighbours [F, 3]) from the
        reference's own builders."""
        faces = _f32(faces)
        vn = np.zeros(n_verts * cap, np.float32)
        fa = np.zeros((faces.shape[0], 3), np.float32)
        md = _u32(0)
        self._err(self.lib.ref_mesh_tables(
            _fp(faces), _u32(faces.shape[0]), _u32(n_verts), _u32(cap),
            _fp(vn), C.byref(md), _fp(fa)), "mesh_tables")
        return vn[: n_verts * md.value].reshape(md.value, n_verts), fa

    def paper_sil_grad(self, pos, faces, vft, mvps, targets, res, radius_px,
                       samples, peels, seed):
        """The paper-path silhouette loss of all views (examples/
        silhouette_optimization/run.cpp:229-396) and d loss / d pos:
        (loss, grad [V, 3], pred [views, R, R])."""
        pos, faces, vft = _f32(pos), _f32(faces), _f32(vft)
        mvps, targets = _f32(mvps), _f32(targets)
        nv, nf = pos.shape[0], faces.shape[0]
        nviews = mvps.reshape(-1, 16).shape[0]
        loss = C.c_float(0.0)
        grad = np.zeros((nv, 3), np.float32)
        pred = np.zeros((nviews, res, res), np.float32)
        self._err(self.lib.ref_paper_sil_grad(
            _u32(nv), _u32(nf), _u32(nviews), _u32(res), C.c_float(radius_px),
            _u32(samples), _u32(peels), _fp(pos), _fp(faces), _fp(vft),
            _u32(vft.shape[0]), _fp(mvps), _fp(targets), C.c_float(seed),
            C.byref(loss), _fp(grad), _fp(pred)), "paper_sil_grad")
        return loss.value, grad, pred

    def screen_coord(self, w, h):
        out = np.zeros((h, w, 2), np.float32)
        self._err(self.lib.ref_screen_coord(_u32(w), _u32(h), _fp(out)),
                  "screen_coord")
        return out

    def lookup_faces(self, attr, faces, vf, corner, gy=None):
        """(out [F, n], g_attr [V, n] or None) through BuildBackward."""
        attr, faces, vf = _f32(attr), _f32(faces), _f32(vf)
        nv = attr.shape[0]
        n = 1 if attr.ndim == 1 else attr.shape[1]
        nf = faces.shape[0]
        out = np.zeros((nf, n), np.float32)
        g = np.zeros((nv, n), np.float32) if gy is not None else None
        keep = _f32(gy) if gy is not None else None
        gyp = _fp(keep) if keep is not None else None
        self._err(self.lib.ref_lookup_faces(
            _fp(attr), _u32(nv), _u32(n), _fp(faces), _u32(nf), _fp(vf),
            _u32(vf.shape[0]), _u32(corner), gyp, _fp(out),
            _fp(g) if g is not None else None), "lookup_faces")
        return out, g

    def face_fetch(self, attr, idx, prj0, prj1, prj2, seed, radius_px,
                   n_samples, gy=None):
        attr, idx = _f32(attr), _f32(idx)
        prj = [_f32(p) for p in (prj0, prj1, prj2)]
        n = 1 if attr.ndim == 1 else attr.shape[1]
        nf = attr.shape[0]
        h, w = idx.shape
        out = np.zeros((h, w, n), np.float32)
        g = np.zeros((nf, n), np.float32) if gy is not None else None
        keep = _f32(gy) if gy is not None else None
        self._err(self.lib.ref_face_fetch(
            _fp(attr), _u32(nf), _u32(n), _fp(idx), _u32(w), _u32(h),
            _fp(prj[0]), _fp(prj[1]), _fp(prj[2]), C.c_float(seed),
            C.c_float(radius_px), _u32(n_samples),
            _fp(keep) if keep is not None else None, _fp(out),
            _fp(g) if g is not None else None), "face_fetch")
        return out, g

    def sum_all(self, x):
        x = _f32(x)
        nc = 1 if x.ndim == 1 else x.shape[-1]
        out = C.c_float(0.0)
        self._err(self.lib.ref_sum_all(_fp(x), _u32(x.size // nc), _u32(nc),
                                       C.byref(out)), "sum_all")
        return np.float32(out.value)

    def regularized_grad(self, pos, faces, g, laplacian, normal):
        pos, faces, g = _f32(pos), _f32(faces), _f32(g)
        out = np.zeros_like(pos)
        self._err(self.lib.ref_regularized_grad(
            _fp(pos), _u32(pos.shape[0]), _fp(faces), _u32(faces.shape[0]),
            _fp(g), C.c_float(laplacian), C.c_float(normal), _fp(out)),
            "regularized_grad")
        return out


def soft_inputs(n_faces: int):
    """face_id {3F} and sequential faces_soft {F,3} (run.cpp:456-466)."""
    fid = np.repeat(np.arange(n_faces, dtype=np.float32), 3)
    fs = np.arange(n_faces * 3, dtype=np.float32).reshape(n_faces, 3)
    return fid, fs
