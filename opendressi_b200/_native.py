"""ctypes binding of libdressi_b200.so (include/dressi_b200.h).

The library is built in-tree by ``opendressi_b200.build``; this module never
falls back to anything else -- if the shared library is missing or fails to
load, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdressi_b200.so")

ABI_VERSION = 1

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_DEVICE = 0, 1, 2, 3, 4
STATUS_INDEX_RANGE = 0x1
STATUS_BIN_OVERFLOW = 0x2

SLOT_PARAM, SLOT_ADAM_M, SLOT_ADAM_V, SLOT_ADAM_T = 0, 1, 2, 3
SLOT_TARGET, SLOT_GRAD, SLOT_LOSS, SLOT_LOSS_HISTORY = 4, 5, 6, 7
SLOT_RASTER, SLOT_MVP = 8, 9

_fp = C.POINTER(C.c_float)
_u32 = C.c_uint32
_vp = C.c_void_p


class SilhouetteDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("n_verts", C.c_uint32), ("n_faces", C.c_uint32),
        ("n_views", C.c_uint32), ("res", C.c_uint32),
        ("radius_px", C.c_float), ("sigma", C.c_float), ("lr", C.c_float),
        ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
        ("faces", _fp), ("mvps", _fp),
        ("loss_history", C.c_uint32),
        ("device", C.c_int),
        ("laplacian", C.c_float), ("normal", C.c_float),
    ]


class AaSilhouetteDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("n_verts", C.c_uint32), ("n_faces", C.c_uint32),
        ("n_views", C.c_uint32), ("res", C.c_uint32),
        ("n_samples", C.c_uint32),
        ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
        ("eps", C.c_float),
        ("faces", _fp), ("mvps", _fp),
        ("loss_history", C.c_uint32),
        ("device", C.c_int),
        ("laplacian", C.c_float), ("normal", C.c_float),
    ]


class PbrDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("n_verts", C.c_uint32), ("n_faces", C.c_uint32),
        ("n_views", C.c_uint32), ("res", C.c_uint32),
        ("tex_size", C.c_uint32), ("env_w", C.c_uint32),
        ("env_h", C.c_uint32), ("levels", C.c_uint32),
        ("lut_size", C.c_uint32), ("lut_samples", C.c_uint32),
        ("loss_kind", C.c_uint32),
        ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
        ("eps", C.c_float),
        ("pos", _fp), ("normal", _fp), ("uv", _fp), ("faces", _fp),
        ("mvps", _fp), ("frames", _fp), ("light", _fp),
        ("loss_history", C.c_uint32),
        ("device", C.c_int),
    ]


class TextureDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("n_verts", C.c_uint32), ("n_faces", C.c_uint32),
        ("n_views", C.c_uint32), ("res", C.c_uint32),
        ("tex_size", C.c_uint32), ("levels", C.c_uint32),
        ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
        ("eps", C.c_float),
        ("pos", _fp), ("uv", _fp), ("faces", _fp), ("mvps", _fp),
        ("loss_history", C.c_uint32),
        ("device", C.c_int),
    ]


# name -> (restype, argtypes); exactly the functions include/dressi_b200.h
# declares.
SIGNATURES = {
    "dressi_abi_version": (C.c_int, []),
    "dressi_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "dressi_soft_clip": (C.c_int, [_vp, _u32, _vp, _u32, _u32, _u32, _u32,
                                   C.c_float, _vp, _vp, _vp]),
    "dressi_rasterize_soft": (C.c_int, [_vp, _u32, _vp, _vp, _u32, _vp, _u32,
                                        _vp, _u32, _u32, _u32, C.c_float, _vp,
                                        _vp, _vp, _vp]),
    "dressi_rasterize_soft_grad": (C.c_int, [_vp, _vp, _vp, _u32, _vp, _u32,
                                             _u32, _u32, _u32, _vp, _vp,
                                             _vp]),
    "dressi_rasterize_face_id": (C.c_int, [_vp, _u32, _vp, _u32, _u32, _u32,
                                           _u32, _vp, _vp, _vp, _vp]),
    "dressi_rasterize_face_id_noalloc": (C.c_int, [_vp, _u32, _vp, _u32, _u32,
                                                   _u32, _u32, _vp, _vp, _vp,
                                                   _vp]),
    "dressi_rasterize": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _u32, _u32,
                                   _u32, _u32, _vp, _vp, _vp]),
    "dressi_antialias": (C.c_int, [_vp, _u32, _vp, _vp, _u32, _vp, _u32,
                                   _u32, _u32, _u32, _vp, _vp, _vp]),
    "dressi_antialias_grad": (C.c_int, [_vp, _vp, _u32, _vp, _vp, _u32, _vp,
                                        _u32, _vp, _u32, C.c_float, _u32,
                                        _u32, _u32, _u32, _vp, _vp, _vp,
                                        _vp]),
    "dressi_silhouette_plan_create": (C.c_int, [C.POINTER(SilhouetteDesc),
                                                C.POINTER(_vp)]),
    "dressi_paper_silhouette_plan_create": (C.c_int, [C.POINTER(SilhouetteDesc),
                                                      _u32, _u32,
                                                      C.POINTER(_vp)]),
    "dressi_aa_silhouette_plan_create": (C.c_int, [C.POINTER(AaSilhouetteDesc),
                                                   C.POINTER(_vp)]),
    "dressi_rasterize_uvzw": (C.c_int, [_vp, _vp, _u32, _vp, _u32, _u32, _u32,
                                        _u32, _vp, _vp, _vp]),
    "dressi_interpolate": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _u32,
                                     _u32, _u32, _u32, _vp, _vp, _vp]),
    "dressi_interpolate_grad": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp,
                                          _u32, _u32, _u32, _u32, _vp, _vp,
                                          _vp]),
    "dressi_texture": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _u32, _u32, _vp,
                                 _vp]),
    "dressi_texture_grad": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _u32, _u32,
                                      _vp, _u32, _vp, _vp]),
    "dressi_vertex_faces_tex": (C.c_int, [_vp, _u32, _u32, _u32, _vp,
                                          C.POINTER(_u32)]),
    "dressi_vertex_neighbors_tex": (C.c_int, [_vp, _u32, _u32, _u32, _vp,
                                              C.POINTER(_u32)]),
    "dressi_face_neighbors_tex": (C.c_int, [_vp, _u32, _vp]),
    "dressi_vertex_neighbor_mean": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _vp,
                                              _vp]),
    "dressi_normal_consistency_face_term": (C.c_int, [_vp, _u32, _vp, _u32,
                                                      _vp, _vp, _vp, _vp]),
    "dressi_normal_consistency_vertex_grad": (C.c_int, [_vp, _vp, _u32, _vp,
                                                        _u32, _vp, _u32, _vp,
                                                        _vp, _vp]),
    "dressi_sum_all": (C.c_int, [_vp, _u32, _u32, _vp, _vp]),
    "dressi_regularized_grad": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _u32,
                                          _vp, _vp, _u32, _vp, C.c_float,
                                          C.c_float, _vp, _vp, _vp]),
    "dressi_equirect_sample": (C.c_int, [_vp, _u32, _u32, _u32, _vp,
                                         C.c_uint64, _vp, _vp]),
    "dressi_equirect_sample_grad": (C.c_int, [_vp, _vp, C.c_uint64, _u32,
                                              _u32, _u32, _vp, _vp]),
    "dressi_irradiance_conv": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _u32,
                                         _vp, _vp]),
    "dressi_irradiance_conv_grad": (C.c_int, [_vp, _u32, _u32, _u32, _u32,
                                              _u32, _vp, _vp]),
    "dressi_prefilter_conv": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _u32,
                                        C.c_float, _vp, _vp]),
    "dressi_prefilter_conv_grad": (C.c_int, [_vp, _u32, _u32, _u32, _u32,
                                             _u32, C.c_float, _vp, _vp]),
    "dressi_brdf_lut": (C.c_int, [_u32, _u32, _u32, _vp, _vp]),
    "dressi_avg_pool2x2": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "dressi_avg_pool2x2_grad": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "dressi_screen_coord": (C.c_int, [_u32, _u32, _vp, _vp]),
    "dressi_lookup_faces": (C.c_int, [_vp, _u32, _u32, _vp, _u32, _u32, _vp,
                                      _vp, _vp]),
    "dressi_lookup_faces_grad": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _u32,
                                           _u32, _u32, _vp, _vp, _vp]),
    "dressi_face_fetch": (C.c_int, [_vp, _u32, _u32, _vp, _u32, _u32, _vp,
                                    _vp]),
    "dressi_face_fetch_grad": (C.c_int, [_vp, _u32, _vp, _u32, _u32, _vp, _vp,
                                         _vp, _u32, C.c_float, C.c_float,
                                         _u32, _vp, _vp]),
    "dressi_pbr_plan_create": (C.c_int, [C.POINTER(PbrDesc), C.POINTER(_vp)]),
    "dressi_texture_plan_create": (C.c_int, [C.POINTER(TextureDesc),
                                             C.POINTER(_vp)]),
    "dressi_image_fit_plan_create": (C.c_int, [_u32, _u32, C.c_float, C.c_int,
                                               C.POINTER(_vp)]),
    "dressi_plan_upload": (C.c_int, [_vp, C.c_int, _vp, C.c_size_t, C.c_int,
                                     _vp]),
    "dressi_plan_download": (C.c_int, [_vp, C.c_int, _vp, C.c_size_t,
                                       C.c_int, _vp]),
    "dressi_plan_slot_bytes": (C.c_int, [_vp, C.c_int,
                                         C.POINTER(C.c_size_t)]),
    "dressi_plan_slot_ptr": (C.c_int, [_vp, C.c_int, C.POINTER(_vp)]),
    "dressi_plan_render_targets": (C.c_int, [_vp, _fp, _vp]),
    "dressi_plan_exec": (C.c_int, [_vp, _u32, _vp]),
    "dressi_plan_exec_phase": (C.c_int, [_vp, C.c_int, _vp]),
    "dressi_plan_record_phase": (C.c_int, [_vp, C.c_int, _vp]),
    "dressi_plan_set_deterministic": (C.c_int, [_vp, C.c_int]),
    "dressi_plan_render": (C.c_int, [_vp, _vp]),
    "dressi_plan_status": (C.c_int, [_vp, C.POINTER(_u32), _vp]),
    "dressi_plan_launches_per_iter": (C.c_int, [_vp, C.POINTER(_u32)]),
    "dressi_plan_profile": (C.c_int, [_vp, _u32, _vp, _u32,
                                      C.POINTER(C.c_char_p), _fp,
                                      C.POINTER(_u32), C.POINTER(_u32)]),
    "dressi_plan_destroy": (C.c_int, [_vp]),
    # graph path
    "dressi_var_create": (C.c_int, [C.c_int, _u32, _u32, C.POINTER(_vp)]),
    "dressi_var_clone": (C.c_int, [_vp, C.POINTER(_vp)]),
    "dressi_var_release": (C.c_int, [_vp]),
    "dressi_var_info": (C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(_u32),
                                  C.POINTER(_u32), C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_int)]),
    "dressi_var_set_requires_grad": (C.c_int, [_vp, C.c_int, C.c_int]),
    "dressi_var_requires_grad": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "dressi_var_set_dirty": (C.c_int, [_vp, C.c_int, C.c_int]),
    "dressi_op": (C.c_int, [C.c_char_p, C.POINTER(_vp), _u32,
                            C.POINTER(C.c_float), _u32,
                            C.POINTER(C.c_int64), _u32, C.POINTER(_vp)]),
    "dressi_ad_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "dressi_ad_destroy": (C.c_int, [_vp]),
    "dressi_ad_set_loss": (C.c_int, [_vp, _vp]),
    "dressi_ad_set_optimizer": (C.c_int, [_vp, _vp, _vp]),
    "dressi_ad_add_update": (C.c_int, [_vp, _vp, _vp]),
    "dressi_ad_mark_output": (C.c_int, [_vp, _vp]),
    "dressi_ad_set_grad_outputs": (C.c_int, [_vp, C.c_int]),
    "dressi_ad_set_rebuild_counts": (C.c_int, [_vp, _u32, _u32]),
    "dressi_ad_set_max_fusion": (C.c_int, [_vp, _u32]),
    "dressi_ad_input_grads": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp),
                                        _u32, C.POINTER(_u32)]),
    "dressi_ad_exec_step": (C.c_int, [_vp, _vp]),
    "dressi_ad_send": (C.c_int, [_vp, _vp, _vp, C.c_size_t, C.c_int, _vp]),
    "dressi_ad_recv": (C.c_int, [_vp, _vp, _vp, C.c_size_t, C.c_int, _vp]),
    "dressi_ad_stats": (C.c_int, [_vp, _vp]),
    "dressi_ad_status": (C.c_int, [_vp, C.POINTER(_u32), C.c_int]),
}

# DressiAD::Optimizer through the C ABI (dressi_optimizer_fn)
OPTIMIZER_FN = C.CFUNCTYPE(C.c_int, _vp, C.POINTER(_vp), C.POINTER(_vp), _u32,
                           C.POINTER(_vp))


class AdStats(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "n_funcs", "n_exec_funcs", "n_steps", "n_programs", "n_fused_ops",
        "n_program_instructions", "max_program_regs", "n_materialized",
        "kernels_per_iter", "rebuilds", "pruning_active")]


class DressiError(RuntimeError):
    """Error reported by libdressi_b200 (the reference's DressiError)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lock = threading.Lock()
_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Loads (once) and returns the shared library; raises if absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise DressiError(
                ERR_INVALID,
                f"{p} is missing: build it with `python -m opendressi_b200."
                "build` (there is no fallback implementation)")
        lib = C.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.dressi_abi_version()
        if ver != ABI_VERSION:
            raise DressiError(ERR_INVALID,
                              f"ABI version {ver} != expected {ABI_VERSION}")
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(4096)
    lib.dressi_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        raise DressiError(rc, f"{what}: {last_error()}" if what
                          else last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
