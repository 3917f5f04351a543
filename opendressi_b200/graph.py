"""The graph API in Python, mirroring the reference's native binding
(python/csrc/module.cpp: ``Variable``, ``VType``, ``DressiAD`` and the ``f``
op namespace) over the C ABI of libdressi_b200 (dressi_var_* / dressi_op /
dressi_ad_*). A graph built here runs through the library's fusion planner
and CUDA-graph executor; there is no other implementation behind it.

Images go in and out as numpy arrays of shape (h, w, c) (a 2-D (h, w) array
for 1-component images), or as CUDA tensors (zero-copy device transfers).
"""

from __future__ import annotations

import ctypes as C
import enum

import numpy as np

from . import _native as N

__all__ = ["VType", "Variable", "DressiAD", "f", "vertex_faces_tex",
           "vertex_neighbors_tex", "face_neighbors_tex"]


class VType(enum.IntEnum):
    """Element types of graph images (the reference's VType order)."""
    FLOAT = 0
    VEC2 = 1
    VEC3 = 2
    VEC4 = 3
    MAT2 = 4
    MAT3 = 5
    MAT4 = 6
    INT = 7
    IVEC2 = 8
    IVEC3 = 9
    IVEC4 = 10
    UINT = 11


NCOMP = {VType.FLOAT: 1, VType.VEC2: 2, VType.VEC3: 3, VType.VEC4: 4,
         VType.MAT2: 4, VType.MAT3: 9, VType.MAT4: 16, VType.INT: 1,
         VType.IVEC2: 2, VType.IVEC3: 3, VType.IVEC4: 4, VType.UINT: 1}


class Variable:
    """A node of the computational graph (a 2-D image)."""

    __slots__ = ("_h",)

    def __init__(self, vtype=VType.FLOAT, width: int = 1, height: int = 1,
                 _handle=None):
        if _handle is not None:
            self._h = _handle
            return
        h = C.c_void_p(0)
        N.call("dressi_var_create", int(vtype), int(width), int(height),
               C.byref(h))
        self._h = h

    @classmethod
    def _adopt(cls, handle) -> "Variable":
        v = cls.__new__(cls)
        v._h = handle if isinstance(handle, C.c_void_p) else C.c_void_p(handle)
        return v

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                N.load().dressi_var_release(h)
            except Exception:
                pass
            self._h = C.c_void_p(0)

    def _info(self):
        vt, w, h = C.c_int(0), C.c_uint32(0), C.c_uint32(0)
        vid, comp = C.c_uint64(0), C.c_int(0)
        N.call("dressi_var_info", self._h, C.byref(vt), C.byref(w),
               C.byref(h), C.byref(vid), C.byref(comp))
        return VType(vt.value), w.value, h.value, vid.value, bool(comp.value)

    @property
    def vtype(self) -> VType:
        return self._info()[0]

    @property
    def width(self) -> int:
        return self._info()[1]

    @property
    def height(self) -> int:
        return self._info()[2]

    @property
    def id(self) -> int:
        return self._info()[3]

    @property
    def ncomp(self) -> int:
        return NCOMP[self.vtype]

    @property
    def is_computed(self) -> bool:
        return self._info()[4]

    def set_requires_grad(self, req: bool = True) -> None:
        N.call("dressi_var_set_requires_grad", self._h, int(bool(req)), 0)

    def set_requires_grad_recursively(self, req: bool = True) -> None:
        N.call("dressi_var_set_requires_grad", self._h, int(bool(req)), 1)

    def requires_grad(self) -> bool:
        r = C.c_int(0)
        N.call("dressi_var_requires_grad", self._h, C.byref(r))
        return bool(r.value)

    def set_dirty(self, dirty: bool = True) -> None:
        N.call("dressi_var_set_dirty", self._h, int(bool(dirty)), 0)

    def __bool__(self):
        return bool(self._h.value)

    def __eq__(self, o):
        return isinstance(o, Variable) and self.id == o.id

    def __hash__(self):
        return self.id

    def __repr__(self):
        vt, w, h, vid, comp = self._info()
        return f"Variable({vt.name}, {w}x{h}, id={vid})"

    # operator overloads (include/dressi/f.h:321-339)
    def __add__(self, b):
        return _op("Add", self, _lift(b))

    def __radd__(self, a):
        return _op("Add", _lift(a), self)

    def __sub__(self, b):
        return _op("Sub", self, _lift(b))

    def __rsub__(self, a):
        return _op("Sub", _lift(a), self)

    def __mul__(self, b):
        return _op("Mul", self, _lift(b))

    def __rmul__(self, a):
        return _op("Mul", _lift(a), self)

    def __truediv__(self, b):
        return _op("Div", self, _lift(b))

    def __rtruediv__(self, a):
        return _op("Div", _lift(a), self)

    def __neg__(self):
        return _op("Neg", self)

    def __lt__(self, b):
        return _op("Less", self, _lift(b))

    def __le__(self, b):
        return _op("LessEqual", self, _lift(b))

    def __gt__(self, b):
        return _op("Greater", self, _lift(b))

    def __ge__(self, b):
        return _op("GreaterEqual", self, _lift(b))


def _lift(x) -> Variable:
    return x if isinstance(x, Variable) else f.constant(float(x))


def _op(name: str, *xs: Variable, fp=(), ip=()) -> Variable:
    n = len(xs)
    arr = (C.c_void_p * max(n, 1))(*[x._h.value for x in xs])
    fa = (C.c_float * max(len(fp), 1))(*[float(v) for v in fp])
    ia = (C.c_int64 * max(len(ip), 1))(*[int(v) for v in ip])
    out = C.c_void_p(0)
    N.call("dressi_op", name.encode(), arr, n, fa, len(fp), ia, len(ip),
           C.byref(out))
    return Variable._adopt(out)


class _F:
    """The op namespace (reference F::, bound as dressi._C.f)."""

    # constants
    def constant(self, v: float) -> Variable:
        return _op("Float", fp=[v])

    def vec2(self, x, y):
        return _op("Vec2", fp=[x, y])

    def vec3(self, x, y, z):
        return _op("Vec3", fp=[x, y, z])

    def vec4(self, x, y, z, w):
        return _op("Vec4", fp=[x, y, z, w])

    def vec2v(self, x, y):
        return _op("Vec2", x, y)

    def vec3v(self, x, y, z):
        return _op("Vec3", x, y, z)

    def vec4v(self, x, y, z, w):
        return _op("Vec4", x, y, z, w)

    def vec3_xy_z(self, xy, z):
        return _op("Vec3", xy, z)

    def vec4_xyz_w(self, xyz, w):
        return _op("Vec4", xyz, w)

    def get_x(self, v):
        return _op("GetX", v)

    def get_y(self, v):
        return _op("GetY", v)

    def get_z(self, v):
        return _op("GetZ", v)

    def get_w(self, v):
        return _op("GetW", v)

    # arithmetic and math
    def add(self, a, b):
        return _op("Add", a, b)

    def sub(self, a, b):
        return _op("Sub", a, b)

    def mul(self, a, b):
        return _op("Mul", a, b)

    def div(self, a, b):
        return _op("Div", a, b)

    def neg(self, x):
        return _op("Neg", x)

    def sin(self, x):
        return _op("Sin", x)

    def cos(self, x):
        return _op("Cos", x)

    def tan(self, x):
        return _op("Tan", x)

    def asin(self, x):
        return _op("Asin", x)

    def acos(self, x):
        return _op("Acos", x)

    def atan(self, x):
        return _op("Atan", x)

    def atan2(self, y, x):
        return _op("Atan2", y, x)

    def exp(self, x):
        return _op("Exp", x)

    def exp2(self, x):
        return _op("Exp2", x)

    def log(self, x):
        return _op("Log", x)

    def log2(self, x):
        return _op("Log2", x)

    def sqrt(self, x):
        return _op("Sqrt", x)

    def inverse_sqrt(self, x):
        return _op("InverseSqrt", x)

    def abs(self, x):
        return _op("Abs", x)

    def sign(self, x):
        return _op("Sign", x)

    def floor(self, x):
        return _op("Floor", x)

    def fract(self, x):
        return _op("Fract", x)

    def mod(self, x, m):
        return _op("Mod", x, m)

    def pow(self, x, p):
        return _op("Pow", x, p)

    def max(self, a, b):
        return _op("Max", a, b)

    def min(self, a, b):
        return _op("Min", a, b)

    def clamp(self, x, lo, hi):
        return _op("Clamp", x, lo, hi)

    def mix(self, a, b, t):
        return _op("Mix", a, b, t)

    def step(self, edge, x):
        return _op("Step", edge, x)

    def smooth_step(self, e0, e1, x):
        return _op("SmoothStep", e0, e1, x)

    def sigmoid(self, x):
        return _op("Sigmoid", x)

    def less(self, a, b):
        return _op("Less", a, b)

    def less_equal(self, a, b):
        return _op("LessEqual", a, b)

    def greater(self, a, b):
        return _op("Greater", a, b)

    def greater_equal(self, a, b):
        return _op("GreaterEqual", a, b)

    # vectors and matrices
    def dot(self, a, b):
        return _op("Dot", a, b)

    def cross(self, a, b):
        return _op("Cross", a, b)

    def length(self, v):
        return _op("Length", v)

    def distance(self, a, b):
        return _op("Distance", a, b)

    def normalize(self, v):
        return _op("Normalize", v)

    def reflect(self, i, n):
        return _op("Reflect", i, n)

    def comp_sum(self, v):
        return _op("CompSum", v)

    def mat_mul(self, a, b):
        return _op("MatMul", a, b)

    def transpose(self, m):
        return _op("Transpose", m)

    def outer_product(self, c, r):
        return _op("OuterProduct", c, r)

    # reductions and broadcast
    def sum_pixel_wise(self, xs):
        return _op("SumPixelWise", *xs)

    def sum(self, x):
        return _op("Sum", x)

    def mean(self, x):
        return _op("Mean", x)

    def sum_all(self, x):
        return _op("SumAll", x)

    def broadcast(self, x, w, h):
        return _op("Broadcast", x, ip=[w, h])

    def stop_gradient(self, x):
        return _op("StopGradient", x)

    def set_frag_depth(self, x):
        return _op("SetFragDepth", x)

    def screen_coord(self, w, h):
        return _op("ScreenCoord", ip=[w, h])

    # rendering
    def rasterize(self, clip, attr, faces, w, h):
        return _op("Rasterize", clip, attr, faces, ip=[w, h])

    def rasterize_face_id(self, clip, attr, faces, w, h):
        return _op("RasterizeFaceId", clip, attr, faces, ip=[w, h])

    def rasterize_soft(self, clip_soft, face_id, faces_soft, clip_hard_tex,
                       faces_tex, vtx_faces_tex, w, h, radius_px):
        return _op("RasterizeSoft", clip_soft, face_id, faces_soft,
                   clip_hard_tex, faces_tex, vtx_faces_tex, fp=[radius_px],
                   ip=[w, h])

    def rasterize_soft_peel(self, clip_soft, face_id, faces_soft,
                            clip_hard_tex, faces_tex, vtx_faces_tex,
                            prev_shifted_depth, w, h, radius_px):
        return _op("RasterizeSoft", clip_soft, face_id, faces_soft,
                   clip_hard_tex, faces_tex, vtx_faces_tex,
                   prev_shifted_depth, fp=[radius_px], ip=[w, h])

    def soft_clip(self, clip_hard_tex, faces_tex, w, h, radius_px):
        return _op("SoftClip", clip_hard_tex, faces_tex, fp=[radius_px],
                   ip=[w, h])

    def anti_alias(self, img, tri_id, vtx_clip, faces, vtx_faces_tex, seed,
                   n_samples=8):
        return _op("AntiAlias", img, tri_id, vtx_clip, faces, vtx_faces_tex,
                   seed, ip=[n_samples])

    def lookup_faces(self, vtx_attr, faces_tex, vtx_faces_tex, corner):
        return _op("LookupFaces", vtx_attr, faces_tex, vtx_faces_tex,
                   ip=[corner])

    def face_fetch(self, tri_attr, idx_img, tri_prj_0, tri_prj_1, tri_prj_2,
                   seed, radius_px, n_samples=4):
        return _op("FaceFetch", tri_attr, idx_img, tri_prj_0, tri_prj_1,
                   tri_prj_2, seed, fp=[radius_px], ip=[n_samples])

    def texture(self, tex, uv, inv_uv):
        return _op("Texture", tex, uv, inv_uv)

    def texture_bilinear(self, tex, uv, inv_uv):
        return _op("TextureBilinear", tex, uv, inv_uv)

    def pixel_fetch(self, tex, x_index, row_idx):
        return _op("PixelFetch", tex, row_idx, ip=[x_index])

    def tile_fetch(self, atlas, tile_idx, tile_h):
        return _op("TileFetch", atlas, tile_idx, ip=[tile_h])

    def vertex_neighbor_mean(self, pos_tex, vtx_neighbors_tex):
        return _op("VertexNeighborMean", pos_tex, vtx_neighbors_tex)

    def normal_consistency_face_term(self, pos_tex, faces_tex, face_adj_tex):
        return _op("NormalConsistencyFaceTerm", pos_tex, faces_tex,
                   face_adj_tex)

    def normal_consistency_vertex_grad(self, face_term, pos_tex, faces_tex,
                                       vtx_faces_tex):
        return _op("NormalConsistencyVertexGrad", face_term, pos_tex,
                   faces_tex, vtx_faces_tex)

    # split-sum IBL
    def equirect_sample(self, env, dir):
        return _op("EquirectSample", env, dir)

    def irradiance_conv(self, env, w, h):
        return _op("IrradianceConv", env, ip=[w, h])

    def prefilter_conv(self, env, w, h, roughness):
        return _op("PrefilterConv", env, fp=[roughness], ip=[w, h])

    def brdf_integration_lut(self, w, h, n_samples=512):
        return _op("BrdfIntegrationLut", ip=[w, h, n_samples])

    def avg_pool2x2(self, x):
        return _op("AvgPool2x2", x)


f = _F()


def _as_float_image(arr, v: Variable):
    a = np.ascontiguousarray(arr, np.float32)
    n = v.width * v.height * v.ncomp
    if a.size != n:
        raise N.DressiError(N.ERR_INVALID, f"image of {a.size} floats for "
                                           f"{v!r} ({n} expected)")
    return a


class DressiAD:
    """The DR-specialised AD driver (reference DressiAD) on one CUDA
    device: set the loss and optimizer, send images, exec_step() per
    iteration, recv images."""

    def __init__(self, device: int = 0):
        h = C.c_void_p(0)
        N.call("dressi_ad_create", int(device), C.byref(h))
        self._h = h
        self.device = int(device)
        self._opt_cb = None  # keeps the ctypes callback alive
        self._opt_err = None

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            N.load().dressi_ad_destroy(self._h)
            self._h = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_loss_var(self, loss: Variable):
        N.call("dressi_ad_set_loss", self._h, loss._h)

    def set_optimizer(self, fn):
        """fn(xs, gxs) -> list of updated Variables, one per input; called
        during the first exec_step (build time only)."""

        def cb(user, xs, gxs, n, out):
            try:
                xv = [Variable._adopt(_clone(xs[i])) for i in range(n)]
                gv = [Variable._adopt(_clone(gxs[i])) for i in range(n)]
                res = list(fn(xv, gv))
                if len(res) != n:
                    raise ValueError("optimizer must return one output per "
                                     "input")
                for i, r in enumerate(res):
                    out[i] = _clone(r._h).value
                return 0
            except Exception as e:  # reported after exec_step returns
                self._opt_err = e
                return 1

        self._opt_cb = N.OPTIMIZER_FN(cb)
        N.call("dressi_ad_set_optimizer", self._h,
               C.cast(self._opt_cb, C.c_void_p), None)

    def add_update(self, input_leaf: Variable, updated: Variable):
        N.call("dressi_ad_add_update", self._h, input_leaf._h, updated._h)

    def mark_output(self, v: Variable):
        N.call("dressi_ad_mark_output", self._h, v._h)

    def set_grad_outputs_enabled(self, enable: bool):
        N.call("dressi_ad_set_grad_outputs", self._h, int(bool(enable)))

    def set_rebuild_counts(self, fast: int, full: int):
        N.call("dressi_ad_set_rebuild_counts", self._h, int(fast), int(full))

    def set_max_fusion(self, max_ops: int):
        """Ops per fused pixel program (1 = one kernel per op)."""
        N.call("dressi_ad_set_max_fusion", self._h, int(max_ops))

    def input_grads(self):
        n = C.c_uint32(0)
        N.call("dressi_ad_input_grads", self._h, None, None, 0, C.byref(n))
        xs = (C.c_void_p * max(n.value, 1))()
        gs = (C.c_void_p * max(n.value, 1))()
        N.call("dressi_ad_input_grads", self._h, xs, gs, n.value, C.byref(n))
        return [(Variable._adopt(xs[i]), Variable._adopt(gs[i]))
                for i in range(n.value)]

    def exec_step(self, stream=None):
        self._opt_err = None
        rc = N.load().dressi_ad_exec_step(self._h, _stream(stream))
        if self._opt_err is not None:
            raise self._opt_err
        N.check(rc, "exec_step")

    def send_img(self, v: Variable, arr, stream=None):
        if _is_cuda_tensor(arr):
            t = arr.detach().float().contiguous()
            N.call("dressi_ad_send", self._h, v._h, t.data_ptr(), t.numel(),
                   1, _stream(stream))
            return
        a = _as_float_image(arr, v)
        N.call("dressi_ad_send", self._h, v._h, a.ctypes.data, a.size, 0,
               _stream(stream))

    def send_imgs(self, items, stream=None):
        for v, arr in items:
            self.send_img(v, arr, stream)

    def exec_step_with_sends(self, items, stream=None):
        self.send_imgs(items, stream)
        self.exec_step(stream)

    def recv_img(self, v: Variable, out=None, stream=None):
        n = v.width * v.height * v.ncomp
        if _is_cuda_tensor(out):
            N.call("dressi_ad_recv", self._h, v._h, out.data_ptr(), n, 1,
                   _stream(stream))
            return out
        a = np.empty(n, np.float32)
        N.call("dressi_ad_recv", self._h, v._h, a.ctypes.data, n, 0,
               _stream(stream))
        c = v.ncomp
        return a.reshape(v.height, v.width, c) if c > 1 else \
            a.reshape(v.height, v.width)

    def recv_imgs(self, vs):
        return [self.recv_img(v) for v in vs]

    def recv_imgs_stacked(self, vs):
        return np.concatenate([self.recv_img(v) for v in vs], 0)

    def exec_step_with_sends_and_recv_imgs_stacked(self, sends, recvs):
        self.exec_step_with_sends(sends)
        return self.recv_imgs_stacked(recvs)

    def stats(self) -> dict:
        s = N.AdStats()
        N.call("dressi_ad_stats", self._h, C.byref(s))
        return {k: int(getattr(s, k)) for k, _ in N.AdStats._fields_}

    def get_func_count(self) -> int:
        return self.stats()["n_funcs"]

    def get_stage_count(self) -> int:
        return self.stats()["n_steps"]

    def get_substage_count(self) -> int:
        return self.stats()["n_steps"]

    def status(self, clear: bool = True) -> int:
        w = C.c_uint32(0)
        N.call("dressi_ad_status", self._h, C.byref(w), int(bool(clear)))
        return w.value


def _clone(h):
    out = C.c_void_p(0)
    src = h if isinstance(h, C.c_void_p) else C.c_void_p(h)
    N.call("dressi_var_clone", src, C.byref(out))
    return out


def _is_cuda_tensor(x) -> bool:
    try:
        import torch
    except ImportError:
        return False
    return isinstance(x, torch.Tensor) and x.is_cuda


def _stream(stream):
    if stream is not None:
        return C.c_void_p(stream.cuda_stream)
    try:
        import torch

        if torch.cuda.is_available():
            return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    except ImportError:
        pass
    return None


# CPU mesh-topology builders (the reference's module-level helpers)
def vertex_faces_tex(faces, n_verts: int) -> np.ndarray:
    from . import ops

    return ops.vertex_faces_tex(np.asarray(faces, np.float32), n_verts)


def vertex_neighbors_tex(faces, n_verts: int) -> np.ndarray:
    from . import ops

    return ops.vertex_neighbors_tex(np.asarray(faces, np.float32), n_verts)


def face_neighbors_tex(faces) -> np.ndarray:
    from . import ops

    return ops.face_neighbors_tex(np.asarray(faces, np.float32))
