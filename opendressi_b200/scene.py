"""Seeded synthetic scenes for the Dressi-AD workloads (no dataset needed).

Everything here is host-side numpy producing float32 arrays in the
reference's layouts (positions {V,1} VEC3, faces {F,1} float-valued VEC3,
column-major 4x4 matrices ``m[col*4+row]`` as in the reference's
examples/common/asset_utils.h:79-85).

* ``icosphere(level)``: 12-vertex icosahedron subdivided ``level`` times with
  normalised edge midpoints -- 10*4^L+2 vertices / 20*4^L faces, the sizes of
  the reference generator (examples/common/geometry_utils.cpp:24-84).
* ``sh_displacement``: r = 1 + amp * f(dir), f a seeded sum of real
  spherical harmonics up to degree 4 with N(0,1) coefficients, normalised to
  max|f| = 1 (the silhouette configs' target shape).
* ``orbit_cameras``: seeded views on a sphere of the given radius looking at
  the origin, fov 45 deg, Vulkan-style perspective (y down, depth in [0,1];
  asset_utils.cpp:733-766).
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "icosphere",
    "real_sh_basis",
    "sh_displacement",
    "look_at",
    "perspective_vk",
    "orbit_cameras",
    "silhouette_radius_px",
    "image_fit_scene",
    "SilhouetteScene",
    "silhouette_scene",
]

_ICO_T = (1.0 + math.sqrt(5.0)) / 2.0
# The regular icosahedron as three orthogonal golden rectangles.
_ICO_V = np.array(
    [
        [-1, _ICO_T, 0], [1, _ICO_T, 0], [-1, -_ICO_T, 0], [1, -_ICO_T, 0],
        [0, -1, _ICO_T], [0, 1, _ICO_T], [0, -1, -_ICO_T], [0, 1, -_ICO_T],
        [_ICO_T, 0, -1], [_ICO_T, 0, 1], [-_ICO_T, 0, -1], [-_ICO_T, 0, 1],
    ],
    dtype=np.float64,
)
_ICO_F = np.array(
    [
        [0, 11, 5], [0, 5, 1], [0, 1, 7], [0, 7, 10], [0, 10, 11],
        [1, 5, 9], [5, 11, 4], [11, 10, 2], [10, 7, 6], [7, 1, 8],
        [3, 9, 4], [3, 4, 2], [3, 2, 6], [3, 6, 8], [3, 8, 9],
        [4, 9, 5], [2, 4, 11], [6, 2, 10], [8, 6, 7], [9, 8, 1],
    ],
    dtype=np.int64,
)


def icosphere(level: int) -> tuple[np.ndarray, np.ndarray]:
    """Unit icosphere: (pos float32 [V,3], faces int64 [F,3])."""
    verts = [v / np.linalg.norm(v) for v in _ICO_V]
    faces = _ICO_F.copy()
    for _ in range(level):
        cache: dict[tuple[int, int], int] = {}

        def mid(a: int, b: int) -> int:
            key = (a, b) if a < b else (b, a)
            hit = cache.get(key)
            if hit is not None:
                return hit
            m = (verts[a] + verts[b]) * 0.5
            verts.append(m / np.linalg.norm(m))
            cache[key] = len(verts) - 1
            return cache[key]

        nxt = np.empty((faces.shape[0] * 4, 3), dtype=np.int64)
        for i, (a, b, c) in enumerate(faces):
            ab, bc, ca = mid(a, b), mid(b, c), mid(c, a)
            nxt[4 * i + 0] = (a, ab, ca)
            nxt[4 * i + 1] = (b, bc, ab)
            nxt[4 * i + 2] = (c, ca, bc)
            nxt[4 * i + 3] = (ab, bc, ca)
        faces = nxt
    return np.asarray(verts, dtype=np.float32), faces


def real_sh_basis(dirs: np.ndarray, lmax: int = 4) -> np.ndarray:
    """Orthonormal real spherical harmonics Y_lm(dir), l <= lmax.

    Returns [N, (lmax+1)^2] (float64). Associated Legendre functions by the
    standard upward recurrences (no Condon-Shortley phase)."""
    d = np.asarray(dirs, dtype=np.float64)
    d = d / np.linalg.norm(d, axis=1, keepdims=True)
    x, y, z = d[:, 0], d[:, 1], d[:, 2]
    ct = np.clip(y, -1.0, 1.0)  # polar axis = +y
    st = np.sqrt(np.maximum(0.0, 1.0 - ct * ct))
    phi = np.arctan2(z, x)
    p = {}
    p[(0, 0)] = np.ones_like(ct)
    for m in range(1, lmax + 1):
        p[(m, m)] = (2 * m - 1) * st * p[(m - 1, m - 1)]
    for m in range(0, lmax):
        p[(m + 1, m)] = (2 * m + 1) * ct * p[(m, m)]
    for m in range(0, lmax + 1):
        for l in range(m + 2, lmax + 1):
            p[(l, m)] = ((2 * l - 1) * ct * p[(l - 1, m)]
                         - (l + m - 1) * p[(l - 2, m)]) / (l - m)
    cols = []
    for l in range(lmax + 1):
        for m in range(-l, l + 1):
            am = abs(m)
            k = math.sqrt((2 * l + 1) / (4 * math.pi)
                          * math.factorial(l - am) / math.factorial(l + am))
            if m == 0:
                cols.append(k * p[(l, 0)])
            elif m > 0:
                cols.append(math.sqrt(2.0) * k * p[(l, am)] * np.cos(am * phi))
            else:
                cols.append(math.sqrt(2.0) * k * p[(l, am)] * np.sin(am * phi))
    return np.stack(cols, axis=1)


def sh_displacement(pos: np.ndarray, seed: int, amp: float = 0.2,
                    lmax: int = 4) -> np.ndarray:
    """Radially displace unit-sphere vertices: r = 1 + amp * f, max|f| = 1."""
    rng = np.random.default_rng(seed)
    basis = real_sh_basis(pos, lmax)
    coef = rng.standard_normal(basis.shape[1])
    f = basis @ coef
    f = f / np.max(np.abs(f))
    dirs = pos.astype(np.float64)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    return (dirs * (1.0 + amp * f)[:, None]).astype(np.float32)


def _normalize(v: np.ndarray) -> np.ndarray:
    return v / np.linalg.norm(v)


def look_at(eye, center, up) -> np.ndarray:
    """Column-major view matrix (float64 [16]) of a right-handed camera."""
    eye = np.asarray(eye, np.float64)
    f = _normalize(np.asarray(center, np.float64) - eye)
    s = _normalize(np.cross(f, np.asarray(up, np.float64)))
    u = np.cross(s, f)
    m = np.zeros(16)
    m[0], m[4], m[8] = s
    m[1], m[5], m[9] = u
    m[2], m[6], m[10] = -f
    m[12], m[13], m[14] = -s @ eye, -u @ eye, f @ eye
    m[15] = 1.0
    return m


def perspective_vk(fovy: float, aspect: float, near: float,
                   far: float) -> np.ndarray:
    """Column-major Vulkan-style projection: y flipped, depth in [0, 1]."""
    t = 1.0 / math.tan(fovy * 0.5)
    m = np.zeros(16)
    m[0] = t / aspect
    m[5] = -t
    m[10] = far / (near - far)
    m[11] = -1.0
    m[14] = near * far / (near - far)
    return m


def _mat_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.reshape(4, 4).T @ b.reshape(4, 4).T).T.reshape(16)


def orbit_cameras(n_views: int, seed: int, radius: float = 3.0,
                  fovy_deg: float = 45.0) -> np.ndarray:
    """Seeded cameras on a sphere of ``radius`` looking at the origin.

    Directions are uniform on the sphere with |elevation| <= 60 deg (keeps
    the +y up vector well-conditioned). Returns float32 [n_views, 16]."""
    rng = np.random.default_rng(seed)
    proj = perspective_vk(math.radians(fovy_deg), 1.0, 0.1, 10.0)
    out = np.empty((n_views, 16), np.float32)
    for v in range(n_views):
        az = rng.uniform(0.0, 2.0 * math.pi)
        el = math.asin(rng.uniform(-math.sin(math.pi / 3), math.sin(math.pi / 3)))
        eye = radius * np.array([math.cos(el) * math.sin(az), math.sin(el),
                                 math.cos(el) * math.cos(az)])
        out[v] = _mat_mul(proj, look_at(eye, (0, 0, 0), (0, 1, 0)))
    return out


def silhouette_radius_px(res: int, sigma: float) -> float:
    """Soft band radius in pixels for a SoftRas-style sigma (NDC^2 units):
    the band ends where d_ndc^2 / sigma = 7 (sigmoid(-7) ~ 1e-3)."""
    return float(math.ceil(math.sqrt(7.0 * sigma) * res / 2.0))


def image_fit_scene(seed: int, w: int = 256, h: int = 256):
    """C1: (param0, target) float32 [h, w, 4].

    param0 ~ U[0,1); target = 0.5 + sum of 8 sinusoids per channel
    (frequencies 1-16 cycles/image, phases U[0, 2pi), amplitudes summing to
    0.5) + N(0, 0.01), clamped to [0, 1]."""
    rng = np.random.default_rng(seed)
    param0 = rng.random((h, w, 4), dtype=np.float32)
    yy, xx = np.meshgrid((np.arange(h) + 0.5) / h, (np.arange(w) + 0.5) / w,
                         indexing="ij")
    target = np.empty((h, w, 4), np.float64)
    for c in range(4):
        amps = rng.random(8)
        amps = amps / amps.sum() * 0.5
        acc = np.full((h, w), 0.5)
        for i in range(8):
            fx, fy = rng.uniform(1.0, 16.0, size=2)
            ph = rng.uniform(0.0, 2.0 * math.pi)
            ang = rng.uniform(0.0, 2.0 * math.pi)
            acc += amps[i] * np.sin(2.0 * math.pi * (fx * xx * math.cos(ang)
                                                     + fy * yy * math.sin(ang))
                                    + ph)
        target[..., c] = acc
    target += rng.normal(0.0, 0.01, size=target.shape)
    return param0, np.clip(target, 0.0, 1.0).astype(np.float32)


class SilhouetteScene:
    """Inputs of one silhouette optimisation (configs C3/C4)."""

    def __init__(self, pos0, target_pos, faces, mvps, res, sigma, radius_px,
                 lr):
        self.pos0 = np.ascontiguousarray(pos0, np.float32)
        self.target_pos = np.ascontiguousarray(target_pos, np.float32)
        self.faces = np.ascontiguousarray(faces, np.int64)
        self.faces_f = self.faces.astype(np.float32)
        self.mvps = np.ascontiguousarray(mvps, np.float32)
        self.res = int(res)
        self.sigma = float(sigma)
        self.radius_px = float(radius_px)
        self.lr = float(lr)

    @property
    def n_verts(self) -> int:
        return self.pos0.shape[0]

    @property
    def n_faces(self) -> int:
        return self.faces.shape[0]

    @property
    def n_views(self) -> int:
        return self.mvps.shape[0]


def silhouette_scene(level: int = 5, n_views: int = 16, res: int = 1024,
                     seed: int = 0, sigma: float = 1e-4,
                     lr: float = 1e-3) -> SilhouetteScene:
    """C3 (level 5, 16 views) / C4 (64 views): optimise the unit icosphere
    toward its SH-displaced copy. Targets are rendered separately (they are
    the hard silhouettes of ``target_pos``)."""
    pos, faces = icosphere(level)
    target = sh_displacement(pos, seed=seed + 1)
    mvps = orbit_cameras(n_views, seed=seed + 2)
    return SilhouetteScene(pos, target, faces, mvps, res, sigma,
                           silhouette_radius_px(res, sigma), lr)


# ------------------------------------------------------------------ C2

def sphere_uv(pos: np.ndarray) -> np.ndarray:
    """Spherical uv of unit-sphere positions: (atan2(z, x) / 2pi + 0.5,
    acos(y) / pi). Triangles across the u seam interpolate through the whole
    texture (the config's spherical mapping has no seam split)."""
    p = pos / np.linalg.norm(pos, axis=1, keepdims=True)
    u = np.arctan2(p[:, 2], p[:, 0]) / (2.0 * math.pi) + 0.5
    v = np.arccos(np.clip(p[:, 1], -1.0, 1.0)) / math.pi
    return np.stack([u, v], 1).astype(np.float32)


def checker_texture(seed: int, size: int = 1024, cells: int = 32) -> np.ndarray:
    """Seeded cells x cells checkerboard with a random RGB per cell, float32
    [size, size, 3]."""
    rng = np.random.default_rng(seed)
    colors = rng.random((cells, cells, 3)).astype(np.float32)
    idx = (np.arange(size) * cells) // size
    return np.ascontiguousarray(colors[idx[:, None], idx[None, :]])


class TextureScene:
    """C2 texture optimisation: a UV-mapped icosphere rendered from seeded
    orbit cameras; the optimised texture starts at 0.5."""

    def __init__(self, pos, faces, uv, mvps, res, tex_size, levels, gt_tex,
                 lr):
        self.pos = pos
        self.faces = faces
        self.faces_f = faces.astype(np.float32)
        self.uv = uv
        self.mvps = mvps
        self.res = res
        self.tex_size = tex_size
        self.levels = levels
        self.gt_tex = gt_tex
        self.tex0 = np.full((tex_size, tex_size, 3), 0.5, np.float32)
        self.lr = lr

    @property
    def n_verts(self):
        return self.pos.shape[0]

    @property
    def n_faces(self):
        return self.faces.shape[0]

    @property
    def n_views(self):
        return self.mvps.shape[0]


def texture_scene(level: int = 4, n_views: int = 8, res: int = 512,
                  tex_size: int = 1024, levels: int = 10, seed: int = 0,
                  lr: float = 1e-2) -> TextureScene:
    """Config C2: icosphere-4 (2562 v / 5120 f) with spherical uv, 8 seeded
    cameras on a radius-3 orbit (fov 45 deg) at 512^2, a 1024^2 x 3 texture
    with 10 mip levels (1024 .. 2), a seeded 32x32 checkerboard target,
    Adam lr 1e-2."""
    pos, faces = icosphere(level)
    return TextureScene(pos.astype(np.float32), faces, sphere_uv(pos),
                        orbit_cameras(n_views, seed), res, tex_size, levels,
                        checker_texture(seed + 1, tex_size), lr)


# ------------------------------------------------------------------ C5 (PBR)

def camera_frame(eye, fovy_deg: float = 45.0, aspect: float = 1.0):
    """The per-view frame of the PBR shader (pbr_material_optimization
    run.cpp:309-318): cam_pos, cam_fwd, cam_right * tan(fov/2) * aspect,
    cam_up * tan(fov/2) (look_at the origin, +y up), float32 [12]."""
    vm = look_at(eye, (0, 0, 0), (0, 1, 0))
    t = math.tan(math.radians(fovy_deg) * 0.5)
    fwd = np.array([-vm[2], -vm[6], -vm[10]])
    right = np.array([vm[0], vm[4], vm[8]]) * t * aspect
    up = np.array([vm[1], vm[5], vm[9]]) * t
    return np.concatenate([np.asarray(eye, np.float64), fwd, right,
                           up]).astype(np.float32)


LIGHT_POS = (2.0, 2.0, 2.0)   # the material example's point light
LIGHT_COL = (20.0, 20.0, 20.0)


def sphere_gbuffer(w: int, h: int, seed: int = 0, radius: float = 3.0):
    """An analytic G-buffer of the unit sphere from a seeded camera on a
    radius-3 orbit (fov 45): (g_n [h][w][3], g_p [h][w][3], mask [h][w],
    frame [18] = camera frame + light position + light colour); background
    pixels hold 0 normals and positions, as the rasterizer writes."""
    rng = np.random.default_rng(seed)
    az = rng.uniform(0, 2 * math.pi)
    el = rng.uniform(-0.6, 0.6)
    eye = radius * np.array([math.cos(el) * math.sin(az), math.sin(el),
                             math.cos(el) * math.cos(az)])
    fr = camera_frame(eye)
    cam, fwd, right, up = fr[0:3], fr[3:6], fr[6:9], fr[9:12]
    ys, xs = np.mgrid[0:h, 0:w]
    ndx = (xs + 0.5) * (2.0 / w) - 1.0
    ndy = (ys + 0.5) * (2.0 / h) - 1.0
    d = (fwd[None, None] + right[None, None] * ndx[..., None] -
         up[None, None] * ndy[..., None]).astype(np.float64)
    d /= np.linalg.norm(d, axis=-1, keepdims=True)
    b = (d * cam).sum(-1)
    disc = b * b - ((cam.astype(np.float64) ** 2).sum() - 1.0)
    hit = disc > 0
    t = -b - np.sqrt(np.maximum(disc, 0.0))
    p = np.where(hit[..., None], cam + d * t[..., None], 0.0)
    frame = np.concatenate([fr, LIGHT_POS, LIGHT_COL]).astype(np.float32)
    return (p.astype(np.float32), p.astype(np.float32),
            hit.astype(np.float32), frame)


def ibl_environment(w: int = 512, h: int = 256, seed: int = 0) -> np.ndarray:
    """The C5 environment: a sky gradient plus 4 seeded Gaussian-lobe
    lights, radiance in [0, 50], stored as fp16 values (float32 [h][w][3])."""
    rng = np.random.default_rng(seed)
    v = (np.arange(h) + 0.5) / h
    u = (np.arange(w) + 0.5) / w
    uu, vv = np.meshgrid(u, v)
    theta, phi = vv * math.pi, (uu - 0.5) * 2 * math.pi
    d = np.stack([np.sin(theta) * np.cos(phi), np.cos(theta),
                  np.sin(theta) * np.sin(phi)], -1)
    sky = np.clip(d[..., 1:2], 0, 1) * np.array([0.4, 0.6, 1.0]) + 0.15
    env = np.broadcast_to(sky, (h, w, 3)).copy()
    for _ in range(4):
        c = rng.standard_normal(3)
        c /= np.linalg.norm(c)
        sharp = rng.uniform(20.0, 200.0)
        col = rng.uniform(0.3, 1.0, 3) * rng.uniform(10.0, 49.0)
        lobe = np.exp(sharp * ((d @ c) - 1.0))
        env += lobe[..., None] * col
    env = np.clip(env, 0.0, 50.0)
    return env.astype(np.float16).astype(np.float32)


def value_noise(size: int, seed: int, cells: int = 8,
                octaves: int = 3) -> np.ndarray:
    """Seeded smooth value noise in [0, 1], float32 [size, size] (bilinear
    interpolation of random lattices, octaves halving the cell size)."""
    rng = np.random.default_rng(seed)
    out = np.zeros((size, size))
    amp, tot = 1.0, 0.0
    for o in range(octaves):
        n = cells * (2 ** o)
        lat = rng.random((n + 1, n + 1))
        x = np.arange(size) * n / size
        i = np.floor(x).astype(int)
        f = x - i
        f = f * f * (3 - 2 * f)
        row = lat[i][:, i] * (1 - f)[None, :] + lat[i][:, i + 1] * f[None, :]
        row2 = (lat[i + 1][:, i] * (1 - f)[None, :] +
                lat[i + 1][:, i + 1] * f[None, :])
        out += amp * (row * (1 - f)[:, None] + row2 * f[:, None])
        tot += amp
        amp *= 0.5
    out /= tot
    return ((out - out.min()) / (out.max() - out.min())).astype(np.float32)


class PbrScene:
    """C5: a UV icosphere (unit radius, spherical uv, normals = positions)
    seen from seeded orbit cameras, GGX Cook-Torrance with split-sum IBL;
    the optimised parameters are the albedo and metallic-roughness maps
    (G = roughness, B = metallic) and the environment."""

    def __init__(self, pos, faces, uv, mvps, frames, res, tex_size, env_gt,
                 levels, albedo_gt, mr_gt, lr):
        self.pos = pos
        self.faces = faces
        self.faces_f = faces.astype(np.float32)
        self.uv = uv
        self.mvps = mvps
        self.frames = frames
        self.res = res
        self.tex_size = tex_size
        self.env_gt = env_gt
        self.levels = levels
        self.albedo_gt = albedo_gt
        self.mr_gt = mr_gt
        self.albedo0 = np.full_like(albedo_gt, 0.5)
        self.mr0 = np.full_like(mr_gt, 0.5)
        self.env0 = np.full_like(env_gt, 0.3)
        self.lr = lr
        self.light = np.concatenate([LIGHT_POS, LIGHT_COL]).astype(np.float32)

    @property
    def n_verts(self):
        return self.pos.shape[0]

    @property
    def n_faces(self):
        return self.faces.shape[0]

    @property
    def n_views(self):
        return self.mvps.shape[0]


def pbr_scene(level: int = 6, n_views: int = 32, res: int = 1024,
              tex_size: int = 1024, env_w: int = 512, env_h: int = 256,
              levels: int = 6, seed: int = 0, lr: float = 1e-2) -> PbrScene:
    """Config C5: icosphere-6 (40962 v / 81920 f) with spherical uv, 32
    seeded cameras on a radius-3 orbit (fov 45) at 1024^2, 1024^2 albedo
    and metallic-roughness maps (seeded value noise, roughness in [0.05,
    1]), a 512x256 fp16-valued environment (4 lobes + sky), 6 prefilter
    levels, Adam lr 1e-2."""
    pos, faces = icosphere(level)
    pos = pos.astype(np.float32)
    rng = np.random.default_rng(seed)
    proj = perspective_vk(math.radians(45.0), 1.0, 0.1, 10.0)
    mvps = np.empty((n_views, 16), np.float32)
    frames = np.empty((n_views, 12), np.float32)
    for v in range(n_views):
        az = rng.uniform(0.0, 2.0 * math.pi)
        el = math.asin(rng.uniform(-math.sin(math.pi / 3),
                                   math.sin(math.pi / 3)))
        eye = 3.0 * np.array([math.cos(el) * math.sin(az), math.sin(el),
                              math.cos(el) * math.cos(az)])
        mvps[v] = _mat_mul(proj, look_at(eye, (0, 0, 0), (0, 1, 0)))
        frames[v] = camera_frame(eye)
    alb = np.stack([value_noise(tex_size, seed + 10 + c) for c in range(3)],
                   -1)
    rough = 0.05 + 0.95 * value_noise(tex_size, seed + 20)
    metal = value_noise(tex_size, seed + 30, cells=4)
    mr = np.stack([np.zeros_like(rough), rough, metal], -1).astype(np.float32)
    return PbrScene(pos, faces, sphere_uv(pos), mvps, frames, res, tex_size,
                    ibl_environment(env_w, env_h, seed + 40), levels,
                    alb.astype(np.float32), mr, lr)
