"""Small seeded scenes shared by the CPU and GPU parity tests."""

from __future__ import annotations

import numpy as np

from opendressi_b200 import scene


def clip_of_screen(sx, sy, z, screen, w=1.0):
    """Clip position of a screen point (tests/softras_scene.h:26-30 of the
    reference): clip = (s / S * 2 - 1) * w."""
    return [(sx / screen * 2.0 - 1.0) * w, (sy / screen * 2.0 - 1.0) * w,
            z * w, w]


def soft_scene(hard_verts, faces, scale, screen):
    """CPU-enlarged soft geometry of the reference's SoftScene fixture
    (tests/softras_scene.h:60-140): soft corners scaled about the screen
    centroid, face_id / sequential soft faces."""
    hc = np.asarray(hard_verts, np.float32)
    faces = np.asarray(faces, np.int64)
    nf = faces.shape[0]
    sc = np.zeros((nf * 3, 4), np.float32)
    for f in range(nf):
        cx = np.float32(0.0)
        cy = np.float32(0.0)
        for k in range(3):
            v = hc[faces[f, k]]
            cx = np.float32(cx + v[0] / v[3] / np.float32(3.0))
            cy = np.float32(cy + v[1] / v[3] / np.float32(3.0))
        for k in range(3):
            v = hc[faces[f, k]]
            w = v[3]
            sc[f * 3 + k, 0] = (cx + (v[0] / w - cx) * np.float32(scale)) * w
            sc[f * 3 + k, 1] = (cy + (v[1] / w - cy) * np.float32(scale)) * w
            sc[f * 3 + k, 2] = v[2]
            sc[f * 3 + k, 3] = w
    fid = np.repeat(np.arange(nf, dtype=np.float32), 3)
    fs = np.arange(nf * 3, dtype=np.float32).reshape(nf, 3)
    return dict(soft_clip=sc, face_id=fid, faces_soft=fs, hard_clip=hc,
                faces_tex=faces.astype(np.float32))


def random_triangles(seed, n_faces, screen, n_verts=None, depth_range=(0.05, 0.95),
                     w_range=(0.5, 2.0), spread=0.9):
    """Random clip-space triangles (shared vertices), several overlapping."""
    rng = np.random.default_rng(seed)
    nv = n_verts or n_faces * 2
    ndc = rng.uniform(-spread, spread, size=(nv, 2))
    z = rng.uniform(*depth_range, size=nv)
    w = rng.uniform(*w_range, size=nv)
    clip = np.stack([ndc[:, 0] * w, ndc[:, 1] * w, z * w, w], 1)
    faces = rng.integers(0, nv, size=(n_faces, 3))
    return clip.astype(np.float32), faces.astype(np.float32)


def sphere_views(level, n_views, res, seed=0, sigma=1e-4):
    """Icosphere silhouette scene with oracle-rendered targets."""
    sc = scene.silhouette_scene(level=level, n_views=n_views, res=res,
                                seed=seed, sigma=sigma)
    return sc
