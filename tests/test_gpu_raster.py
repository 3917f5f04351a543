"""GPU parity of the rasterizer ops against the C restatement and the
reference's golden outputs. Triangle IDs, coverage, distances and depths are
compared BIT-EXACT; gradients within 1e-4 abs + 1e-3 rel (the reference's
SoftRasGpu.BackwardParityCpu bar)."""

import os

import numpy as np
import pytest

from conftest import GOLDEN
import scenes as S

from oracle import pyoracle
from opendressi_b200 import scene

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def T(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)


def npy(t):
    return t.detach().cpu().numpy()


def assert_bitexact(gpu, cpu, what):
    g, c = bits(gpu), bits(cpu)
    if not np.array_equal(g, c):
        bad = np.argwhere(g != c)
        i = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatching words, first at "
                             f"{i}: gpu={np.asarray(gpu)[i]!r} "
                             f"cpu={np.asarray(cpu)[i]!r}")


def _soft_case(port, seed, w, h, n_faces=60, radius=3.0, spread=1.1):
    clip, faces = S.random_triangles(seed, n_faces, max(w, h), spread=spread,
                                     w_range=(0.2, 3.0))
    clip[:2, 3] = -clip[:2, 3]          # behind the camera
    faces[3] = faces[4]                 # duplicate face (depth tie)
    faces[5, 1] = faces[5, 0]           # degenerate face
    soft = port.soft_clip(clip, faces, w, h, radius)
    fid, fs = pyoracle.soft_inputs(faces.shape[0])
    return clip, faces, soft, fid, fs


def test_golden_raster_small(cuda, port):
    from opendressi_b200 import ops

    g = np.load(os.path.join(GOLDEN, "raster_small.npz"))
    w, h, radius = 48, 40, 3.0
    clip, faces = S.random_triangles(1, 40, 48)
    soft = ops.soft_clip(T(clip, cuda), T(faces, cuda), w, h, radius)
    assert_bitexact(npy(soft), g["soft_clip"], "SoftClip")
    fid, fs = pyoracle.soft_inputs(faces.shape[0])
    rs = ops.rasterize_soft(soft, T(fid, cuda), T(fs, cuda), T(clip, cuda),
                            T(faces, cuda), w, h, radius)
    assert_bitexact(npy(rs), g["rs"], "RasterizeSoft")
    assert_bitexact(npy(ops.rasterize_face_id(T(clip, cuda), T(faces, cuda),
                                              w, h)), g["face_id"], "FaceId")
    attr = np.random.default_rng(8).random((clip.shape[0], 3)).astype(np.float32)
    assert_bitexact(npy(ops.rasterize(T(clip, cuda), T(attr, cuda),
                                      T(faces, cuda), w, h)), g["hard"],
                    "Rasterize")
    grad = ops.rasterize_soft_grad(T(g["gy"], cuda), rs, T(clip, cuda),
                                   T(faces, cuda))
    np.testing.assert_allclose(npy(grad), g["grad"], atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("seed,w,h", [(21, 16, 16), (22, 33, 17), (23, 64, 48),
                                      (24, 1, 1), (25, 130, 70)])
def test_rasterize_soft_random_bitexact(cuda, port, seed, w, h):
    from opendressi_b200 import ops

    radius = 2.5 + seed % 3
    clip, faces, soft, fid, fs = _soft_case(port, seed, w, h, radius=radius)
    cpu = port.rasterize_soft(soft, fid, fs, clip, faces, w, h, radius)
    gpu = ops.rasterize_soft(T(soft, cuda), T(fid, cuda), T(fs, cuda),
                             T(clip, cuda), T(faces, cuda), w, h, radius)
    assert_bitexact(npy(gpu), cpu, "RasterizeSoft")
    # depth-peeling variant with the previous layer's shifted depth
    prev = np.where(cpu[..., 3] > 0, 0.3, 0.0).astype(np.float32)
    cpu2 = port.rasterize_soft(soft, fid, fs, clip, faces, w, h, radius, prev)
    gpu2 = ops.rasterize_soft(T(soft, cuda), T(fid, cuda), T(fs, cuda),
                              T(clip, cuda), T(faces, cuda), w, h, radius,
                              prev_depth=T(prev, cuda))
    assert_bitexact(npy(gpu2), cpu2, "RasterizeSoft peel")
    assert_bitexact(npy(ops.rasterize_face_id(T(clip, cuda), T(faces, cuda),
                                              w, h)),
                    port.rasterize_face_id(clip, faces, w, h), "FaceId")


def test_rasterize_soft_views_batched(cuda, port):
    from opendressi_b200 import ops

    w, h, radius = 40, 40, 3.0
    cases = [_soft_case(port, 30 + v, w, h) for v in range(3)]
    clip, faces = cases[0][0], cases[0][1]
    # views share faces: re-use view 0's faces, different geometry
    softs, clips = [], []
    for v in range(3):
        c = S.random_triangles(40 + v, 60, 40)[0]
        clips.append(c)
        softs.append(port.soft_clip(c, faces, w, h, radius))
    fid, fs = pyoracle.soft_inputs(faces.shape[0])
    gpu = ops.rasterize_soft(T(np.stack(softs), cuda),
                             T(np.stack([fid] * 3), cuda), T(fs, cuda),
                             T(np.stack(clips), cuda), T(faces, cuda), w, h,
                             radius)
    for v in range(3):
        cpu = port.rasterize_soft(softs[v], fid, fs, clips[v], faces, w, h,
                                  radius)
        assert_bitexact(npy(gpu[v]), cpu, f"view {v}")


def test_sphere_256_bitexact_and_grad(cuda, port):
    from opendressi_b200 import ops

    sc = scene.silhouette_scene(level=4, n_views=2, res=256, seed=3)
    for v in range(2):
        clip = port.transform_clip(sc.pos0, sc.mvps[v])
        soft_c = port.soft_clip(clip, sc.faces_f, 256, 256, sc.radius_px)
        soft_g = ops.soft_clip(T(clip, cuda), T(sc.faces_f, cuda), 256, 256,
                               sc.radius_px)
        assert_bitexact(npy(soft_g), soft_c, "SoftClip")
        fid, fs = pyoracle.soft_inputs(sc.n_faces)
        cpu = port.rasterize_soft(soft_c, fid, fs, clip, sc.faces_f, 256,
                                  256, sc.radius_px)
        gpu = ops.rasterize_soft(soft_g, T(fid, cuda), T(fs, cuda),
                                 T(clip, cuda), T(sc.faces_f, cuda), 256, 256,
                                 sc.radius_px)
        assert_bitexact(npy(gpu), cpu, "RasterizeSoft sphere")
        gy = np.random.default_rng(v).standard_normal((256, 256)).astype(
            np.float32)
        g_cpu = port.dist_grad(gy, cpu, clip, sc.faces_f, 256, 256)
        g_gpu = ops.rasterize_soft_grad(T(gy, cuda), gpu, T(clip, cuda),
                                        T(sc.faces_f, cuda))
        np.testing.assert_allclose(npy(g_gpu), g_cpu, atol=1e-4, rtol=1e-3)


def test_empty_mesh_and_index_errors(cuda, port):
    import torch
    from opendressi_b200 import ops
    from opendressi_b200._native import DressiError

    empty = torch.zeros((0, 3), device=cuda)
    out = ops.rasterize_soft(torch.zeros((0, 4), device=cuda),
                             torch.zeros((0,), device=cuda), empty,
                             torch.zeros((3, 4), device=cuda), empty, 8, 8,
                             2.0)
    assert float(out.abs().sum()) == 0.0
    clip, faces = S.random_triangles(5, 4, 16)
    bad = faces.copy()
    bad[2, 1] = 1e6  # vertex index out of range: the reference throws
    with pytest.raises(DressiError):
        ops.rasterize_face_id(T(clip, cuda), T(bad, cuda), 16, 16)
        ops.check_status()
    with pytest.raises(DressiError):
        ops.soft_clip(T(clip, cuda), T(bad, cuda), 16, 16, 2.0)
        ops.check_status()


@pytest.mark.parametrize("spill_cap", [None, "0"])
def test_bin_overflow_fallback_is_exact(cuda, port, monkeypatch, spill_cap):
    """A tile-list capacity too small for the scene sends the excess entries
    to the spill lists (spill_cap None) or, with no spill room, makes the
    device fall back to exhaustive (all-faces) sweeps: bit-exact either way,
    and flagged in the status word."""
    from opendressi_b200 import ops
    from opendressi_b200 import _native as N

    monkeypatch.setenv("DRESSI_B200_BIN_CAP", "64")
    if spill_cap is not None:
        monkeypatch.setenv("DRESSI_B200_SPILL_CAP", spill_cap)
    sc = scene.silhouette_scene(level=3, n_views=1, res=128, seed=9)
    clip = port.transform_clip(sc.pos0, sc.mvps[0])
    soft = port.soft_clip(clip, sc.faces_f, 128, 128, sc.radius_px)
    fid, fs = pyoracle.soft_inputs(sc.n_faces)
    cpu = port.rasterize_soft(soft, fid, fs, clip, sc.faces_f, 128, 128,
                              sc.radius_px)
    import torch

    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty((1, 128, 128, 4), device=cuda)
    args = [T(soft, cuda), T(fid, cuda), T(fs, cuda), T(clip, cuda),
            T(sc.faces_f, cuda)]
    N.call("dressi_rasterize_soft", args[0].data_ptr(), soft.shape[0],
           args[1].data_ptr(), args[2].data_ptr(), sc.n_faces,
           args[3].data_ptr(), clip.shape[0], args[4].data_ptr(), 1, 128, 128,
           float(sc.radius_px), None, out.data_ptr(), st.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert int(st.item()) & N.STATUS_BIN_OVERFLOW
    assert_bitexact(npy(out[0]), cpu, "RasterizeSoft (overflow fallback)")
    fi = ops.rasterize_face_id(T(clip, cuda), T(sc.faces_f, cuda), 128, 128,
                               check=False)
    assert_bitexact(npy(fi), port.rasterize_face_id(clip, sc.faces_f, 128,
                                                    128), "FaceId fallback")
