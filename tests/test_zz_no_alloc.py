"""dressi_rasterize_face_id_noalloc (fixed library-owned scratch, no device
allocation) against dressi_rasterize_face_id on the same inputs, two calls
in a row, through the C ABI. Runs last so that it also covers the state left
by every other test; it must pass alone in a fresh process too."""

import numpy as np
import pytest

import scenes as S
from opendressi_b200 import scene

pytestmark = pytest.mark.gpu


def _call(name, clip, faces, views, w, h, out, depth, status, stream):
    from opendressi_b200 import _native as N

    return getattr(N.load(), name)(
        clip.data_ptr(), clip.shape[-2], faces.data_ptr(), faces.shape[0],
        views, w, h, out.data_ptr(), depth.data_ptr(), status.data_ptr(),
        stream)


def _run_pair(clip_np, faces_np, views, w, h):
    import torch
    from opendressi_b200 import _native as N

    dev = torch.device("cuda:0")
    clip = torch.as_tensor(clip_np, device=dev).contiguous()
    faces = torch.as_tensor(faces_np, device=dev).contiguous()
    stream = torch.cuda.current_stream().cuda_stream
    res = {}
    for name in ("dressi_rasterize_face_id", "dressi_rasterize_face_id_noalloc"):
        outs = []
        for _ in range(2):
            out = torch.full((views, h, w), -7.0, device=dev)
            depth = torch.full((views, h, w), -7.0, device=dev)
            st = torch.zeros(1, dtype=torch.int32, device=dev)
            rc = _call(name, clip, faces, views, w, h, out, depth, st, stream)
            assert rc == 0, N.last_error()
            torch.cuda.synchronize()
            outs.append((out.cpu().numpy(), depth.cpu().numpy(),
                         int(st.item())))
        res[name] = outs
    return res


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", ["random", "sphere"])
def test_noalloc_matches_allocating_entry(cuda, port, case):
    if case == "random":
        clip, faces = S.random_triangles(71, 300, 96, spread=1.1,
                                         w_range=(0.2, 3.0))
        clip[:2, 3] = -clip[:2, 3]
        clip = np.stack([clip, clip * np.float32(0.9)])
        views, w, h = 2, 97, 61
    else:
        sc = scene.silhouette_scene(level=5, n_views=2, res=512, seed=4)
        from oracle import pyoracle

        port = pyoracle.Port()
        clip = np.stack([port.transform_clip(sc.pos0, sc.mvps[v])
                         for v in range(2)])
        faces, views, w, h = sc.faces_f, 2, 512, 512
    res = _run_pair(clip.astype(np.float32), faces.astype(np.float32), views,
                    w, h)
    ref = res["dressi_rasterize_face_id"][0]
    assert (ref[0] > 0).any()
    # and both against the C restatement of RasterizeFaceId
    for v in range(views):
        exp = port.rasterize_face_id(clip[v], faces, w, h)
        assert np.array_equal(_bits(ref[0][v]), _bits(exp)), f"view {v}"
    for k, (out, depth, st) in enumerate(res["dressi_rasterize_face_id_noalloc"]):
        assert np.array_equal(_bits(out), _bits(ref[0])), f"face id, call {k}"
        assert np.array_equal(_bits(depth), _bits(ref[1])), f"depth, call {k}"
        assert st == ref[2] == 0


def test_noalloc_rejects_oversize(cuda):
    import torch
    from opendressi_b200 import _native as N

    # 1 view of 200k faces needs ~32 MB of scratch, over the fixed 16 MiB
    dev = torch.device("cuda:0")
    clip = torch.zeros((3, 4), device=dev)
    faces = torch.zeros((200_000, 3), device=dev)
    out = torch.zeros((1, 8, 8), device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _call("dressi_rasterize_face_id_noalloc", clip, faces, 1, 8, 8, out,
               out, st, torch.cuda.current_stream().cuda_stream)
    assert rc == N.ERR_INVALID
    assert "16777216" in N.last_error()
