"""The C++ graph API (include/dressi/dressi.h) drives the silhouette
optimisation (config C3's graph, icosphere-4, 4 views at 256^2, the
example's regulariser) through DressiAD::execStep from a C++ program
(tests/cpp/graph_silhouette.cpp, built here against libdressi_b200.so): its
loss trace and positions match the fused SilhouettePlan on the same scene
and the C restatement's run (trace 1e-3 rel)."""

import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from opendressi_b200 import ops, scene

pytestmark = pytest.mark.gpu


def _build(tmp_path):
    exe = str(tmp_path / "graph_silhouette")
    cxx = os.environ.get("CXX", "g++")
    lib = os.path.join(ROOT, "opendressi_b200")
    subprocess.run([cxx, "-std=c++17", "-O2", "-I", os.path.join(ROOT,
                                                                 "include"),
                    os.path.join(ROOT, "tests", "cpp",
                                 "graph_silhouette.cpp"),
                    "-o", exe, "-L", lib, "-ldressi_b200",
                    f"-Wl,-rpath,{lib}"], check=True)
    return exe


def test_cpp_graph_silhouette_matches_plan(cuda, port, tmp_path):
    from opendressi_b200 import _native as N
    from opendressi_b200.plans import SilhouettePlan

    sc = scene.silhouette_scene(level=4, n_views=4, res=256, seed=5)
    targets = np.stack([(port.rasterize_face_id(
        port.transform_clip(sc.target_pos, m), sc.faces_f, 256, 256)
        > 0).astype(np.float32) for m in sc.mvps])
    n, lap, nrm = 10, 0.15, 0.4
    vft = ops.vertex_faces_tex(sc.faces_f, sc.n_verts)
    vnb = ops.vertex_neighbors_tex(sc.faces_f, sc.n_verts)
    fadj = ops.face_neighbors_tex(sc.faces_f)
    hdr = np.array([sc.n_verts, sc.faces_f.shape[0], 4, 256, n,
                    vft.shape[0], vnb.shape[0]], np.uint32)
    par = np.array([sc.radius_px, sc.sigma, sc.lr, lap, nrm], np.float32)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as fp:
        for a in (hdr, par, sc.pos0, sc.faces_f, sc.mvps, targets, vft, vnb,
                  fadj):
            fp.write(np.ascontiguousarray(a).tobytes())
    out = tmp_path / "out.bin"
    exe = _build(tmp_path)
    r = subprocess.run([exe, str(inp), str(out)], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    res = np.fromfile(out, np.float32)
    trace, pos = res[:n], res[n:].reshape(-1, 3)
    # the fused plan on the same scene
    plan = SilhouettePlan.from_scene(sc, laplacian=lap, normal=nrm)
    plan.upload(N.SLOT_PARAM, sc.pos0)
    plan.upload(N.SLOT_TARGET, targets)
    plan.step(n)
    np.testing.assert_allclose(trace, plan.loss_history(n), rtol=1e-3)
    trace_cpu, pos_cpu = port.silhouette_run(
        sc.pos0, sc.faces_f, sc.mvps, targets, 256, sc.radius_px, sc.sigma,
        sc.lr, n, laplacian=lap, normal=nrm)
    np.testing.assert_allclose(trace, trace_cpu, rtol=1e-3)
    for p in (plan.download(N.SLOT_PARAM).reshape(-1, 3), pos_cpu):
        assert np.isclose(pos, p, atol=1e-4, rtol=1e-3).mean() > 0.99
    assert "kernels" in r.stdout
