"""The C-ABI library loads without a GPU and exports exactly what
include/dressi_b200.h declares; argument errors are reported through the
status code + dressi_last_error() before any CUDA call."""

import ctypes as C
import os
import re

import pytest

from conftest import ROOT
from opendressi_b200 import _native as N

HEADER = os.path.join(ROOT, "include", "dressi_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dressi_[a-z0-9_]+)\s*\(", text)))


def test_library_built_and_loads():
    assert os.path.exists(N.LIB_PATH), "run python -m opendressi_b200.build"
    lib = N.load()
    assert lib.dressi_abi_version() == N.ABI_VERSION


def test_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 20
    raw = C.CDLL(N.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), f"{n} declared but not exported"
    # the ctypes binding covers the same set
    assert sorted(N.SIGNATURES) == names


def test_invalid_arguments_report_errors_without_gpu():
    lib = N.load()
    rc = lib.dressi_rasterize_soft(None, 0, None, None, 0, None, 0, None, 1,
                                   16, 16, 3.0, None, None, None, None)
    assert rc == N.ERR_INVALID
    assert "null pointer" in N.last_error()
    rc = lib.dressi_plan_exec(None, 1, None)
    assert rc == N.ERR_INVALID and "null plan" in N.last_error()
    desc = N.SilhouetteDesc()
    desc.struct_size = 3  # wrong size must be rejected
    h = C.c_void_p(0)
    rc = lib.dressi_silhouette_plan_create(C.byref(desc), C.byref(h))
    assert rc == N.ERR_INVALID and "struct_size" in N.last_error()
    with pytest.raises(N.DressiError):
        N.call("dressi_plan_destroy", None) or N.call("dressi_plan_exec",
                                                      None, 1, None)


def test_last_error_truncates():
    lib = N.load()
    lib.dressi_plan_exec(None, 1, None)
    buf = C.create_string_buffer(5)
    full = lib.dressi_last_error(buf, 5)
    assert full > 4 and len(buf.value) == 4


def test_mesh_tables_host_builders_match_oracle(port):
    """The library's VertexFacesTex / VertexNeighborsTex / FaceNeighborsTex
    (host code, no GPU) equal the C restatement, itself pinned to the
    reference's builders."""
    import numpy as np

    from opendressi_b200 import ops, scene

    cases = []
    for lvl in (1, 3):
        sc = scene.silhouette_scene(level=lvl, n_views=1, res=16, seed=1)
        cases.append((sc.faces_f, sc.n_verts))
    for seed in (0, 1):
        rng = np.random.default_rng(seed)
        nv = int(rng.integers(8, 300))
        f = rng.integers(0, nv, (int(rng.integers(4, 600)), 3))
        f = f[(f[:, 0] != f[:, 1]) & (f[:, 1] != f[:, 2]) &
              (f[:, 0] != f[:, 2])]
        cases.append((f.astype(np.float32), nv))
    for f, nv in cases:
        assert np.array_equal(ops.vertex_faces_tex(f, nv),
                              port.vertex_faces_tex(f, nv))
        assert np.array_equal(ops.vertex_neighbors_tex(f, nv),
                              port.vertex_neighbors_tex(f, nv))
        assert np.array_equal(ops.face_neighbors_tex(f),
                              port.face_neighbors_tex(f))
    with pytest.raises(N.DressiError, match="out of range"):
        ops.vertex_faces_tex(np.array([[0, 1, 5]], np.float32), 3)
    with pytest.raises(N.DressiError, match="above cap"):
        ops.vertex_neighbors_tex(cases[1][0], cases[1][1], cap=3)


@pytest.mark.parametrize("name", ["dressi_rasterize_face_id",
                                  "dressi_rasterize_face_id_noalloc"])
def test_face_id_rejects_counts_above_int_max(name):
    """Face or vertex counts above INT_MAX are argument errors, reported
    before any CUDA call (the pointers are never dereferenced)."""
    lib = N.load()
    fake = C.c_void_p(256)
    big = 2**31
    for nv, nf in ((3, big), (big, 1)):
        rc = getattr(lib, name)(fake, nv, fake, nf, 1, 8, 8, fake, None,
                                fake, None)
        assert rc == N.ERR_INVALID
        assert "INT_MAX" in N.last_error()
