"""The graph path's host side, without a GPU: Variables and F:: ops through
the C ABI (dressi_var_* / dressi_op), output type and size inference and
the reference's argument errors; and the recorded op lists that the parity
tests replay on the compiled reference."""

import numpy as np
import pytest

import graph_programs as gp
from opendressi_b200 import _native as N
from opendressi_b200 import graph as G

f = G.f
VT = G.VType


def test_inference_follows_the_reference():
    a = G.Variable(VT.VEC3, 8, 4)
    s = G.Variable(VT.FLOAT, 8, 4)
    u = G.Variable(VT.FLOAT, 1, 1)
    assert (a + s).vtype == VT.VEC3             # scalars broadcast
    assert (a * u).width == 8                   # {1,1} broadcasts spatially
    assert f.dot(a, a).vtype == VT.FLOAT
    assert f.cross(a, a).vtype == VT.VEC3
    assert f.get_y(a).vtype == VT.FLOAT
    assert f.vec4_xyz_w(a, s).vtype == VT.VEC4
    assert f.sum(a).width == 1 and f.sum(a).vtype == VT.VEC3
    assert f.mean(a).vtype == VT.FLOAT
    b = f.broadcast(u, 5, 7)
    assert (b.width, b.height) == (5, 7)
    sc = f.screen_coord(9, 3)
    assert sc.vtype == VT.VEC2 and (sc.width, sc.height) == (9, 3)
    c = f.comp_sum(a)
    assert c.vtype == VT.FLOAT


@pytest.mark.parametrize("bad", [
    lambda: f.dot(G.Variable(VT.VEC3, 2, 2), G.Variable(VT.VEC2, 2, 2)),
    lambda: G.Variable(VT.VEC3, 3, 2) + G.Variable(VT.VEC3, 2, 2),
    lambda: G.Variable(VT.VEC2, 2, 2) + G.Variable(VT.VEC3, 2, 2),
    lambda: G.Variable(VT.INT, 2, 2) + G.Variable(VT.FLOAT, 2, 2),
    lambda: f.less(G.Variable(VT.VEC2, 2, 2), G.Variable(VT.VEC2, 2, 2)),
    lambda: f.broadcast(G.Variable(VT.FLOAT, 2, 2), 4, 4),
    lambda: f.cross(G.Variable(VT.VEC4, 2, 2), G.Variable(VT.VEC4, 2, 2)),
])
def test_reference_argument_errors(bad):
    with pytest.raises(N.DressiError) as e:
        bad()
    assert e.value.code == N.ERR_INVALID


def test_rendering_op_checks():
    clip = G.Variable(VT.VEC4, 10, 1)
    faces = G.Variable(VT.IVEC3, 4, 1)
    ftex = G.Variable(VT.VEC3, 4, 1)
    vft = G.Variable(VT.FLOAT, 10, 6)
    r = f.rasterize(clip, G.Variable(VT.VEC2, 10, 1), faces, 32, 16)
    assert r.vtype == VT.VEC2 and (r.width, r.height) == (32, 16)
    soft = f.soft_clip(clip, ftex, 32, 32, 2.0)
    assert (soft.width, soft.height, soft.vtype) == (12, 1, VT.VEC4)
    rs = f.rasterize_soft(soft, G.Variable(VT.FLOAT, 12, 1), faces, clip,
                          ftex, vft, 32, 32, 2.0)
    assert rs.vtype == VT.VEC4
    with pytest.raises(N.DressiError, match="unwelded"):
        f.rasterize_soft(clip, G.Variable(VT.FLOAT, 10, 1), faces, clip,
                         ftex, vft, 32, 32, 2.0)
    with pytest.raises(N.DressiError, match="unknown"):
        G._op("NoSuchOp", clip)


def test_handles_and_requires_grad():
    x = G.Variable(VT.FLOAT, 4, 4)
    y = f.sin(x) * 2.0
    assert not y.requires_grad()
    x.set_requires_grad_recursively(True)
    assert x.requires_grad() and y.requires_grad()
    assert y.is_computed and not x.is_computed
    z = f.exp(y)                      # created after: not marked
    assert not z.requires_grad()
    ids = [x.id, y.id, z.id]
    assert ids == sorted(ids)         # creation order = topological order


def test_random_programs_replay_on_the_reference(ref):
    """The recorded op lists are valid reference graphs: the compiled
    reference builds, differentiates and evaluates them (the GPU parity
    tests compare the library against exactly these values)."""
    for seed in range(4):
        r, leaves = gp.random_program(seed, 7, 5)
        vals = gp.ref_eval(ref, r, grads_of=leaves)
        assert len(vals) == 2 + len(leaves)
        assert np.isfinite(vals[1]).all()
