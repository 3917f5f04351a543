"""Test helper: builds a graph with the library's graph API
(opendressi_b200.graph) while recording it as an op list that the compiled
reference evaluates with its own F:: ops, BuildBackward and CpuEvaluator
(oracle/ref_driver.cpp ref_graph_eval); random elementwise programs over
every pixel-wise op; and the evaluation of a recorded program on both
sides."""

from __future__ import annotations

import ctypes as C

import numpy as np

from opendressi_b200 import graph as G

# ops with their arity and the input domain they need
UNARY = ["Neg", "Sin", "Cos", "Exp", "Abs", "Sign", "Floor", "Fract",
         "Sigmoid", "Atan", "Tan"]
UNARY_POS = ["Log", "Log2", "Sqrt", "InverseSqrt"]       # inputs > 0
UNARY_UNIT = ["Asin", "Acos"]                           # inputs in (-1, 1)
BINARY = ["Add", "Sub", "Mul", "Max", "Min", "Step", "Atan2"]
BINARY_DIV = ["Div", "Mod"]                             # divisor away from 0
TERNARY = ["Clamp", "Mix", "SmoothStep"]


class Recorder:
    def __init__(self):
        self.lines: list[str] = []
        self.leaves: list[tuple[int, G.Variable, np.ndarray, bool]] = []
        self.next = 1
        self.evals: list[int] = []
        self.loss_id = None

    def _id(self):
        i = self.next
        self.next += 1
        return i

    def leaf(self, vtype, w, h, data, rg=False):
        v = G.Variable(vtype, w, h)
        i = self._id()
        self.lines.append(f"leaf {i} {int(vtype)} {w} {h} {int(rg)}")
        data = np.ascontiguousarray(data, np.float32).reshape(
            h, w, G.NCOMP[G.VType(vtype)])
        self.leaves.append((i, v, data, rg))
        return (i, v)

    def op(self, name, *ins, fp=(), ip=()):
        v = G._op(name, *[x[1] for x in ins], fp=fp, ip=ip)
        i = self._id()
        fps = " ".join("%.9g" % float(x) for x in fp)
        ips = " ".join(str(int(x)) for x in ip)
        self.lines.append(
            f"op {i} {name} {len(ins)} {' '.join(str(x[0]) for x in ins)} "
            f"{len(fp)} {fps} {len(ip)} {ips}")
        return (i, v)

    def set_loss(self, x):
        self.loss_id = x
        self.lines.append(f"loss {x[0]}")

    def eval(self, x):
        self.evals.append(x)

    def program(self, grads_of=()) -> tuple[str, list]:
        """The reference-side text: the recorded ops, the gradients of the
        given leaves, then the values to return (evals first)."""
        lines = list(self.lines)
        outs = []
        for x in self.evals:
            outs.append(("value", x))
        for j, x in enumerate(grads_of):
            gid = 10_000_000 + j
            lines.append(f"grad {gid} {x[0]}")
            outs.append(("grad", x, gid))
        for o in outs:
            lines.append(f"eval {o[1][0] if o[0] == 'value' else o[2]}")
        return "\n".join(lines) + "\n", outs


def ref_eval(ref, rec: Recorder, grads_of=()):
    """Runs the recorded program on the compiled reference; returns the
    values then the gradients, each as an (h, w, c) array."""
    text, outs = rec.program(grads_of)
    data = np.concatenate([d.reshape(-1) for _, _, d, _ in rec.leaves]
                          or [np.zeros(1, np.float32)])
    shapes = []
    for o in outs:
        v = o[1][1]
        shapes.append((v.height, v.width, v.ncomp))
    total = sum(a * b * c for a, b, c in shapes)
    out = np.zeros(max(total, 1), np.float32)
    fn = ref.lib.ref_graph_eval
    fn.restype = C.c_int
    rc = fn(text.encode(), data.ctypes.data_as(C.POINTER(C.c_float)),
            out.ctypes.data_as(C.POINTER(C.c_float)))
    if rc != 0:
        ref.lib.ref_last_error.restype = C.c_char_p
        raise RuntimeError(ref.lib.ref_last_error().decode())
    res, o = [], 0
    for s in shapes:
        n = s[0] * s[1] * s[2]
        res.append(out[o:o + n].reshape(s))
        o += n
    return res


def ours_eval(rec: Recorder, grads_of=(), device=0, steps=1):
    """Runs the recorded graph on the library (DressiAD on `device`):
    the eval values, then the gradients of `grads_of`."""
    ad = G.DressiAD(device)
    for _, v, _, rg in rec.leaves:
        if rg:
            v.set_requires_grad_recursively(True)
    ad.set_loss_var(rec.loss_id[1])
    ad.set_grad_outputs_enabled(True)
    for x in rec.evals:
        ad.mark_output(x[1])
    for _, v, d, _ in rec.leaves:
        ad.send_img(v, d)
    for _ in range(steps):
        ad.exec_step()
    vals = [ad.recv_img(x[1]).reshape(x[1].height, x[1].width, x[1].ncomp)
            for x in rec.evals]
    pairs = {x.id: g for x, g in ad.input_grads()}
    grads = []
    for x in grads_of:
        g = pairs[x[1].id]
        grads.append(ad.recv_img(g).reshape(g.height, g.width, g.ncomp))
    return vals + grads, ad


def leaf_values(rng, vtype, w, h, lo=-1.5, hi=1.5):
    n = w * h * G.NCOMP[G.VType(vtype)]
    return rng.uniform(lo, hi, n).astype(np.float32)


def random_program(seed: int, w: int, h: int, n_ops: int = 24,
                   vec: bool = True):
    """A random pixel-wise graph over a few leaves (FLOAT / VEC3 images and
    a {1,1} uniform), every op of the library's pixel-wise set, domain-safe
    by construction; loss = Mean of the last value (and the sum of the
    others, so every value reaches the loss)."""
    rng = np.random.default_rng(seed)
    r = Recorder()
    leaves = [r.leaf(G.VType.FLOAT, w, h, leaf_values(rng, 0, w, h), True),
              r.leaf(G.VType.FLOAT, w, h, leaf_values(rng, 0, w, h), True),
              r.leaf(G.VType.FLOAT, 1, 1, leaf_values(rng, 0, 1, 1), True)]
    if vec:
        leaves.append(r.leaf(G.VType.VEC3, w, h,
                             leaf_values(rng, 2, w, h), True))
    scal = [leaves[0], leaves[1]]
    vecs = [leaves[3]] if vec else []
    uni = leaves[2]

    def pick(pool):
        return pool[int(rng.integers(len(pool)))]

    def positive(x):
        # Add(Mul(x, x), 0.5) > 0
        return r.op("Add", r.op("Mul", x, x), r.op("Float", fp=[0.5]))

    def unit(x):
        # 0.9 * sin(x) in (-1, 1)
        return r.op("Mul", r.op("Sin", x), r.op("Float", fp=[0.9]))

    for _ in range(n_ops):
        kind = rng.random()
        if vec and kind < 0.15:
            a, b = pick(vecs), pick(vecs)
            name = ["Dot", "Cross", "Normalize", "Length", "CompSum", "Add",
                    "Mul"][int(rng.integers(7))]
            if name in ("Dot",):
                scal.append(r.op(name, a, b))
            elif name == "Cross":
                vecs.append(r.op(name, a, b))
            elif name == "Normalize":
                vecs.append(r.op(name, r.op("Add", a, r.op(
                    "Vec3", fp=[2.0, 2.0, 2.0]))))
            elif name in ("Length", "CompSum"):
                scal.append(r.op(name, a))
            else:
                vecs.append(r.op(name, a, pick(scal + vecs)))
            continue
        if vec and kind < 0.22:
            # compose / extract
            if rng.random() < 0.5:
                vecs.append(r.op("Vec3", pick(scal), pick(scal), pick(scal)))
            else:
                scal.append(r.op(["GetX", "GetY", "GetZ"][int(rng.integers(3))],
                                 pick(vecs)))
            continue
        x = pick(scal)
        if kind < 0.5:
            name = UNARY[int(rng.integers(len(UNARY)))]
            if name == "Tan":
                x = unit(x)
            scal.append(r.op(name, x))
        elif kind < 0.58:
            scal.append(r.op(UNARY_POS[int(rng.integers(len(UNARY_POS)))],
                             positive(x)))
        elif kind < 0.62:
            scal.append(r.op(UNARY_UNIT[int(rng.integers(2))], unit(x)))
        elif kind < 0.82:
            y = pick(scal + [uni])
            scal.append(r.op(BINARY[int(rng.integers(len(BINARY)))], x, y))
        elif kind < 0.88:
            y = positive(pick(scal + [uni]))
            scal.append(r.op(BINARY_DIV[int(rng.integers(2))], x, y))
        elif kind < 0.92:
            scal.append(r.op("Pow", positive(x), pick(scal + [uni])))
        else:
            name = TERNARY[int(rng.integers(len(TERNARY)))]
            if name == "SmoothStep":
                e0 = r.op("Float", fp=[-0.5])
                e1 = r.op("Float", fp=[0.7])
                scal.append(r.op(name, e0, e1, x))
            elif name == "Clamp":
                scal.append(r.op(name, x, r.op("Float", fp=[-0.4]),
                                 r.op("Float", fp=[0.6])))
            else:
                scal.append(r.op(name, x, pick(scal), pick(scal + [uni])))
    # every leaf reaches the loss
    terms = scal[2:] + [r.op("CompSum", v) for v in vecs] + [
        r.op("Mul", leaves[0], leaves[1]), r.op("Mul", leaves[0], uni)]
    total = r.op("SumPixelWise", *terms) if len(terms) > 1 else terms[0]
    loss = r.op("Mean", r.op("Mul", total, total))
    r.set_loss(loss)
    r.eval(total)
    r.eval(loss)
    return r, leaves
