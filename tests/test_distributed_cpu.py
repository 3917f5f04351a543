"""Host logic of the view-sharded iteration (opendressi_b200.distributed) on
2 gloo ranks on CPU: each rank owns a slice of the views, runs phase 0, the
ranks sum their gradients with an all-reduce, and every rank applies the
same Adam step. A CPU stand-in for the plan (the C restatement computing
its views' loss and gradient, orc_adam for the update) must reproduce the
single-process run over all views."""

import os
import socket

import numpy as np
import pytest

from opendressi_b200 import scene
from opendressi_b200.distributed import shard_views


def test_shard_views_partitions():
    for n, world in [(16, 1), (16, 2), (16, 3), (64, 8), (5, 5)]:
        parts = [shard_views(n, world, r) for r in range(world)]
        assert np.array_equal(np.concatenate(parts), np.arange(n))
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_views(3, 4, 0)
    with pytest.raises(ValueError):
        shard_views(8, 2, 2)


class OraclePlan:
    """CPU stand-in exposing the plan interface ShardedStep drives."""

    def __init__(self, sc, targets, views, lr):
        import torch
        from oracle import pyoracle

        self.port = pyoracle.Port()
        self.sc, self.lr = sc, lr
        self.mvps = np.ascontiguousarray(sc.mvps[views])
        self.targets = np.ascontiguousarray(targets[views])
        self.pos = sc.pos0.astype(np.float32).copy()
        self.m = np.zeros_like(self.pos)
        self.v = np.zeros_like(self.pos)
        self.t = 0.0
        self.grad = torch.zeros(self.pos.shape, dtype=torch.float32)
        self.loss_t = torch.zeros(1, dtype=torch.float32)

    def forward_backward(self):
        import torch

        sc = self.sc
        loss, g, _ = self.port.silhouette_loss_grad(
            self.pos, sc.faces_f, self.mvps, self.targets, sc.res,
            sc.radius_px, sc.sigma)
        self.grad.copy_(torch.from_numpy(g))
        self.loss_t[0] = loss

    def grad_tensor(self):
        return self.grad

    def loss_tensor(self):
        return self.loss_t

    def apply_update(self):
        g = np.ascontiguousarray(self.grad.numpy(), np.float32)
        self.t = self.port.adam(self.pos, self.m, self.v, self.t, g, self.lr)


def _scene():
    from oracle import pyoracle

    sc = scene.silhouette_scene(level=2, n_views=4, res=48, seed=8)
    port = pyoracle.Port()
    targets = np.stack([(port.rasterize_face_id(
        port.transform_clip(sc.target_pos, m), sc.faces_f, 48, 48)
        > 0).astype(np.float32) for m in sc.mvps])
    return sc, targets


def _worker(rank, world, port_no, out_dir, iters):
    import torch.distributed as dist
    from opendressi_b200.distributed import ShardedStep

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            init_method=f"tcp://127.0.0.1:{port_no}")
    try:
        sc, targets = _scene()
        plan = OraclePlan(sc, targets, shard_views(sc.n_views, world, rank),
                          lr=1e-2)
        step = ShardedStep(plan)
        losses = []
        for _ in range(iters):
            step()
            losses.append(step.loss())
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), pos=plan.pos,
                 losses=np.array(losses, np.float64))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_step_two_gloo_ranks_match_single_process(tmp_path, port):
    import torch.multiprocessing as mp

    iters = 3
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), iters), nprocs=2,
             join=True)
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    # replicated Adam: the ranks' parameters are bit-identical
    assert np.array_equal(r0["pos"], r1["pos"])
    assert np.array_equal(r0["losses"], r1["losses"])
    sc, targets = _scene()
    trace, pos = port.silhouette_run(sc.pos0, sc.faces_f, sc.mvps, targets,
                                     48, sc.radius_px, sc.sigma, 1e-2, iters)
    np.testing.assert_allclose(r0["losses"], trace, rtol=1e-5)
    close = np.isclose(r0["pos"], pos, atol=1e-5, rtol=1e-4)
    assert close.mean() > 0.99
