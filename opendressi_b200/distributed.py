"""View-sharded data parallelism for the plans (one process per GPU,
torch.distributed over NCCL).

The views of a silhouette optimisation are independent and the loss is their
sum (examples/silhouette_optimization/run.cpp:386-396 of the reference), so
each rank holds a plan over a contiguous slice of the views; one iteration
is the plan's phase 0 (forward + backward of its views, local gradient in the
GRAD slot), a sum all-reduce of that gradient, and phase 1 (the replicated
Adam step, identical on every rank because its inputs are). The position
gradient is 12 B per vertex (123 KB for icosphere-5).

With ``graph=True`` the three parts are captured once into one CUDA graph
(the phases' kernels and the NCCL all-reduce on one stream) and each
iteration is a single graph replay: no host round trip between the phases.
"""

from __future__ import annotations

import numpy as np

__all__ = ["shard_views", "ShardedStep"]


def shard_views(n_views: int, world: int, rank: int) -> np.ndarray:
    """The views rank `rank` of `world` owns: contiguous, sizes differing by
    at most one (numpy.array_split order)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_views < world:
        raise ValueError(f"{n_views} views cannot be sharded over {world} "
                         "ranks")
    return np.array_split(np.arange(n_views), world)[rank]


class ShardedStep:
    """One view-sharded iteration over any plan exposing forward_backward(),
    grad_tensor(), apply_update(), loss_tensor() and record_phase()
    (SilhouettePlan, AaSilhouettePlan, TexturePlan, PbrPlan). With world
    size 1 it runs the same two phases without a collective. Every rank must
    call it the same number of times.

    graph=True captures phase 0, the all-reduce and phase 1 into one CUDA
    graph on first use (after one uncaptured iteration, which sets up the
    communicator); call close() before destroy_process_group()."""

    def __init__(self, plan, group=None, graph: bool = False):
        import torch.distributed as dist

        self.plan = plan
        self.group = group
        self.world = (dist.get_world_size(group)
                      if dist.is_available() and dist.is_initialized() else 1)
        self.grad = plan.grad_tensor()
        self._dist = dist
        self._use_graph = graph
        self._graph = None
        self._calls = 0

    def _eager(self) -> None:
        self.plan.forward_backward()
        if self.world > 1:
            self._dist.all_reduce(self.grad, group=self.group)
        self.plan.apply_update()

    def _capture(self) -> None:
        import torch

        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=side):
            self.plan.record_phase(0)
            if self.world > 1:
                self._dist.all_reduce(self.grad, group=self.group)
            self.plan.record_phase(1)
        torch.cuda.current_stream().wait_stream(side)
        self._graph = g

    def __call__(self) -> None:
        self._calls += 1
        if not self._use_graph or self._calls == 1:
            self._eager()
            return
        if self._graph is None:
            self._capture()
        self._graph.replay()

    def phase_times(self, n: int = 10) -> dict:
        """Milliseconds per iteration of phase 0, the all-reduce and phase 1
        (CUDA events around each, uncaptured; collective)."""
        import torch

        s = torch.cuda.current_stream()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        tot = [0.0, 0.0, 0.0]
        for _ in range(n):
            ev[0].record(s)
            self.plan.forward_backward()
            ev[1].record(s)
            if self.world > 1:
                self._dist.all_reduce(self.grad, group=self.group)
            ev[2].record(s)
            self.plan.apply_update()
            ev[3].record(s)
            torch.cuda.synchronize()
            for i in range(3):
                tot[i] += ev[i].elapsed_time(ev[i + 1])
        return {"forward_backward": tot[0] / n, "all_reduce": tot[1] / n,
                "update": tot[2] / n}

    def loss(self) -> float:
        """Total loss of the last iteration over every rank's views (a sum
        all-reduce; collective)."""
        t = self.plan.loss_tensor().clone()
        if self.world > 1:
            self._dist.all_reduce(t, group=self.group)
        return float(t.item())

    def close(self) -> None:
        """Releases the captured graph (it holds an NCCL call)."""
        self._graph = None
