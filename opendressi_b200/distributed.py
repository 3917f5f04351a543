"""View-sharded data parallelism for the silhouette plans (one process per
GPU, torch.distributed over NCCL).

The views of a silhouette optimisation are independent and the loss is their
sum (examples/silhouette_optimization/run.cpp:386-396 of the reference), so
each rank holds a plan over a contiguous slice of the views; one iteration
is the plan's phase 0 (forward + backward of its views, local position
gradient in the GRAD slot), a sum all-reduce of that gradient, and phase 1
(the replicated Adam step, identical on every rank because its inputs are).
The gradient is 12 B per vertex (123 KB for icosphere-5).
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
    grad_tensor(), apply_update() and loss_tensor() (SilhouettePlan,
    AaSilhouettePlan). With world size 1 it runs the same two phases without
    a collective. Every rank must call it the same number of times."""

    def __init__(self, plan, group=None):
        import torch.distributed as dist

        self.plan = plan
        self.group = group
        self.world = (dist.get_world_size(group)
                      if dist.is_available() and dist.is_initialized() else 1)
        self.grad = plan.grad_tensor()
        self._dist = dist

    def __call__(self) -> None:
        self.plan.forward_backward()
        if self.world > 1:
            self._dist.all_reduce(self.grad, group=self.group)
        self.plan.apply_update()

    def loss(self) -> float:
        """Total loss of the last iteration over every rank's views (a sum
        all-reduce; collective)."""
        t = self.plan.loss_tensor().clone()
        if self.world > 1:
            self._dist.all_reduce(t, group=self.group)
        return float(t.item())
