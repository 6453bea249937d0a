"""Data-parallel training over several GPUs: one process per GPU, each rank
renders its own view of the replicated model per step, the gradient arenas
are summed with one all-reduce, and every rank applies the same Adam step.

This is the reference's gradient accumulation over several views
(Orchestrator::train_step with accumulate_grad_steps = N,
tinygs/src/orchestrator.cu:343-403: N backward passes add into one gradient
arena, then one optimizer step with gradient scale 1/(grad_scaler * N)),
with the N views of one optimizer step rendered on N GPUs at once.  Any
torch.distributed backend works (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DataParallel:
    world: int = 1
    rank: int = 0
    group: object = None

    @classmethod
    def from_env(cls, group=None) -> "DataParallel":
        if dist.is_available() and dist.is_initialized():
            return cls(dist.get_world_size(group), dist.get_rank(group), group)
        return cls()

    def view_index(self, step: int, n_views: int) -> int:
        """View rendered by this rank at `step`: the N ranks of one step take
        N consecutive views of the orbit, so one step covers the same views
        the reference's accumulation loop would take in N iterations."""
        return (step * self.world + self.rank) % n_views

    def gradient_scale(self, grad_scaler: float) -> float:
        """Adam's gradient scale after the sum over ranks."""
        return 1.0 / (grad_scaler * self.world)

    def reduce_gradients(self, grads: torch.Tensor) -> torch.Tensor:
        """Sum the gradient arena over the ranks in place (one collective)."""
        if self.world > 1:
            dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=self.group)
        return grads

    def max_over_ranks(self, value: float, device) -> float:
        """Largest value over the ranks (timings are reported as the max)."""
        if self.world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())
