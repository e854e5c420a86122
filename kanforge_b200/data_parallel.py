"""Batch data parallelism for KAN layers: one process per GPU, replicated
coefficients, one NCCL all-reduce of the parameter gradients per step.

The reference has no distributed code; tokens (and collocation points) are
independent, so the hot path shards by batch and the only exchange is the
gradient sum of training.  ``edge_derivative`` needs no collective.
"""

from __future__ import annotations

from collections import defaultdict

import torch
import torch.distributed as dist


def allreduce_gradients(params, group=None, average: bool = False) -> None:
    """Sum (or average) ``p.grad`` over the ranks of ``group`` in one collective
    per dtype: gradients are flattened into one buffer, reduced, and copied back."""
    by_dtype = defaultdict(list)
    for p in params:
        if p.grad is not None:
            by_dtype[p.grad.dtype].append(p.grad)
    world = dist.get_world_size(group)
    for grads in by_dtype.values():
        flat = torch.cat([g.reshape(-1) for g in grads])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        if average:
            flat.div_(world)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off: off + n].view_as(g))
            off += n


def max_over_ranks(value: float, device, group=None) -> float:
    """The maximum of a per-rank scalar (step times are reported as the max over ranks)."""
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
