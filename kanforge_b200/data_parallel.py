"""Batch data parallelism for KAN layers: one process per GPU, replicated
coefficients, the parameter gradients summed over the ranks each step.

The reference has no distributed code; tokens (and collocation points) are
independent, so the hot path shards by batch and the only exchange is the
gradient sum of training.  ``edge_derivative`` needs no collective.

Two ways to sum the gradients, both in place (no flattened copy):

* ``allreduce_gradients(params)`` after the backward: one NCCL all-reduce per
  gradient tensor, issued together;
* ``GradientSync(params)`` around the backward: the tensor-core layers hand
  over their parameter gradients as soon as the coefficient-gradient kernel
  has written them, and their all-reduce runs on NCCL's stream while the
  input-gradient kernel runs (kernels.set_grad_ready_hook); what no layer
  handed over is reduced when the context exits.  With
  ``reserved_sms`` the persistent kernels launched after the first all-reduce
  was issued (the input gradients) leave that many SMs to NCCL
  (kernels.set_reserved_sms); a persistent kernel holding every SM would
  otherwise keep NCCL's kernel waiting until it ends.  It needs ``p.grad is None`` at the start of the
  backward (no gradient accumulation across micro-batches).

The sum runs in the gradients' dtype (bf16 for bf16 layers): NCCL adds the
ranks' bf16 values, so each element carries about one bf16 rounding per rank
of relative error; the 2-GPU test holds the result to 2e-2 of the one-GPU
full-batch gradient.

Grid updates (``update_grid``) adapt each layer's grid to its input samples;
on sharded batches every rank would adapt to its own shard and the replicas
would drift apart.  ``update_grid(model, x)`` gathers the ranks' samples
first, so every rank computes the same grids and refit from the whole batch.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels as _kernels


def allreduce_gradients(params, group=None, average: bool = False) -> None:
    """Sum (or average) ``p.grad`` over the ranks of ``group`` in place."""
    grads = [p.grad for p in params if p.grad is not None]
    works = [dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group, async_op=True) for g in grads]
    for w in works:
        w.wait()
    if average:
        world = dist.get_world_size(group)
        for g in grads:
            g.div_(world)


class GradientSync:
    """Context manager around one backward: all-reduces every parameter
    gradient of ``params`` exactly once, overlapped with the backward where a
    layer hands its gradients over early."""

    def __init__(self, params, group=None, reserved_sms: int = 0):
        self.params = [p for p in params]
        self.group = group
        self.reserved_sms = reserved_sms
        self._done: set[int] = set()
        self._works = []

    def _ready(self, pairs):
        works = []
        for p, g in pairs:
            if id(p) in self._done or p.grad is not None:
                continue  # reduced already, or will accumulate into an existing gradient: left to the exit
            self._done.add(id(p))
            works.append(dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
        if works and self.reserved_sms:
            _kernels.set_reserved_sms(self.reserved_sms)  # from the next launch on, beside the all-reduce
        return works

    def __enter__(self):
        self._done.clear()
        _kernels.set_grad_ready_hook(self._ready)
        return self

    def __exit__(self, exc_type, exc, tb):
        _kernels.set_grad_ready_hook(None)
        if self.reserved_sms:
            _kernels.set_reserved_sms(0)
        if exc_type is not None:
            return False
        rest = [p for p in self.params if p.grad is not None and id(p) not in self._done]
        allreduce_gradients(rest, group=self.group)
        return False


def gather_samples(x: torch.Tensor, group=None) -> torch.Tensor:
    """The ranks' sample batches concatenated along the first dimension, in rank
    order, on every rank (one all-gather; every rank passes the same shape)."""
    world = dist.get_world_size(group)
    x = x.contiguous()
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out


def update_grid(model, x: torch.Tensor, group=None, **kwargs) -> None:
    """``model.update_grid`` on the samples of all ranks (a KANLinear or a KAN):
    the replicas keep identical grids and coefficients."""
    model.update_grid(gather_samples(x, group), **kwargs)


def max_over_ranks(value: float, device, group=None) -> float:
    """The maximum of a per-rank scalar (step times are reported as the max over ranks)."""
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
