"""Multi-rank plumbing on CPU (gloo, world size 2): the gradient all-reduce and
the max-over-ranks timing used by bench.py, the sample gather of the
data-parallel grid update, and a rank that fails before the collective, which
the other rank must see as an error within the process-group timeout instead
of hanging."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kanforge_b200.data_parallel import allreduce_gradients, max_over_ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _allreduce_worker(rank, world, port, out):
    _init(rank, world, port)
    try:
        p1 = torch.nn.Parameter(torch.zeros(3, 4))
        p2 = torch.nn.Parameter(torch.zeros(5, dtype=torch.bfloat16))
        p3 = torch.nn.Parameter(torch.zeros(2))  # no gradient this step
        p1.grad = torch.full((3, 4), float(rank + 1))
        p2.grad = torch.arange(5, dtype=torch.bfloat16) * (rank + 1)
        allreduce_gradients([p1, p2, p3])
        t = max_over_ranks(10.0 * (rank + 1), "cpu")
        out[rank] = (p1.grad.clone(), p2.grad.float().clone(), p3.grad, t)
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_and_max_over_ranks():
    world, port = 2, _free_port()
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    mp.spawn(_allreduce_worker, args=(world, port, out), nprocs=world, join=True)
    for rank in range(world):
        g1, g2, g3, t = out[rank]
        assert torch.equal(g1, torch.full((3, 4), 3.0))  # 1 + 2
        assert torch.equal(g2, torch.arange(5, dtype=torch.float32) * 3)
        assert g3 is None
        assert t == 20.0


def _failing_worker(rank, world, port, out):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        out[rank] = "left"
        os._exit(0)  # leaves between steps, before its collective, without cleanup
    p = torch.nn.Parameter(torch.zeros(4))
    p.grad = torch.ones(4)
    try:
        allreduce_gradients([p])
        out[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - any collective failure is the expected outcome
        out[rank] = f"error: {type(e).__name__}"


def test_lost_rank_is_an_error_not_a_hang():
    world, port = 2, _free_port()
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung on the collective of a lost peer")
    assert out[1] == "left"
    assert str(out[0]).startswith("error"), out[0]


def _sync_worker(rank, world, port, out):
    """GradientSync: gradients handed over during the backward are reduced once
    (there), the others when the context exits; the hook is removed after."""
    _init(rank, world, port)
    try:
        import kanforge_b200.kernels as kk
        from kanforge_b200.data_parallel import GradientSync

        early = torch.nn.Parameter(torch.zeros(3))
        late = torch.nn.Parameter(torch.zeros(2))
        sync = GradientSync([early, late])
        with sync:
            g = torch.full((3,), float(rank + 1))
            works = kk._grads_ready([(early, g), (None, None)])  # as the fused backward does
            for w in works:
                w.wait()
            kk._grads_ready([(early, g)])  # a second hand-over of the same parameter is ignored
            early.grad = g
            late.grad = torch.full((2,), 10.0 * (rank + 1))
        out[rank] = (early.grad.clone(), late.grad.clone(), kk._grad_hook is None)
    finally:
        dist.destroy_process_group()


def test_gradient_sync_reduces_every_gradient_once():
    world, port = 2, _free_port()
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    mp.spawn(_sync_worker, args=(world, port, out), nprocs=world, join=True)
    for rank in range(world):
        e, l_, unhooked = out[rank]
        assert torch.equal(e, torch.full((3,), 3.0))
        assert torch.equal(l_, torch.full((2,), 30.0))
        assert unhooked


class _RecordingModel:
    """Stands in for a KAN model: records the samples its grid update sees."""

    def __init__(self):
        self.seen = None
        self.kwargs = None

    def update_grid(self, x, **kwargs):
        self.seen = x.clone()
        self.kwargs = kwargs


def _gather_worker(rank, world, port, out):
    """update_grid on sharded batches: every rank adapts to all ranks' samples,
    in rank order, so the replicas keep identical grids."""
    _init(rank, world, port)
    try:
        from kanforge_b200.data_parallel import gather_samples, update_grid

        x = torch.arange(12, dtype=torch.float32).reshape(3, 4) + 100.0 * rank
        full = gather_samples(x)
        model = _RecordingModel()
        update_grid(model, x[:, :2], margin=0.5)
        out[rank] = (full.clone(), model.seen, model.kwargs)
    finally:
        dist.destroy_process_group()


def test_update_grid_gathers_every_ranks_samples():
    world, port = 2, _free_port()
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    mp.spawn(_gather_worker, args=(world, port, out), nprocs=world, join=True)
    base = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    want = torch.cat([base + 100.0 * r for r in range(world)])
    for rank in range(world):
        full, seen, kwargs = out[rank]
        assert torch.equal(full, want)
        assert torch.equal(seen, want[:, :2])
        assert kwargs == {"margin": 0.5}
