"""Data parallelism on two GPUs over NCCL: the batch split across ranks, the
gradients summed by an all-reduce that overlaps the backward
(data_parallel.GradientSync), must equal the gradients of the whole batch on
one GPU.  The ranks add bf16 gradients, so the bound is the bf16 tolerance
2e-2 (metric max|a-b| / max(1, max|b|)).  Skipped with fewer than two GPUs."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import kan_oracle as ko

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(kind: str):
    import kanforge_b200 as kb

    torch.manual_seed(0)
    if kind == "cheb":
        layer = kb.KANLinear(256, 512, kb.Chebyshev(12), edge_scale=True)
    elif kind == "bspline":
        layer = kb.KANLinear(128, 256, kb.BSpline(8, 3))
    else:
        layer = kb.GRKAN(256, 512, groups=8)
    with torch.no_grad():
        layer.coef.normal_(0, 0.05)
    return layer


def _batch(n_in: int, n_out: int):
    g = torch.Generator().manual_seed(1)
    return torch.randn(4096, n_in, generator=g).clamp(-3, 3), torch.randn(4096, n_out, generator=g) * 0.1


def _grads(layer, x, dy, sync=None):
    for p in layer.parameters():
        p.grad = None
    y = layer(x)
    if sync is None:
        y.backward(dy)
    else:
        with sync:
            y.backward(dy)
    return {n: p.grad.detach().float().cpu() for n, p in layer.named_parameters()}


def _worker(rank, world, port, kind, reserve, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        from kanforge_b200.data_parallel import GradientSync, allreduce_gradients

        layer = _layer(kind).to(device=dev, dtype=torch.bfloat16)
        x, dy = _batch(layer.in_features, layer.out_features)
        shard = slice(rank * 2048, (rank + 1) * 2048)
        xs, dys = x[shard].to(dev, torch.bfloat16), dy[shard].to(dev, torch.bfloat16)
        overlapped = _grads(layer, xs, dys, GradientSync(list(layer.parameters()), reserved_sms=reserve))
        _grads(layer, xs, dys)
        allreduce_gradients(list(layer.parameters()))
        after = {n: p.grad.detach().float().cpu() for n, p in layer.named_parameters()}
        torch.cuda.synchronize()
        out[rank] = (overlapped, after)
        if rank == 0:
            out["full"] = _grads(layer, x.to(dev, torch.bfloat16), dy.to(dev, torch.bfloat16))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("kind,reserve", [("cheb", 0), ("cheb", 16), ("bspline", 0), ("grkan", 0)])
def test_two_gpu_gradients_equal_full_batch(kind, reserve):
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    mp.spawn(_worker, args=(2, _free_port(), kind, reserve, out), nprocs=2, join=True)
    full = out["full"]
    for rank in range(2):
        overlapped, after = out[rank]
        for name, want in full.items():
            for got, how in ((overlapped, "overlapped"), (after, "after the backward")):
                err = ko.max_rel_err(got[name].double().numpy(), want.double().numpy())
                assert err <= 2e-2, f"rank {rank} {name} ({how}): max rel err {err:.3e}"
        for name in full:  # both ranks hold the same sum
            assert torch.equal(out[0][0][name], out[1][0][name])


def _grid_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        import kanforge_b200 as kb
        from kanforge_b200.data_parallel import update_grid

        def model():
            torch.manual_seed(0)
            return kb.KAN([64, 32, 16], kb.BSpline(8, 3), device=dev)

        g = torch.Generator().manual_seed(2)
        x = (torch.randn(4096, 64, generator=g) * 1.5).to(dev)
        dp = model()
        update_grid(dp, x[rank * 2048:(rank + 1) * 2048])
        out[rank] = {n: t.detach().cpu().clone() for n, t in dp.state_dict().items()}
        if rank == 0:
            full = model()
            full.update_grid(x)
            out["full"] = {n: t.detach().cpu().clone() for n, t in full.state_dict().items()}
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_gpu_grid_update_equals_full_batch():
    """data_parallel.update_grid on a batch split over two ranks leaves both
    replicas with the grids and coefficients of the whole-batch update on one
    GPU, bit for bit (the device update is deterministic)."""
    out = mp.get_context("spawn").Manager().dict()  # no fork after CUDA is up
    mp.spawn(_grid_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    full = out["full"]
    for rank in range(2):
        for name, want in full.items():
            assert torch.equal(out[rank][name], want), f"rank {rank} {name}"
