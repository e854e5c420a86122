"""Sparse B-spline kernels (kf_sparse_fwd / dgrad / wgrad; the k+1-coefficient
gather of kanforge/bases/base.py:15-16) against the float64 oracle: float32
KANLinear layers whose outputs are few, forward and every gradient, tolerance
1e-5 (max|a-b| / max(1, max|b|)), plus BASELINE config 0 (KAN([2,5,1])) and
the dispatch rule."""

from __future__ import annotations

import contextlib

import numpy as np
import pytest
import torch
from test_gpu_parity import FP32_TOL, close, layer_numpy

import kan_oracle as ko
import kanforge_b200 as kb
from kanforge_b200 import kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"


@contextlib.contextmanager
def launches():
    names = []

    @contextlib.contextmanager
    def observe(name):
        names.append(name)
        yield

    K.set_launch_observer(observe)
    try:
        yield names
    finally:
        K.set_launch_observer(None)


CASES = [
    # (B, I, O, basis, base, edge_scale, x range)
    (1024, 2, 5, kb.BSpline(5, 3, (-2.0, 2.0)), True, False, 2.0),
    (1024, 5, 1, kb.BSpline(5, 3, (-2.0, 2.0)), True, False, 2.0),
    (4096, 64, 16, kb.BSpline(8, 3), True, True, 1.5),
    (3001, 37, 64, kb.BSpline(4, 1), False, True, 1.2),
    (777, 9, 33, kb.BSpline(6, 2), True, False, 1.3),
    (2048, 20, 7, kb.BSpline(3, 4), True, True, 1.4),
    (513, 130, 3, kb.BSpline(10, 5), True, False, 1.1),
    (70, 3, 201, kb.BSpline(5, 3), True, True, 1.3),  # O > 64 with O % 4 != 0: sparse by shape
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}x{c[1]}->{c[2]}_{c[3]!r}")
def test_sparse_layer_matches_oracle(case, monkeypatch):
    monkeypatch.setattr(K, "SPARSE_MAX_OUT", 1 << 30)  # every output tile width, whatever the dispatch threshold
    n_b, n_in, n_out, basis, base, scaled, rng_x = case
    torch.manual_seed(n_in * 7 + n_out)
    layer = kb.KANLinear(n_in, n_out, basis, edge_scale=scaled, base_activation=torch.nn.functional.silu if base else None,
                         device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.3)
        layer.bias.uniform_(-0.2, 0.2)
        layer.edge_mask[n_out // 2, n_in // 2] = 0
        if scaled:
            layer.edge_scale.uniform_(0.5, 1.5)
    if n_in >= 5:  # non-uniform per-input grids
        layer.update_grid(torch.randn(4000, n_in, device=DEV) * 0.5)
    x0 = (torch.rand(n_b, n_in, device=DEV) * 2 - 1) * rng_x
    x = x0.clone().requires_grad_()
    with launches() as names:
        y = layer(x)
        g = torch.randn_like(y)
        grads = torch.autograd.grad(y, [x] + [p for p in layer.parameters()], g)
    assert "kf_sparse_fwd" in names and "kf_sparse_dgrad" in names and "kf_sparse_wgrad" in names, names
    K.check_device_errors()
    n = layer_numpy(layer)
    xs, gs = x0.double().cpu().numpy(), g.double().cpu().numpy()
    close(y, ko.kan_linear(xs, n["coef"], n["base_weight"], n["bias"], n["spec"], n["params"], n["edge_scale"],
                           n["edge_mask"]), FP32_TOL, "y")
    want = ko.kan_linear_backward(xs, gs, n["coef"], n["base_weight"], n["bias"], n["spec"], n["params"], n["edge_scale"],
                                  n["edge_mask"])
    close(grads[0], want["dx"], FP32_TOL, "dx")
    names_p = [name for name, _ in layer.named_parameters()]
    for name, got in zip(names_p, grads[1:]):
        key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias", "edge_scale": "dedge_scale"}[name]
        close(got, want[key], FP32_TOL, name)


def test_sparse_gradients_are_deterministic():
    torch.manual_seed(0)
    layer = kb.KANLinear(48, 12, kb.BSpline(8, 3), edge_scale=True, device=DEV)
    x = torch.randn(20000, 48, device=DEV).requires_grad_()
    g = torch.randn(20000, 12, device=DEV)
    a = torch.autograd.grad(layer(x), [x, layer.coef, layer.base_weight, layer.edge_scale, layer.bias], g)
    b = torch.autograd.grad(layer(x), [x, layer.coef, layer.base_weight, layer.edge_scale, layer.bias], g)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_dispatch_wide_layers_stay_on_the_tensor_cores():
    layer = kb.KANLinear(64, 128, kb.BSpline(8, 3), device=DEV)
    with launches() as names:
        layer(torch.randn(256, 64, device=DEV))
    assert "kf_sparse_fwd" not in names and "kf_gemm_tf32x3" in names, names
    narrow = kb.KANLinear(64, K.SPARSE_MAX_OUT, kb.BSpline(8, 3), device=DEV)
    with launches() as names:
        narrow(torch.randn(256, 64, device=DEV))
    assert "kf_sparse_fwd" in names, names


def test_config0_training_step_matches_oracle():
    """KAN([2,5,1]) BSpline(5,3) on [-2,2], float32, batch 1024,
    MSE against exp(sin(pi x0) + x1^2): loss and every gradient."""
    torch.manual_seed(0)
    model = kb.KAN([2, 5, 1], kb.BSpline(5, 3, (-2.0, 2.0)), coef_init="lecun", device=DEV)
    x = torch.rand(1024, 2, device=DEV) * 4 - 2
    target = torch.exp(torch.sin(torch.pi * x[:, :1]) + x[:, 1:] ** 2)
    with launches() as names:
        loss = ((model(x) - target) ** 2).mean()
        loss.backward()
    assert names.count("kf_sparse_fwd") == 2, names
    # oracle: the two layers in float64 on the same parameters
    l0, l1 = (layer_numpy(m) for m in model)
    xs = x.double().cpu().numpy()
    h = ko.kan_linear(xs, l0["coef"], l0["base_weight"], l0["bias"], l0["spec"], l0["params"], None, l0["edge_mask"])
    y = ko.kan_linear(h, l1["coef"], l1["base_weight"], l1["bias"], l1["spec"], l1["params"], None, l1["edge_mask"])
    t = target.double().cpu().numpy()
    close(loss, np.mean((y - t) ** 2), FP32_TOL, "loss")
    dy = 2 * (y - t) / y.size
    g1 = ko.kan_linear_backward(h, dy, l1["coef"], l1["base_weight"], l1["bias"], l1["spec"], l1["params"], None,
                                l1["edge_mask"])
    g0 = ko.kan_linear_backward(xs, g1["dx"], l0["coef"], l0["base_weight"], l0["bias"], l0["spec"], l0["params"], None,
                                l0["edge_mask"])
    for m, gw in ((model[0], g0), (model[1], g1)):
        close(m.coef.grad, gw["dcoef"], FP32_TOL, "dcoef")
        close(m.base_weight.grad, gw["dbase_weight"], FP32_TOL, "dbase")
        close(m.bias.grad, gw["dbias"], FP32_TOL, "dbias")


def test_sparse_double_backward_matches_primitives():
    """create_graph=True: the input gradient is itself differentiable (PINN losses)."""
    torch.manual_seed(3)
    layer = kb.KANLinear(6, 4, kb.BSpline(5, 3), device=DEV)
    x = (torch.rand(300, 6, device=DEV) * 1.6 - 0.8).requires_grad_()
    (gx,) = torch.autograd.grad(layer(x).sum(), x, create_graph=True)
    (gxx,) = torch.autograd.grad(gx.sum(), x)
    n = layer_numpy(layer)
    xs = x.detach().double().cpu().numpy()
    ed1 = ko.edge_derivative(xs, n["coef"], n["base_weight"], n["spec"], n["params"], 1, None, n["edge_mask"])
    ed2 = ko.edge_derivative(xs, n["coef"], n["base_weight"], n["spec"], n["params"], 2, None, n["edge_mask"])
    close(gx, ed1.sum(-2), FP32_TOL, "dx")
    close(gxx, ed2.sum(-2), FP32_TOL, "d2x")


@pytest.mark.parametrize("grid_size,n_out", [(40, 64), (100, 24), (5, 5)])
def test_bf16_layers_outside_the_fused_kernels_run_sparse(grid_size, n_out):
    """bf16 B-spline layers with more than 31 features per input or an output
    count the fused kernels do not tile compute in float32 on the sparse
    kernels (tolerance: bf16, 2e-2, against the oracle on the bf16 values)."""
    torch.manual_seed(grid_size)
    layer = kb.KANLinear(12, n_out, kb.BSpline(grid_size, 3), device=DEV, dtype=torch.bfloat16)
    x = ((torch.rand(2000, 12, device=DEV) * 2.4 - 1.2).bfloat16()).requires_grad_()
    with launches() as names:
        y = layer(x)
        g = torch.randn_like(y)
        gx, gc = torch.autograd.grad(y, [x, layer.coef], g)
    assert "kf_sparse_fwd" in names and y.dtype == torch.bfloat16, names
    n = layer_numpy(layer)
    xs, gs = x.detach().double().cpu().numpy(), g.double().cpu().numpy()
    close(y, ko.kan_linear(xs, n["coef"], n["base_weight"], n["bias"], n["spec"], n["params"], None, n["edge_mask"]),
          2e-2, "y")
    want = ko.kan_linear_backward(xs, gs, n["coef"], n["base_weight"], n["bias"], n["spec"], n["params"], None,
                                  n["edge_mask"])
    close(gx, want["dx"], 2e-2, "dx")
    close(gc, want["dcoef"], 2e-2, "dcoef")
