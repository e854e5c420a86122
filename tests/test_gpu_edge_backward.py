"""Backward of KANLinear.edge_derivative (reference kanforge/torch/layers.py:206-226,
an autograd graph there): a loss on the edge derivatives of order m trains the
layer.  With L = sum g * d^m phi / dx^m, against the float64 oracle:
  dL/dx[b,i]       = sum_o g[b,o,i] (order m+1 edge derivative)[b,o,i]
  dL/dcoef[o,i,k]  = sum_b g[b,o,i] phi_k^(m)(x[b,i]) edge_scale[o,i] mask[o,i]
  dL/dbase[o,i]    = sum_b g[b,o,i] silu^(m)(x[b,i]) mask[o,i]
  dL/dscale[o,i]   = sum_b,k g[b,o,i] phi_k^(m)(x[b,i]) coef[o,i,k] mask[o,i]
float32 kernels, tolerance 1e-5 (max|a-b| / max(1, max|b|))."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from test_gpu_parity import FP32_TOL, close, layer_numpy

import kan_oracle as ko
import kanforge_b200 as kb

pytestmark = pytest.mark.gpu
DEV = "cuda"

BASES = [kb.Chebyshev(6), kb.Jacobi(6, 0.5, 0.5), kb.BSpline(8, 3), kb.Fourier(3), kb.RBF(6), kb.Chebyshev(20)]


@pytest.mark.parametrize("basis", BASES, ids=repr)
@pytest.mark.parametrize("order", [0, 1, 2])
@pytest.mark.parametrize("shape", [(64, 24, 301), (37, 5, 1000), (5, 7, 4097)], ids=str)
def test_edge_derivative_gradients_match_oracle(basis, order, shape):
    n_in, n_out, n_b = shape
    torch.manual_seed(order)
    layer = kb.KANLinear(n_in, n_out, basis, edge_scale=True, device=DEV)
    with torch.no_grad():
        layer.edge_scale.uniform_(0.5, 1.5)
        layer.edge_mask[n_out // 2, n_in // 2] = 0
        layer.coef.normal_(0, 0.3)
    x0 = torch.rand(n_b, n_in, device=DEV) * 2.4 - 1.2
    x = x0.clone().requires_grad_()
    d = layer.edge_derivative(x, order)
    g = torch.randn_like(d)
    grads = torch.autograd.grad(d, [x, layer.coef, layer.base_weight, layer.edge_scale], g)
    kb.kernels.check_device_errors()
    n = layer_numpy(layer)
    xs, gs = x0.double().cpu().numpy(), g.double().cpu().numpy()
    args = (n["coef"], n["base_weight"], n["spec"], n["params"])
    ed1 = ko.edge_derivative(xs, *args, order + 1, n["edge_scale"], n["edge_mask"])
    close(grads[0], np.einsum("boi,boi->bi", gs, ed1), FP32_TOL, "dx")
    phi = ko.basis_eval(n["spec"], xs, order, n["params"])  # (B, I, K)
    mask, scale = n["edge_mask"], n["edge_scale"]
    dce = np.einsum("boi,bik->oik", gs, phi)
    close(grads[1], dce * (scale * mask)[..., None], FP32_TOL, "dcoef")
    close(grads[2], np.einsum("boi,bi->oi", gs, ko.silu_derivative(xs, order)) * mask, FP32_TOL, "dbase")
    close(grads[3], (dce * n["coef"]).sum(-1) * mask, FP32_TOL, "dedge_scale")


def test_pinn_style_training_step_on_edge_derivatives():
    """A residual on the second edge derivatives backpropagates through the
    kernels into every parameter and the collocation points."""
    torch.manual_seed(0)
    layer = kb.KANLinear(16, 16, kb.Jacobi(6, 0.5, 0.5), device=DEV)
    x = (torch.rand(2048, 16, device=DEV) * 2 - 1).requires_grad_()
    loss = (layer.edge_derivative(x, 2) ** 2).mean()
    loss.backward()
    for p in [x, layer.coef, layer.base_weight]:
        assert p.grad is not None and torch.isfinite(p.grad).all() and p.grad.abs().sum() > 0
