"""KAN convolutions on the implicit patch matrix (reference kanforge/torch/conv.py).

The bf16 tensor-core path gathers every receptive field from the image inside
the kernels (kf_conv_fwd / kf_conv_features / kf_conv_dgrad / kf_conv_wgrad)
and folds the patch-matrix gradient back onto the image (kf_conv_fold); other
layers materialise the patch matrix with kf_conv_patches.  Checked against the
float64 oracle applied to patches built in the test with numpy, and the two
paths against each other (the same arithmetic on the same values, so the
same bits).  Tolerances (max|a-b| / max(1, max|b|)): bf16 2e-2, float32 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from test_gpu_parity import BF16_TOL, FP32_TOL, close, layer_numpy

import kan_oracle as ko
import kanforge_b200 as kb
from kanforge_b200 import conv as kconv

pytestmark = pytest.mark.gpu
DEV = "cuda"


def numpy_patches(x, kernel, stride, padding, dilation, c0, cg):
    """(N * prod(out), cg * prod(kernel)) receptive fields of x (N, C, *L) in
    float64, zero padding, columns ordered (channel, kernel offsets)."""
    x = np.asarray(x, np.float64)
    n = x.ndim - 2
    xp = np.pad(x, [(0, 0), (0, 0)] + [(p, p) for p in padding])
    out = [(x.shape[2 + d] + 2 * padding[d] - dilation[d] * (kernel[d] - 1) - 1) // stride[d] + 1 for d in range(n)]
    rows = []
    for idx in np.ndindex(x.shape[0], *out):
        b, o = idx[0], idx[1:]
        sl = [b, slice(c0, c0 + cg)] + [slice(o[d] * stride[d], o[d] * stride[d] + dilation[d] * (kernel[d] - 1) + 1,
                                              dilation[d]) for d in range(n)]
        rows.append(xp[tuple(sl)].reshape(-1))
    return np.stack(rows), out


def oracle_conv(layer, x, dy):
    """Oracle forward and gradients of a KAN convolution (zero padding)."""
    n = layer.n_dims
    cg, og = layer.in_channels // layer.groups, layer.out_channels // layer.groups
    ys, dxs, grads = [], np.zeros(x.shape), []
    for g, kan in enumerate(layer.kans):
        p, out = numpy_patches(x, layer.kernel_size, layer.stride, layer.padding, layer.dilation, g * cg, cg)
        k = layer_numpy(kan)
        kw = dict(coef=k["coef"], base_weight=k["base_weight"], bias=k["bias"], spec=k["spec"], params=k["params"],
                  edge_scale=k["edge_scale"], edge_mask=k["edge_mask"])
        ys.append(ko.kan_linear(p, **kw))
        dyg = np.moveaxis(dy[:, g * og:(g + 1) * og], 1, -1).reshape(-1, og)
        back = ko.kan_linear_backward(p, dyg, **kw)
        grads.append(back)
        # fold the patch gradient onto the image
        dp = back["dx"]
        xp = np.zeros((x.shape[0], x.shape[1]) + tuple(x.shape[2 + d] + 2 * layer.padding[d] for d in range(n)))
        for r, idx in enumerate(np.ndindex(x.shape[0], *out)):
            b, o = idx[0], idx[1:]
            sl = [b, slice(g * cg, (g + 1) * cg)] + [slice(o[d] * layer.stride[d],
                                                          o[d] * layer.stride[d] + layer.dilation[d] * (layer.kernel_size[d] - 1) + 1,
                                                          layer.dilation[d]) for d in range(n)]
            xp[tuple(sl)] += dp[r].reshape(xp[tuple(sl)].shape)
        crop = (slice(None), slice(None)) + tuple(slice(layer.padding[d], layer.padding[d] + x.shape[2 + d]) for d in range(n))
        dxs = dxs + xp[crop]
    y = np.concatenate(ys, -1).reshape(x.shape[0], *out, layer.out_channels)
    return np.moveaxis(y, -1, 1), dxs, grads


def make_conv(cls, cin, cout, k, basis, dtype, seed=0, **kw):
    torch.manual_seed(seed)
    layer = cls(cin, cout, k, basis=basis, **kw)
    with torch.no_grad():
        for kan in layer.kans:
            kan.coef.normal_(0, 0.3)
            kan.bias.normal_(0, 0.1)
            kan.edge_mask[0, -1] = 0
    return layer.to(device=DEV, dtype=dtype)


CONV_CASES = [
    # cls, C_in, C_out, kernel, kwargs, input spatial size, batch
    (kb.KANConv2d, 3, 8, 3, dict(padding=1), (9, 7), 2),
    (kb.KANConv2d, 4, 16, (3, 2), dict(stride=(2, 1), padding=(1, 0), dilation=(1, 2), groups=2), (11, 8), 3),
    (kb.KANConv2d, 8, 8, 1, dict(), (5, 5), 4),
    (kb.KANConv1d, 5, 24, 5, dict(padding=2, stride=2), (33,), 3),
    (kb.KANConv3d, 2, 8, 3, dict(padding=1), (4, 5, 3), 2),
]


@pytest.mark.parametrize("basis", [kb.Chebyshev(6), kb.BSpline(5, 3, (-1.5, 1.5))], ids=repr)
@pytest.mark.parametrize("case", range(len(CONV_CASES)))
def test_bf16_implicit_conv_matches_oracle(case, basis):
    cls, cin, cout, k, kw, size, nb = CONV_CASES[case]
    layer = make_conv(cls, cin, cout, k, basis, torch.bfloat16, **kw)
    x0 = (torch.rand(nb, cin, *size, device=DEV) * 3 - 1.5).to(torch.bfloat16)
    assert all(layer._implicit(kan, x0) for kan in layer.kans)
    x = x0.clone().requires_grad_()
    y = layer(x)
    dy = torch.randn_like(y)
    params = [p for _, p in layer.named_parameters()]
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + params, dy)
    kb.kernels.check_device_errors()
    want_y, want_dx, want_g = oracle_conv(layer, x0.double().cpu().numpy(), dy.double().cpu().numpy())
    close(y, want_y, BF16_TOL, "y")
    close(grads[0], want_dx, BF16_TOL, "dx")
    key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias"}
    for nme, gr in zip(names, grads[1:]):
        g, leaf = int(nme.split(".")[1]), nme.split(".")[2]
        close(gr, want_g[g][key[leaf]], BF16_TOL, nme)


@pytest.mark.parametrize("basis", [kb.Chebyshev(6), kb.BSpline(5, 3)], ids=repr)
def test_implicit_conv_equals_explicit_patch_path(basis, monkeypatch):
    """The kernels' gather and the materialised patch matrix give the same bits."""
    layer = make_conv(kb.KANConv2d, 4, 16, 3, basis, torch.bfloat16, seed=2, padding=1, stride=2, groups=2)
    x = (torch.rand(3, 4, 13, 10, device=DEV) * 3 - 1.5).to(torch.bfloat16).requires_grad_()
    dy = None
    params = [p for _, p in layer.named_parameters()]

    def run():
        y = layer(x)
        nonlocal dy
        if dy is None:
            dy = torch.randn(y.shape, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV).to(y.dtype)
        return (y.detach(),) + torch.autograd.grad(y, [x] + params, dy)

    implicit = run()
    monkeypatch.setattr(kconv._KANConvNd, "_implicit", lambda self, kan, x: False)
    explicit = run()
    for a, b in zip(implicit, explicit):
        assert torch.equal(a, b)


@pytest.mark.parametrize("case", [0, 1, 3, 4])
def test_float32_conv_patch_path_matches_oracle(case):
    cls, cin, cout, k, kw, size, nb = CONV_CASES[case]
    layer = make_conv(cls, cin, cout, k, kb.BSpline(5, 3), torch.float32, **kw)
    x0 = torch.rand(nb, cin, *size, device=DEV) * 2.4 - 1.2
    x = x0.clone().requires_grad_()
    y = layer(x)
    dy = torch.randn_like(y)
    grads = torch.autograd.grad(y, [x, layer.kans[0].coef], dy)
    want_y, want_dx, want_g = oracle_conv(layer, x0.double().cpu().numpy(), dy.double().cpu().numpy())
    close(y, want_y, FP32_TOL, "y")
    close(grads[0], want_dx, FP32_TOL, "dx")
    close(grads[1], want_g[0]["dcoef"], FP32_TOL, "dcoef")


@pytest.mark.parametrize("mode", ["reflect", "replicate", "circular"])
def test_conv_padding_modes_match_torch_padding(mode):
    """Non-zero padding modes pad the image (F.pad) and convolve without padding."""
    layer = make_conv(kb.KANConv2d, 3, 4, 3, kb.Chebyshev(5), torch.float32, padding=2, padding_mode=mode)
    x = torch.rand(2, 3, 8, 9, device=DEV) * 2 - 1
    with torch.no_grad():
        y = layer(x)
        ref_layer = make_conv(kb.KANConv2d, 3, 4, 3, kb.Chebyshev(5), torch.float32, padding=0)
        ref_layer.load_state_dict(layer.state_dict())
        want = ref_layer(torch.nn.functional.pad(x, [2, 2, 2, 2], mode=mode))
    close(y, want.double().cpu().numpy(), 1e-6, mode)


def test_from_conv_reproduces_the_convolution():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(4, 6, 3, stride=2, padding=1, groups=2).to(DEV)
    layer = kb.KANConv2d.from_conv(conv, basis=kb.Chebyshev(4))
    x = torch.randn(2, 4, 9, 10, device=DEV)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        with torch.no_grad():
            want = conv(x)
            got = layer(x)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    close(got, want.double().cpu().numpy(), FP32_TOL, "from_conv")
