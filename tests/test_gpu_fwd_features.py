"""kf_fwd_emit_features: the forward that also writes the feature matrix for
the coefficient gradient.  Through the C ABI its output y must equal kf_fwd's
bit for bit, and its feature matrix kf_features' bit for bit (the same feature
rows, evaluated by the forward's producer warps); through the layer, the
gradients of a layer whose forward kept the matrix must equal those of one
whose backward made it."""

from __future__ import annotations

import ctypes

import pytest
import torch

import kanforge_b200 as kb
import kanforge_b200.kernels as kk

pytestmark = pytest.mark.gpu


def _layer(basis, n_in, n_out):
    torch.manual_seed(0)
    layer = kb.KANLinear(n_in, n_out, basis, device="cuda")
    with torch.no_grad():
        layer.coef.normal_(0, 0.05)
    return layer.to(torch.bfloat16)


@pytest.mark.parametrize("basis,n_in,n_out,batch", [
    (kb.Chebyshev(12), 256, 512, 777),   # a ragged last token tile, one 512-output tile
    (kb.Chebyshev(5), 100, 264, 300),    # tail K step (inputs not a multiple of 4)
    (kb.Fourier(6), 128, 1024, 513),     # two output tiles: only the first stores features
])
def test_emitted_features_equal_kf_features_and_y_equals_kf_fwd(basis, n_in, n_out, batch):
    layer = _layer(basis, n_in, n_out)
    plan = layer._plan
    has_base = layer.base_weight is not None
    nt, f_pad = kk.fused_layout(plan, has_base)
    x = (torch.randn(batch, n_in, device="cuda") * 1.5).to(torch.bfloat16)
    packed = kk.pack_coef(layer.coef, layer.base_weight, getattr(layer, "edge_scale", None), None, plan, f_pad)
    desc = plan.desc()
    s = kk._stream(x)
    b = kk._bf16_or_none(layer.bias)
    y0 = torch.empty(batch, n_out, device="cuda", dtype=torch.bfloat16)
    y1 = torch.empty_like(y0)
    f0 = torch.empty(batch, n_in * f_pad, device="cuda", dtype=torch.bfloat16)
    f1 = torch.full_like(f0, float("nan"))
    kk._launch("kf_fwd", kk._ptr(x), None, kk._ptr(packed), kk._ptr(b), None, kk._ptr(y0), batch, n_in, n_out, nt, f_pad,
               int(has_base), ctypes.byref(desc), s)
    kk._launch("kf_features", kk._ptr(x), None, kk._ptr(f0), batch, n_in, nt, f_pad, int(has_base), ctypes.byref(desc), s)
    for _ in range(2):  # a second call over the same buffers
        kk._launch("kf_fwd_emit_features", kk._ptr(x), kk._ptr(packed), kk._ptr(b), None, kk._ptr(y1), kk._ptr(f1), batch,
                   n_in, n_out, nt, f_pad, int(has_base), ctypes.byref(desc), s)
        torch.cuda.synchronize()
        assert torch.equal(y1, y0)
        assert torch.equal(f1.view(torch.int16), f0.view(torch.int16))


def test_layer_gradients_unchanged_by_kept_features(monkeypatch):
    layer = _layer(kb.Chebyshev(12), 512, 512)
    x = (torch.randn(1024, 512, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(1024, 512, device="cuda").to(torch.bfloat16)

    def grads():
        for p in layer.parameters():
            p.grad = None
        x.grad = None
        layer(x).backward(dy)
        torch.cuda.synchronize()
        return [x.grad.clone()] + [p.grad.clone() for p in layer.parameters() if p.grad is not None]

    kept = grads()
    monkeypatch.setattr(kk, "FORWARD_FEATURE_BYTES_MAX", 0)  # the backward makes the matrix instead
    made = grads()
    for a, b in zip(kept, made):
        assert torch.equal(a, b)


def test_emit_features_rejects_other_plans():
    layer = _layer(kb.BSpline(8, 3), 64, 64)
    plan = layer._plan
    nt, f_pad = kk.fused_layout(plan, True)
    x = torch.randn(32, 64, device="cuda").to(torch.bfloat16)
    y = torch.empty(32, 64, device="cuda", dtype=torch.bfloat16)
    feat = torch.empty(32, 64 * f_pad, device="cuda", dtype=torch.bfloat16)
    g = layer.basis_grid.detach().float().contiguous()
    tab = kk.knot_tables(g, plan)
    packed = kk.pack_coef(layer.coef, layer.base_weight, None, None, plan, f_pad)
    desc = plan.desc()
    with pytest.raises(RuntimeError, match="Chebyshev-feature or Fourier"):
        kk._launch("kf_fwd_emit_features", kk._ptr(x), kk._ptr(packed), None, kk._ptr(tab), kk._ptr(y), kk._ptr(feat), 32,
                   64, 64, nt, f_pad, 1, ctypes.byref(desc), kk._stream(x))
