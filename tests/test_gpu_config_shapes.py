"""Parity at the benchmark configurations' own shapes.

Each configuration the bench measures runs here at its full size, and its
results are checked two ways:

* against the float64 oracle on sampled rows, outputs and inputs (the oracle
  is too slow for the whole tensors): y and dx on sampled rows, the
  coefficient and base-weight gradients on sampled (output, input) blocks
  summed over EVERY row, so the contractions run at their full depth
  (K = I * F in the forward, O in the input gradient, the whole batch in the
  coefficient gradient);
* on the whole tensors against the float32 CUDA-core primitives (kf_prim),
  an independent float32 evaluation of the same sums.

Tolerances (metric max|a-b| / max(1, max|b|), reference tests/test_kernels.py:96-99):
bf16 2e-2 against the float64 oracle evaluated on the same bf16-valued inputs
and parameters; float32 1e-5 against the float64 oracle.  Two float32 results
that both round differ by more than either from float64, so the whole-tensor
float32 comparison allows 1e-4.

Configurations (synthetic, seeded; shapes and value distributions of the
bench's configurations):
  0  KAN([2, 5, 1]) B-spline(5, 3) on [-2, 2], float32, batch 1024, MSE loss
  1  KANLinear 1024 -> 1024 B-spline(8, 3) + SiLU, batch 65536, bf16 and float32
  2  KANLinear 4096 -> 4096 Chebyshev(12) + SiLU, bf16, 16384 tokens (the headline)
  3  KANFFN GR-KAN 768 -> 3072 -> 768, groups 8, bf16, 32 x 1024 tokens
  4  edge_derivative order 2, KANLinear 64 -> 64 Jacobi(6, 0.5, 0.5), float32,
     262144 points
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import kan_oracle as ko
import kanforge_b200 as kb

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16_TOL = 2e-2
FP32_TOL = 1e-5
FP32_PAIR_TOL = 1e-4


def np64(t):
    return t.detach().double().cpu().numpy()


def close(got, want, tol, what):
    got = np64(got) if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    want = np64(want) if isinstance(want, torch.Tensor) else np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    err = ko.max_rel_err(got, want)
    assert err <= tol, f"{what}: max rel err {err:.3e} > {tol:.0e}"


def spec_of(layer) -> dict:
    cfg = layer.basis.config()
    if cfg["name"] == "bspline":
        return {"kind": "bspline", "grid_size": cfg["grid_size"], "order": cfg["order"], "grid_range": cfg["grid_range"]}
    if cfg["name"] == "rational":
        return {"kind": "rational", "num_degree": cfg["num_degree"], "den_degree": cfg["den_degree"]}
    out = {"kind": "poly", "family": cfg["name"], "degree": cfg["degree"], "input_map": cfg["input_map"]}
    for k in ("alpha", "beta", "lam"):
        if k in cfg:
            out[k] = cfg[k]
    return out


def sample(n: int, k: int, gen: np.random.Generator) -> np.ndarray:
    """k sorted indices of range(n), always holding the first and the last."""
    pick = gen.choice(np.arange(1, n - 1), size=k - 2, replace=False)
    return np.sort(np.concatenate([[0, n - 1], pick]))


def sampled_oracle(layer, x, dy, rows, outs, ins):
    """The float64 oracle's y and dx on `rows`, and the coefficient and
    base-weight gradients of the (outs x ins) block summed over every row."""
    spec = spec_of(layer)
    grid = getattr(layer, "basis_grid", None)
    params = {} if grid is None else {"grid": np64(grid)}
    coef, mask = np64(layer.coef), np64(layer.edge_mask)
    base = None if layer.base_weight is None else np64(layer.base_weight)
    bias = None if layer.bias is None else np64(layer.bias)
    c, w = ko.effective(coef, base, None, mask)
    n_out, n_in, k = c.shape
    xr, dyr = np64(x[rows]), np64(dy[rows])
    phi = ko.basis_eval(spec, xr, 0, params)
    y = phi.reshape(len(rows), -1) @ c.reshape(n_out, -1).T
    h = (dyr @ c.reshape(n_out, -1)).reshape(len(rows), n_in, k)
    dx = (h * ko.basis_eval(spec, xr, 1, params)).sum(-1)
    if w is not None:
        y = y + ko.silu(xr) @ w.T
        dx = dx + (dyr @ w) * ko.silu_derivative(xr, 1)
    if bias is not None:
        y = y + bias
    # the coefficient gradient of the sampled block: a sum over every row
    xi = np64(x[:, ins])
    dyo = np64(dy[:, outs])
    sub = {} if grid is None else {"grid": params["grid"][ins]}
    phi_i = ko.basis_eval(spec, xi, 0, sub)  # (B, len(ins), K)
    dceff = (dyo.T @ phi_i.reshape(len(xi), -1)).reshape(len(outs), len(ins), k)
    msub = mask[np.ix_(outs, ins)]
    out = {"y": y[:, outs], "dx": dx, "dcoef": dceff * msub[..., None]}
    if w is not None:
        out["dbase_weight"] = (dyo.T @ ko.silu(xi)) * msub
    return out


def primitive_reference(layer, x, dy):
    """Whole-tensor y, dx, dcoef, dbase of the layer from the float32 CUDA-core
    primitives (kf_prim) and float32 torch products for the SiLU branch."""
    plan = layer._plan
    xf, dyf = x.detach().float(), dy.float()
    grid = getattr(layer, "basis_grid", None)
    g = xf.new_zeros(1) if grid is None else grid.detach().float()
    mask = layer.edge_mask.float()
    ce = layer.coef.detach().float() * mask[..., None]
    ones = torch.ones_like(xf)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            y = kb.kernels.prim_F(xf, ce, ones, g, plan, 0)
            dx = kb.kernels.prim_P(xf, dyf, ce, g, plan, 1)
            dcoef = kb.kernels.prim_G(xf, dyf, ones, g, plan, 0) * mask[..., None]
            out = {"y": y, "dx": dx, "dcoef": dcoef}
            if layer.base_weight is not None:
                be = layer.base_weight.detach().float() * mask
                s = torch.sigmoid(xf)
                out["y"] = y + torch.nn.functional.silu(xf) @ be.T
                out["dx"] = dx + (dyf @ be) * (s * (1 + xf * (1 - s)))
                out["dbase_weight"] = (dyf.T @ torch.nn.functional.silu(xf)) * mask
            if layer.bias is not None:
                out["y"] = out["y"] + layer.bias.detach().float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out


def run_layer(layer, x0, dy):
    x = x0.clone().requires_grad_()
    y = layer(x)
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + [p for _, p in layer.named_parameters()], dy)
    torch.cuda.synchronize()
    kb.kernels.check_device_errors()
    got = {"y": y.detach(), "dx": grads[0]}
    key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias"}
    for n, g in zip(names, grads[1:]):
        got[key[n]] = g
    return got


def check_layer(layer, x0, dy, tol, pair_tol, n_rows=12, n_outs=24, n_ins=24, seed=0):
    got = run_layer(layer, x0, dy)
    gen = np.random.default_rng(seed)
    rows = sample(x0.shape[0], n_rows, gen)
    outs = sample(layer.out_features, n_outs, gen)
    ins = sample(layer.in_features, n_ins, gen)
    want = sampled_oracle(layer, x0, dy, rows, outs, ins)
    close(got["y"][rows][:, outs], want["y"], tol, "y (oracle, sampled rows)")
    close(got["dx"][rows], want["dx"], tol, "dx (oracle, sampled rows)")
    close(got["dcoef"][outs][:, ins], want["dcoef"], tol, "dcoef (oracle, every row)")
    if "dbase_weight" in want:
        close(got["dbase_weight"][outs][:, ins], want["dbase_weight"], tol, "dbase (oracle, every row)")
    if layer.bias is not None:
        close(got["dbias"], np64(dy).sum(0), tol, "dbias")
    ref = primitive_reference(layer, x0, dy)
    for k in ("y", "dx", "dcoef", "dbase_weight"):
        if k in ref:
            close(got[k].float(), ref[k], pair_tol, f"{k} (float32 primitives, whole tensor)")


# --- configurations 1 and 2: one KANLinear, forward + backward ------------------


def config_layer(cfg: int, dtype):
    torch.manual_seed(0)
    if cfg == 1:
        n, basis, std = 1024, kb.BSpline(8, 3), 0.1 / np.sqrt(1024 * 11)
    else:
        n, basis, std = 4096, kb.Chebyshev(12), 1.0 / np.sqrt(4096 * 13)
    layer = kb.KANLinear(n, n, basis, device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, std)
        layer.bias.normal_(0, 0.1)
        layer.edge_mask[3, 5] = 0  # one pruned edge
    return layer.to(dtype)


def config_inputs(cfg: int, n_b: int, n_in: int, n_out: int, dtype):
    g = torch.Generator(device=DEV).manual_seed(cfg)
    x = torch.randn(n_b, n_in, device=DEV, generator=g)
    if cfg == 1:
        x = x.clamp(-3, 3)
    dy = torch.randn(n_b, n_out, device=DEV, generator=g) * 0.5
    return x.to(dtype), dy.to(dtype)


def test_config2_headline_chebyshev12_4096_bf16_16384_tokens():
    layer = config_layer(2, torch.bfloat16)
    x0, dy = config_inputs(2, 16384, 4096, 4096, torch.bfloat16)
    assert kb.kernels.fused_ok(layer._plan, x0, 4096, True, layer.coef.dtype)
    check_layer(layer, x0, dy, BF16_TOL, BF16_TOL)


def test_config1_bspline8_1024_bf16_65536_tokens():
    layer = config_layer(1, torch.bfloat16)
    x0, dy = config_inputs(1, 65536, 1024, 1024, torch.bfloat16)
    assert kb.kernels.fused_ok(layer._plan, x0, 1024, True, layer.coef.dtype)
    check_layer(layer, x0, dy, BF16_TOL, BF16_TOL)


def test_config1_bspline8_1024_float32_65536_tokens():
    """The float32 tensor-core path (three TF32 products): the coefficient
    gradient accumulates over all 65536 tokens."""
    layer = config_layer(1, torch.float32)
    x0, dy = config_inputs(1, 65536, 1024, 1024, torch.float32)
    assert kb.kernels.tf32_ok(layer._plan, x0, 1024, True, layer.coef.dtype)
    check_layer(layer, x0, dy, FP32_TOL, FP32_PAIR_TOL)


# --- configuration 0: KAN([2, 5, 1]) regression step ----------------------------


def test_config0_kan_2_5_1_bspline_float32_mse_step():
    torch.manual_seed(0)
    model = kb.KAN([2, 5, 1], kb.BSpline(5, 3, (-2.0, 2.0)), coef_init="lecun").to(DEV)
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.rand(1024, 2, device=DEV, generator=g) * 4 - 2
    target = torch.exp(torch.sin(torch.pi * x[:, :1]) + x[:, 1:] ** 2)
    xg = x.clone().requires_grad_()
    y = model(xg)
    loss = ((y - target) ** 2).mean()
    params = list(model.parameters())
    grads = torch.autograd.grad(loss, [xg] + params)

    l1, l2 = model[0], model[1]
    n1 = dict(coef=np64(l1.coef), base_weight=np64(l1.base_weight), bias=np64(l1.bias), spec=spec_of(l1),
              params={"grid": np64(l1.basis_grid)}, edge_mask=np64(l1.edge_mask))
    n2 = dict(coef=np64(l2.coef), base_weight=np64(l2.base_weight), bias=np64(l2.bias), spec=spec_of(l2),
              params={"grid": np64(l2.basis_grid)}, edge_mask=np64(l2.edge_mask))
    xs, ts = np64(x), np64(target)
    h = ko.kan_linear(xs, **n1)
    yy = ko.kan_linear(h, **n2)
    close(y, yy, FP32_TOL, "y")
    dyy = 2 * (yy - ts) / yy.size
    b2 = ko.kan_linear_backward(h, dyy, **n2)
    b1 = ko.kan_linear_backward(xs, b2["dx"], **n1)
    close(grads[0], b1["dx"], FP32_TOL, "dx")
    want = [b1["dcoef"], b1["dbase_weight"], b1["dbias"], b2["dcoef"], b2["dbase_weight"], b2["dbias"]]
    names = [n for n, _ in model.named_parameters()]
    assert names == ["0.coef", "0.base_weight", "0.bias", "1.coef", "1.base_weight", "1.bias"]
    for n, gr, w in zip(names, grads[1:], want):
        close(gr, w, FP32_TOL, f"d{n}")


# --- configuration 3: the GR-KAN FFN --------------------------------------------


def rational64(x, num, den):
    """P(x) / (1 + |Q(x)|) in float64 torch, per-group parameters repeated over
    the inputs (num (I, p+1), den (I, q)); autograd gives d/dx and d/dparams
    (sign(0) = 0 through |.|)."""
    p = torch.zeros_like(x)
    for j in range(num.shape[1] - 1, -1, -1):
        p = p * x + num[:, j]
    q = torch.zeros_like(x)
    for j in range(den.shape[1] - 1, -1, -1):
        q = (q + den[:, j]) * x
    return p / (1 + q.abs())


def grkan_reference64(layer, x, dy):
    """Float64 torch reference of one GR-KAN layer on the bf16-valued input x
    (B, I) and upstream gradient dy (B, O): its output, the input gradient and
    the gradients of coef, bias and the per-group rational parameters."""
    ipg = layer.in_features // layer.groups
    leaves = {n: p.detach().double().requires_grad_() for n, p in layer.named_parameters()}
    xr = x.detach().double().requires_grad_()
    r = rational64(xr, leaves["basis_numerator"].repeat_interleave(ipg, 0),
                   leaves["basis_denominator"].repeat_interleave(ipg, 0))
    y = r @ leaves["coef"][..., 0].T + leaves["bias"]
    grads = torch.autograd.grad(y, [xr] + list(leaves.values()), dy.double())
    return y.detach(), grads[0], dict(zip(leaves, grads[1:]))


def test_config3_grkan_ffn_768_3072_bf16_32k_tokens():
    """Each layer against a float64 reference evaluated on the same bf16
    activations and upstream gradients the bf16 path produced: the rational's
    |Q| has kinks (sign(Q) flips where Q = 0, e.g. near h = 4.44 for the GELU
    fit), so rounding the hidden activation to bf16 before comparing is part
    of the computation, not an error of the kernels."""
    torch.manual_seed(0)
    ffn = kb.KANFFN(768, 3072, kind="grkan", groups=8).to(device=DEV, dtype=torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(3)
    x0 = torch.randn(32768, 768, device=DEV, generator=g).to(torch.bfloat16)
    dy = torch.randn(32768, 768, device=DEV, generator=g).to(torch.bfloat16)
    x = x0.clone().requires_grad_()
    h = ffn.fc1(x)
    h.retain_grad()
    y = ffn.fc2(h)
    y.backward(dy)
    torch.cuda.synchronize()
    kb.kernels.check_device_errors()

    for layer, inp, out, up, dinp in ((ffn.fc2, h, y, dy, h.grad), (ffn.fc1, x0, h, h.grad, x.grad)):
        y_ref, dx_ref, g_ref = grkan_reference64(layer, inp, up)
        close(out, y_ref, BF16_TOL, f"{layer.in_features}->{layer.out_features} y")
        close(dinp, dx_ref, BF16_TOL, f"{layer.in_features}->{layer.out_features} dx")
        for n, p in layer.named_parameters():
            # rational parameter gradients are sums over 32768 x 96 or x 384 inputs
            tol = 5e-2 if n.startswith("basis_") else BF16_TOL
            close(p.grad, g_ref[n], tol, f"{layer.in_features}->{layer.out_features} d{n}")

    # the float64 torch reference itself against the oracle on sampled rows
    gen = np.random.default_rng(3)
    rows = sample(32768, 8, gen)
    n1, ipg1 = ffn.fc1, 768 // 8
    p1 = {"numerator": np.repeat(np64(n1.basis_numerator), ipg1, 0),
          "denominator": np.repeat(np64(n1.basis_denominator), ipg1, 0)}
    h_ref, _, _ = grkan_reference64(n1, x0[rows], torch.zeros(len(rows), 3072, device=DEV))
    h_or = ko.kan_linear(np64(x0[rows]), np64(n1.coef), None, np64(n1.bias), spec_of(n1), p1, None, np64(n1.edge_mask))
    close(h_ref, h_or, 1e-10, "float64 torch reference vs oracle (fc1)")


# --- configuration 4: edge_derivative ---------------------------------------------


def test_config4_edge_derivative_order2_jacobi6_262144_points():
    torch.manual_seed(0)
    layer = kb.KANLinear(64, 64, kb.Jacobi(6, 0.5, 0.5), device=DEV)
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.rand(262144, 64, device=DEV, generator=g) * 2 - 1
    with torch.no_grad():
        d = layer.edge_derivative(x, 2)
    torch.cuda.synchronize()
    kb.kernels.check_device_errors()
    assert d.shape == (262144, 64, 64) and d.dtype == torch.float32
    gen = np.random.default_rng(4)
    rows = np.sort(np.concatenate([sample(262144, 64, gen), np.arange(262144 - 40, 262144 - 2)]))
    n = dict(coef=np64(layer.coef), base_weight=np64(layer.base_weight), spec=spec_of(layer), params={},
             edge_mask=np64(layer.edge_mask))
    want = ko.edge_derivative(np64(x[rows]), order=2, **n)
    close(d[rows], want, FP32_TOL, "edge_derivative (sampled rows)")
    assert torch.isfinite(d).all()
