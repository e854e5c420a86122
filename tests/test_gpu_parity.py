"""Parity of the sm_100a kernels with the oracle and the reference's golden vectors.

Tolerances (metric max|a-b| / max(1, max|b|), reference tests/test_kernels.py:96-99):
  float32 kernels vs float64 oracle ........ 1e-5 (layer values and gradients)
  float32 primitives vs reference Triton ... 2e-5 (both float32)
  bf16 fused tensor-core path .............. 2e-2, against the float64 oracle evaluated
                                             on the same bf16-valued inputs and parameters
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from conftest import load_golden, params_of, spec_of

import kan_oracle as ko
import kanforge_b200 as kb

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 2e-2
DEV = "cuda"


def close(got, want, tol, what=""):
    got = got.detach().double().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    err = ko.max_rel_err(got, want)
    assert got.shape == np.shape(want), (what, got.shape, np.shape(want))
    assert err <= tol, f"{what}: max rel err {err:.3e} > {tol:.0e}"


def spec_of_basis(basis) -> dict:
    cfg = basis.config()
    if cfg["name"] == "bspline":
        return {"kind": "bspline", "grid_size": cfg["grid_size"], "order": cfg["order"], "grid_range": cfg["grid_range"]}
    if cfg["name"] == "rational":
        return {"kind": "rational", "num_degree": cfg["num_degree"], "den_degree": cfg["den_degree"]}
    if cfg["name"] == "fourier":
        return {"kind": "fourier", "frequencies": cfg["frequencies"], "period": cfg["period"]}
    if cfg["name"] in ("rbf", "mexican_hat", "dog", "rswaf"):
        return {"kind": "bump", "family": cfg["name"], "count": cfg["count"], "grid_range": cfg["grid_range"]}
    out = {"kind": "poly", "family": cfg["name"], "degree": cfg["degree"], "input_map": cfg["input_map"]}
    for k in ("alpha", "beta", "lam"):
        if k in cfg:
            out[k] = cfg[k]
    return out


def layer_numpy(layer) -> dict:
    n_in = layer.in_features
    params = {}
    for k, v in layer.basis_params().items():
        v = v.detach().double().cpu().numpy()
        params[k] = v if v.shape[0] == n_in else np.repeat(v, n_in // v.shape[0], axis=0)
    g = lambda t: None if t is None else t.detach().double().cpu().numpy()  # noqa: E731
    return dict(coef=g(layer.coef), base_weight=g(layer.base_weight), bias=g(layer.bias), spec=spec_of_basis(layer.basis),
                params=params, edge_scale=g(layer.edge_scale), edge_mask=g(layer.edge_mask))


# ---------------------------------------------------------------------------
# primitives F/G/P vs the reference's own Triton kernels and the oracle
# ---------------------------------------------------------------------------

PRIMS = load_golden("prims.npz")
PRIM_BASES = {"bspline_5_3": kb.BSpline(5, 3), "chebyshev_5": kb.Chebyshev(5), "jacobi_4": kb.Jacobi(4, 0.5, 1.5),
              "fourier_3": kb.Fourier(3), "rbf_6": kb.RBF(6), "dog_5": kb.DoG(5, learnable=False), "rswaf_6": kb.RSWAF(6)}


@pytest.mark.parametrize("case", sorted(PRIM_BASES))
@pytest.mark.parametrize("m", [0, 1, 2])
def test_primitives_match_reference_triton(case, m):
    plan = kb.plan_for(PRIM_BASES[case])
    t = {k.split("/", 1)[1]: torch.as_tensor(v, device=DEV) for k, v in PRIMS.items() if k.startswith(case + "/")}
    with torch.no_grad():
        f = kb.kernels.prim_F(t["x"], t["c"], t["w"], t["grid"], plan, m)
        g = kb.kernels.prim_G(t["x"], t["g"], t["w"], t["grid"], plan, m)
        p = kb.kernels.prim_P(t["x"], t["g"], t["c"], t["grid"], plan, m)
    for got, key in [(f, "F"), (g, "G"), (p, "P")]:
        close(got, PRIMS[f"{case}/{key}{m}"], 2e-5, f"{case} {key}{m}")


PRIM_SWEEP = [
    (kb.BSpline(8, 3), 300, 37, 70),
    (kb.BSpline(4, 1), 65, 5, 3),
    (kb.BSpline(3, 2), 129, 9, 65),
    (kb.BSpline(6, 5), 40, 6, 9),
    (kb.Chebyshev(12), 200, 33, 66),
    (kb.Chebyshev(4, input_map="identity"), 17, 3, 2),
    (kb.Jacobi(6, 0.5, 0.5), 99, 12, 31),
    (kb.Fourier(5, 3.0), 150, 11, 20),
    (kb.RBF(8), 100, 9, 17),
    (kb.MexicanHat(6, learnable=False), 77, 5, 9),
    (kb.DoG(5, (-2.0, 2.0), learnable=False), 64, 7, 5),
    (kb.RSWAF(7), 64, 10, 12),
]


@pytest.mark.parametrize("basis,n_b,n_in,n_out", PRIM_SWEEP, ids=lambda v: repr(v) if isinstance(v, kb.Basis) else str(v))
@pytest.mark.parametrize("m", [0, 1, 2, 3])
def test_primitives_match_oracle_ragged_shapes(basis, n_b, n_in, n_out, m):
    plan = kb.plan_for(basis)
    spec = spec_of_basis(basis)
    rng = np.random.default_rng(7 + m)
    lo, hi = spec.get("grid_range", (-1.0, 1.0))
    x = rng.uniform(1.3 * lo - 0.2, 1.3 * hi + 0.2, (n_b, n_in))
    w = rng.uniform(0.5, 1.5, (n_b, n_in))
    g = rng.standard_normal((n_b, n_out))
    c = rng.standard_normal((n_out, n_in, basis.size)) * 0.3
    params = None
    grid = np.zeros(1)
    if spec["kind"] in ("bspline", "bump"):  # non-uniform per-input grids / centres
        grid = ko.default_grid(spec, n_in)
        grid[:, 1:-1] += rng.uniform(-0.2, 0.2, (n_in, grid.shape[1] - 2)) * (grid[0, 1] - grid[0, 0])
        params = {"grid": grid}
    T = lambda a: torch.as_tensor(a, dtype=torch.float32, device=DEV)  # noqa: E731
    x32 = x.astype(np.float32).astype(np.float64)
    grid32 = grid.astype(np.float32).astype(np.float64)
    p64 = None if params is None else {"grid": grid32}
    with torch.no_grad():
        f = kb.kernels.prim_F(T(x), T(c), T(w), T(grid), plan, m)
        gg = kb.kernels.prim_G(T(x), T(g), T(w), T(grid), plan, m)
        p = kb.kernels.prim_P(T(x), T(g), T(c), T(grid), plan, m)
    close(f, ko.prim_F(x32, c, w, spec, m, p64), 5e-5, "F")
    close(gg, ko.prim_G(x32, g, w, spec, m, p64), 5e-5, "G")
    close(p, ko.prim_P(x32, g, c, spec, m, p64), 5e-5, "P")


# ---------------------------------------------------------------------------
# float32 layers: forward, all gradients, edge_derivative vs golden + oracle
# ---------------------------------------------------------------------------

LAYERS = load_golden("layers.npz")
LAYER_BASES = {
    "bspline_5_3": (kb.BSpline(5, 3), {}),
    "bspline_8_3": (kb.BSpline(8, 3), {}),
    "chebyshev_12": (kb.Chebyshev(12), {}),
    "jacobi_6": (kb.Jacobi(6, 0.5, 0.5), {}),
    "chebyshev_4_id_nobase": (kb.Chebyshev(4, input_map="identity"), {"base_activation": None}),
    "rational_gelu_g2": (kb.Rational(5, 4, "gelu"), {"base_activation": None, "groups": 2}),
    "rational_identity_g1": (kb.Rational(5, 4, "identity"), {"base_activation": None, "groups": 1}),
    "fourier_3": (kb.Fourier(3), {}),
    "rbf_6": (kb.RBF(6), {}),
    "mexican_hat_5": (kb.MexicanHat(5, learnable=False), {"base_activation": None}),
    "rswaf_6": (kb.RSWAF(6), {}),
}


def golden_layer(case, dtype=torch.float32):
    pre = f"{case}/state/"
    state = {k[len(pre):]: v for k, v in LAYERS.items() if k.startswith(pre)}
    basis, kw = LAYER_BASES[case]
    n_out, n_in = state["coef"].shape[:2]
    layer = kb.KANLinear(n_in, n_out, basis, edge_scale="edge_scale" in state, **kw)
    layer.load_state_dict({k: torch.as_tensor(v) for k, v in state.items()})
    return layer.to(device=DEV, dtype=dtype)


@pytest.mark.parametrize("case", sorted(LAYER_BASES))
def test_float32_layer_matches_reference_values_and_gradients(case):
    layer = golden_layer(case)
    x = torch.as_tensor(LAYERS[f"{case}/x"], dtype=torch.float32, device=DEV).requires_grad_()
    y = layer(x)
    close(y, LAYERS[f"{case}/y"], FP32_TOL, "y")
    dy = torch.as_tensor(LAYERS[f"{case}/dy"], dtype=torch.float32, device=DEV)
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad((y * dy).sum(), [x] + [p for _, p in layer.named_parameters()])
    close(grads[0], LAYERS[f"{case}/grad/x"], FP32_TOL, "dx")
    for n, gr in zip(names, grads[1:]):
        close(gr, LAYERS[f"{case}/grad/{n}"], FP32_TOL, f"d{n}")


@pytest.mark.parametrize("case", sorted(LAYER_BASES))
@pytest.mark.parametrize("order", [0, 1, 2])
def test_edge_derivative_matches_reference(case, order):
    layer = golden_layer(case)
    x = torch.as_tensor(LAYERS[f"{case}/x"], dtype=torch.float32, device=DEV)
    with torch.no_grad():
        d = layer.edge_derivative(x, order)
    close(d, LAYERS[f"{case}/edge{order}"], FP32_TOL, f"edge{order}")


# (n_in, n_out, batch): even I (two inputs per lane: one or several 64-input
# chunks, I < 64 with several outputs per warp) and odd I (one input per lane:
# partial 32-input chunks, I < 32), outputs idle when O is small, ragged row groups.
EDGE_SHAPES = [(64, 24, 301), (37, 3, 133), (5, 7, 1000), (2, 1, 4096), (130, 9, 50), (24, 40, 99), (66, 5, 17)]


@pytest.mark.parametrize("basis", [kb.Jacobi(6, 0.5, 0.5), kb.BSpline(8, 3), kb.Chebyshev(5), kb.Fourier(4), kb.RBF(6), kb.RSWAF(5)], ids=repr)
@pytest.mark.parametrize("order", [0, 2, 3])
@pytest.mark.parametrize("shape", EDGE_SHAPES, ids=str)
def test_edge_derivative_streaming_kernel_matches_oracle(basis, order, shape):
    n_in, n_out, n_b = shape
    torch.manual_seed(0)
    layer = kb.KANLinear(n_in, n_out, basis, edge_scale=True, device=DEV)
    with torch.no_grad():
        layer.edge_scale.uniform_(0.5, 1.5)
        layer.edge_mask[n_out // 2, n_in // 2] = 0
        layer.coef.normal_(0, 0.3)
    x = torch.rand(n_b, n_in, device=DEV) * 2.4 - 1.2
    with torch.no_grad():
        d = layer.edge_derivative(x, order)
    n = layer_numpy(layer)
    want = ko.edge_derivative(x.double().cpu().numpy(), n["coef"], n["base_weight"], n["spec"], n["params"], order,
                              n["edge_scale"], n["edge_mask"])
    close(d, want, FP32_TOL, "edge")


@pytest.mark.parametrize("order", [0, 2])
def test_edge_derivative_many_features_scalar_kernel(order):
    """More than 16 features per input takes the one-thread-per-(b, i) kernel."""
    torch.manual_seed(0)
    layer = kb.KANLinear(33, 6, kb.BSpline(20, 3), device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.3)
    x = torch.rand(77, 33, device=DEV) * 1.8 - 0.9
    with torch.no_grad():
        d = layer.edge_derivative(x, order)
    n = layer_numpy(layer)
    want = ko.edge_derivative(x.double().cpu().numpy(), n["coef"], n["base_weight"], n["spec"], n["params"], order,
                              n["edge_scale"], n["edge_mask"])
    close(d, want, FP32_TOL, "edge")


@pytest.mark.parametrize("n_out", [5, 8])
def test_higher_order_input_derivatives_and_gradient_penalty(n_out):
    """Closure of F/G/P: 1st-3rd input derivatives and the double backward into
    coef (reference tests/test_kernels.py:102-121), against the oracle.  With
    8 outputs the float32 forward runs on the tensor cores and the
    differentiable backward on the primitives."""
    torch.manual_seed(0)
    for basis in (kb.BSpline(5, 3), kb.Chebyshev(5), kb.Jacobi(4, 0.5, 1.5)):
        layer = kb.KANLinear(4, n_out, basis, edge_scale=True, device=DEV)
        with torch.no_grad():
            layer.coef.normal_(0, 0.5)
            layer.edge_scale.uniform_(0.5, 1.5)
            layer.bias.normal_()
        x0 = torch.rand(37, 4, device=DEV) * 1.8 - 0.9
        wts = torch.linspace(-1, 1, n_out, device=DEV)
        x = x0.clone().requires_grad_()
        y = layer(x)
        loss = (y * wts).sum()
        (gx,) = torch.autograd.grad(loss, x, create_graph=True)
        (gxx,) = torch.autograd.grad(gx.sum(), x, create_graph=True)
        (gxxx,) = torch.autograd.grad(gxx.sum(), x, create_graph=True)
        (gc,) = torch.autograd.grad((gx**2).sum(), layer.coef)
        n = layer_numpy(layer)
        xs = x0.double().cpu().numpy()
        w = wts.double().cpu().numpy()
        eds = [ko.edge_derivative(xs, n["coef"], n["base_weight"], n["spec"], n["params"], m, n["edge_scale"], n["edge_mask"])
               for m in (1, 2, 3)]
        for got, ed, what in zip((gx, gxx, gxxx), eds, ("gx", "gxx", "gxxx")):
            close(got, np.einsum("boi,o->bi", ed, w), 2e-5, f"{basis!r} {what}")
        # d/dcoef sum_b,i gx^2 = 2 sum_b gx[b,i] w_o phi'_k(x_bi) s_oi m_oi
        gx_np = np.einsum("boi,o->bi", eds[0], w)
        dphi = ko.basis_eval(n["spec"], xs, 1, n["params"])
        scale = n["edge_scale"] * n["edge_mask"]
        want = 2 * np.einsum("bi,o,bik->oik", gx_np, w, dphi) * scale[..., None]
        close(gc, want, 2e-5, f"{basis!r} gradient penalty")


def test_reference_model_file_forward():
    import kanforge_b200.convert as cv
    from conftest import GOLDEN

    model = cv.load(GOLDEN / "ref_model.npz").to(DEV)
    io = load_golden("ref_model_io.npz")
    with torch.no_grad():
        y = model(torch.as_tensor(io["x"], device=DEV))
    close(y, io["y"], FP32_TOL, "model file")


# ---------------------------------------------------------------------------
# bf16 fused tensor-core path
# ---------------------------------------------------------------------------

FUSED_CASES = [
    # basis, B, I, O, base, bias, edge_scale
    (kb.Chebyshev(12), 300, 40, 264, True, True, False),
    (kb.BSpline(8, 3), 257, 37, 136, True, True, True),
    (kb.Jacobi(6, 0.5, 0.5), 130, 64, 256, True, True, False),
    (kb.Chebyshev(20), 200, 20, 64, True, True, False),         # f_pad 32
    (kb.Chebyshev(5), 129, 9, 24, False, False, False),          # no base, no bias
    (kb.BSpline(5, 3, (-2.0, 2.0)), 1030, 16, 520, True, True, False),
    (kb.BSpline(4, 1), 64, 8, 8, True, True, False),
    (kb.Chebyshev(4, input_map="identity"), 77, 12, 40, True, True, False),
    (kb.BSpline(6, 2), 200, 24, 72, True, True, False),
    (kb.BSpline(4, 4), 99, 10, 16, False, True, False),
    (kb.BSpline(7, 5), 150, 20, 48, True, False, False),
    (kb.BSpline(20, 3), 140, 12, 40, True, True, False),       # f_pad 32
    (kb.Fourier(4), 300, 40, 264, True, True, False),
    (kb.Fourier(7), 257, 37, 136, True, False, True),
    (kb.Fourier(12, 3.0), 129, 9, 24, True, True, False),        # f_pad 32
]


def make_bf16_layer(basis, n_in, n_out, base, bias, scale, seed=0):
    torch.manual_seed(seed)
    kw = {} if base else {"base_activation": None}
    layer = kb.KANLinear(n_in, n_out, basis, bias=bias, edge_scale=scale, **kw)
    with torch.no_grad():
        layer.coef.normal_(0, 1.0 / np.sqrt(n_in * basis.size))
        if layer.bias is not None:
            layer.bias.normal_(0, 0.1)
        if scale:
            layer.edge_scale.uniform_(0.5, 1.5)
        layer.edge_mask[0, -1] = 0
        if hasattr(layer, "basis_grid"):  # non-uniform per-input grids
            g = layer.basis_grid
            step = (g[:, 1] - g[:, 0])[:, None]
            g[:, 1:-1] += (torch.rand_like(g[:, 1:-1]) - 0.5) * 0.4 * step
    return layer.to(device=DEV, dtype=torch.bfloat16)


@pytest.mark.parametrize("basis,n_b,n_in,n_out,base,bias,scale", FUSED_CASES, ids=lambda v: repr(v) if isinstance(v, kb.Basis) else str(v))
def test_bf16_fused_layer_forward_and_gradients(basis, n_b, n_in, n_out, base, bias, scale):
    layer = make_bf16_layer(basis, n_in, n_out, base, bias, scale)
    x0 = (torch.randn(n_b, n_in, device=DEV) * 1.2).clamp(-3, 3).to(torch.bfloat16)
    assert kb.kernels.fused_ok(layer._plan, x0, n_out, base)
    x = x0.clone().requires_grad_()
    y = layer(x)
    assert y.dtype == torch.bfloat16
    dy = (torch.randn(n_b, n_out, device=DEV) * 0.5).to(torch.bfloat16)
    params = [p for _, p in layer.named_parameters()]
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + params, dy)
    n = layer_numpy(layer)
    xs = x0.double().cpu().numpy()
    kw = dict(coef=n["coef"], base_weight=n["base_weight"], bias=n["bias"], spec=n["spec"], params=n["params"],
              edge_scale=n["edge_scale"], edge_mask=n["edge_mask"])
    close(y, ko.kan_linear(xs, **kw), BF16_TOL, "y")
    want = ko.kan_linear_backward(xs, dy.double().cpu().numpy(), **kw)
    close(grads[0], want["dx"], BF16_TOL, "dx")
    key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias", "edge_scale": "dedge_scale"}
    for nme, gr in zip(names, grads[1:]):
        close(gr, want[key[nme]], BF16_TOL, f"d{nme}")


@pytest.mark.parametrize("case", [0, 1, 3, 5, 6, 7, 8, 9, 10, 11])
def test_bf16_wgrad_feature_matrix_path_equals_self_evaluating_path(monkeypatch, case):
    """kf_wgrad (and, for B-splines, kf_fwd) reading the kf_features matrix by
    TMA and the same kernels evaluating the features themselves (no feature
    buffer) give bit-identical outputs and gradients: the same bf16 features
    meet the same MMA accumulation order."""
    basis, n_b, n_in, n_out, base, bias, scale = FUSED_CASES[case]
    layer = make_bf16_layer(basis, n_in, n_out, base, bias, scale, seed=3)
    x = (torch.randn(n_b, n_in, device=DEV) * 1.2).clamp(-3, 3).to(torch.bfloat16).requires_grad_()
    dy = (torch.randn(n_b, n_out, device=DEV) * 0.5).to(torch.bfloat16)
    params = [p for _, p in layer.named_parameters()]

    def run():
        y = layer(x)
        return (y.detach(),) + torch.autograd.grad(y, [x] + params, dy)

    fast = run()
    monkeypatch.setattr(kb.kernels, "WGRAD_FEATURE_BYTES_MAX", 0)
    slow = run()
    for a, b in zip(fast, slow):
        assert torch.equal(a, b)


# ---------------------------------------------------------------------------
# float32 layers on the tensor cores (kf_gemm_tf32x3, three TF32 products)
# ---------------------------------------------------------------------------

# (M, N, K, A MN-major, B MN-major, bias): ragged tiles and K steps, every major
# combination, several persistent tiles per CTA
GEMM_CASES = [
    (300, 200, 100, False, False, True),
    (129, 260, 37, True, True, False),
    (513, 64, 1000, False, True, True),
    (64, 513, 999, True, False, False),
    (1, 4, 1, False, False, True),
    (9, 80, 4, False, True, False),
    (4096, 1024, 512, False, False, False),
    (1024, 4096, 3000, True, True, False),
]


@pytest.mark.parametrize("m,n,k,a_mn,b_mn,bias", GEMM_CASES)
def test_gemm_tf32x3_matches_float64(m, n, k, a_mn, b_mn, bias):
    g = torch.Generator(device="cpu").manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, dtype=torch.float64)
    b = torch.randn(n, k, generator=g, dtype=torch.float64)
    bv = torch.randn(n, generator=g, dtype=torch.float64) if bias else None
    pad4 = lambda v: (v + 3) // 4 * 4  # noqa: E731
    # operands in padded storage (row pitch a multiple of 4 floats), as the kernel takes them
    sa = torch.zeros((k, pad4(m)) if a_mn else (m, pad4(k)), dtype=torch.float32, device=DEV)
    sb = torch.zeros((k, pad4(n)) if b_mn else (n, pad4(k)), dtype=torch.float32, device=DEV)
    if a_mn:
        sa[:, :m] = a.T.float().to(DEV)
    else:
        sa[:, :k] = a.float().to(DEV)
    if b_mn:
        sb[:, :n] = b.T.float().to(DEV)
    else:
        sb[:, :k] = b.float().to(DEV)
    out = torch.full((m, pad4(n)), float("nan"), dtype=torch.float32, device=DEV)
    bias_d = None if bv is None else bv.float().to(DEV)
    kb.kernels.gemm_tf32x3(sa, a_mn, sb, b_mn, out, m, n, k, bias=bias_d)
    want = a.float().double() @ b.float().double().T + (0 if bv is None else bv.float().double())
    close(out[:, :n], want.numpy(), FP32_TOL, "C")
    assert torch.isnan(out[:, n:]).all()  # nothing written past N


FP32_LAYER_CASES = [
    # basis, B, I, O, base, bias, edge_scale
    (kb.BSpline(8, 3), 257, 37, 136, True, True, True),
    (kb.Chebyshev(12), 300, 40, 264, True, True, False),
    (kb.Jacobi(6, 0.5, 0.5), 130, 64, 256, True, True, False),
    (kb.BSpline(5, 3, (-2.0, 2.0)), 1030, 16, 520, True, False, False),
    (kb.BSpline(20, 3), 140, 12, 40, True, True, False),      # 32-wide feature rows
    (kb.Chebyshev(5), 129, 9, 24, False, False, False),
    (kb.Chebyshev(4, input_map="identity"), 77, 12, 40, True, True, True),
    (kb.Fourier(5), 257, 37, 136, True, True, True),
    (kb.RBF(8), 300, 24, 64, True, True, False),
    (kb.RSWAF(6), 129, 9, 24, False, False, False),
    (kb.MexicanHat(5, learnable=False), 77, 12, 40, True, True, True),
]


@pytest.mark.parametrize("basis,n_b,n_in,n_out,base,bias,scale", FP32_LAYER_CASES,
                         ids=lambda v: repr(v) if isinstance(v, kb.Basis) else str(v))
def test_float32_layer_on_tensor_cores_matches_oracle(basis, n_b, n_in, n_out, base, bias, scale):
    layer = make_bf16_layer(basis, n_in, n_out, base, bias, scale).float()
    x0 = (torch.randn(n_b, n_in, device=DEV) * 1.2).clamp(-3, 3)
    assert kb.kernels.tf32_ok(layer._plan, x0, n_out, base, layer.coef.dtype)
    x = x0.clone().requires_grad_()
    y = layer(x)
    nodes = [y.grad_fn] + [f for f, _ in y.grad_fn.next_functions if f is not None]
    assert any("Tf32" in type(f).__name__ for f in nodes)  # the tensor-core path served the call
    dy = torch.randn(n_b, n_out, device=DEV) * 0.5
    params = [p for _, p in layer.named_parameters()]
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + params, dy)
    n = layer_numpy(layer)
    xs = x0.double().cpu().numpy()
    kw = dict(coef=n["coef"], base_weight=n["base_weight"], bias=n["bias"], spec=n["spec"], params=n["params"],
              edge_scale=n["edge_scale"], edge_mask=n["edge_mask"])
    close(y, ko.kan_linear(xs, **kw), FP32_TOL, "y")
    want = ko.kan_linear_backward(xs, dy.double().cpu().numpy(), **kw)
    close(grads[0], want["dx"], FP32_TOL, "dx")
    key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias", "edge_scale": "dedge_scale"}
    for nme, gr in zip(names, grads[1:]):
        close(gr, want[key[nme]], FP32_TOL, f"d{nme}")


@pytest.mark.parametrize("order,grid_size,base,n_b", [(1, 6, True, 1000), (2, 9, False, 1000), (3, 8, True, 1000),
                                                      (4, 5, True, 1000), (5, 7, False, 1000), (3, 20, True, 1000),
                                                      (3, 8, True, 30011), (2, 9, False, 40003)])
def test_float32_spline_features_from_knot_tables_match_grid_kernel(order, grid_size, base, n_b):
    """kf_features_spline_f32 (knot tables) against kf_features_f32 (raw grid) on
    non-uniform grids, with inputs on knots, outside the grid and at its ends.
    The 30011- and 40003-row cases run the row loop's later grid-stride passes
    and end on a partial group of rows."""
    n_in = 37
    layer = make_bf16_layer(kb.BSpline(grid_size, order), n_in, 8, base, False, False).float()
    plan, g = layer._plan, layer.basis_grid.float().contiguous()
    nt, f_pad = kb.kernels.fused_layout(plan, base)
    x = (torch.randn(n_b, n_in, device=DEV) * 1.2).clamp(-3, 3)
    x[:64] = g[:, torch.randint(0, g.shape[1], (64,))].T  # exactly on knots (ends included)
    x[64:80] = 5.0
    x[80:96] = -5.0
    x = x.contiguous()
    desc = plan.desc()
    want = torch.full((n_b, n_in * f_pad), float("nan"), device=DEV)
    got = torch.full_like(want, float("nan"))
    kb.kernels._launch("kf_features_f32", x.data_ptr(), g.data_ptr(), want.data_ptr(), n_b, n_in, nt, f_pad, int(base),
                       ctypes.byref(desc), kb.kernels._stream(x))
    tab = kb.kernels.knot_tables(g, plan)
    kb.kernels._launch("kf_features_spline_f32", x.data_ptr(), tab.data_ptr(), got.data_ptr(), n_b, n_in, nt, f_pad,
                       int(base), ctypes.byref(desc), kb.kernels._stream(x))
    torch.cuda.synchronize()
    assert not torch.isnan(got).any()
    torch.testing.assert_close(got, want, rtol=1e-5, atol=2e-6)


@pytest.mark.parametrize("basis", [kb.Chebyshev(6), kb.BSpline(5, 2)], ids=repr)
def test_float32_feature_kernels_past_the_grid_y_limit(basis):
    """More rows than 65535 row blocks of 64 (4,194,240): kf_features_f32 and
    kf_features_dot_f32 stride over the row blocks; the rows past the limit
    equal the same rows computed by a small launch."""
    n_b, n_in = 65535 * 64 + 777, 1
    plan = kb.plan_for(basis)
    nt, f_pad = kb.kernels.fused_layout(plan, True)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = (torch.randn(n_b, n_in, device=DEV, generator=g) * 1.2).clamp(-3, 3)
    grid = torch.linspace(-1, 1, basis.size - plan.consts[1] + 1, device=DEV)[None] if plan.kind == "bspline" else \
        x.new_zeros(1)
    desc = plan.desc()
    feat = torch.empty(n_b, n_in * f_pad, device=DEV)
    kb.kernels._launch("kf_features_f32", x.data_ptr(), grid.data_ptr(), feat.data_ptr(), n_b, n_in, nt, f_pad, 1,
                       ctypes.byref(desc), kb.kernels._stream(x))
    dfeat = torch.randn(n_b, n_in * f_pad, device=DEV, generator=g)
    dx = torch.empty_like(x)
    kb.kernels._launch("kf_features_dot_f32", x.data_ptr(), grid.data_ptr(), dfeat.data_ptr(), dx.data_ptr(), n_b, n_in,
                       nt, f_pad, 1, ctypes.byref(desc), kb.kernels._stream(x))
    tail = slice(n_b - 5000, n_b)
    xt = x[tail].contiguous()
    ft = torch.empty(5000, n_in * f_pad, device=DEV)
    kb.kernels._launch("kf_features_f32", xt.data_ptr(), grid.data_ptr(), ft.data_ptr(), 5000, n_in, nt, f_pad, 1,
                       ctypes.byref(desc), kb.kernels._stream(x))
    dft = dfeat[tail].contiguous()
    dxt = torch.empty_like(xt)
    kb.kernels._launch("kf_features_dot_f32", xt.data_ptr(), grid.data_ptr(), dft.data_ptr(), dxt.data_ptr(), 5000, n_in,
                       nt, f_pad, 1, ctypes.byref(desc), kb.kernels._stream(x))
    torch.cuda.synchronize()
    assert torch.equal(feat[tail], ft)
    assert torch.equal(dx[tail], dxt)


def test_bf16_fused_multi_tile_persistent_against_float32_primitives():
    """Enough tiles that every persistent CTA runs several (both TMEM accumulators,
    every pipeline phase); checked against the float32 primitive kernels."""
    torch.manual_seed(1)
    n_b, n_in, n_out = 16384 + 77, 64, 1024
    layer = make_bf16_layer(kb.Chebyshev(12), n_in, n_out, True, True, False, seed=1)
    x0 = torch.randn(n_b, n_in, device=DEV).clamp(-3, 3).to(torch.bfloat16)
    x = x0.clone().requires_grad_()
    y = layer(x)
    dy = (torch.randn(n_b, n_out, device=DEV) * 0.1).to(torch.bfloat16)
    gx, gc, gb = torch.autograd.grad(y, [x, layer.coef, layer.base_weight], dy)
    plan = layer._plan
    xf, dyf = x0.float(), dy.float()
    ce, be = layer.effective_coef().float().detach(), layer.effective_base_weight().float().detach()
    ones = torch.ones_like(xf)
    g0 = xf.new_zeros(1)
    with torch.no_grad():
        y_ref = kb.kernels.prim_F(xf, ce, ones, g0, plan, 0) + torch.nn.functional.silu(xf) @ be.T + layer.bias.float()
        s = torch.sigmoid(xf)
        gx_ref = kb.kernels.prim_P(xf, dyf, ce, g0, plan, 1) + (dyf @ be) * (s * (1 + xf * (1 - s)))
        mask = layer.edge_mask.float()
        gc_ref = kb.kernels.prim_G(xf, dyf, ones, g0, plan, 0) * mask[..., None]
        gb_ref = (dyf.T @ torch.nn.functional.silu(xf)) * mask
    for got, ref, what in ((y, y_ref, "y"), (gx, gx_ref, "dx"), (gc, gc_ref, "dcoef"), (gb, gb_ref, "dbase")):
        close(got.float(), ref.double().cpu().numpy(), BF16_TOL, what)
    kb.kernels.check_device_errors()


def test_bf16_layer_double_backward_uses_differentiable_path():
    layer = make_bf16_layer(kb.Chebyshev(6), 8, 16, True, True, False)
    x = (torch.rand(33, 8, device=DEV) * 2 - 1).to(torch.bfloat16).requires_grad_()
    y = layer(x)
    (gx,) = torch.autograd.grad(y.float().sum(), x, create_graph=True)
    (gc,) = torch.autograd.grad((gx.float() ** 2).sum(), layer.coef)
    assert gc.shape == layer.coef.shape and torch.isfinite(gc).all()
    n = layer_numpy(layer)
    xs = x.detach().double().cpu().numpy()
    ed = ko.edge_derivative(xs, n["coef"], n["base_weight"], n["spec"], n["params"], 1, n["edge_scale"], n["edge_mask"])
    close(gx, ed.sum(1), BF16_TOL, "gx")


# ---------------------------------------------------------------------------
# GR-KAN (rational) and KAN blocks
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dtype,tol", [(torch.float32, FP32_TOL), (torch.bfloat16, BF16_TOL)])
def test_grkan_forward_and_gradients(dtype, tol):
    torch.manual_seed(0)
    layer = kb.GRKAN(64, 48, groups=8)
    with torch.no_grad():
        layer.basis_numerator.add_(0.05 * torch.randn_like(layer.basis_numerator))
        layer.basis_denominator.add_(0.05 * torch.randn_like(layer.basis_denominator))
    layer = layer.to(device=DEV, dtype=dtype)
    x0 = (torch.randn(513, 64, device=DEV) * 1.5).to(dtype)
    x = x0.clone().requires_grad_()
    y = layer(x)
    dy = torch.randn_like(y)
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + [p for _, p in layer.named_parameters()], dy)
    n = layer_numpy(layer)
    xs = x0.double().cpu().numpy()
    kw = dict(coef=n["coef"], base_weight=None, bias=n["bias"], spec=n["spec"], params=n["params"], edge_scale=None,
              edge_mask=n["edge_mask"])
    close(y, ko.kan_linear(xs, **kw), tol, "y")
    want = ko.kan_linear_backward(xs, dy.double().cpu().numpy(), groups=8, **kw)
    close(grads[0], want["dx"], tol, "dx")
    key = {"coef": "dcoef", "bias": "dbias", "basis_numerator": "dnumerator", "basis_denominator": "ddenominator"}
    for nme, gr in zip(names, grads[1:]):
        # parameter gradients are sums over 513 x 8 inputs: scale the bf16 bound by their size
        close(gr, want[key[nme]], tol if dtype == torch.float32 else 5e-2, f"d{nme}")


# (B, I, O, groups): the bf16 GR-KAN tensor-core path (inputs per group a
# multiple of 32): ragged row and output tiles, groups spanning several 256-input
# tiles and several groups per tile, 512- and 256-output forward tiles
GRKAN_TC_CASES = [(1000, 256, 136, 8), (513, 512, 64, 4), (300, 64, 24, 2), (4097, 768, 520, 8), (2048, 1024, 768, 8)]


@pytest.mark.parametrize("n_b,n_in,n_out,groups", GRKAN_TC_CASES)
def test_grkan_bf16_tensor_core_path_matches_oracle(n_b, n_in, n_out, groups):
    torch.manual_seed(n_in)
    layer = kb.GRKAN(n_in, n_out, groups=groups)
    with torch.no_grad():
        layer.basis_numerator.add_(0.05 * torch.randn_like(layer.basis_numerator))
        layer.basis_denominator.add_(0.05 * torch.randn_like(layer.basis_denominator))
        layer.bias.normal_(0, 0.1)
        layer.edge_mask[1, 3] = 0
    layer = layer.to(device=DEV, dtype=torch.bfloat16)
    x0 = (torch.randn(n_b, n_in, device=DEV) * 1.5).to(torch.bfloat16)
    assert kb.kernels.grkan_ok(layer._plan, x0, n_in, n_out, groups, layer.coef.dtype) == "bf16"
    x = x0.clone().requires_grad_()
    y = layer(x)
    nodes = [y.grad_fn] + [f for f, _ in y.grad_fn.next_functions if f is not None]
    assert any(type(f).__name__ == "_GRKANLinearBackward" for f in nodes)  # the tensor-core path served the call
    dy = torch.randn_like(y)
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + [p for _, p in layer.named_parameters()], dy)
    kb.kernels.check_device_errors()
    n = layer_numpy(layer)
    xs = x0.double().cpu().numpy()
    kw = dict(coef=n["coef"], base_weight=None, bias=n["bias"], spec=n["spec"], params=n["params"], edge_scale=None,
              edge_mask=n["edge_mask"])
    close(y, ko.kan_linear(xs, **kw), BF16_TOL, "y")
    want = ko.kan_linear_backward(xs, dy.double().cpu().numpy(), groups=groups, **kw)
    close(grads[0], want["dx"], BF16_TOL, "dx")
    key = {"coef": "dcoef", "bias": "dbias", "basis_numerator": "dnumerator", "basis_denominator": "ddenominator"}
    for nme, gr in zip(names, grads[1:]):
        close(gr, want[key[nme]], BF16_TOL if nme in ("coef", "bias") else 5e-2, f"d{nme}")


def test_grkan_bf16_tensor_core_gradients_are_deterministic():
    torch.manual_seed(1)
    layer = kb.GRKAN(768, 520, groups=8).to(device=DEV, dtype=torch.bfloat16)
    x = (torch.randn(3001, 768, device=DEV) * 1.5).to(torch.bfloat16).requires_grad_()
    dy = torch.randn(3001, 520, device=DEV).to(torch.bfloat16)
    params = [p for _, p in layer.named_parameters()]
    first = torch.autograd.grad(layer(x), [x] + params, dy)
    second = torch.autograd.grad(layer(x), [x] + params, dy)
    for a, b in zip(first, second):
        assert torch.equal(a, b)


# (B, I, groups, p, q, misaligned x): the vector kernels (16-byte forward, paired
# backward for degrees (5, 4)), their row and chunk tails, and the one-element
# kernels (odd inputs per group, other degrees, x one element off alignment).
RATIONAL_CASES = [
    (1003, 64, 8, 5, 4, False),
    (4096, 768, 8, 5, 4, False),
    (20000, 256, 8, 5, 4, False),
    (3, 64, 8, 5, 4, False),
    (77, 320, 8, 5, 4, False),
    (37, 24, 8, 5, 4, False),
    (129, 64, 2, 3, 3, False),
    (200, 520, 8, 5, 4, False),
    (77, 64, 8, 5, 4, True),
]


@pytest.mark.parametrize("dtype,tol,ptol", [(torch.float32, FP32_TOL, FP32_TOL), (torch.bfloat16, BF16_TOL, 5e-2)])
@pytest.mark.parametrize("n_b,n_in,groups,p,q,offset", RATIONAL_CASES)
def test_rational_kernels_match_oracle_on_every_launch_path(n_b, n_in, groups, p, q, offset, dtype, tol, ptol):
    g = torch.Generator(device="cpu").manual_seed(n_b + n_in)
    a, b = kb.fit_rational("gelu", p, q)
    num = torch.as_tensor(np.tile(a, (groups, 1)), dtype=torch.float32) + 0.05 * torch.randn(groups, p + 1, generator=g)
    den = torch.as_tensor(np.tile(b, (groups, 1)), dtype=torch.float32) + 0.05 * torch.randn(groups, q, generator=g)
    x0 = (torch.randn(n_b, n_in, generator=g) * 1.5).to(dtype)
    dr = torch.randn(n_b, n_in, generator=g).to(dtype)
    if offset:  # a view one element past an aligned allocation
        buf = torch.empty(n_b * n_in + 1, device=DEV, dtype=dtype)
        x = buf[1:].view(n_b, n_in)
        x.copy_(x0)
        assert x.data_ptr() % 16 != 0
    else:
        x = x0.to(DEV)
    numd, dend = num.to(DEV).requires_grad_(), den.to(DEV).requires_grad_()
    x.requires_grad_()
    plan = kb.plan_for(kb.Rational(p, q))
    r = kb.kernels.rational_act(x, numd, dend, plan, groups)
    gx, gnum, gden = torch.autograd.grad(r, [x, numd, dend], dr.to(DEV))

    xs = x0.double().numpy()
    ipg = n_in // groups
    num_i, den_i = np.repeat(num.double().numpy(), ipg, 0), np.repeat(den.double().numpy(), ipg, 0)
    drs = dr.double().numpy()
    close(r, ko.rational(xs, num_i, den_i, 0)[..., 0], tol, "R")
    close(gx, drs * ko.rational(xs, num_i, den_i, 1)[..., 0], tol, "dx")
    dn, dq = ko.rational_param_partials(xs, num_i, den_i)
    want_n = (drs[..., None] * dn).sum(0).reshape(groups, ipg, p + 1).sum(1)
    want_q = (drs[..., None] * dq).sum(0).reshape(groups, ipg, q).sum(1)
    close(gnum, want_n, ptol, "dnum")
    close(gden, want_q, ptol, "dden")


def test_grkan_starts_as_gelu_and_keeps_variance():
    """reference tests/test_layers.py:84-96, on the CUDA kernels."""
    torch.manual_seed(0)
    layer = kb.GRKAN(64, 64, groups=8).to(DEV)
    x = torch.randn(4096, 64, device=DEV)
    with torch.no_grad():
        assert 0.7 < layer(x).std().item() < 1.4
        z = torch.linspace(-3, 3, 301, device=DEV)[:, None].expand(301, 64).contiguous()
        acts = kb.kernels.rational_act(z, layer.basis_numerator, layer.basis_denominator, layer._plan, 8)
    assert (acts[:, 0] - torch.nn.functional.gelu(z[:, 0])).abs().max() < 2e-2


def test_kanffn_and_conv2d_match_oracle():
    torch.manual_seed(0)
    ffn = kb.KANFFN(32, 64, kind="grkan", groups=8).to(DEV)
    x = torch.randn(3, 5, 32, device=DEV)
    with torch.no_grad():
        y = ffn(x)
        h = ffn.fc1(x)
    n1, n2 = layer_numpy(ffn.fc1), layer_numpy(ffn.fc2)
    xs = x.double().cpu().numpy()
    h_ref = ko.kan_linear(xs, n1["coef"], None, n1["bias"], n1["spec"], n1["params"], None, n1["edge_mask"])
    close(h, h_ref, FP32_TOL, "fc1")
    y_ref = ko.kan_linear(h.double().cpu().numpy(), n2["coef"], None, n2["bias"], n2["spec"], n2["params"], None, n2["edge_mask"])
    close(y, y_ref, FP32_TOL, "fc2")

    conv = kb.KANConv2d(3, 4, 3, padding=1, basis=kb.BSpline(5, 3)).to(DEV)
    img = torch.rand(2, 3, 6, 7, device=DEV) * 2 - 1
    with torch.no_grad():
        out = conv(img)
    assert out.shape == (2, 4, 6, 7)
    n = layer_numpy(conv.kans[0])
    patches = torch.nn.functional.unfold(img, 3, padding=1).transpose(1, 2).double().cpu().numpy()  # (2, 42, 27)
    ref = ko.kan_linear(patches, n["coef"], n["base_weight"], n["bias"], n["spec"], n["params"], None, n["edge_mask"])
    close(out.permute(0, 2, 3, 1).reshape(2, 42, 4), ref, FP32_TOL, "conv2d")


def test_no_device_errors_recorded():
    kb.kernels.check_device_errors()


@pytest.mark.parametrize("kind", ["bf16_bspline", "bf16_cheb", "f32_bspline", "grkan_bf16"])
def test_training_step_in_cuda_graph_matches_eager(kind):
    """A forward + backward captured into a CUDA graph (the bench's --graph
    mode) and replayed gives bit-identical outputs and gradients to the eager
    step: the library's launches follow torch's current stream and allocate
    through torch."""
    torch.manual_seed(0)
    if kind == "grkan_bf16":
        layer = kb.GRKAN(64, 48, groups=8).to(device=DEV, dtype=torch.bfloat16)
        dtype = torch.bfloat16
    else:
        basis = kb.Chebyshev(12) if kind == "bf16_cheb" else kb.BSpline(8, 3)
        dtype = torch.float32 if kind.startswith("f32") else torch.bfloat16
        layer = make_bf16_layer(basis, 40, 264, True, True, True).to(dtype)
    x = (torch.randn(300, layer.in_features, device=DEV) * 1.2).clamp(-3, 3).to(dtype).requires_grad_()
    params = [p for _, p in layer.named_parameters()]
    dy = torch.randn(300, layer.out_features, device=DEV).to(dtype)

    def step():
        for p in params:
            p.grad = None
        x.grad = None
        y = layer(x)
        y.backward(dy)
        return y.detach()

    want_y = step().clone()
    want = [x.grad.clone()] + [p.grad.clone() for p in params]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    graph.replay()
    torch.cuda.synchronize()
    # the library's own kernels are deterministic; GR-KAN's linear maps are
    # cuBLAS, whose algorithm choice may differ under capture
    same = (lambda a, b: torch.testing.assert_close(a, b)) if kind == "grkan_bf16" else \
        (lambda a, b: torch.testing.assert_close(a, b, rtol=0, atol=0))
    same(out, want_y)
    for got, w in zip([x.grad] + [p.grad for p in params], want):
        same(got, w)
    del graph


@pytest.mark.parametrize("basis", [kb.RBF(8), kb.RSWAF(6)], ids=repr)
def test_bf16_bump_layer_on_float32_tensor_cores_matches_oracle(basis):
    """bf16 bump layers (centres per input) run the float32 three-TF32 path."""
    layer = make_bf16_layer(basis, 24, 64, True, True, True)
    x0 = (torch.randn(300, 24, device=DEV) * 1.2).clamp(-3, 3).to(torch.bfloat16)
    x = x0.clone().requires_grad_()
    y = layer(x)
    assert y.dtype == torch.bfloat16
    dy = (torch.randn(300, 64, device=DEV) * 0.5).to(torch.bfloat16)
    params = [p for _, p in layer.named_parameters()]
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad(y, [x] + params, dy)
    n = layer_numpy(layer)
    xs = x0.double().cpu().numpy()
    kw = dict(coef=n["coef"], base_weight=n["base_weight"], bias=n["bias"], spec=n["spec"], params=n["params"],
              edge_scale=n["edge_scale"], edge_mask=n["edge_mask"])
    close(y, ko.kan_linear(xs, **kw), BF16_TOL, "y")
    want = ko.kan_linear_backward(xs, dy.double().cpu().numpy(), **kw)
    close(grads[0], want["dx"], BF16_TOL, "dx")
    key = {"coef": "dcoef", "base_weight": "dbase_weight", "bias": "dbias", "edge_scale": "dedge_scale"}
    for nme, gr in zip(names, grads[1:]):
        close(gr, want[key[nme]], BF16_TOL, f"d{nme}")
