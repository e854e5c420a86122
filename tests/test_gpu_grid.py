"""Grid tools on the GPU against the oracle and the reference's own results
(tests/golden/grid.npz): kf_adaptive_grid, kf_resample_grid and kf_refit
through KANLinear.update_grid / refine_grid / change_basis and KAN.update_grid
(reference kanforge/grid.py:19-85, kanforge/_layer.py:107-183).

Bars: grids bit-exact (float64 against the oracle, float32 against the
reference's layer buffers); refit coefficients in float64 within 1e-9 of the
oracle's lstsq (metric max|a-b| / max(1, max|b|)); float32 layer coefficients
within the float32 tolerance 1e-5 of the reference's."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from conftest import load_golden

import kan_oracle as ko
import kanforge_b200 as kb
from kanforge_b200 import kernels as K
from kanforge_b200.plan import plan_for

pytestmark = pytest.mark.gpu
DEV = "cuda"
GRID = load_golden("grid.npz")
FP32_TOL = 1e-5


def _sub(prefix):
    return {k[len(prefix):]: v for k, v in GRID.items() if k.startswith(prefix)}


def _columns(x):
    return K.sample_columns(torch.as_tensor(np.ascontiguousarray(x), device=DEV))


@pytest.mark.parametrize("case", sorted({k.split("/")[1] for k in GRID if k.startswith("adaptive/") and k.endswith("/args")}))
def test_adaptive_grid_bit_exact(case):
    n, margin, eps = GRID[f"adaptive/{case}/args"]
    got = K.adaptive_grid(_columns(GRID["adaptive/x"]), int(n), margin, eps).cpu().numpy()
    assert np.array_equal(got, GRID[f"adaptive/{case}/grid"])


def test_adaptive_grid_one_sample_nan_and_bf16():
    got = K.adaptive_grid(_columns(GRID["adaptive/x1"]), 5).cpu().numpy()
    assert np.array_equal(got, GRID["adaptive/x1/grid"])
    rng = np.random.default_rng(3)
    x = rng.standard_normal((777, 9)).astype(np.float32)
    x[5, 2] = np.nan
    xb = torch.as_tensor(x, device=DEV).bfloat16()
    got = K.adaptive_grid(K.sample_columns(xb), 7, 0.03, 0.1).cpu().numpy()
    want = ko.adaptive_grid(xb.float().cpu().numpy(), 7, 0.03, 0.1)
    assert np.array_equal(got, want, equal_nan=True)


@pytest.mark.parametrize("shape", [(100_000, 37), (4096, 1024), (3, 5)], ids=str)
@pytest.mark.parametrize("n_points", [2, 9, 192])
def test_adaptive_grid_sizes(shape, n_points):
    """Many samples (several CTAs per input), many inputs, ties and the largest grid."""
    rng = np.random.default_rng(shape[0] + n_points)
    x = (rng.standard_normal(shape) * rng.uniform(0.1, 3, shape[1])).astype(np.float32)
    x[: shape[0] // 3, 0] = 1.25  # a third of one input ties
    got = K.adaptive_grid(_columns(x), n_points).cpu().numpy()
    assert np.array_equal(got, ko.adaptive_grid(x, n_points))


def test_adaptive_grid_rejects_bad_arguments():
    xt = _columns(GRID["adaptive/x"])
    with pytest.raises(ValueError):
        K.adaptive_grid(xt, 9, grid_eps=0.0)
    with pytest.raises(ValueError):
        K.adaptive_grid(xt, 193)


@pytest.mark.parametrize("n", [2, 5, 9, 17, 33])
def test_resample_grid_bit_exact(n):
    g = torch.as_tensor(GRID["resample/grid"], device=DEV)
    got = K.resample_grid(g, n).cpu().numpy()
    assert np.array_equal(got, ko.resample_grid(GRID["resample/grid"], n))


def _fit(spec_cfg, params, dev=DEV):
    from kanforge_b200.bases import make_basis

    basis = make_basis(json.loads(str(spec_cfg)))
    grid = params.get("grid")
    grid = None if grid is None else torch.as_tensor(grid, device=dev)
    return basis, K.fit_basis(plan_for(basis), grid, dev)


@pytest.mark.parametrize("case", sorted({k.split("/")[1] for k in GRID if k.startswith("refit/")}))
@pytest.mark.parametrize("from_ranges", [False, True])
def test_refit_matches_oracle(case, from_ranges):
    pre = f"refit/{case}/"
    old_p, new_p = _sub(pre + "old/"), _sub(pre + "new/")
    _, (old_fb, k1) = _fit(GRID[pre + "old_config"], old_p)
    _, (new_fb, k2) = _fit(GRID[pre + "new_config"], new_p)
    coef = GRID[pre + "coef"].astype(np.float32)
    ridge = float(GRID[pre + "ridge"])
    x = GRID[pre + "x"]
    if from_ranges:  # evenly spaced samples over per-input ranges, generated on the device
        ranges = np.stack([x.min(0), x.max(0)], -1)
        n = 333
        got, _ = K.refit(None, torch.as_tensor(ranges, device=DEV), n, old_fb, new_fb,
                         torch.as_tensor(coef, device=DEV), None, ridge)
        xs = ko.sample_inputs(ranges, n)
    else:
        got, _ = K.refit(_columns(x.astype(np.float32)), None, x.shape[0], old_fb, new_fb,
                         torch.as_tensor(coef, device=DEV), None, ridge)
        xs = x
    old = ko.spec_from_config(json.loads(str(GRID[pre + "old_config"])))
    new = ko.spec_from_config(json.loads(str(GRID[pre + "new_config"])))
    want = ko.refit(old, old_p, coef, new, new_p, xs, ridge)
    err = ko.max_rel_err(got.cpu().numpy(), want)
    assert err <= 1e-9, f"{case}: {err:.3e}"
    if not from_ranges:
        assert ko.max_rel_err(got.cpu().numpy(), GRID[pre + "out"]) <= 1e-6  # the reference's own lstsq, float32 coef


def _layer_from_state(cfg, state):
    from kanforge_b200.bases import make_basis

    basis = make_basis(json.loads(str(cfg)))
    layer = kb.KANLinear(state["coef"].shape[1], state["coef"].shape[0], basis, edge_scale="edge_scale" in state,
                         device=DEV)
    layer.load_state_dict({k: torch.as_tensor(v) for k, v in state.items()})
    return layer


LAYER_OPS = {
    "update_bspline": lambda m, x: m.update_grid(x),
    "update_bspline_margin": lambda m, x: m.update_grid(x, margin=0.05, grid_eps=0.2, ridge=0.01),
    "update_rbf": lambda m, x: m.update_grid(x),
    "update_rswaf": lambda m, x: m.update_grid(x),
    "refine_bspline": lambda m, x: m.refine_grid(10),
    "refine_bspline_x": lambda m, x: m.refine_grid(7, x),
    "refine_rbf": lambda m, x: m.refine_grid(9),
    "change_bspline_cheb": lambda m, x: m.change_basis(kb.Chebyshev(8)),
    "change_cheb_bspline_x": lambda m, x: m.change_basis(kb.BSpline(6, 3), x),
    "change_bspline_rbf": lambda m, x: m.change_basis(kb.RBF(10)),
}


@pytest.mark.parametrize("case", sorted(LAYER_OPS))
def test_layer_grid_tools_match_reference(case):
    before, after = _sub(f"layer/{case}/before/state/"), _sub(f"layer/{case}/after/state/")
    layer = _layer_from_state(GRID[f"layer/{case}/before/config"], before)
    x = torch.as_tensor(GRID["layer/x"], device=DEV)
    y_before = layer(x)
    LAYER_OPS[case](layer, x)
    kb.kernels.check_device_errors()
    assert json.loads(json.dumps(layer.basis.config())) == json.loads(str(GRID[f"layer/{case}/after/config"]))
    got = {k: v.detach().cpu().numpy() for k, v in layer.state_dict().items()}
    assert set(got) == set(after)
    if "basis_grid" in after:
        assert np.array_equal(got["basis_grid"], after["basis_grid"])
    if "edge_scale" in after:
        assert np.array_equal(got["edge_scale"], after["edge_scale"])
    err = ko.max_rel_err(got["coef"], after["coef"])
    assert err <= FP32_TOL, f"coef: {err:.3e}"
    assert layer.coef.is_contiguous() and layer.coef.shape == after["coef"].shape
    y_after = layer(x)  # the layer runs on its new basis
    assert torch.isfinite(y_after).all() and y_after.shape == y_before.shape


def test_kan_update_grid_matches_reference():
    torch.manual_seed(0)
    model = kb.KAN([5, 4, 3], kb.BSpline(5, 3), device=DEV)
    for j, layer in enumerate(model):
        layer.load_state_dict({k: torch.as_tensor(v) for k, v in _sub(f"kan/before/{j}/").items()})
    model.update_grid(torch.as_tensor(GRID["kan/x"], device=DEV))
    for j, layer in enumerate(model):
        want = _sub(f"kan/after/{j}/")
        assert np.array_equal(layer.basis_grid.cpu().numpy(), want["basis_grid"]) if j == 0 else \
            np.allclose(layer.basis_grid.cpu().numpy(), want["basis_grid"], rtol=0, atol=1e-5)
        assert ko.max_rel_err(layer.coef.detach().cpu().numpy(), want["coef"]) <= 1e-4


def test_refine_nested_bspline_grid_keeps_function():
    """A spline on a grid is exactly a spline on the grid with every interval
    halved (reference tests/test_phase2.py:92-102)."""
    torch.manual_seed(0)
    layer = kb.KANLinear(3, 2, kb.BSpline(5, 3), edge_scale=True, device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.5)
        layer.edge_scale.uniform_(0.5, 2)
    x = torch.linspace(-1, 1, 301, device=DEV)[:, None].repeat(1, 3)
    before = layer(x)
    layer.refine_grid(10)
    assert layer.basis.grid_size == 10 and layer.coef.shape == (2, 3, 13)
    assert ko.max_rel_err(layer(x).detach().cpu().numpy(), before.detach().cpu().numpy()) <= FP32_TOL


def test_update_grid_outside_the_grid_keeps_function():
    torch.manual_seed(1)
    layer = kb.KANLinear(3, 2, kb.BSpline(5, 3), device=DEV)
    x = torch.rand(500, 3, device=DEV) * 2 + 3  # the spline part is zero here
    before = layer(x)
    layer.update_grid(x)
    assert ko.max_rel_err(layer(x).detach().cpu().numpy(), before.detach().cpu().numpy()) <= FP32_TOL
    assert layer.basis_grid.min() > 2.9


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_update_grid_at_scale_matches_oracle(dtype):
    """65536 samples of a 256-input layer: grid bit-exact, refit within tolerance."""
    torch.manual_seed(2)
    layer = kb.KANLinear(256, 64, kb.BSpline(8, 3), edge_scale=True, device=DEV, dtype=dtype)
    with torch.no_grad():
        layer.edge_scale.uniform_(0.5, 1.5)
    x = (torch.randn(65536, 256, device=DEV) * 0.8).to(dtype)
    coef0 = layer.coef.detach().double().cpu().numpy()
    scale0 = layer.edge_scale.detach().double().cpu().numpy()
    grid0 = layer.basis_grid.detach().double().cpu().numpy()
    layer.update_grid(x)
    xs = x.float().cpu().numpy()
    cols = slice(0, 256, 37)  # the float64 oracle on a column subset
    grid = ko.adaptive_grid(xs[:, cols], 9)
    assert torch.equal(layer.basis_grid[cols].cpu(), torch.as_tensor(grid).to(dtype))
    spec = {"kind": "bspline", "grid_size": 8, "order": 3, "grid_range": (-1.0, 1.0)}
    coef, _ = ko.refit_layer(spec, {"grid": grid0[cols]}, coef0[:, cols], scale0[:, cols], spec, {"grid": grid},
                             xs[:, cols])
    tol = FP32_TOL if dtype == torch.float32 else 2e-2
    assert ko.max_rel_err(layer.coef.detach().double().cpu().numpy()[:, cols], coef) <= tol


def test_grid_tool_errors():
    layer = kb.KANLinear(3, 2, kb.Chebyshev(4), device=DEV)
    x = torch.rand(400, 3, device=DEV) * 2 - 1
    with pytest.raises(TypeError, match="no grid"):
        layer.update_grid(x)
    with pytest.raises(ValueError, match="pass samples"):
        layer.change_basis(kb.Legendre(4))
    before = layer(x)
    layer.change_basis(kb.Legendre(4), x)  # the same polynomial space: exact
    assert ko.max_rel_err(layer(x).detach().cpu().numpy(), before.detach().cpu().numpy()) <= FP32_TOL
    with pytest.raises(ValueError):
        kb.KANLinear(3, 2, kb.BSpline(4, 3), device=DEV).update_grid(x, grid_eps=0.0)
    with pytest.raises(NotImplementedError):
        kb.GRKAN(8, 8, groups=2, device=DEV).change_basis(kb.Chebyshev(3), torch.rand(10, 8, device=DEV))


def _bspline_spec(g, k, rng=(-1.0, 1.0)):
    return {"kind": "bspline", "grid_size": g, "order": k, "grid_range": rng}


def test_refine_to_a_fine_grid_uses_the_large_solver():
    """Grid extension 5 -> 100 intervals (103 functions per edge: the Cholesky
    path above 64): nested grids keep the function, coefficients match lstsq."""
    torch.manual_seed(4)
    layer = kb.KANLinear(6, 5, kb.BSpline(5, 3), edge_scale=True, device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.5)
        layer.edge_scale.uniform_(0.5, 2)
    old_grid = layer.basis_grid.double().cpu().numpy()
    coef0 = layer.coef.detach().double().cpu().numpy()
    scale0 = layer.edge_scale.detach().double().cpu().numpy()
    x = torch.linspace(-1, 1, 401, device=DEV)[:, None].repeat(1, 6)
    before = layer(x)
    layer.refine_grid(100)
    kb.kernels.check_device_errors()
    assert layer.coef.shape == (5, 6, 103)
    assert ko.max_rel_err(layer(x).detach().cpu().numpy(), before.detach().cpu().numpy()) <= FP32_TOL
    new_grid = ko.resample_grid(old_grid, 101)
    xs = ko.sample_inputs(np.stack([old_grid[:, 0], old_grid[:, -1]], -1), 8 * 103 + 64)
    want, _ = ko.refit_layer(_bspline_spec(5, 3), {"grid": old_grid}, coef0, scale0, _bspline_spec(100, 3),
                             {"grid": new_grid}, xs)
    assert ko.max_rel_err(layer.coef.detach().double().cpu().numpy(), want) <= FP32_TOL


def test_large_refit_drops_functions_no_sample_reaches():
    """Samples in [-0.5, 0.5] only: the B-splines of a 150-interval grid outside
    that range get coefficient 0, as in the reference's minimum-norm lstsq."""
    torch.manual_seed(5)
    layer = kb.KANLinear(3, 2, kb.BSpline(6, 3), device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.5)
    old_grid = layer.basis_grid.double().cpu().numpy()
    coef0 = layer.coef.detach().double().cpu().numpy()
    x = torch.rand(6000, 3, device=DEV) - 0.5
    layer.refine_grid(150, x)
    kb.kernels.check_device_errors()
    got = layer.coef.detach().double().cpu().numpy()
    want, _ = ko.refit_layer(_bspline_spec(6, 3), {"grid": old_grid}, coef0, None, _bspline_spec(150, 3),
                             {"grid": ko.resample_grid(old_grid, 151)}, x.double().cpu().numpy())
    assert ko.max_rel_err(got, want) <= FP32_TOL
    assert (got[..., :30] == 0).all() and (got[..., -30:] == 0).all()


def test_update_grid_on_a_fine_grid_matches_oracle():
    torch.manual_seed(6)
    layer = kb.KANLinear(8, 4, kb.BSpline(120, 3), device=DEV)
    with torch.no_grad():
        layer.coef.normal_(0, 0.3)
    old_grid = layer.basis_grid.double().cpu().numpy()
    coef0 = layer.coef.detach().double().cpu().numpy()
    x = torch.randn(20000, 8, device=DEV) * 0.5
    layer.update_grid(x)
    kb.kernels.check_device_errors()
    xs = x.double().cpu().numpy()
    grid = ko.adaptive_grid(xs, 121)
    assert torch.equal(layer.basis_grid.cpu(), torch.as_tensor(grid).float())
    want, _ = ko.refit_layer(_bspline_spec(120, 3), {"grid": old_grid}, coef0, None, _bspline_spec(120, 3),
                             {"grid": grid}, xs)
    assert ko.max_rel_err(layer.coef.detach().double().cpu().numpy(), want) <= FP32_TOL
