"""Pin the CPU oracle against golden vectors produced by the reference itself.

Every fixture was written by ``tests/golden/make_golden.py`` from the
reference package (NumPy bases, torch ops path in float64, Triton F/G/P under
the CPU interpreter).  Agreement here is what makes the oracle a valid checker
for the CUDA kernels in the ``gpu`` tests.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden_cases, load_golden, params_of, spec_of

import kan_oracle as ko

BASES = load_golden("bases.npz")
LAYERS = load_golden("layers.npz")
PRIMS = load_golden("prims.npz")

LAYER_SPECS = {
    "bspline_5_3": {"kind": "bspline", "grid_size": 5, "order": 3, "grid_range": (-1.0, 1.0)},
    "bspline_8_3": {"kind": "bspline", "grid_size": 8, "order": 3, "grid_range": (-1.0, 1.0)},
    "chebyshev_12": {"kind": "poly", "family": "chebyshev", "degree": 12, "input_map": "tanh"},
    "jacobi_6": {"kind": "poly", "family": "jacobi", "degree": 6, "alpha": 0.5, "beta": 0.5, "input_map": "tanh"},
    "chebyshev_4_id_nobase": {"kind": "poly", "family": "chebyshev", "degree": 4, "input_map": "identity"},
    "rational_gelu_g2": {"kind": "rational", "num_degree": 5, "den_degree": 4},
    "rational_identity_g1": {"kind": "rational", "num_degree": 5, "den_degree": 4},
}
PRIM_SPECS = {
    "bspline_5_3": {"kind": "bspline", "grid_size": 5, "order": 3, "grid_range": (-1.0, 1.0)},
    "chebyshev_5": {"kind": "poly", "family": "chebyshev", "degree": 5, "input_map": "tanh"},
    "jacobi_4": {"kind": "poly", "family": "jacobi", "degree": 4, "alpha": 0.5, "beta": 1.5, "input_map": "tanh"},
}


def layer_state(case):
    pre = f"{case}/state/"
    return {k[len(pre):]: v for k, v in LAYERS.items() if k.startswith(pre)}


def layer_params(case, state, n_in):
    groups = int(LAYERS[f"{case}/groups"])
    out = {}
    for k, v in state.items():
        if k.startswith("basis_"):
            name = k[len("basis_"):]
            out[name] = v if v.shape[0] == n_in else np.repeat(v, n_in // v.shape[0], axis=0)
    return out, groups


@pytest.mark.parametrize("case", golden_cases(BASES))
@pytest.mark.parametrize("m", [0, 1, 2, 3])
def test_basis_derivatives_match_reference(case, m):
    spec = spec_of(BASES, case)
    got = ko.basis_eval(spec, BASES[f"{case}/x"], m, params_of(BASES, case))
    want = BASES[f"{case}/d{m}"]
    assert got.shape == want.shape
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-10 * max(1.0, np.abs(want).max()))


@pytest.mark.parametrize("case", [c for c in golden_cases(BASES) if f"{c}/fold0" in BASES])
@pytest.mark.parametrize("m", [0, 1, 2, 3])
def test_fold_matrices_match_reference(case, m):
    spec = spec_of(BASES, case)
    if f"{case}/cheb" in BASES:
        np.testing.assert_allclose(ko.cheb_matrix(spec), BASES[f"{case}/cheb"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ko.fold(spec, m), BASES[f"{case}/fold{m}"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("case", [c for c in golden_cases(BASES) if f"{c}/fold0" in BASES])
@pytest.mark.parametrize("m", [0, 1, 2, 3])
def test_folded_features_reproduce_derivatives(case, m):
    """phi^(m) = T-features @ R_m^T: the identity the fused kernels rely on (plan.py:1-12)."""
    spec = spec_of(BASES, case)
    x = BASES[f"{case}/x"]
    feats = ko.kernel_features(spec, x, m)
    want = BASES[f"{case}/d{m}"]
    np.testing.assert_allclose(feats @ ko.fold(spec, m).T, want, atol=1e-9 * max(1.0, np.abs(want).max()))


@pytest.mark.parametrize("case", sorted(LAYER_SPECS))
def test_layer_forward_backward_edge_derivative_match_reference(case):
    spec = LAYER_SPECS[case]
    st = layer_state(case)
    x = LAYERS[f"{case}/x"]
    params, groups = layer_params(case, st, x.shape[-1])
    kw = dict(
        coef=st["coef"], base_weight=st.get("base_weight"), bias=st.get("bias"), spec=spec, params=params,
        edge_scale=st.get("edge_scale"), edge_mask=st["edge_mask"],
    )
    y = ko.kan_linear(x, **kw)
    np.testing.assert_allclose(y, LAYERS[f"{case}/y"], rtol=1e-10, atol=1e-12)
    grads = ko.kan_linear_backward(x, LAYERS[f"{case}/dy"], groups=groups, **kw)
    np.testing.assert_allclose(grads["dx"], LAYERS[f"{case}/grad/x"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(grads["dcoef"], LAYERS[f"{case}/grad/coef"], rtol=1e-9, atol=1e-11)
    for name, key in [("base_weight", "dbase_weight"), ("bias", "dbias"), ("edge_scale", "dedge_scale"),
                      ("basis_numerator", "dnumerator"), ("basis_denominator", "ddenominator")]:
        ref_key = f"{case}/grad/{name}"
        if ref_key in LAYERS:
            np.testing.assert_allclose(grads[key], LAYERS[ref_key], rtol=1e-9, atol=1e-11, err_msg=name)
    for m in range(3):
        d = ko.edge_derivative(x, order=m, **{k: v for k, v in kw.items() if k != "bias"})
        np.testing.assert_allclose(d, LAYERS[f"{case}/edge{m}"], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("case", sorted(PRIM_SPECS))
@pytest.mark.parametrize("m", [0, 1, 2])
def test_primitives_match_reference_triton_kernels(case, m):
    """F/G/P closure (kernels/__init__.py:5-13) vs the reference's own Triton kernels (float32)."""
    spec = PRIM_SPECS[case]
    g = {k.split("/", 1)[1]: v for k, v in PRIMS.items() if k.startswith(case + "/")}
    params = {"grid": g["grid"].astype(np.float64)} if spec["kind"] == "bspline" else None
    f = ko.prim_F(g["x"], g["c"], g["w"], spec, m, params)
    gg = ko.prim_G(g["x"], g["g"], g["w"], spec, m, params)
    p = ko.prim_P(g["x"], g["g"], g["c"], spec, m, params)
    for got, key in [(f, "F"), (gg, "G"), (p, "P")]:
        assert ko.max_rel_err(got, g[f"{key}{m}"]) < 2e-5, key


def test_parity_metric_matches_reference_definition():
    a = np.array([1.0, 2.0, 3.0])
    assert ko.max_rel_err(a, a) == 0.0
    assert ko.max_rel_err(a + 0.3, a) == pytest.approx(0.1)  # scaled by max|b| = 3
    assert ko.max_rel_err(np.array([0.1]), np.array([0.0])) == pytest.approx(0.1)  # floor of 1


def test_planted_oracle_mistake_is_caught():
    """A deliberately wrong oracle (B-spline without the half-open interval rule)
    disagrees with the golden vectors: the pin has teeth."""
    case = "bspline_5_3"
    spec = spec_of(BASES, case)
    x = BASES[f"{case}/x"].copy()
    params = params_of(BASES, case)
    good = ko.basis_eval(spec, x, 0, params)
    t = ko.extend_grid(params["grid"], 3)
    xe = x[..., None]
    b = ((xe >= t[..., :-1]) & (xe <= t[..., 1:])).astype(np.float64)  # closed intervals: wrong
    for q in range(1, 4):
        left = (xe - t[..., : -(q + 1)]) / (t[..., q:-1] - t[..., : -(q + 1)])
        right = (t[..., q + 1:] - xe) / (t[..., q + 1:] - t[..., 1:-q])
        b = left * b[..., :-1] + right * b[..., 1:]
    assert np.abs(b - BASES[f"{case}/d0"]).max() > 1e-3
    assert np.abs(good - BASES[f"{case}/d0"]).max() < 1e-12
