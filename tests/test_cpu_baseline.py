"""Pins the timed CPU baseline (oracle/cpu_baseline.py) to the reference.

The bench's CPU baseline and its ``--impl reference`` arm time
``cpu_baseline``, a float32 NumPy restatement of the reference's plain-ops
path.  These CPU tests check that restatement against the reference's own
float64 torch-ops outputs in ``tests/golden/layers.npz`` (forward and every
gradient of a weighted-sum loss) and against the float64 oracle, at float32
tolerance (metric max|a-b| / max(1, max|b|), reference tests/test_kernels.py:96-99).
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import load_golden

import cpu_baseline as cb
import kan_oracle as ko

LAYERS = load_golden("layers.npz")
TOL = 2e-5  # float32 arithmetic against float64 results


def err(a, b) -> float:
    return ko.max_rel_err(np.asarray(a, np.float64), np.asarray(b, np.float64))


def golden_state(case):
    pre = f"{case}/state/"
    return {k[len(pre):]: v for k, v in LAYERS.items() if k.startswith(pre)}


def features_for(case, st):
    f32 = np.float32
    if case.startswith("bspline"):
        grid = st["basis_grid"].astype(f32)
        k = st["coef"].shape[-1] - (grid.shape[1] - 1)
        return lambda v: cb.bspline_features(v, grid, k)
    if case == "chebyshev_12":
        return lambda v: cb.cheb_features(v, 12, None)
    if case == "jacobi_6":
        a = ko.cheb_matrix({"kind": "poly", "family": "jacobi", "degree": 6, "alpha": 0.5, "beta": 0.5})
        return lambda v: cb.cheb_features(v, 6, a)
    raise KeyError(case)


@pytest.mark.parametrize("case", ["bspline_5_3", "bspline_8_3", "chebyshev_12", "jacobi_6"])
def test_cpu_baseline_layer_step_matches_reference_golden(case):
    st = golden_state(case)
    f32 = np.float32
    scale = st["edge_mask"] * st.get("edge_scale", 1.0)
    coef = (st["coef"] * scale[..., None]).astype(f32)
    base = (st["base_weight"] * st["edge_mask"]).astype(f32)
    x = LAYERS[f"{case}/x"].astype(f32)
    dy = LAYERS[f"{case}/dy"].astype(f32)
    _, g = cb.kan_linear_step(x, coef, base, st["bias"].astype(f32), features_for(case, st), dy=dy)
    assert err(g["y"], LAYERS[f"{case}/y"]) <= TOL
    assert err(g["x"], LAYERS[f"{case}/grad/x"]) <= TOL
    assert err(g["coef"] * scale[..., None], LAYERS[f"{case}/grad/coef"]) <= TOL
    assert err(g["base_weight"] * st["edge_mask"], LAYERS[f"{case}/grad/base_weight"]) <= TOL
    assert err(g["bias"], LAYERS[f"{case}/grad/bias"]) <= TOL


@pytest.mark.parametrize("case", ["bspline_8_3", "chebyshev_12"])
def test_cpu_baseline_layer_step_matches_oracle_at_bench_distribution(case):
    """The bench's sample: x ~ N(0, 1) clipped to [-3, 3] (points outside the
    extended grid included), mean-square loss."""
    rng = np.random.default_rng(1)
    f32 = np.float32
    n_b, n_in, n_out = 64, 24, 16
    if case.startswith("bspline"):
        grid = np.broadcast_to(np.linspace(-1, 1, 9), (n_in, 9)).copy()
        spec, params, k = {"kind": "bspline", "grid_size": 8, "order": 3, "grid_range": (-1.0, 1.0)}, {"grid": grid}, 11
        feats = lambda v: cb.bspline_features(v, grid.astype(f32), 3)  # noqa: E731
    else:
        spec, params, k = {"kind": "poly", "family": "chebyshev", "degree": 12, "input_map": "tanh"}, {}, 13
        feats = lambda v: cb.cheb_features(v, 12, None)  # noqa: E731
    x = rng.standard_normal((n_b, n_in)).clip(-3, 3).astype(f32)
    coef = (rng.standard_normal((n_out, n_in, k)) / np.sqrt(n_in * k)).astype(f32)
    base = (rng.standard_normal((n_out, n_in)) / np.sqrt(n_in)).astype(f32)
    bias = (rng.standard_normal(n_out) * 0.1).astype(f32)
    loss, g = cb.kan_linear_step(x, coef, base, bias, feats)
    y = ko.kan_linear(x, coef, base, bias, spec, params)
    assert abs(loss - np.mean(y * y)) <= TOL * max(1.0, abs(np.mean(y * y)))
    want = ko.kan_linear_backward(x, 2 * y / y.size, coef, base, bias, spec, params)
    assert err(g["y"], y) <= TOL
    assert err(g["x"], want["dx"]) <= TOL
    assert err(g["coef"], want["dcoef"]) <= TOL
    assert err(g["base_weight"], want["dbase_weight"]) <= TOL
    assert err(g["bias"], want["dbias"]) <= TOL


def test_cpu_baseline_grkan_ffn_matches_oracle():
    rng = np.random.default_rng(2)
    f32 = np.float32
    n_b, d, h, groups = 40, 32, 64, 8
    a = np.array([0.0, 0.5, 0.3, 0.05, -0.01, 0.002])  # a GELU-like starting rational
    b = np.array([0.1, 0.2, 0.02, 0.01])

    def mk(i, o):
        return {"w": (rng.standard_normal((o, i)) / np.sqrt(i)).astype(f32), "b": (rng.standard_normal(o) * 0.1).astype(f32),
                "num": (np.tile(a, (groups, 1)) + 0.05 * rng.standard_normal((groups, 6))).astype(f32),
                "den": (np.tile(b, (groups, 1)) + 0.05 * rng.standard_normal((groups, 4))).astype(f32)}

    l1, l2 = mk(d, h), mk(h, d)
    x = (rng.standard_normal((n_b, d)) * 1.5).astype(f32)
    _, g = cb.grkan_ffn_step(x, l1, l2, groups)
    spec = {"kind": "rational", "num_degree": 5, "den_degree": 4}

    def params(l, n_in):
        return {"numerator": np.repeat(l["num"], n_in // groups, 0), "denominator": np.repeat(l["den"], n_in // groups, 0)}

    p1, p2 = params(l1, d), params(l2, h)
    hid = ko.kan_linear(x, l1["w"][..., None], None, l1["b"], spec, p1)
    y = ko.kan_linear(hid, l2["w"][..., None], None, l2["b"], spec, p2)
    assert err(g["y"], y) <= TOL
    b2 = ko.kan_linear_backward(hid, 2 * y / y.size, l2["w"][..., None], None, l2["b"], spec, p2, groups=groups)
    b1 = ko.kan_linear_backward(x, b2["dx"], l1["w"][..., None], None, l1["b"], spec, p1, groups=groups)
    assert err(g["x"], b1["dx"]) <= TOL
    assert err(g["w1"], b1["dcoef"][..., 0]) <= TOL
    assert err(g["w2"], b2["dcoef"][..., 0]) <= TOL


@pytest.mark.parametrize("order", [0, 1, 2])
def test_cpu_baseline_edge_derivative_matches_oracle(order):
    rng = np.random.default_rng(3)
    f32 = np.float32
    spec = {"kind": "poly", "family": "jacobi", "degree": 6, "input_map": "tanh", "alpha": 0.5, "beta": 0.5}
    n_b, n_in, n_out = 50, 16, 12
    x = rng.uniform(-1, 1, (n_b, n_in)).astype(f32)
    coef = (rng.standard_normal((n_out, n_in, 7)) * 0.3).astype(f32)
    base = (rng.standard_normal((n_out, n_in)) * 0.3).astype(f32)
    coef_fold = (coef.astype(np.float64) @ ko.fold(spec, order)).astype(f32)
    got = cb.edge_derivative_order(x, coef_fold, base, order)
    want = ko.edge_derivative(x, coef, base, spec, {}, order)
    assert err(got, want) <= TOL
