"""Pin the oracle's grid tools (adaptive quantile grid, resampling, samples,
least-squares refit) against ``tests/golden/grid.npz``, which the reference's
own kanforge/grid.py and float32 torch layers wrote (update_grid, refine_grid,
change_basis: kanforge/_layer.py:148-183)."""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import load_golden

import kan_oracle as ko

GRID = load_golden("grid.npz")
REFITS = sorted({k.split("/")[1] for k in GRID if k.startswith("refit/")})
LAYER_OPS = sorted({k.split("/")[1] for k in GRID if k.startswith("layer/") and k.count("/") > 1})


def _cfg(key):
    return json.loads(str(GRID[key]))


def _sub(prefix):
    return {k[len(prefix):]: v for k, v in GRID.items() if k.startswith(prefix)}


@pytest.mark.parametrize("case", sorted({k.split("/")[1] for k in GRID if k.startswith("adaptive/") and k.endswith("/args")}))
def test_adaptive_grid_bit_exact(case):
    n, margin, eps = GRID[f"adaptive/{case}/args"]
    got = ko.adaptive_grid(GRID["adaptive/x"], int(n), margin, eps)
    assert np.array_equal(got, GRID[f"adaptive/{case}/grid"])


def test_adaptive_grid_single_sample_and_bad_eps():
    assert np.array_equal(ko.adaptive_grid(GRID["adaptive/x1"], 5), GRID["adaptive/x1/grid"])
    with pytest.raises(ValueError):
        ko.adaptive_grid(GRID["adaptive/x"], 5, grid_eps=0.0)


@pytest.mark.parametrize("n", [5, 9, 17, 33])
def test_resample_and_samples_bit_exact(n):
    assert np.array_equal(ko.resample_grid(GRID["resample/grid"], n), GRID[f"resample/{n}"])
    assert np.array_equal(ko.sample_inputs(GRID["samples/ranges"], 100), GRID["samples/100"])


@pytest.mark.parametrize("case", REFITS)
def test_refit_matches_reference(case):
    pre = f"refit/{case}/"
    old = ko.spec_from_config(_cfg(pre + "old_config"))
    new = ko.spec_from_config(_cfg(pre + "new_config"))
    got = ko.refit(old, _sub(pre + "old/"), GRID[pre + "coef"], new, _sub(pre + "new/"), GRID[pre + "x"],
                   float(GRID[pre + "ridge"]))
    want = GRID[pre + "out"]
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-9 * max(1.0, np.abs(want).max()))


def _grid_params(state):
    return {k[len("basis_"):]: v.astype(np.float64) for k, v in state.items() if k.startswith("basis_")}


@pytest.mark.parametrize("case", LAYER_OPS)
def test_layer_grid_tools_match_reference(case):
    """Recompute the reference layer's new coefficients from its state before
    the call: the float64 solution rounds to the reference's float32 values."""
    before, after = _sub(f"layer/{case}/before/state/"), _sub(f"layer/{case}/after/state/")
    old = ko.spec_from_config(_cfg(f"layer/{case}/before/config"))
    new = ko.spec_from_config(_cfg(f"layer/{case}/after/config"))
    x = GRID["layer/x"].astype(np.float64)
    old_p, new_p = _grid_params(before), _grid_params(after)
    new_size = ko.basis_size(new)
    if case.startswith("update"):
        n_points = before["basis_grid"].shape[-1]
        kw = {"margin": 0.05, "grid_eps": 0.2} if case.endswith("margin") else {}
        grid = ko.adaptive_grid(x, n_points, **kw)
        np.testing.assert_array_equal(grid.astype(np.float32), after["basis_grid"])
        new_p = {"grid": grid}
        xs = x
    elif case.startswith("refine"):
        grid = ko.resample_grid(old_p["grid"], after["basis_grid"].shape[-1])
        np.testing.assert_array_equal(grid.astype(np.float32), after["basis_grid"])
        new_p = {"grid": grid}
        xs = x if case.endswith("_x") else ko.sample_inputs(np.stack([old_p["grid"][:, 0], old_p["grid"][:, -1]], -1),
                                                            8 * new_size + 64)
    else:
        if case.endswith("_x"):
            xs = x
        else:
            g = old_p["grid"]
            xs = ko.sample_inputs(np.stack([g[:, 0], g[:, -1]], -1), 8 * max(new_size, ko.basis_size(old)) + 64)
        if "grid" in new_p and "grid" in old_p:  # the new grid spans each input's old range
            g = old_p["grid"]
            new_p = {"grid": g[:, :1] + (g[:, -1:] - g[:, :1]) * np.linspace(0, 1, new_p["grid"].shape[-1])}
            np.testing.assert_array_equal(new_p["grid"].astype(np.float32), after["basis_grid"])
    ridge = 0.01 if case.endswith("margin") else 0.0
    coef, scale = ko.refit_layer(old, old_p, before["coef"], before.get("edge_scale"), new, new_p, xs, ridge)
    np.testing.assert_allclose(coef.astype(np.float32), after["coef"], rtol=2e-6, atol=2e-6)
    if scale is not None:
        np.testing.assert_array_equal(scale.astype(np.float32), after["edge_scale"])


def test_kan_update_grid_feeds_each_layer_its_inputs():
    """KAN.update_grid (kanforge/torch/layers.py:389-393): layer 0 adapts to x,
    layer 1 to layer 0's output after its update."""
    x = GRID["kan/x"].astype(np.float64)
    grid0 = ko.adaptive_grid(x, GRID["kan/before/0/basis_grid"].shape[-1])
    np.testing.assert_array_equal(grid0.astype(np.float32), GRID["kan/after/0/basis_grid"])
    a0 = _sub("kan/after/0/")
    spec = {"kind": "bspline", "grid_size": 5, "order": 3, "grid_range": (-1.0, 1.0)}
    h = ko.kan_linear(x.astype(np.float32), a0["coef"], a0["base_weight"], a0["bias"], spec,
                      {"grid": a0["basis_grid"].astype(np.float64)}, a0.get("edge_scale"), a0["edge_mask"])
    grid1 = ko.adaptive_grid(h, GRID["kan/before/1/basis_grid"].shape[-1])
    np.testing.assert_allclose(grid1, GRID["kan/after/1/basis_grid"], rtol=0, atol=1e-5)
