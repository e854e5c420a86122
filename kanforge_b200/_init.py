"""Initial values of a KAN layer's parameters (host side, float64, run once).

The quantities the reference layer draws at construction
(kanforge/_layer.py:18-83), computed here from their definitions:

* parameter groups: ``None`` means one group per input, otherwise the count
  must divide the inputs;
* the basis state: trainable basis parameters once per group, buffers (the
  B-spline grids) once per input, a grid optionally respread uniformly over a
  per-input range with the same number of knots;
* coefficient / base-weight standard deviations for the named schemes, which
  need E[sum_b B_b(Z)^2] and E[silu(Z)^2] for Z ~ N(0, 1): both are taken with
  the 96-point Gauss-Hermite rule of the normal density (the reference's
  quadrature, so the standard deviations agree to rounding);
* the polynomials in sigmoid(x) of silu's derivatives, for edge_derivative.

Nothing here runs in a forward or backward pass.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from functools import lru_cache

import numpy as np
from numpy.polynomial import hermite_e
from numpy.polynomial import polynomial as npoly

from .bases import Basis

COEF_INITS = ("normal", "zero", "variance", "lecun", "glorot")
QUADRATURE_POINTS = 96


def resolve_groups(in_features: int, groups: int | None) -> int:
    """Number of basis-parameter groups of a layer with ``in_features`` inputs."""
    n = in_features if groups is None else groups
    if n < 1 or in_features % n != 0:
        raise ValueError(f"groups={groups} must divide in_features={in_features}")
    return n


@dataclass
class BasisState:
    """Initial basis tensors of a layer: trainable (groups, *shape), buffers (in, *shape)."""

    trainable: dict[str, np.ndarray] = field(default_factory=dict)
    buffers: dict[str, np.ndarray] = field(default_factory=dict)


def _uniform_grids(ranges, n_inputs: int, n_knots: int) -> np.ndarray:
    """(n_inputs, n_knots) knots spread evenly over each input's [lo, hi]:
    lo + (hi - lo) t, t = linspace(0, 1, n_knots), the reference's rounding
    (kanforge/_layer.py:40-42)."""
    lo_hi = np.broadcast_to(np.asarray(ranges, dtype=np.float64), (n_inputs, 2))
    frac = np.linspace(0.0, 1.0, n_knots)
    return lo_hi[:, 0:1] + (lo_hi[:, 1:2] - lo_hi[:, 0:1]) * frac


def initial_basis_state(basis: Basis, groups: int, in_features: int, grid_ranges=None) -> BasisState:
    """The basis tensors a new layer registers (reference kanforge/_layer.py:27-44)."""
    state = BasisState()
    grids = set(basis.grid_names())
    for name, spec in basis.param_specs().items():
        rows, target = (groups, state.trainable) if spec.trainable else (in_features, state.buffers)
        value = np.array(np.broadcast_to(np.asarray(spec.value, dtype=np.float64), (rows, *spec.shape)))
        if not spec.trainable and grid_ranges is not None and name in grids:
            value = _uniform_grids(grid_ranges, in_features, spec.shape[-1])
        target[name] = value
    return state


@lru_cache(maxsize=None)
def _normal_rule(points: int = QUADRATURE_POINTS) -> tuple[np.ndarray, np.ndarray]:
    """Nodes and weights with sum(w f(z)) ~ E[f(Z)], Z ~ N(0, 1)."""
    z, w = hermite_e.hermegauss(points)
    return z, w / math.sqrt(2.0 * math.pi)


def normal_expectation(fn) -> float:
    """E[fn(Z)] for Z ~ N(0, 1); fn maps (n,) nodes to (n,) values."""
    z, w = _normal_rule()
    return float(np.dot(w, fn(z)))


def basis_second_moment(basis: Basis) -> float:
    """E[sum_b B_b(Z)^2], Z ~ N(0, 1), at the basis' default parameters."""
    return normal_expectation(lambda z: np.square(basis.host_eval(z)).sum(axis=-1))


@lru_cache(maxsize=None)
def silu_second_moment() -> float:
    """E[silu(Z)^2], Z ~ N(0, 1)."""
    return normal_expectation(lambda z: np.square(z / (1.0 + np.exp(-z))))


def init_stds(basis: Basis, in_features: int, out_features: int, coef_init: str, coef_init_std: float, has_base: bool):
    """(coef std, base-weight std or None) for a coefficient scheme; None means
    torch's default kaiming-uniform base weight (reference kanforge/_layer.py:61-83).

    normal:   coef_init_std / sqrt(in)
    zero:     0 (the layer starts as its base branch)
    variance: unit output variance from the spline branch alone
    lecun / glorot: unit output variance for N(0, 1) inputs, half from each
              branch when the base branch exists, fan = in or (in + out) / 2
    """
    if coef_init not in COEF_INITS:
        raise ValueError(f"coef_init must be one of {COEF_INITS}")
    if coef_init in ("normal", "zero"):
        return (coef_init_std / math.sqrt(in_features) if coef_init == "normal" else 0.0), None
    moment = max(basis_second_moment(basis), 1e-12)
    if coef_init == "variance":
        return 1.0 / math.sqrt(in_features * moment), None
    fan = float(in_features) if coef_init == "lecun" else 0.5 * (in_features + out_features)
    branch_share = 0.5 if has_base else 1.0
    coef_std = math.sqrt(branch_share / (fan * moment))
    base_std = math.sqrt(branch_share / (fan * silu_second_moment())) if has_base else None
    return coef_std, base_std


def silu_derivative_polys(m: int, n: int = 8) -> np.ndarray:
    """[h_m, h_{m-1}] as polynomials in s = sigmoid(x), n coefficients each, with
    silu^(m)(x) = x h_m(s) + m h_{m-1}(s) (kanforge/_calculus.py:35-44, 90-96)."""
    polys = [np.array([0.0, 1.0])]
    factor = np.array([0.0, 1.0, -1.0])  # s - s^2
    for _ in range(max(m, 1)):
        polys.append(npoly.polymul(npoly.polyder(polys[-1]), factor))
    out = np.zeros((2, n))
    if m >= 1:
        hm, hm1 = polys[m], polys[m - 1]
        if len(hm) > n or len(hm1) > n:
            raise ValueError(f"silu derivative of order {m} needs more than {n} coefficients")
        out[0, : len(hm)] = hm
        out[1, : len(hm1)] = hm1
    return out
