"""Layer parameter layout and initialisation (reference kanforge/_layer.py:18-83).

Host-side float64 statistics used once at construction; nothing here runs in
the forward or backward pass.
"""

from __future__ import annotations

import math

import numpy as np

from .bases import Basis

COEF_INITS = ("normal", "zero", "variance", "lecun", "glorot")


def resolve_groups(in_features: int, groups: int | None) -> int:
    """Parameter groups: None = one group per input (_layer.py:18-24)."""
    if groups is None:
        return in_features
    if groups < 1 or in_features % groups:
        raise ValueError(f"groups={groups} must divide in_features={in_features}")
    return groups


def basis_param_values(basis: Basis, groups: int, in_features: int, grid_ranges=None):
    """Initial basis state: trainable (groups, *shape), buffers (in, *shape) (_layer.py:27-44)."""
    trainable, buffers = {}, {}
    for name, spec in basis.param_specs().items():
        if spec.trainable:
            trainable[name] = np.broadcast_to(spec.value, (groups, *spec.shape)).copy()
            continue
        value = np.broadcast_to(spec.value, (in_features, *spec.shape)).astype(np.float64)
        if grid_ranges is not None and name in basis.grid_names():
            r = np.broadcast_to(np.asarray(grid_ranges, dtype=np.float64), (in_features, 2))
            value = r[:, :1] + (r[:, 1:] - r[:, :1]) * np.linspace(0, 1, spec.shape[-1])
        buffers[name] = value.copy()
    return trainable, buffers


def _gauss_hermite(points: int = 96):
    """Probabilists' Gauss-Hermite rule normalised to the N(0, 1) density."""
    x, w = np.polynomial.hermite_e.hermegauss(points)
    return x, w / math.sqrt(2 * math.pi)


def basis_second_moment(basis: Basis) -> float:
    """E[sum_b B_b(x)^2], x ~ N(0, 1), default parameters (_layer.py:52-55)."""
    x, w = _gauss_hermite()
    return float(w @ (basis.host_eval(x) ** 2).sum(-1))


def _silu_np(x):
    return x / (1.0 + np.exp(-x))


SILU_SECOND_MOMENT = float(_gauss_hermite()[1] @ _silu_np(_gauss_hermite()[0]) ** 2)


def init_stds(basis: Basis, in_features: int, out_features: int, coef_init: str, coef_init_std: float, has_base: bool):
    """(coef std, base weight std or None for kaiming-uniform) (_layer.py:61-83)."""
    if coef_init not in COEF_INITS:
        raise ValueError(f"coef_init must be one of {COEF_INITS}")
    if coef_init == "normal":
        return coef_init_std / math.sqrt(in_features), None
    if coef_init == "zero":
        return 0.0, None
    m2 = max(basis_second_moment(basis), 1e-12)
    if coef_init == "variance":
        return 1.0 / math.sqrt(in_features * m2), None
    fan = in_features if coef_init == "lecun" else (in_features + out_features) / 2
    share = 0.5 if has_base else 1.0
    return math.sqrt(share / (fan * m2)), (math.sqrt(share / (fan * SILU_SECOND_MOMENT)) if has_base else None)


def silu_derivative_polys(m: int, n: int = 8) -> np.ndarray:
    """[h_m, h_{m-1}] as polynomials in s = sigmoid(x), n coefficients each, with
    silu^(m)(x) = x h_m(s) + m h_{m-1}(s) (kanforge/_calculus.py:35-44, 90-96)."""
    p = np.polynomial.polynomial
    polys = [np.array([0.0, 1.0])]
    factor = np.array([0.0, 1.0, -1.0])  # s - s^2
    for _ in range(max(m, 1)):
        polys.append(p.polymul(p.polyder(polys[-1]), factor))
    out = np.zeros((2, n))
    if m >= 1:
        hm, hm1 = polys[m], polys[m - 1]
        if len(hm) > n or len(hm1) > n:
            raise ValueError(f"silu derivative of order {m} needs more than {n} coefficients")
        out[0, : len(hm)] = hm
        out[1, : len(hm1)] = hm1
    return out
