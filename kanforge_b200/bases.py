"""Edge-function bases of the KAN layer hot path (host side).

These classes carry the configuration, the per-input / per-group parameter
specs and the float64 host algebra the kernels need (Chebyshev coefficient
matrices, rational initial fits, initialisation moments).  Evaluation on
tensors happens only in the CUDA kernels of ``libkanb200``.

Names, constructor arguments, ``size``, ``param_specs`` and ``config`` follow
the reference (kanforge/bases/base.py:48-128, spline.py:33-92,
polynomial.py:30-262, rational.py:27-104) so that models, state dicts and
``.npz`` files carry over unchanged.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from functools import cached_property, lru_cache
from typing import Any

import numpy as np
from numpy.polynomial import chebyshev as npcheb
from numpy.polynomial import hermite as nphermite
from numpy.polynomial import laguerre as nplaguerre
from numpy.polynomial import legendre as nplegendre


@dataclass(frozen=True)
class ParamSpec:
    """Default value of one basis parameter for a single input (bases/base.py:29-42).

    ``trainable=False`` marks state such as grids: one buffer row per input.
    """

    value: np.ndarray
    trainable: bool = True

    @property
    def shape(self) -> tuple[int, ...]:
        return np.shape(self.value)


BASES: dict[str, type[Basis]] = {}


class Basis:
    """A family of edge functions phi(x) = sum_b c_b B_b(x; theta)."""

    name: str = ""
    local: bool = False

    def __init_subclass__(cls, **kwargs):
        super().__init_subclass__(**kwargs)
        if cls.__dict__.get("name"):
            BASES[cls.name] = cls

    @property
    def size(self) -> int:
        raise NotImplementedError

    @property
    def support(self) -> int:
        return self.size

    def param_specs(self) -> dict[str, ParamSpec]:
        return {}

    def grid_names(self) -> list[str]:
        return [k for k, s in self.param_specs().items() if not s.trainable and k.endswith("grid")]

    def config(self) -> dict[str, Any]:
        raise NotImplementedError

    def host_eval(self, x: np.ndarray, params: dict | None = None) -> np.ndarray:
        """Order-0 values (..., size) at float64 points; used only for initialisation statistics."""
        raise NotImplementedError

    def __repr__(self) -> str:
        args = ", ".join(f"{k}={v!r}" for k, v in self.config().items() if k != "name")
        return f"{type(self).__name__}({args})"

    def __eq__(self, other) -> bool:
        return isinstance(other, Basis) and self.config() == other.config()

    def __hash__(self) -> int:
        return hash(repr(self.config()))

    @classmethod
    def from_config(cls, cfg: dict) -> Basis:
        cfg = {k: tuple(v) if k == "grid_range" else v for k, v in cfg.items()}
        return cls(**cfg)


def _check_range(grid_range) -> tuple[float, float]:
    lo, hi = float(grid_range[0]), float(grid_range[1])
    if not hi > lo:
        raise ValueError("grid_range must be increasing")
    return lo, hi


def make_basis(spec: str | dict | Basis = "bspline", **kwargs) -> Basis:
    """A basis from a name, a ``config()`` dict or an instance (bases/base.py:112-128)."""
    if isinstance(spec, Basis):
        if kwargs:
            raise TypeError("kwargs are not allowed with a Basis instance")
        return spec
    if isinstance(spec, dict):
        spec = dict(spec)
        name = spec.pop("name")
        cls = BASES.get(name)
        if cls is None:
            raise ValueError(f"unknown basis {name!r}; available: {sorted(BASES)}")
        return cls.from_config({**spec, **kwargs})
    cls = BASES.get(spec)
    if cls is None:
        raise ValueError(f"unknown basis {spec!r}; available: {sorted(BASES)}")
    return cls(**kwargs)


# ---------------------------------------------------------------------------
# B-splines
# ---------------------------------------------------------------------------


def extend_grid_np(grid: np.ndarray, k: int) -> np.ndarray:
    """``k`` extra knots per side at the mean grid step (spline.py:22-30)."""
    grid = np.asarray(grid, dtype=np.float64)
    if k == 0:
        return grid
    h = (grid[..., -1:] - grid[..., :1]) / (grid.shape[-1] - 1)
    steps = np.arange(k, dtype=np.float64)
    return np.concatenate([grid[..., :1] - h * (k - steps), grid, grid[..., -1:] + h * (steps + 1)], -1)


class BSpline(Basis):
    """B-splines of ``order`` on ``grid_size`` intervals of a per-input grid.

    ``grid_size + order`` functions; zero outside the extended grid
    (spline.py:199-228).  The grid is a per-input buffer (I, grid_size + 1).
    """

    name = "bspline"
    local = True

    def __init__(self, grid_size: int = 5, order: int = 3, grid_range: tuple[float, float] = (-1.0, 1.0)):
        if grid_size < 1 or order < 0:
            raise ValueError("grid_size must be >= 1 and order >= 0")
        self.grid_size = int(grid_size)
        self.order = int(order)
        self.grid_range = _check_range(grid_range)

    @property
    def size(self) -> int:
        return self.grid_size + self.order

    @property
    def support(self) -> int:
        return self.order + 1

    def param_specs(self):
        return {"grid": ParamSpec(np.linspace(*self.grid_range, self.grid_size + 1), trainable=False)}

    def config(self):
        return {"name": self.name, "grid_size": self.grid_size, "order": self.order, "grid_range": self.grid_range}

    def host_eval(self, x, params=None):
        grid = np.linspace(*self.grid_range, self.grid_size + 1) if params is None else params["grid"]
        t = extend_grid_np(grid, self.order)
        xe = np.asarray(x, dtype=np.float64)[..., None]
        b = ((xe >= t[..., :-1]) & (xe < t[..., 1:])).astype(np.float64)
        for q in range(1, self.order + 1):
            b = (xe - t[..., : -(q + 1)]) / (t[..., q:-1] - t[..., : -(q + 1)]) * b[..., :-1] + (t[..., q + 1:] - xe) / (
                t[..., q + 1:] - t[..., 1:-q]
            ) * b[..., 1:]
        return b


# ---------------------------------------------------------------------------
# polynomial families as Chebyshev coefficient matrices
# ---------------------------------------------------------------------------

INPUT_MAPS = ("tanh", "identity", "fractional")


class PolynomialBasis(Basis):
    """family_k(z) = sum_j T_j(z) A[j, k] of z = g(x), g = tanh or identity
    (polynomial.py:30-111).  The kernels evaluate T_j(g(x)); A and every
    derivative order are folded into the coefficients."""

    default_input_map = "tanh"
    _is_chebyshev = False

    def __init__(self, degree: int = 5, input_map: str | None = None):
        if degree < 0:
            raise ValueError("degree must be >= 0")
        input_map = input_map or self.default_input_map
        if input_map not in INPUT_MAPS:
            raise ValueError(f"input_map must be one of {INPUT_MAPS}")
        self.degree = int(degree)
        self.input_map = input_map

    @property
    def size(self) -> int:
        return self.degree + 1

    def _family(self, z: np.ndarray) -> np.ndarray:
        raise NotImplementedError

    @cached_property
    def _cheb(self) -> np.ndarray:
        """Chebyshev coefficients (D+1, size): interpolation at the D+1 Chebyshev nodes."""
        d = self.degree
        nodes = np.cos(np.pi * (np.arange(d + 1) + 0.5) / (d + 1))
        return np.linalg.solve(npcheb.chebvander(nodes, d), self._family(nodes))

    def param_specs(self):
        if self.input_map == "fractional":
            return {"exponent_logit": ParamSpec(np.zeros(1))}
        return {}

    def config(self):
        return {"name": self.name, "degree": self.degree, "input_map": self.input_map}

    def host_eval(self, x, params=None):
        x = np.asarray(x, dtype=np.float64)
        z = np.tanh(x) if self.input_map == "tanh" else x
        return npcheb.chebvander(z, self.degree) @ self._cheb


class Chebyshev(PolynomialBasis):
    """T_n(tanh x) (ChebyKAN)."""

    name = "chebyshev"
    _is_chebyshev = True

    def _family(self, z):
        return npcheb.chebvander(z, self.degree)


class Chebyshev2(PolynomialBasis):
    """Chebyshev polynomials of the second kind U_n."""

    name = "chebyshev2"

    def _family(self, z):
        u = [np.ones_like(z), 2 * z]
        for _ in range(2, self.degree + 1):
            u.append(2 * z * u[-1] - u[-2])
        return np.stack(u[: self.degree + 1], -1)


class Legendre(PolynomialBasis):
    name = "legendre"

    def _family(self, z):
        return nplegendre.legvander(z, self.degree)


class Jacobi(PolynomialBasis):
    """Jacobi polynomials P_n^(alpha, beta) by their three-term recurrence."""

    name = "jacobi"

    def __init__(self, degree: int = 5, alpha: float = 1.0, beta: float = 1.0, input_map: str | None = None):
        if alpha <= -1 or beta <= -1:
            raise ValueError("alpha and beta must be > -1")
        super().__init__(degree, input_map)
        self.alpha, self.beta = float(alpha), float(beta)

    def _family(self, z):
        a, b = self.alpha, self.beta
        vals = [np.ones_like(z), (a + 1) + (a + b + 2) * (z - 1) / 2]
        for n in range(2, self.degree + 1):
            c = 2 * n + a + b
            num = (c - 1) * (c * (c - 2) * z + a * a - b * b) * vals[-1] - 2 * (n + a - 1) * (n + b - 1) * c * vals[-2]
            vals.append(num / (2 * n * (n + a + b) * (c - 2)))
        return np.stack(vals[: self.degree + 1], -1)

    def config(self):
        return {**super().config(), "alpha": self.alpha, "beta": self.beta}


class Gegenbauer(PolynomialBasis):
    """Gegenbauer polynomials C_n^(lam)."""

    name = "gegenbauer"

    def __init__(self, degree: int = 5, lam: float = 1.0, input_map: str | None = None):
        if lam <= -0.5 or lam == 0:
            raise ValueError("lam must be > -1/2 and non-zero")
        super().__init__(degree, input_map)
        self.lam = float(lam)

    def _family(self, z):
        lam = self.lam
        vals = [np.ones_like(z), 2 * lam * z]
        for n in range(2, self.degree + 1):
            vals.append((2 * z * (n + lam - 1) * vals[-1] - (n + 2 * lam - 2) * vals[-2]) / n)
        return np.stack(vals[: self.degree + 1], -1)

    def config(self):
        return {**super().config(), "lam": self.lam}


class Hermite(PolynomialBasis):
    """Physicists' Hermite polynomials H_n."""

    name = "hermite"

    def _family(self, z):
        return nphermite.hermvander(z, self.degree)


class Laguerre(PolynomialBasis):
    name = "laguerre"

    def _family(self, z):
        return nplaguerre.lagvander(z, self.degree)


class Bernstein(PolynomialBasis):
    """C(n, j) t^j (1 - t)^(n - j) of t = (z + 1) / 2."""

    name = "bernstein"

    def _family(self, z):
        t, n = (z + 1) / 2, self.degree
        return np.stack([math.comb(n, j) * t**j * (1 - t) ** (n - j) for j in range(n + 1)], -1)


class Gram(PolynomialBasis):
    """Polynomials orthonormal on ``points`` equally spaced points of [-1, 1]."""

    name = "gram"

    def __init__(self, degree: int = 5, points: int | None = None, input_map: str | None = None):
        super().__init__(degree, input_map)
        self.points = int(points) if points is not None else 2 * (self.degree + 1)
        if self.points <= self.degree:
            raise ValueError("points must be > degree")

    @cached_property
    def _cheb(self):
        grid = np.linspace(-1, 1, self.points)
        _q, r = np.linalg.qr(npcheb.chebvander(grid, self.degree))
        sign = np.sign(np.diag(r))
        return np.linalg.inv(r) * sign * math.sqrt(self.points)

    def config(self):
        return {**super().config(), "points": self.points}


class Taylor(PolynomialBasis):
    """Monomials 1, x, ..., x^degree; identity input map by default."""

    name = "taylor"
    default_input_map = "identity"

    def _family(self, z):
        return np.stack([z**j for j in range(self.degree + 1)], -1)


# ---------------------------------------------------------------------------
# KAT group rational
# ---------------------------------------------------------------------------


def _erf(x):
    return np.vectorize(math.erf)(x)


TARGETS = {
    "identity": lambda x: x,
    "silu": lambda x: x / (1 + np.exp(-x)),
    "gelu": lambda x: 0.5 * x * (1 + _erf(x / math.sqrt(2))),
    "tanh": np.tanh,
}


@lru_cache(maxsize=None)
def fit_rational(target: str, num_degree: int, den_degree: int, lim: float = 3.0):
    """(a, b) of P/(1+|Q|) fitting ``target`` on [-lim, lim] (rational.py:27-61).

    Start from the linear least-squares solution of P - f Q = f, then
    Levenberg-Marquardt on the true residual (damping x1/3 on success, x4 on
    failure, stop above 1e8, at most 200 iterations).
    """
    f = TARGETS[target]
    xs = np.linspace(-lim, lim, 2001)
    ys = f(xs)
    vp = xs[:, None] ** np.arange(num_degree + 1)
    vq = xs[:, None] ** np.arange(1, den_degree + 1)
    theta = np.linalg.lstsq(np.hstack([vp, -ys[:, None] * vq]), ys, rcond=None)[0]
    damping = 1e-3
    npar = num_degree + 1

    def resid(th):
        s = vq @ th[npar:]
        return (vp @ th[:npar]) / (1 + np.abs(s)) - ys, s

    r, s = resid(theta)
    for _ in range(200):
        den = 1 + np.abs(s)
        num = vp @ theta[:npar]
        jac = np.hstack([vp / den[:, None], (-num / den**2 * np.sign(s))[:, None] * vq])
        grad = jac.T @ r
        jtj = jac.T @ jac
        step = np.linalg.solve(jtj + damping * np.diag(np.diag(jtj) + 1e-12), -grad)
        r_new, s_new = resid(theta + step)
        if r_new @ r_new < r @ r:
            theta, r, s, damping = theta + step, r_new, s_new, damping / 3
        else:
            damping *= 4
        if damping > 1e8:
            break
    return theta[:npar].copy(), theta[npar:].copy()


class Rational(Basis):
    """P(x) / (1 + |Q(x)|), size 1, trainable numerator / denominator (rational.py:64-104)."""

    name = "rational"

    def __init__(self, num_degree: int = 5, den_degree: int = 4, init: str = "silu"):
        if num_degree < 0 or den_degree < 1:
            raise ValueError("num_degree must be >= 0 and den_degree >= 1")
        if init not in TARGETS:
            raise ValueError(f"init must be one of {sorted(TARGETS)}")
        self.num_degree = int(num_degree)
        self.den_degree = int(den_degree)
        self.init = init

    @property
    def size(self) -> int:
        return 1

    def param_specs(self):
        a, b = fit_rational(self.init, self.num_degree, self.den_degree)
        return {"numerator": ParamSpec(a), "denominator": ParamSpec(b)}

    def config(self):
        return {"name": self.name, "num_degree": self.num_degree, "den_degree": self.den_degree, "init": self.init}

    def host_eval(self, x, params=None):
        if params is None:
            a, b = fit_rational(self.init, self.num_degree, self.den_degree)
        else:
            a, b = params["numerator"], params["denominator"]
        x = np.asarray(x, dtype=np.float64)
        p = np.polynomial.polynomial.polyval(x, np.asarray(a))
        q = x * np.polynomial.polynomial.polyval(x, np.asarray(b))
        return (p / (1 + np.abs(q)))[..., None]


__all__ = [
    "BASES",
    "Basis",
    "BSpline",
    "Bernstein",
    "Chebyshev",
    "Chebyshev2",
    "Gegenbauer",
    "Gram",
    "Hermite",
    "Jacobi",
    "Laguerre",
    "Legendre",
    "ParamSpec",
    "PolynomialBasis",
    "Rational",
    "Taylor",
    "fit_rational",
    "make_basis",
]
