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


def chebyshev_gauss_nodes(n: int) -> np.ndarray:
    """The n zeros of T_n, cos(pi (m + 1/2) / n)."""
    return np.cos(np.pi * (np.arange(n) + 0.5) / n)


def chebyshev_projection(values: np.ndarray) -> np.ndarray:
    """Chebyshev coefficients (n, k) of k polynomials of degree < n from their
    values (n, k) at the n Chebyshev-Gauss nodes, by the discrete orthogonality
    of T_0 .. T_{n-1} on those nodes (exact for that degree: a DCT-II)."""
    n = values.shape[0]
    theta = np.pi * (np.arange(n) + 0.5) / n
    t = np.cos(np.outer(np.arange(n), theta))  # t[j, m] = T_j(node m)
    coef = (2.0 / n) * (t @ values)
    coef[0] *= 0.5
    return coef


def _convert_to_chebyshev(series_cls, degree: int) -> np.ndarray:
    """(degree+1, degree+1): column k = the Chebyshev coefficients of basis
    polynomial k of a numpy polynomial series class (exact conversion)."""
    out = np.zeros((degree + 1, degree + 1))
    for k in range(degree + 1):
        c = series_cls.basis(k).convert(kind=npcheb.Chebyshev).coef
        out[: len(c), k] = c
    return out


class PolynomialBasis(Basis):
    """family_k(z) = sum_j T_j(z) A[j, k] of z = g(x), g = tanh or identity
    (reference kanforge/bases/polynomial.py:30-111).  ``_cheb`` is A, built by
    each family from its definition; the kernels evaluate T_j(g(x)) and fold
    A and every derivative order into the coefficients."""

    default_input_map = "tanh"
    _is_chebyshev = False

    def __init__(self, degree: int = 5, input_map: str | None = None):
        if degree < 0:
            raise ValueError("degree must be >= 0")
        self.degree = int(degree)
        self.input_map = input_map or self.default_input_map
        if self.input_map not in INPUT_MAPS:
            raise ValueError(f"input_map must be one of {INPUT_MAPS}")

    @property
    def size(self) -> int:
        return self.degree + 1

    def family_values(self, z: np.ndarray) -> np.ndarray:
        """(len(z), degree + 1) values of the family at float64 points z."""
        raise NotImplementedError

    def _chebyshev_matrix(self) -> np.ndarray:
        return chebyshev_projection(self.family_values(chebyshev_gauss_nodes(self.degree + 1)))

    @cached_property
    def _cheb(self) -> np.ndarray:
        """A, (degree + 1, size)."""
        a = np.asarray(self._chebyshev_matrix(), dtype=np.float64)
        a.setflags(write=False)
        return a

    def param_specs(self):
        return {"exponent_logit": ParamSpec(np.zeros(1))} if self.input_map == "fractional" else {}

    def config(self):
        return {"name": self.name, "degree": self.degree, "input_map": self.input_map}

    def host_eval(self, x, params=None):
        x = np.asarray(x, dtype=np.float64)
        z = np.tanh(x) if self.input_map == "tanh" else x
        return np.moveaxis(npcheb.chebval(z, self._cheb), 0, -1)


class Chebyshev(PolynomialBasis):
    """T_n(tanh x) (ChebyKAN): A is the identity."""

    name = "chebyshev"
    _is_chebyshev = True

    def _chebyshev_matrix(self):
        return np.eye(self.degree + 1)


class Chebyshev2(PolynomialBasis):
    """Chebyshev polynomials of the second kind:
    U_n = 2 (T_n + T_{n-2} + ...) ending in T_1, or in T_0 counted once."""

    name = "chebyshev2"

    def _chebyshev_matrix(self):
        d = self.degree
        a = np.zeros((d + 1, d + 1))
        for n in range(d + 1):
            a[n % 2 : n + 1 : 2, n] = 2.0
            if n % 2 == 0:
                a[0, n] = 1.0
        return a


class Legendre(PolynomialBasis):
    name = "legendre"

    def _chebyshev_matrix(self):
        return _convert_to_chebyshev(np.polynomial.Legendre, self.degree)


class Jacobi(PolynomialBasis):
    """Jacobi polynomials P_n^(alpha, beta), P_n(1) = C(n + alpha, n), from the
    three-term recurrence P_{n+1} = (a_n z + b_n) P_n - c_n P_{n-1} (DLMF 18.9.2)."""

    name = "jacobi"

    def __init__(self, degree: int = 5, alpha: float = 1.0, beta: float = 1.0, input_map: str | None = None):
        if alpha <= -1 or beta <= -1:
            raise ValueError("alpha and beta must be > -1")
        super().__init__(degree, input_map)
        self.alpha, self.beta = float(alpha), float(beta)

    def family_values(self, z):
        al, be = self.alpha, self.beta
        out = np.empty(z.shape + (self.degree + 1,))
        out[..., 0] = 1.0
        if self.degree >= 1:
            out[..., 1] = 0.5 * (al - be) + 0.5 * (al + be + 2.0) * z
        for n in range(1, self.degree):
            s = 2.0 * n + al + be
            denom = 2.0 * (n + 1) * (n + al + be + 1) * s
            a_n = (s + 1) * (s + 2) * s / denom
            b_n = (s + 1) * (al * al - be * be) / denom
            c_n = 2.0 * (n + al) * (n + be) * (s + 2) / denom
            out[..., n + 1] = (a_n * z + b_n) * out[..., n] - c_n * out[..., n - 1]
        return out

    def config(self):
        return {**super().config(), "alpha": self.alpha, "beta": self.beta}


class Gegenbauer(PolynomialBasis):
    """Gegenbauer (ultraspherical) polynomials C_n^(lam):
    (n + 1) C_{n+1} = 2 (n + lam) z C_n - (n + 2 lam - 1) C_{n-1}."""

    name = "gegenbauer"

    def __init__(self, degree: int = 5, lam: float = 1.0, input_map: str | None = None):
        if lam <= -0.5 or lam == 0:
            raise ValueError("lam must be > -1/2 and non-zero")
        super().__init__(degree, input_map)
        self.lam = float(lam)

    def family_values(self, z):
        lam = self.lam
        out = np.empty(z.shape + (self.degree + 1,))
        out[..., 0] = 1.0
        if self.degree >= 1:
            out[..., 1] = 2.0 * lam * z
        for n in range(1, self.degree):
            out[..., n + 1] = (2.0 * (n + lam) * z * out[..., n] - (n + 2.0 * lam - 1.0) * out[..., n - 1]) / (n + 1)
        return out

    def config(self):
        return {**super().config(), "lam": self.lam}


class Hermite(PolynomialBasis):
    """Physicists' Hermite polynomials H_n."""

    name = "hermite"

    def _chebyshev_matrix(self):
        return _convert_to_chebyshev(np.polynomial.Hermite, self.degree)


class Laguerre(PolynomialBasis):
    name = "laguerre"

    def _chebyshev_matrix(self):
        return _convert_to_chebyshev(np.polynomial.Laguerre, self.degree)


class Bernstein(PolynomialBasis):
    """Bernstein polynomials C(n, j) t^j (1 - t)^(n - j) of t = (z + 1) / 2."""

    name = "bernstein"

    def family_values(self, z):
        n = self.degree
        t = 0.5 * (z + 1.0)
        j = np.arange(n + 1)
        binom = np.array([math.comb(n, k) for k in j], dtype=np.float64)
        return binom * t[..., None] ** j * (1.0 - t)[..., None] ** (n - j)


class Gram(PolynomialBasis):
    """Gram polynomials: orthonormal for the mean over ``points`` equally spaced
    points of [-1, 1] (mean of each square = 1), positive leading coefficient;
    built by Gram-Schmidt on z * p_k, carried on those points and the Chebyshev
    nodes together."""

    name = "gram"

    def __init__(self, degree: int = 5, points: int | None = None, input_map: str | None = None):
        super().__init__(degree, input_map)
        self.points = int(points) if points is not None else 2 * (self.degree + 1)
        if self.points <= self.degree:
            raise ValueError("points must be > degree")

    def _chebyshev_matrix(self):
        d, n_pts = self.degree, self.points
        z = np.concatenate([np.linspace(-1.0, 1.0, n_pts), chebyshev_gauss_nodes(d + 1)])
        mean = lambda f, g: float(np.dot(f[:n_pts], g[:n_pts])) / n_pts  # noqa: E731
        family = [np.ones_like(z)]
        for _ in range(d):
            q = z * family[-1]
            for _sweep in range(2):  # re-orthogonalise once for accuracy
                for p in family:
                    q = q - mean(q, p) * p
            family.append(q / math.sqrt(mean(q, q)))
        return chebyshev_projection(np.stack(family, -1)[n_pts:])

    def config(self):
        return {**super().config(), "points": self.points}


class Taylor(PolynomialBasis):
    """Monomials 1, x, ..., x^degree; identity input map by default."""

    name = "taylor"
    default_input_map = "identity"

    def _chebyshev_matrix(self):
        return _convert_to_chebyshev(np.polynomial.Polynomial, self.degree)


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


class _RationalLeastSquares:
    """Least-squares fit of R = P / (1 + |Q|) to samples (x_n, y_n): P of degree
    p (coefficients a_0..a_p), Q = sum_{j=1..q} b_j x^j; theta = (a, b)."""

    def __init__(self, xs: np.ndarray, ys: np.ndarray, p: int, q: int):
        self.ys = ys
        self.n_num = p + 1
        self.pow_num = xs[:, None] ** np.arange(p + 1)      # x^0 .. x^p
        self.pow_den = xs[:, None] ** np.arange(1, q + 1)   # x^1 .. x^q

    def linearised_start(self) -> np.ndarray:
        """theta minimising |P - y Q - y|: the fit of P = y (1 + Q), which a
        rational reaches exactly when it interpolates."""
        design = np.concatenate([self.pow_num, -self.ys[:, None] * self.pow_den], axis=1)
        return np.linalg.lstsq(design, self.ys, rcond=None)[0]

    def evaluate(self, theta):
        """(residual R - y, Q) at theta."""
        q = self.pow_den @ theta[self.n_num:]
        return (self.pow_num @ theta[: self.n_num]) / (1 + np.abs(q)) - self.ys, q

    def jacobian(self, theta, q):
        """dR/dtheta: x^j / D for a_j and -P sign(Q) x^j / D^2 for b_j, D = 1 + |Q|."""
        d = 1 + np.abs(q)
        p_val = self.pow_num @ theta[: self.n_num]
        return np.concatenate([self.pow_num / d[:, None], (-p_val / d**2 * np.sign(q))[:, None] * self.pow_den], axis=1)


@lru_cache(maxsize=None)
def fit_rational(target: str, num_degree: int, den_degree: int, lim: float = 3.0):
    """(a, b) of the rational P / (1 + |Q|) closest to ``target`` on [-lim, lim].

    The reference's initial fit (kanforge/bases/rational.py:27-61), whose
    steps are kept so the coefficients agree to rounding: samples at 2001
    evenly spaced points, the linearised least-squares start, then
    Levenberg-Marquardt with Marquardt's diagonal scaling (system
    J^T J + mu (diag(J^T J) + 1e-12)): mu starts at 1e-3, a step that lowers
    the squared residual is taken and divides mu by 3, a rejected one
    multiplies it by 4, and the search ends once mu exceeds 1e8 or after 200
    trials.  Exact for ``identity``.
    """
    xs = np.linspace(-lim, lim, 2001)
    ls = _RationalLeastSquares(xs, TARGETS[target](xs), num_degree, den_degree)
    theta = ls.linearised_start()
    resid, q = ls.evaluate(theta)
    mu, trials = 1e-3, 0
    while trials < 200 and mu <= 1e8:
        trials += 1
        jac = ls.jacobian(theta, q)
        normal = jac.T @ jac
        delta = np.linalg.solve(normal + mu * np.diag(np.diag(normal) + 1e-12), -(jac.T @ resid))
        cand_resid, cand_q = ls.evaluate(theta + delta)
        if cand_resid @ cand_resid < resid @ resid:
            theta, resid, q = theta + delta, cand_resid, cand_q
            mu /= 3
        else:
            mu *= 4
    return theta[: num_degree + 1].copy(), theta[num_degree + 1:].copy()


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


# ---------------------------------------------------------------------------
# periodic and bump bases (the reference's "fourier" and "bump" kernel plans)
# ---------------------------------------------------------------------------


class Fourier(Basis):
    """cos(w_j x), then sin(w_j x), w_j = 2 pi j / period, j = 1..frequencies
    (FourierKAN; the constant term is the layer bias), reference
    kanforge/bases/fourier.py:13-52.  ``learnable_frequency`` adds a trainable
    per-group frequency scale (no kernel plan then)."""

    name = "fourier"

    def __init__(self, frequencies: int = 5, period: float = 2 * math.pi, learnable_frequency: bool = False):
        if frequencies < 1 or not period > 0:
            raise ValueError("frequencies must be >= 1 and period > 0")
        self.frequencies = int(frequencies)
        self.period = float(period)
        self.learnable_frequency = bool(learnable_frequency)

    @property
    def size(self) -> int:
        return 2 * self.frequencies

    def param_specs(self):
        return {"frequency_scale": ParamSpec(np.ones(1))} if self.learnable_frequency else {}

    def config(self):
        return {"name": self.name, "frequencies": self.frequencies, "period": self.period,
                "learnable_frequency": self.learnable_frequency}

    def host_eval(self, x, params=None):
        w = (2.0 * math.pi / self.period) * np.arange(1, self.frequencies + 1)
        arg = np.asarray(x, dtype=np.float64)[..., None] * w
        return np.concatenate([np.cos(arg), np.sin(arg)], axis=-1)


def gaussian_bump_polys(p, max_order: int) -> list[np.ndarray]:
    """P_0 .. P_max_order with d^m/du^m [p(u) exp(-u^2/2)] = P_m(u) exp(-u^2/2):
    P_{m+1} = P_m' - u P_m."""
    out = [np.asarray(p, dtype=np.float64)]
    for _ in range(max_order):
        q = out[-1]
        out.append(np.polynomial.polynomial.polysub(np.polynomial.polynomial.polyder(q),
                                                    np.polynomial.polynomial.polymulx(q)))
    return out


def tanh_bump_polys(max_order: int) -> list[np.ndarray]:
    """P_0 .. P_max_order in t = tanh(v) with d^m/dv^m (1 - tanh(v)^2) = P_m(t):
    P_0 = 1 - t^2, P_{m+1} = P_m'(t) (1 - t^2)."""
    sech2 = np.array([1.0, 0.0, -1.0])
    out = [sech2]
    for _ in range(max_order):
        out.append(np.polynomial.polynomial.polymul(np.polynomial.polynomial.polyder(out[-1]), sech2))
    return out


class _Bump(Basis):
    """psi(u_scale (x - c_j) / h) on ``count`` centres spread over ``grid_range``,
    h = the centre spacing, psi(u) = norm p(u) exp(-u^2/2) (reference
    kanforge/bases/radial.py:35-74).  Fixed centres are a per-input grid
    buffer; ``learnable`` centres and width are trainable (no kernel plan)."""

    p: tuple = (1.0,)
    norm = 1.0
    u_scale = 1.0

    def __init__(self, count: int = 8, grid_range: tuple[float, float] = (-1.0, 1.0), learnable: bool = False):
        if count < 2:
            raise ValueError("count must be >= 2")
        self.count = int(count)
        self.grid_range = _check_range(grid_range)
        self.learnable = bool(learnable)

    @property
    def size(self) -> int:
        return self.count

    def param_specs(self):
        lo, hi = self.grid_range
        centres = np.linspace(lo, hi, self.count)
        if not self.learnable:
            return {"grid": ParamSpec(centres, trainable=False)}
        return {"centers": ParamSpec(centres), "log_scale": ParamSpec(np.array([math.log((hi - lo) / (self.count - 1))]))}

    def config(self) -> dict[str, Any]:
        return {"name": self.name, "count": self.count, "grid_range": self.grid_range, "learnable": self.learnable}

    def host_eval(self, x, params=None):
        c = np.linspace(*self.grid_range, self.count) if params is None else np.asarray(params["grid"])
        k = self.u_scale * (self.count - 1) / (c[..., -1:] - c[..., :1])
        u = (np.asarray(x, dtype=np.float64)[..., None] - c) * k
        return self.norm * np.polynomial.polynomial.polyval(u, np.asarray(self.p)) * np.exp(-0.5 * u * u)


class RBF(_Bump):
    """Gaussian RBF exp(-((x - c) / h)^2) on a uniform grid of centres (FastKAN)."""

    name = "rbf"
    u_scale = math.sqrt(2.0)


class MexicanHat(_Bump):
    """Mexican-hat wavelet 2 / (sqrt(3) pi^(1/4)) (1 - u^2) exp(-u^2 / 2)."""

    name = "mexican_hat"
    p = (1.0, 0.0, -1.0)
    norm = 2.0 / (math.sqrt(3.0) * math.pi**0.25)

    def __init__(self, count: int = 8, grid_range: tuple[float, float] = (-1.0, 1.0), learnable: bool = True):
        super().__init__(count, grid_range, learnable)


class DoG(_Bump):
    """Derivative-of-Gaussian wavelet -u exp(-u^2 / 2)."""

    name = "dog"
    p = (0.0, -1.0)

    def __init__(self, count: int = 8, grid_range: tuple[float, float] = (-1.0, 1.0), learnable: bool = True):
        super().__init__(count, grid_range, learnable)


class RSWAF(Basis):
    """Reflectional switch activation 1 - tanh((x - c) / h)^2 on a uniform grid
    of centres, h = their spacing (FasterKAN), reference kanforge/bases/radial.py:120-147."""

    name = "rswaf"

    def __init__(self, count: int = 8, grid_range: tuple[float, float] = (-1.0, 1.0)):
        if count < 2:
            raise ValueError("count must be >= 2")
        self.count = int(count)
        self.grid_range = _check_range(grid_range)

    @property
    def size(self) -> int:
        return self.count

    def param_specs(self):
        return {"grid": ParamSpec(np.linspace(*self.grid_range, self.count), trainable=False)}

    def config(self):
        return {"name": self.name, "count": self.count, "grid_range": self.grid_range}

    def host_eval(self, x, params=None):
        c = np.linspace(*self.grid_range, self.count) if params is None else np.asarray(params["grid"])
        h = (c[..., -1:] - c[..., :1]) / (self.count - 1)
        return 1.0 - np.tanh((np.asarray(x, dtype=np.float64)[..., None] - c) / h) ** 2


__all__ = [
    "BASES",
    "Basis",
    "BSpline",
    "Bernstein",
    "Chebyshev",
    "Chebyshev2",
    "DoG",
    "Fourier",
    "MexicanHat",
    "RBF",
    "RSWAF",
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
