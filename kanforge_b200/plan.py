"""What the kernels compute for a basis (reference kanforge/kernels/plan.py:39-121).

A ``KernelPlan`` names the features the CUDA kernels evaluate per input and how
derivatives are obtained:

* ``cheb``: every polynomial family with a tanh or identity input map is
  evaluated as Chebyshev features T_j(g(x)); the family matrix and the m-th
  x-derivative are *folded* into the coefficients, phi_k^(m) = sum_j R_m[k,j] T_j,
  so kernels never differentiate (kanforge/kernels/plan.py:75-101).
* ``fourier``: cos / sin features of the harmonics; the m-th derivative of
  every feature is a rotation of its (cos, sin) pair scaled by w^m, folded into
  the coefficients like ``cheb`` (kanforge/kernels/plan.py:76-87);
* ``bspline``: the derivative order is evaluated natively from the per-input grid.
* ``bump``: RBF / wavelet / RSWAF bumps on a per-input grid of centres,
  natively at every order from derivative polynomials (plan.py:33-73, 112-120).
* ``rational``: the KAT group rational; trainable per-group parameters, so the
  reference has no fused plan for it (plan.py:107-108).  This package runs it on
  its own elementwise kernels plus the layer contraction.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
from numpy.polynomial import chebyshev as npcheb

from . import _lib
from .bases import RBF, RSWAF, BSpline, DoG, Fourier, MexicanHat, PolynomialBasis, Rational, gaussian_bump_polys, tanh_bump_polys

ONE_MINUS_Z2 = np.array([0.5, 0.0, -0.5])  # 1 - z^2 in the Chebyshev basis


@dataclass(frozen=True)
class KernelPlan:
    kind: str             # "cheb" | "fourier" | "bspline" | "bump" | "rational"
    consts: tuple         # cheb: (degree, input_map); fourier: (frequencies, period); bspline: (grid_size, order);
                          # bump: (mode, count, u_scale, norm, p); rational: (p, q)
    size: int             # basis functions per edge
    fold_key: tuple = ()  # cheb: the Chebyshev coefficient matrix, flattened
    grid: bool = False    # the kernels read the per-input grid

    @property
    def folded(self) -> bool:
        return self.kind in ("cheb", "fourier")

    def n_features(self, m: int) -> int:
        """Features evaluated for derivative order m (plan.py:52-56)."""
        if self.kind == "cheb":
            d, input_map = self.consts
            return d + 1 + m if input_map == "tanh" else d + 1
        return self.size

    def native_order(self, m: int) -> int:
        return 0 if self.folded else m

    def fold(self, m: int) -> np.ndarray | None:
        """R_m (size, n_features(m)) for folded plans, else None."""
        if not self.folded:
            return None
        if self.kind == "fourier":
            return _fourier_fold(self.consts, m)
        return _fold(self.consts, self.fold_key, m)

    def bump_poly(self, m: int) -> np.ndarray:
        """Coefficients (lowest first) of the bump's m-th derivative polynomial:
        in u for gauss bumps, in tanh for RSWAF."""
        mode, _count, _u_scale, _norm, p = self.consts
        return (gaussian_bump_polys(p, m) if mode == "gauss" else tanh_bump_polys(m))[m]

    def is_identity_fold(self) -> bool:
        """R_0 is the identity (plain Chebyshev): the coefficients need no fold."""
        if not self.folded:
            return True
        r = self.fold(0)
        return r.shape[0] == r.shape[1] and bool(np.allclose(r, np.eye(r.shape[0]), rtol=0.0, atol=1e-12))

    def desc(self, groups: int = 1) -> _lib.BasisDesc:
        """The ``kf_basis_desc`` of this plan."""
        d = _lib.BasisDesc()
        d.size = self.size
        d.groups = groups
        if self.kind == "cheb":
            d.kind = _lib.KF_BASIS_CHEB
            d.degree = self.consts[0]
            d.input_map = _lib.KF_MAP_TANH if self.consts[1] == "tanh" else _lib.KF_MAP_IDENTITY
        elif self.kind == "bspline":
            d.kind = _lib.KF_BASIS_BSPLINE
            d.grid_size, d.order = self.consts
        elif self.kind == "fourier":
            d.kind = _lib.KF_BASIS_FOURIER
            d.degree, d.period = self.consts
        elif self.kind == "bump":
            d.kind = _lib.KF_BASIS_BUMP
            mode, _count, d.u_scale, d.norm, _p = self.consts
            d.bump_mode = _lib.KF_BUMP_GAUSS if mode == "gauss" else _lib.KF_BUMP_TANH
            for m in range(_lib.KF_BUMP_MAX_ORDER + 1):
                poly = self.bump_poly(m)
                if len(poly) > 8:
                    raise ValueError(f"bump derivative polynomial of order {m} has more than 8 coefficients")
                for e, v in enumerate(poly):
                    d.bump_poly[m][e] = float(v)
        else:
            d.kind = _lib.KF_BASIS_RATIONAL
            d.degree, d.den_degree = self.consts
        return d

    def supported(self, op: int, dtype: int) -> bool:
        d = self.desc()
        return bool(_lib.load().kf_query(ctypes.byref(d), op, dtype))


@lru_cache(maxsize=None)
def _fold(consts, fold_key, m):
    d, input_map = consts
    a = np.asarray(fold_key, dtype=np.float64).reshape(d + 1, -1)
    n_t = d + 1 + m if input_map == "tanh" else d + 1
    cols = []
    for k in range(a.shape[1]):
        col = a[:, k]
        for _ in range(m):
            col = npcheb.chebder(col) if len(col) > 1 else np.zeros(1)
            if input_map == "tanh":  # d/dx T(tanh x) = T'(z) (1 - z^2)
                col = npcheb.chebmul(col, ONE_MINUS_Z2)
        out = np.zeros(n_t)
        out[: min(len(col), n_t)] = col[:n_t]
        cols.append(out)
    r = np.stack(cols)
    r.setflags(write=False)
    return r


@lru_cache(maxsize=None)
def _fourier_fold(consts, m):
    """R_m (2n, 2n): cos(w x)^(m) = w^m (cos(m pi/2) cos(w x) - sin(m pi/2) sin(w x)),
    sin(w x)^(m) = w^m (sin(m pi/2) cos(w x) + cos(m pi/2) sin(w x))."""
    n, period = consts
    wm = (2.0 * np.pi / period * np.arange(1, n + 1)) ** m
    c, s = (1.0, 0.0, -1.0, 0.0)[m % 4], (0.0, 1.0, 0.0, -1.0)[m % 4]
    eye = np.eye(n)
    r = np.block([[eye * (wm * c), eye * (-wm * s)], [eye * (wm * s), eye * (wm * c)]])
    r.setflags(write=False)
    return r


def plan_for(basis) -> KernelPlan | None:
    """The kernel plan of ``basis``, or None when no kernel exists (plan.py:104-121)."""
    if isinstance(basis, PolynomialBasis) and basis.input_map in ("tanh", "identity"):
        return KernelPlan("cheb", (basis.degree, basis.input_map), basis.size, tuple(basis._cheb.ravel().tolist()))
    if type(basis) is BSpline:
        return KernelPlan("bspline", (basis.grid_size, basis.order), basis.size, grid=True)
    if type(basis) is Rational:
        return KernelPlan("rational", (basis.num_degree, basis.den_degree), 1)
    if any(spec.trainable for spec in basis.param_specs().values()):
        return None  # learnable frequencies / centres: no kernel plan (plan.py:107-108)
    if type(basis) is Fourier:
        return KernelPlan("fourier", (basis.frequencies, basis.period), basis.size)
    if type(basis) in (RBF, MexicanHat, DoG):
        return KernelPlan("bump", ("gauss", basis.count, basis.u_scale, basis.norm, tuple(basis.p)), basis.size, grid=True)
    if type(basis) is RSWAF:
        return KernelPlan("bump", ("tanh", basis.count, 1.0, 1.0, (1.0, 0.0, -1.0)), basis.size, grid=True)
    return None
