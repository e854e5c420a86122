"""What the kernels compute for a basis (reference kanforge/kernels/plan.py:39-121).

A ``KernelPlan`` names the features the CUDA kernels evaluate per input and how
derivatives are obtained:

* ``cheb``: every polynomial family with a tanh or identity input map is
  evaluated as Chebyshev features T_j(g(x)); the family matrix and the m-th
  x-derivative are *folded* into the coefficients, phi_k^(m) = sum_j R_m[k,j] T_j,
  so kernels never differentiate (kanforge/kernels/plan.py:75-101).
* ``bspline``: the derivative order is evaluated natively from the per-input grid.
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
from .bases import BSpline, PolynomialBasis, Rational

ONE_MINUS_Z2 = np.array([0.5, 0.0, -0.5])  # 1 - z^2 in the Chebyshev basis


@dataclass(frozen=True)
class KernelPlan:
    kind: str             # "cheb" | "bspline" | "rational"
    consts: tuple         # cheb: (degree, input_map); bspline: (grid_size, order); rational: (p, q)
    size: int             # basis functions per edge
    fold_key: tuple = ()  # cheb: the Chebyshev coefficient matrix, flattened
    grid: bool = False    # the kernels read the per-input grid

    @property
    def folded(self) -> bool:
        return self.kind == "cheb"

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
        return _fold(self.consts, self.fold_key, m)

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


def plan_for(basis) -> KernelPlan | None:
    """The kernel plan of ``basis``, or None when no kernel exists (plan.py:104-121)."""
    if isinstance(basis, PolynomialBasis) and basis.input_map in ("tanh", "identity"):
        return KernelPlan("cheb", (basis.degree, basis.input_map), basis.size, tuple(basis._cheb.ravel().tolist()))
    if type(basis) is BSpline:
        return KernelPlan("bspline", (basis.grid_size, basis.order), basis.size, grid=True)
    if type(basis) is Rational:
        return KernelPlan("rational", (basis.num_degree, basis.den_degree), 1)
    return None
