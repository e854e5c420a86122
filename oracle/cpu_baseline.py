"""CPU baseline of the KANLinear step -- TEST / BENCHMARK INFRASTRUCTURE ONLY.

A float32 NumPy restatement of the reference's plain-ops path
(kanforge/torch/layers.py:184-191 forward, autograd of the same graph
backward): materialise the basis tensor (B, I, K), one GEMM against the
coefficients, the SiLU base GEMM and the bias; backward through the same
graph.  ``bench.py`` times it on the GPU box's host cores as the CPU baseline
and as the ``--impl reference`` arm (the reference is Python and cannot travel
to the box; this port of its algorithm can).  NumPy's BLAS uses every host
thread.
"""

from __future__ import annotations

import os
import time

import numpy as np
from numpy.polynomial import chebyshev as npcheb


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _dsilu(x):
    s = 1.0 / (1.0 + np.exp(-x))
    return s * (1.0 + x * (1.0 - s))


def cheb_features(x, degree, a_mat):
    """phi (B, I, K) and dphi/dx of family polynomials of tanh(x) (polynomial.py:87-106)."""
    z = np.tanh(x)
    t = [np.ones_like(z), z]
    dt = [np.zeros_like(z), np.ones_like(z)]
    for _ in range(2, degree + 1):
        t.append(2 * z * t[-1] - t[-2])
        dt.append(2 * t[-2] + 2 * z * dt[-1] - dt[-2])
    t = np.stack(t[: degree + 1], -1)
    dt = np.stack(dt[: degree + 1], -1) * (1 - z * z)[..., None]
    if a_mat is not None:
        t, dt = t @ a_mat, dt @ a_mat
    return t.astype(np.float32), dt.astype(np.float32)


def bspline_features(x, grid, k):
    """phi and dphi/dx of order-k B-splines on per-input grids (spline.py:74-92)."""
    h = (grid[:, -1:] - grid[:, :1]) / (grid.shape[1] - 1)
    steps = np.arange(k, dtype=np.float32)
    t = np.concatenate([grid[:, :1] - h * (k - steps), grid, grid[:, -1:] + h * (steps + 1)], 1).astype(np.float32)
    xe = x[..., None]
    b = ((xe >= t[:, :-1]) & (xe < t[:, 1:])).astype(np.float32)
    for q in range(1, k):
        b = (xe - t[:, : -(q + 1)]) / (t[:, q:-1] - t[:, : -(q + 1)]) * b[..., :-1] + (t[:, q + 1:] - xe) / (
            t[:, q + 1:] - t[:, 1:-q]) * b[..., 1:]
    n = b.shape[-1] - 1
    db = k * (b[..., :-1] / (t[:, k: k + n] - t[:, :n]) - b[..., 1:] / (t[:, k + 1: k + 1 + n] - t[:, 1: 1 + n]))
    q = k
    phi = (xe - t[:, : -(q + 1)]) / (t[:, q:-1] - t[:, : -(q + 1)]) * b[..., :-1] + (t[:, q + 1:] - xe) / (
        t[:, q + 1:] - t[:, 1:-q]) * b[..., 1:]
    return phi.astype(np.float32), db.astype(np.float32)


def kan_linear_step(x, coef, base_w, bias, feats, dy=None):
    """One fwd+bwd of loss = mean(y^2), or of sum(dy * y) when dy is given;
    returns (loss, grads) with grads["y"] the forward output."""
    bsz, n_in = x.shape
    n_out = coef.shape[0]
    phi, dphi = feats(x)
    y = phi.reshape(bsz, -1) @ coef.reshape(n_out, -1).T
    if base_w is not None:
        y += _silu(x) @ base_w.T
    if bias is not None:
        y += bias
    if dy is None:
        loss = float(np.mean(y * y))
        dy = (2.0 / y.size) * y
    else:
        loss = float(np.sum(dy * y))
    dphi_in = (dy @ coef.reshape(n_out, -1)).reshape(bsz, n_in, -1)
    dx = (dphi_in * dphi).sum(-1)
    dcoef = (dy.T @ phi.reshape(bsz, -1)).reshape(coef.shape)
    grads = {"x": dx, "coef": dcoef, "y": y}
    if base_w is not None:
        dx += (dy @ base_w) * _dsilu(x)
        grads["base_weight"] = dy.T @ _silu(x)
    if bias is not None:
        grads["bias"] = dy.sum(0)
    return loss, grads


def rational_features(x, num, den, groups):
    """R(x) per group and R'(x) (rational.py:84-101), float32."""
    ipg = x.shape[1] // groups
    a = np.repeat(num, ipg, axis=0)
    b = np.repeat(den, ipg, axis=0)
    p = np.zeros_like(x) + a[:, -1]
    dp = np.zeros_like(x)
    for j in range(a.shape[1] - 2, -1, -1):
        dp = dp * x + p
        p = p * x + a[:, j]
    qs = np.zeros_like(x) + b[:, -1]
    dqs = np.zeros_like(x)
    for j in range(b.shape[1] - 2, -1, -1):
        dqs = dqs * x + qs
        qs = qs * x + b[:, j]
    q = x * qs
    dq = qs + x * dqs
    d = 1 + np.abs(q)
    r = p / d
    dr = (dp - np.sign(q) * dq * r) / d
    return r[..., None].astype(np.float32), dr[..., None].astype(np.float32)


def grkan_ffn_step(x, l1, l2, groups):
    """fwd+bwd of fc2(fc1(x)) with GR-KAN layers (transformer.py:25-52), loss = mean(y^2)."""
    r1, dr1 = rational_features(x, l1["num"], l1["den"], groups)
    h = r1[..., 0] @ l1["w"].T + l1["b"]
    r2, dr2 = rational_features(h, l2["num"], l2["den"], groups)
    y = r2[..., 0] @ l2["w"].T + l2["b"]
    loss = float(np.mean(y * y))
    dy = (2.0 / y.size) * y
    dw2 = dy.T @ r2[..., 0]
    dh = (dy @ l2["w"]) * dr2[..., 0]
    dw1 = dh.T @ r1[..., 0]
    dx = (dh @ l1["w"]) * dr1[..., 0]
    return loss, {"x": dx, "w1": dw1, "w2": dw2, "y": y}


def edge_derivative_order(x, coef_fold, base_w, m):
    """(B, O, I) edge derivatives from folded Chebyshev coefficients, float32."""
    z = np.tanh(x)
    t = npcheb.chebvander(z, coef_fold.shape[-1] - 1).astype(np.float32)
    out = np.einsum("bij,oij->boi", t, coef_fold, optimize=True)
    s = 1 / (1 + np.exp(-x))
    if m == 2:
        sm = x * (1 - 2 * s) * (s - s * s) + 2 * (s - s * s)
    elif m == 1:
        sm = x * (s - s * s) + s
    else:
        sm = _silu(x)
    return out + sm[:, None, :] * base_w


def host_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def time_steps(step, warmup: int, steps: int) -> float:
    """Median seconds per call after warm-up (the reference's timing method,
    benchmarks/bench_kernels.py:19-29)."""
    for _ in range(warmup):
        step()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))
