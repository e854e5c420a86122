"""Generate the golden fixtures in this folder by running the REFERENCE package.

    KANFORGE_REFERENCE=/path/to/kanforge TRITON_INTERPRET=1 python tests/golden/make_golden.py [names]

Imports fx-xf/kanforge v0.8.0 from the directory in ``KANFORGE_REFERENCE`` and
records, on small seeded inputs:

* ``bases.npz``    -- ``Basis.derivative(x, m, params)`` for every hot-path basis,
                      orders 0..3 (kanforge/bases/*.py), and the fold matrices
                      ``KernelPlan.fold(m)`` (kanforge/kernels/plan.py:75-101);
* ``layers.npz``   -- torch ``KANLinear`` (backend="ops", float64) forward, the
                      gradients of a weighted-sum loss into the input and every
                      parameter, and ``edge_derivative`` orders 0..2
                      (kanforge/torch/layers.py:171-226);
* ``prims.npz``    -- the reference Triton primitives F_m/G_m/P_m run by the
                      Triton CPU interpreter (kanforge/torch/kernels.py:131-140);
* ``init.npz``     -- ``fit_rational`` coefficients, basis second moments and
                      ``init_stds`` (kanforge/bases/rational.py:27-61, _layer.py:47-83);
* ``ref_model.npz`` + ``ref_model_io.npz`` -- a model file written by
                      ``kanforge.save`` and its outputs (kanforge/convert.py:313-325);
* ``grid.npz``     -- the grid tools: ``adaptive_grid``, ``resample_grid``,
                      ``sample_inputs``, ``refit`` (kanforge/grid.py) and float32
                      layers before and after ``update_grid`` / ``refine_grid`` /
                      ``change_basis`` (kanforge/_layer.py:148-183).

Pass file names (``bases layers prims init model_file grid``) to regenerate a subset.

The fixtures are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = os.environ.get("KANFORGE_REFERENCE")
if not REF:
    sys.exit("set KANFORGE_REFERENCE to the directory that holds the reference's kanforge package")
sys.path.insert(0, REF)
os.environ.setdefault("TRITON_INTERPRET", "1")

import kanforge as kf  # noqa: E402
import torch  # noqa: E402

from kanforge.kernels import plan_for  # noqa: E402

# (name, reference basis, oracle spec)
BASIS_CASES = [
    ("bspline_5_3", kf.BSpline(5, 3), {"kind": "bspline", "grid_size": 5, "order": 3, "grid_range": (-1.0, 1.0)}),
    ("bspline_5_3_r2", kf.BSpline(5, 3, (-2.0, 2.0)), {"kind": "bspline", "grid_size": 5, "order": 3, "grid_range": (-2.0, 2.0)}),
    ("bspline_8_3", kf.BSpline(8, 3), {"kind": "bspline", "grid_size": 8, "order": 3, "grid_range": (-1.0, 1.0)}),
    ("bspline_4_1", kf.BSpline(4, 1), {"kind": "bspline", "grid_size": 4, "order": 1, "grid_range": (-1.0, 1.0)}),
    ("bspline_3_2", kf.BSpline(3, 2), {"kind": "bspline", "grid_size": 3, "order": 2, "grid_range": (-1.0, 1.0)}),
    ("chebyshev_5", kf.Chebyshev(5), {"kind": "poly", "family": "chebyshev", "degree": 5, "input_map": "tanh"}),
    ("chebyshev_12", kf.Chebyshev(12), {"kind": "poly", "family": "chebyshev", "degree": 12, "input_map": "tanh"}),
    ("chebyshev_4_id", kf.Chebyshev(4, input_map="identity"), {"kind": "poly", "family": "chebyshev", "degree": 4, "input_map": "identity"}),
    ("jacobi_6", kf.Jacobi(6, 0.5, 0.5), {"kind": "poly", "family": "jacobi", "degree": 6, "alpha": 0.5, "beta": 0.5, "input_map": "tanh"}),
    ("jacobi_4", kf.Jacobi(4, 0.5, 1.5), {"kind": "poly", "family": "jacobi", "degree": 4, "alpha": 0.5, "beta": 1.5, "input_map": "tanh"}),
    ("legendre_4_id", kf.Legendre(4, input_map="identity"), {"kind": "poly", "family": "legendre", "degree": 4, "input_map": "identity"}),
    ("gegenbauer_5", kf.Gegenbauer(5, 0.75), {"kind": "poly", "family": "gegenbauer", "degree": 5, "lam": 0.75, "input_map": "tanh"}),
    ("taylor_3", kf.Taylor(3), {"kind": "poly", "family": "taylor", "degree": 3, "input_map": "identity"}),
    ("rational_gelu", kf.Rational(5, 4, "gelu"), {"kind": "rational", "num_degree": 5, "den_degree": 4}),
    ("rational_identity", kf.Rational(5, 4, "identity"), {"kind": "rational", "num_degree": 5, "den_degree": 4}),
    ("fourier_3", kf.Fourier(3), {"kind": "fourier", "frequencies": 3, "period": 2 * np.pi}),
    ("fourier_4_p3", kf.Fourier(4, 3.0), {"kind": "fourier", "frequencies": 4, "period": 3.0}),
    ("rbf_6", kf.RBF(6), {"kind": "bump", "family": "rbf", "count": 6, "grid_range": (-1.0, 1.0)}),
    ("mexican_hat_5", kf.MexicanHat(5, learnable=False),
     {"kind": "bump", "family": "mexican_hat", "count": 5, "grid_range": (-1.0, 1.0)}),
    ("dog_5", kf.DoG(5, (-2.0, 2.0), learnable=False), {"kind": "bump", "family": "dog", "count": 5, "grid_range": (-2.0, 2.0)}),
    ("rswaf_6", kf.RSWAF(6), {"kind": "bump", "family": "rswaf", "count": 6, "grid_range": (-1.0, 1.0)}),
]


def perturbed(basis, n_in, seed):
    rng = np.random.default_rng(seed)
    out = {}
    for name, spec in basis.param_specs().items():
        v = np.broadcast_to(spec.value, (n_in, *spec.shape)).astype(np.float64)
        if name == "grid":  # keep knots increasing: jitter the interior only
            jit = 0.15 * (v[:, 1:] - v[:, :-1]).min() * rng.uniform(-1, 1, v.shape)
            jit[:, 0] = jit[:, -1] = 0.0
            v = v + jit
        else:
            v = v + 0.05 * rng.standard_normal(v.shape)
        out[name] = v
    return out


def make_bases():
    rec = {}
    n_in = 3
    for ci, (name, basis, spec) in enumerate(BASIS_CASES):
        rng = np.random.default_rng(100 + ci)
        lo, hi = spec.get("grid_range", (-1.0, 1.0))
        x = rng.uniform(1.6 * lo, 1.6 * hi, (24, n_in))
        params = perturbed(basis, n_in, 200 + ci)
        if spec["kind"] == "bspline":
            # exact knots and points outside the extended grid (half-open intervals)
            knots = kf.bases.spline.extend_grid(params["grid"], spec["order"])
            x[0] = knots[np.arange(n_in), 1]
            x[1] = knots[np.arange(n_in), spec["order"] + 1]
            x[2] = knots[:, -1]
            x[3] = knots[:, 0] - 0.01
        rec[f"{name}/spec"] = np.array(json.dumps(spec))
        rec[f"{name}/x"] = x
        for k, v in params.items():
            rec[f"{name}/param/{k}"] = v
        for m in range(4):
            rec[f"{name}/d{m}"] = np.asarray(basis.derivative(x, m, params))
        plan = plan_for(basis)
        if plan is not None and plan.folded:
            if plan.kind == "cheb":
                rec[f"{name}/cheb"] = basis._cheb
            for m in range(4):
                rec[f"{name}/fold{m}"] = plan.fold(m)
    np.savez_compressed(HERE / "bases.npz", **rec)


LAYER_CASES = [
    # name, basis, n_in, n_out, groups, base, edge_scale, x-range
    ("bspline_5_3", kf.BSpline(5, 3), 4, 3, None, True, True, 1.4),
    ("bspline_8_3", kf.BSpline(8, 3), 5, 4, None, True, False, 2.5),
    ("chebyshev_12", kf.Chebyshev(12), 4, 3, None, True, True, 2.0),
    ("jacobi_6", kf.Jacobi(6, 0.5, 0.5), 4, 5, None, True, False, 1.0),
    ("chebyshev_4_id_nobase", kf.Chebyshev(4, input_map="identity"), 3, 2, None, False, True, 0.9),
    ("rational_gelu_g2", kf.Rational(5, 4, "gelu"), 4, 3, 2, False, False, 2.5),
    ("rational_identity_g1", kf.Rational(5, 4, "identity"), 4, 2, 1, False, True, 2.0),
    ("fourier_3", kf.Fourier(3), 4, 3, None, True, True, 2.5),
    ("rbf_6", kf.RBF(6), 4, 3, None, True, False, 1.4),
    ("mexican_hat_5", kf.MexicanHat(5, learnable=False), 3, 4, None, False, True, 1.2),
    ("rswaf_6", kf.RSWAF(6), 4, 2, None, True, False, 1.3),
]


def make_layers():
    from kanforge.torch import KANLinear

    rec = {}
    for ci, (name, basis, n_in, n_out, groups, base, scale, xr) in enumerate(LAYER_CASES):
        torch.manual_seed(10 + ci)
        kw = {"groups": groups, "edge_scale": scale, "backend": "ops", "dtype": torch.float64}
        if not base:
            kw["base_activation"] = None
        layer = KANLinear(n_in, n_out, basis, **kw)
        with torch.no_grad():
            for p in layer.parameters():
                p.add_(0.1 * torch.randn_like(p))
            mask = torch.ones_like(layer.edge_mask)
            mask[0, -1] = 0.0  # one pruned edge
            layer.edge_mask.copy_(mask)
        if hasattr(layer, "basis_grid"):
            x_fit = torch.randn(200, n_in, dtype=torch.float64) * 0.5
            layer.update_grid(x_fit)  # non-uniform per-input grids
        x = (torch.rand(9, n_in, dtype=torch.float64) * 2 - 1) * xr
        x.requires_grad_(True)
        y = layer(x)
        wts = torch.linspace(-1, 1, n_out, dtype=torch.float64)
        loss = (y * wts).sum()
        names = [n for n, _ in layer.named_parameters()]
        grads = torch.autograd.grad(loss, [x] + [p for _, p in layer.named_parameters()])
        rec[f"{name}/x"] = x.detach().numpy()
        rec[f"{name}/y"] = y.detach().numpy()
        rec[f"{name}/dy"] = wts.expand_as(y).numpy()
        rec[f"{name}/grad/x"] = grads[0].numpy()
        for n, g in zip(names, grads[1:]):
            rec[f"{name}/grad/{n}"] = g.numpy()
        for n, t in list(layer.named_parameters()) + list(layer.named_buffers()):
            rec[f"{name}/state/{n}"] = t.detach().numpy()
        rec[f"{name}/groups"] = np.array(layer.groups)
        with torch.no_grad():
            for m in range(3):
                rec[f"{name}/edge{m}"] = layer.edge_derivative(x.detach(), m).numpy()
    np.savez_compressed(HERE / "layers.npz", **rec)


PRIM_CASES = [("bspline_5_3", kf.BSpline(5, 3)), ("chebyshev_5", kf.Chebyshev(5)), ("jacobi_4", kf.Jacobi(4, 0.5, 1.5)),
              ("fourier_3", kf.Fourier(3)), ("rbf_6", kf.RBF(6)), ("dog_5", kf.DoG(5, learnable=False)),
              ("rswaf_6", kf.RSWAF(6))]


def make_prims():
    from kanforge.torch import kernels as tk

    rec = {}
    for ci, (name, basis) in enumerate(PRIM_CASES):
        plan = plan_for(basis)
        torch.manual_seed(50 + ci)
        n_b, n_in, n_out, size = 13, 3, 4, basis.size
        x = torch.rand(n_b, n_in) * 1.8 - 0.9
        w = torch.rand(n_b, n_in) + 0.5
        g = torch.randn(n_b, n_out)
        c = torch.randn(n_out, n_in, size) * 0.5
        grid = torch.as_tensor(perturbed(basis, n_in, 300 + ci).get("grid", np.zeros((1,))), dtype=torch.float32)
        rec[f"{name}/x"], rec[f"{name}/w"], rec[f"{name}/g"], rec[f"{name}/c"] = x.numpy(), w.numpy(), g.numpy(), c.numpy()
        rec[f"{name}/grid"] = grid.numpy()
        with torch.no_grad():
            for m in range(3):
                rec[f"{name}/F{m}"] = tk.prim_F(x, c, w, grid, plan, m).numpy()
                rec[f"{name}/G{m}"] = tk.prim_G(x, g, w, grid, plan, m).numpy()
                rec[f"{name}/P{m}"] = tk.prim_P(x, g, c, grid, plan, m).numpy()
    np.savez_compressed(HERE / "prims.npz", **rec)


def make_init():
    from kanforge._layer import basis_second_moment, init_stds
    from kanforge.bases.rational import fit_rational

    rec = {}
    for target in ("identity", "gelu", "silu", "tanh"):
        a, b = fit_rational(target, 5, 4)
        rec[f"fit/{target}/num"], rec[f"fit/{target}/den"] = a, b
    for name, basis, _spec in BASIS_CASES:
        rec[f"m2/{name}"] = np.array(basis_second_moment(basis))
    cases = [
        ("lecun_bspline_5_3_r2", kf.BSpline(5, 3, (-2.0, 2.0)), 2, 5, "lecun", True),
        ("glorot_chebyshev_12", kf.Chebyshev(12), 7, 3, "glorot", True),
        ("variance_rational_gelu", kf.Rational(5, 4, "gelu"), 768, 3072, "variance", False),
        ("normal_bspline_8_3", kf.BSpline(8, 3), 1024, 1024, "normal", True),
    ]
    for key, basis, n_in, n_out, how, base in cases:
        c, b = init_stds(basis, n_in, n_out, how, 0.1, base)
        rec[f"std/{key}"] = np.array([c, np.nan if b is None else b])
    np.savez_compressed(HERE / "init.npz", **rec)


def make_model_file():
    from kanforge.torch import KAN

    torch.manual_seed(3)
    model = KAN([2, 3, 1], kf.BSpline(4, 3), dtype=torch.float64)
    model[0].update_grid(torch.randn(100, 2, dtype=torch.float64) * 0.4)
    kf.save(model, HERE / "ref_model.npz")
    x = torch.rand(6, 2, dtype=torch.float64) * 1.6 - 0.8
    with torch.no_grad():
        y = model(x)
    np.savez(HERE / "ref_model_io.npz", x=x.numpy(), y=y.numpy())


GRID_REFITS = [
    # name, old basis, new basis (None = same basis on an adaptive grid), ridge, with edge_scale
    ("bspline_adapt", kf.BSpline(5, 3), None, 0.0, False),
    ("bspline_adapt_ridge", kf.BSpline(5, 3), None, 0.1, True),
    ("bspline_to_cheb", kf.BSpline(5, 3), kf.Chebyshev(8), 0.0, False),
    ("bspline_refine", kf.BSpline(4, 2), kf.BSpline(9, 2), 0.0, True),
    ("rbf_adapt", kf.RBF(6), None, 0.0, False),
    ("cheb_to_legendre", kf.Chebyshev(4), kf.Legendre(6, input_map="identity"), 0.0, False),
    ("fourier_to_bspline", kf.Fourier(2), kf.BSpline(6, 3), 0.01, False),
    ("rswaf_to_mexican_hat", kf.RSWAF(5), kf.MexicanHat(7, learnable=False), 0.0, False),
]


def make_grid():
    """``grid.npz``: the reference grid tools (kanforge/grid.py) on float32-valued
    samples, and float32 KANLinear layers after update_grid / refine_grid /
    change_basis (kanforge/_layer.py:148-183)."""
    from kanforge import grid as gridlib
    from kanforge._layer import basis_param_values
    from kanforge.torch import KAN, KANLinear

    rec = {}
    rng = np.random.default_rng(7)
    x = rng.standard_normal((1000, 6)).astype(np.float32)
    x[:, 1] = np.round(x[:, 1] * 2) / 2  # many ties
    x[:, 2] = 0.375  # flat column
    x[:, 3] = rng.uniform(3, 5, 1000).astype(np.float32)
    x[:7, 4] = -0.0
    cases = [(9, 0.0, 0.02), (12, 0.1, 0.5), (2, 0.0, 1.0), (6, 0.0, 0.02)]
    rec["adaptive/x"] = x
    for j, (n, margin, eps) in enumerate(cases):
        rec[f"adaptive/{j}/args"] = np.array([n, margin, eps])
        rec[f"adaptive/{j}/grid"] = gridlib.adaptive_grid(x.astype(np.float64), n, margin, eps)
    rec["adaptive/x1"] = x[:1]
    rec["adaptive/x1/grid"] = gridlib.adaptive_grid(x[:1].astype(np.float64), 5, 0.0, 0.02)
    g = gridlib.adaptive_grid(x.astype(np.float64), 9, 0.0, 0.02)
    rec["resample/grid"] = g
    for n in (5, 9, 17, 33):
        rec[f"resample/{n}"] = gridlib.resample_grid(g, n)
    rec["samples/ranges"] = np.stack([g[:, 0], g[:, -1]], -1)
    rec["samples/100"] = gridlib.sample_inputs(rec["samples/ranges"], 100)

    for name, old, new, ridge, scaled in GRID_REFITS:
        n_in, n_out = 4, 3
        xs = (rng.standard_normal((400, n_in)) * 0.6).astype(np.float32).astype(np.float64)
        _, old_buf = basis_param_values(old, n_in, n_in)
        coef = rng.standard_normal((n_out, n_in, old.size)) * 0.3
        if new is None:
            new_basis, new_buf = old, {k: gridlib.adaptive_grid(xs, v.shape[-1], 0.0, 0.02) for k, v in old_buf.items()}
        else:
            ranges = gridlib.grid_ranges(old, old_buf)
            new_basis = new
            _, new_buf = basis_param_values(new, n_in, n_in, ranges)
        out = gridlib.refit(old, old_buf, coef, new_basis, new_buf, xs, ridge)
        rec[f"refit/{name}/x"] = xs
        rec[f"refit/{name}/coef"] = coef
        rec[f"refit/{name}/ridge"] = np.array(ridge)
        rec[f"refit/{name}/old_config"] = np.array(json.dumps(old.config()))
        rec[f"refit/{name}/new_config"] = np.array(json.dumps(new_basis.config()))
        for k, v in old_buf.items():
            rec[f"refit/{name}/old/{k}"] = v
        for k, v in new_buf.items():
            rec[f"refit/{name}/new/{k}"] = v
        rec[f"refit/{name}/out"] = out

    # float32 layers through the reference's own methods
    def layer(basis, scaled, seed):
        torch.manual_seed(seed)
        lay = KANLinear(5, 4, basis, edge_scale=scaled)
        with torch.no_grad():
            lay.coef.normal_(0, 0.4)
            if scaled:
                lay.edge_scale.uniform_(0.5, 1.5)
                lay.edge_scale[1, 2] = 0.0
        return lay

    def dump(prefix, lay):
        for k, v in lay.state_dict().items():
            rec[f"{prefix}/state/{k}"] = v.detach().numpy()
        rec[f"{prefix}/config"] = np.array(json.dumps(lay.basis.config()))

    xl = (torch.randn(3000, 5) * 0.7 + 0.2).float()
    xl[:, 4] = xl[:, 4] * 4
    ops = [
        ("update_bspline", kf.BSpline(6, 3), True, lambda m: m.update_grid(xl)),
        ("update_bspline_margin", kf.BSpline(4, 2), False, lambda m: m.update_grid(xl, margin=0.05, grid_eps=0.2, ridge=0.01)),
        ("update_rbf", kf.RBF(8), False, lambda m: m.update_grid(xl)),
        ("update_rswaf", kf.RSWAF(6), True, lambda m: m.update_grid(xl)),
        ("refine_bspline", kf.BSpline(5, 3), True, lambda m: m.refine_grid(10)),
        ("refine_bspline_x", kf.BSpline(5, 3), False, lambda m: m.refine_grid(7, xl)),
        ("refine_rbf", kf.RBF(5), False, lambda m: m.refine_grid(9)),
        ("change_bspline_cheb", kf.BSpline(5, 3), True, lambda m: m.change_basis(kf.Chebyshev(8))),
        ("change_cheb_bspline_x", kf.Chebyshev(5), False, lambda m: m.change_basis(kf.BSpline(6, 3), xl)),
        ("change_bspline_rbf", kf.BSpline(5, 3), False, lambda m: m.change_basis(kf.RBF(10))),
    ]
    rec["layer/x"] = xl.numpy()
    for j, (name, basis, scaled, op) in enumerate(ops):
        lay = layer(basis, scaled, 20 + j)
        dump(f"layer/{name}/before", lay)
        op(lay)
        dump(f"layer/{name}/after", lay)

    torch.manual_seed(5)
    model = KAN([5, 4, 3], kf.BSpline(5, 3))
    rec["kan/x"] = xl.numpy()
    for j, lay in enumerate(model):
        for k, v in lay.state_dict().items():
            rec[f"kan/before/{j}/{k}"] = v.detach().numpy()
    model.update_grid(xl)
    for j, lay in enumerate(model):
        for k, v in lay.state_dict().items():
            rec[f"kan/after/{j}/{k}"] = v.detach().numpy()
    np.savez_compressed(HERE / "grid.npz", **rec)


if __name__ == "__main__":
    which = sys.argv[1:] or ["bases", "layers", "prims", "init", "model_file", "grid"]
    for name in which:
        globals()[f"make_{name}"]()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
