"""Host-side checks that need no GPU: the C-ABI library loads and exports every
entry point of include/kanforge_b200.h, the host algebra (fold matrices,
rational fits, init statistics) matches the reference's golden values, and the
layer layout / .npz format match the reference."""

from __future__ import annotations

import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import GOLDEN, load_golden

import kanforge_b200 as kb
from kanforge_b200 import _lib
from kanforge_b200._init import basis_second_moment, init_stds, silu_derivative_polys

ROOT = Path(__file__).resolve().parents[1]
BASES = load_golden("bases.npz")
INIT = load_golden("init.npz")
LAYERS = load_golden("layers.npz")


def declared_symbols() -> list[str]:
    text = "\n".join(p.read_text() for p in (ROOT / "include").glob("*.h"))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kf_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(_lib.PROTOTYPES), set(names) - set(_lib.PROTOTYPES)


def test_version_and_query():
    lib = _lib.load()
    assert lib.kf_version() == 2
    cheb = kb.plan_for(kb.Chebyshev(12))
    spline = kb.plan_for(kb.BSpline(8, 3))
    rat = kb.plan_for(kb.Rational())
    assert cheb.supported(_lib.KF_OP_F, _lib.KF_DTYPE_F32)
    assert spline.supported(_lib.KF_QUERY_FUSED, _lib.KF_DTYPE_BF16)
    assert cheb.supported(_lib.KF_QUERY_FUSED, _lib.KF_DTYPE_BF16)
    assert not rat.supported(_lib.KF_QUERY_FUSED, _lib.KF_DTYPE_BF16)
    assert rat.supported(_lib.KF_QUERY_EDGE, _lib.KF_DTYPE_F32)
    assert not kb.plan_for(kb.BSpline(40, 3)).supported(_lib.KF_OP_F, _lib.KF_DTYPE_F32)  # 43 features > 32


def test_bad_arguments_fail_without_a_gpu():
    """Argument validation happens on the host, before any CUDA call."""
    d = kb.plan_for(kb.Chebyshev(3)).desc()
    rc = _lib.load().kf_prim(7, 0, None, None, None, None, None, 4, 2, 2, 4, ctypes.byref(d), None)
    assert rc == 1 and "bad op" in _lib.last_error()
    rc = _lib.load().kf_fwd(None, None, None, None, None, None, 4, 2, 2, 4, 16, 1, ctypes.byref(d), None)
    assert rc == 1 and "null" in _lib.last_error()
    rc = _lib.load().kf_features(None, None, None, 4, 2, 4, 16, 1, ctypes.byref(d), None)
    assert rc == 1 and "null" in _lib.last_error()


CHEB_CASES = [c for c in sorted({k.split("/")[0] for k in BASES}) if f"{c}/fold0" in BASES]


def _basis_from_spec(spec):
    if spec["kind"] == "bspline":
        return kb.BSpline(spec["grid_size"], spec["order"], tuple(spec["grid_range"]))
    if spec["kind"] == "rational":
        return kb.Rational(spec["num_degree"], spec["den_degree"])
    if spec["kind"] == "fourier":
        return kb.Fourier(spec["frequencies"], spec["period"])
    if spec["kind"] == "bump":
        cls = {"rbf": kb.RBF, "mexican_hat": kb.MexicanHat, "dog": kb.DoG, "rswaf": kb.RSWAF}[spec["family"]]
        kw = {} if spec["family"] in ("rbf", "rswaf") else {"learnable": False}
        return cls(spec["count"], tuple(spec["grid_range"]), **kw)
    fam = spec["family"]
    kw = {"input_map": spec["input_map"]}
    if fam == "jacobi":
        return kb.Jacobi(spec["degree"], spec["alpha"], spec["beta"], **kw)
    if fam == "gegenbauer":
        return kb.Gegenbauer(spec["degree"], spec["lam"], **kw)
    cls = {"chebyshev": kb.Chebyshev, "legendre": kb.Legendre, "taylor": kb.Taylor}[fam]
    return cls(spec["degree"], **kw)


@pytest.mark.parametrize("case", CHEB_CASES)
@pytest.mark.parametrize("m", [0, 1, 2, 3])
def test_package_fold_matrices_match_reference(case, m):
    basis = _basis_from_spec(json.loads(str(BASES[f"{case}/spec"])))
    plan = kb.plan_for(basis)
    if f"{case}/cheb" in BASES:
        np.testing.assert_allclose(basis._cheb, BASES[f"{case}/cheb"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(plan.fold(m), BASES[f"{case}/fold{m}"], rtol=1e-12, atol=1e-12)
    assert plan.n_features(m) == BASES[f"{case}/fold{m}"].shape[1]


@pytest.mark.parametrize("target", ["identity", "gelu", "silu", "tanh"])
def test_rational_initial_fit_matches_reference(target):
    a, b = kb.fit_rational(target, 5, 4)
    np.testing.assert_allclose(a, INIT[f"fit/{target}/num"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(b, INIT[f"fit/{target}/den"], rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("case", sorted({k.split("/")[1] for k in INIT if k.startswith("m2/")}))
def test_basis_second_moment_matches_reference(case):
    spec = json.loads(str(BASES[f"{case}/spec"]))
    basis = _basis_from_spec(spec)
    if spec["kind"] == "rational":
        basis = kb.Rational(5, 4, "gelu" if "gelu" in case else "identity")
    assert basis_second_moment(basis) == pytest.approx(float(INIT[f"m2/{case}"]), rel=1e-10)


def test_init_stds_match_reference():
    cases = {
        "lecun_bspline_5_3_r2": (kb.BSpline(5, 3, (-2.0, 2.0)), 2, 5, "lecun", True),
        "glorot_chebyshev_12": (kb.Chebyshev(12), 7, 3, "glorot", True),
        "variance_rational_gelu": (kb.Rational(5, 4, "gelu"), 768, 3072, "variance", False),
        "normal_bspline_8_3": (kb.BSpline(8, 3), 1024, 1024, "normal", True),
    }
    for key, (basis, n_in, n_out, how, base) in cases.items():
        c, b = init_stds(basis, n_in, n_out, how, 0.1, base)
        want = INIT[f"std/{key}"]
        assert c == pytest.approx(want[0], rel=1e-10)
        assert (b is None and np.isnan(want[1])) or b == pytest.approx(want[1], rel=1e-10)


def test_silu_derivative_polynomials_match_oracle():
    import kan_oracle as ko

    x = np.linspace(-4, 4, 33)
    s = 1 / (1 + np.exp(-x))
    for m in range(1, 5):
        h = silu_derivative_polys(m)
        got = x * np.polyval(h[0][::-1], s) + m * np.polyval(h[1][::-1], s)
        np.testing.assert_allclose(got, ko.silu_derivative(x, m), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("case", sorted({k.split("/")[0] for k in LAYERS}))
def test_layer_state_layout_matches_reference(case):
    """Same parameter/buffer names and shapes as the reference layer of the fixture."""
    pre = f"{case}/state/"
    ref = {k[len(pre):]: v for k, v in LAYERS.items() if k.startswith(pre)}
    specs = {
        "bspline_5_3": (kb.BSpline(5, 3), {}),
        "bspline_8_3": (kb.BSpline(8, 3), {}),
        "chebyshev_12": (kb.Chebyshev(12), {}),
        "jacobi_6": (kb.Jacobi(6, 0.5, 0.5), {}),
        "chebyshev_4_id_nobase": (kb.Chebyshev(4, input_map="identity"), {"base_activation": None}),
        "rational_gelu_g2": (kb.Rational(5, 4, "gelu"), {"base_activation": None, "groups": 2}),
        "rational_identity_g1": (kb.Rational(5, 4, "identity"), {"base_activation": None, "groups": 1}),
        "fourier_3": (kb.Fourier(3), {}),
        "rbf_6": (kb.RBF(6), {}),
        "mexican_hat_5": (kb.MexicanHat(5, learnable=False), {"base_activation": None}),
        "rswaf_6": (kb.RSWAF(6), {}),
    }
    basis, kw = specs[case]
    n_out, n_in = ref["coef"].shape[:2]
    layer = kb.KANLinear(n_in, n_out, basis, edge_scale="edge_scale" in ref, dtype=torch.float64, **kw)
    mine = {**dict(layer.named_parameters()), **dict(layer.named_buffers())}
    assert set(mine) == set(ref)
    for k, v in ref.items():
        assert tuple(mine[k].shape) == v.shape, k
    layer.load_state_dict({k: torch.as_tensor(v) for k, v in ref.items()})
    for k, v in ref.items():
        assert np.array_equal(mine[k].detach().numpy(), v), k


def test_reference_npz_loads_bit_exact(tmp_path):
    """A model file written by the reference loads with identical arrays, and a
    save / load round trip here is bit-exact (reference tests/test_export.py:67-76)."""
    model = kb.load(GOLDEN / "ref_model.npz")
    with np.load(GOLDEN / "ref_model.npz") as data:
        arrays = {k: data[k] for k in data.files if k != "__spec__"}
    state = {k: v.numpy() for k, v in model.state_dict().items()}
    assert set(state) == set(arrays)
    for k, v in arrays.items():
        assert np.array_equal(state[k], v), k
    assert model[0].coef.dtype == torch.float64
    kb.save(model, tmp_path / "m.npz")
    back = kb.load(tmp_path / "m.npz")
    for k, v in back.state_dict().items():
        assert torch.equal(v, model.state_dict()[k]), k


def test_cpu_tensors_fail_loudly():
    layer = kb.KANLinear(3, 2, "chebyshev")
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.zeros(4, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.edge_derivative(torch.zeros(4, 3), 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        kb.kernels.prim_F(torch.zeros(2, 3), torch.zeros(2, 3, 4), torch.ones(2, 3), torch.zeros(1),
                          kb.plan_for(kb.Chebyshev(3)), 0)


def test_backend_argument_and_errors():
    with pytest.raises(ValueError):
        kb.KANLinear(3, 2, backend="fast")
    with pytest.raises(ValueError, match="must divide"):
        kb.KANLinear(5, 2, "rational", groups=2)
    layer = kb.KANLinear(3, 2, "bspline", backend="ops")
    assert not layer.uses_kernel(torch.device("cpu"))
    with pytest.raises(RuntimeError, match="device"):
        kb.KANLinear(3, 2, "bspline", backend="kernel").uses_kernel(torch.device("cpu"))


@pytest.mark.parametrize("basis", [kb.Chebyshev(12), kb.BSpline(8, 3), kb.Chebyshev(4, input_map="identity")], ids=repr)
def test_float32_packed_operand_layout(basis):
    """The float32 tensor-core operand has the column layout of kf_pack_coef:
    per input, the basis columns (coef * edge_scale * edge_mask, folded into
    Chebyshev features), zeros, and base_weight * edge_mask last."""
    torch.manual_seed(0)
    plan = kb.plan_for(basis)
    n_out, n_in, k = 6, 5, basis.size
    nt, f_pad = kb.kernels.fused_layout(plan, True)
    coef = torch.randn(n_out, n_in, k)
    base = torch.randn(n_out, n_in)
    scale = torch.rand(n_out, n_in) + 0.5
    mask = (torch.rand(n_out, n_in) > 0.3).float()
    packed = kb.kernels.packed_f32(coef, base, scale, mask, plan, f_pad).view(n_out, n_in, f_pad)
    ce = (coef * (scale * mask)[..., None]).double().numpy()
    fold = plan.fold(0)
    want = ce @ fold if (plan.folded and not plan.is_identity_fold()) else ce
    np.testing.assert_allclose(packed[..., :nt].double().numpy(), want[..., :nt], rtol=1e-5, atol=1e-6)
    assert torch.all(packed[..., nt:f_pad - 1] == 0)
    np.testing.assert_allclose(packed[..., f_pad - 1].numpy(), (base * mask).numpy(), rtol=1e-6)


def test_float32_tensor_core_dispatch_rules():
    """CPU tensors, bf16 inputs, rational plans and outputs that are not a
    multiple of 4 never take the float32 tensor-core path."""
    plan = kb.plan_for(kb.BSpline(8, 3))
    x = torch.zeros(3, 4)
    assert not kb.kernels.tf32_ok(plan, x, 8, True, torch.float32)  # CPU
    assert not kb.kernels.tf32_ok(plan, x.to(torch.bfloat16), 8, True)
    assert not kb.kernels.tf32_ok(kb.plan_for(kb.Rational(5, 4)), x, 8, False)
    assert not kb.kernels.tf32_ok(None, x, 8, False)


def test_float32_tensor_core_path_respects_its_memory_budget(monkeypatch):
    """Above FP32_FEATURE_BYTES_MAX the float32 layer takes the primitives
    (checked on the dispatch rule; the CPU tensor itself never qualifies)."""
    plan = kb.plan_for(kb.BSpline(8, 3))
    x = torch.zeros(1000, 64)
    monkeypatch.setattr(kb.kernels, "FP32_FEATURE_BYTES_MAX", 0)
    assert not kb.kernels.tf32_ok(plan, x, 8, True, torch.float32)


@pytest.mark.parametrize("basis,first", [(kb.BSpline(8, 3), ["kf_knot_tables", "kf_features_spline_f32"]),
                                         (kb.Chebyshev(12), ["kf_features_f32"])])
def test_float32_tensor_core_forward_launch_sequence(monkeypatch, basis, first):
    """The float32 layer's forward launches: B-spline features from the knot
    tables, other bases from kf_features_f32, then one GEMM with the bias
    (launches recorded, nothing executed)."""
    calls = []
    monkeypatch.setattr(kb.kernels, "_launch", lambda name, *args: calls.append((name, args)))
    monkeypatch.setattr(kb.kernels, "_stream", lambda t: None)
    layer = kb.KANLinear(16, 8, basis)
    x = torch.zeros(5, 16)
    with torch.no_grad():
        y = kb.kernels.kan_linear_tf32(x, layer.coef, layer.base_weight, layer.bias, layer.edge_scale, layer.edge_mask,
                                       layer._grid(), layer._plan)
    assert y.shape == (5, 8)
    assert [n for n, _ in calls] == first + ["kf_gemm_tf32x3"]
    nt, f_pad = kb.kernels.fused_layout(layer._plan, True)
    feat_args = calls[len(first) - 1][1]
    assert feat_args[3:8] == (5, 16, nt, f_pad, 1)  # B, I, nt, f_pad, has_base
    gemm = calls[-1][1]
    assert gemm[-4:-1] == (5, 8, 16 * f_pad)  # M = tokens, N = outputs, K = I * f_pad
    assert gemm[6].value == layer.bias.data_ptr()


def test_polynomial_family_matrices_match_independent_evaluations():
    """Every family's Chebyshev matrix A reproduces the family evaluated
    independently (scipy.special, or the definition): family_k(z) =
    sum_j T_j(z) A[j, k]; Gram polynomials are orthonormal on their points."""
    from scipy import special

    z = np.linspace(-1, 1, 41)
    d = 7

    def via_a(basis):
        return np.polynomial.chebyshev.chebvander(z, basis.degree) @ basis._cheb

    cases = [
        (kb.Chebyshev(d), lambda n: special.eval_chebyt(n, z)),
        (kb.Chebyshev2(d), lambda n: special.eval_chebyu(n, z)),
        (kb.Legendre(d), lambda n: special.eval_legendre(n, z)),
        (kb.Jacobi(d, 0.5, 1.5), lambda n: special.eval_jacobi(n, 0.5, 1.5, z)),
        (kb.Jacobi(d, -0.3, 2.0), lambda n: special.eval_jacobi(n, -0.3, 2.0, z)),
        (kb.Gegenbauer(d, 0.7), lambda n: special.eval_gegenbauer(n, 0.7, z)),
        (kb.Hermite(d), lambda n: special.eval_hermite(n, z)),
        (kb.Laguerre(d), lambda n: special.eval_genlaguerre(n, 0.0, z)),
        (kb.Bernstein(d), lambda n: special.comb(d, n) * ((z + 1) / 2) ** n * ((1 - z) / 2) ** (d - n)),
        (kb.Taylor(d), lambda n: z**n),
    ]
    for basis, fn in cases:
        want = np.stack([fn(n) for n in range(d + 1)], -1)
        np.testing.assert_allclose(via_a(basis), want, rtol=1e-11, atol=1e-11 * max(1.0, np.abs(want).max()),
                                   err_msg=repr(basis))
    g = kb.Gram(5, points=11)
    pts = np.linspace(-1, 1, 11)
    v = np.polynomial.chebyshev.chebvander(pts, 5) @ g._cheb
    np.testing.assert_allclose(v.T @ v / 11, np.eye(6), atol=1e-12)
    assert (np.diag(g._cheb) > 0).all()


def test_grid_tools_validate_arguments_without_a_gpu():
    """kf_adaptive_grid / kf_refit reject bad sizes on the host, before any CUDA call."""
    lib = _lib.load()
    ws = ctypes.c_void_p(16)
    rc = lib.kf_adaptive_grid(ws, 10, 3, 1, 0.0, 0.02, ws, ws, None)
    assert rc == 1 and "n_points" in _lib.last_error()
    rc = lib.kf_adaptive_grid(ws, 10, 3, 9, 0.0, 0.0, ws, ws, None)
    assert rc == 1 and "grid_eps" in _lib.last_error()
    rc = lib.kf_adaptive_grid(ws, 0, 3, 9, 0.0, 0.02, ws, ws, None)
    assert rc == 1 and "samples" in _lib.last_error()
    assert lib.kf_grid_workspace(1000, 6, 9) == 6 * 9 * (8 + 1024)
    big, keep = kb.kernels.fit_basis(kb.plan_for(kb.Chebyshev(5)), None, "cpu")
    rat = _lib.FitBasis(kind=_lib.KF_BASIS_RATIONAL, size=1)
    rc = lib.kf_refit(ws, None, 10, 3, 2, ctypes.byref(rat), ctypes.byref(big), ws, None, 0, 0.0, ws, None, ws, None)
    assert rc == 2 and "no refit" in _lib.last_error()
    with pytest.raises(ValueError, match="up to 256"):
        kb.kernels.fit_basis(kb.plan_for(kb.BSpline(300, 3)), torch.zeros(3, 301, dtype=torch.float64), "cpu")


def test_grid_tools_fail_loudly_on_cpu():
    layer = kb.KANLinear(3, 2, kb.BSpline(5, 3))
    with pytest.raises(ValueError, match="samples"):
        layer.update_grid(None)
    with pytest.raises(TypeError, match="no grid"):
        kb.KANLinear(3, 2, kb.Chebyshev(4)).update_grid(torch.zeros(8, 3))
    with pytest.raises(TypeError, match="grid size"):
        kb.KANLinear(3, 2, kb.Chebyshev(4)).refine_grid(8)
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.update_grid(torch.zeros(8, 3))
    with pytest.raises(ValueError, match="pass samples"):
        kb.KANLinear(3, 2, kb.Chebyshev(4)).change_basis(kb.Legendre(4))
