"""KAN layers on the sm_100a kernels: KANLinear, KAN, GRKAN.

Same constructor arguments, parameter names, shapes, buffers and state-dict
layout as the reference torch layers (kanforge/torch/layers.py:28-398), so
state dicts and ``.npz`` files move between the two unchanged.  The compute
differs: every forward and backward runs ``libkanb200`` kernels on CUDA.

Dispatch of ``KANLinear.forward`` (reference kanforge/torch/layers.py:171-192):

* bfloat16 B-spline / polynomial layers -> one fused tcgen05 contraction per
  pass (basis features + SiLU base branch + bias, ``kernels.kan_linear_fused``);
* other dtypes and shapes -> the closed float32 primitive family
  (``kernels.spline_forward``) plus the base branch and bias;
* rational (GRKAN) layers -> the group-rational kernel, then the contraction
  with the layer coefficients.

CPU tensors raise: there is no CPU fallback.
"""

from __future__ import annotations

import functools
import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from . import kernels as _kernels
from ._init import init_stds, initial_basis_state, resolve_groups
from .bases import Basis, Rational, make_basis
from .plan import plan_for

BACKENDS = ("auto", "ops", "kernel")


def _require_cuda(x: torch.Tensor) -> None:
    if x.device.type != "cuda":
        raise RuntimeError(
            f"kanforge_b200 layers run on CUDA devices only (got a {x.device} tensor); there is no CPU fallback"
        )


@dataclass(frozen=True)
class LayerOptions:
    """The constructor choices a layer keeps for re-initialisation and export
    (the ``.npz`` layer spec of kanforge/convert.py:108-160)."""

    bias: bool
    base_activation: Callable[[torch.Tensor], torch.Tensor] | None
    groups: int | None  # as given: None = one group per input
    edge_scale: bool
    coef_init: str
    coef_init_std: float
    edge_dropout: float
    backend: str
    grid_ranges: object = None


class KANLinear(nn.Module):
    """One KAN layer: y_o = sum_i s_oi phi_oi(x_i) + sum_i w_oi act(x_i) + b_o.

    Parameters (reference names, kanforge/torch/layers.py:52-118): ``coef``
    (out, in, basis.size), ``base_weight`` (out, in), ``bias`` (out,),
    ``edge_scale`` (out, in), trainable basis parameters ``basis_<name>``
    (groups, *shape).  Buffers: ``basis_<name>`` grids (in, *shape),
    ``edge_mask``, ``sym_code``, ``sym_params``.

    ``backend`` is accepted for compatibility ("auto", "ops", "kernel"); every
    value runs the CUDA kernels.  ``"kernel"`` raises for a basis without one.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        basis: str | dict | Basis = "bspline",
        *,
        bias: bool = True,
        base_activation: Callable[[torch.Tensor], torch.Tensor] | None = F.silu,
        groups: int | None = None,
        edge_scale: bool = False,
        grid_ranges=None,
        coef_init: str = "normal",
        coef_init_std: float = 0.1,
        edge_dropout: float = 0.0,
        backend: str = "auto",
        device=None,
        dtype=None,
    ):
        super().__init__()
        if backend not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS}")
        if not 0.0 <= edge_dropout < 1.0:
            raise ValueError("edge_dropout must be in [0, 1)")
        self.options = LayerOptions(bias, base_activation, groups, edge_scale, coef_init, coef_init_std, edge_dropout,
                                    backend, grid_ranges)
        self.in_features, self.out_features = in_features, out_features
        self.basis = make_basis(basis)
        self.base_activation = base_activation
        self.groups = resolve_groups(in_features, groups)
        self.coef_init, self.coef_init_std = coef_init, coef_init_std
        self.edge_dropout, self.backend = edge_dropout, backend
        # rejects an unknown scheme before any tensor exists
        init_stds(self.basis, in_features, out_features, coef_init, coef_init_std, base_activation is not None)

        edge = (out_features, in_features)
        tensor = functools.partial(torch.empty, device=device, dtype=dtype)
        optional = {
            "coef": edge + (self.basis.size,),
            "base_weight": edge if base_activation is not None else None,
            "bias": (out_features,) if bias else None,
            "edge_scale": edge if edge_scale else None,
        }
        for name, shape in optional.items():
            self.register_parameter(name, None if shape is None else nn.Parameter(tensor(shape)))
        self.register_buffer("edge_mask", tensor(edge))
        self.register_buffer("sym_code", torch.empty(edge, dtype=torch.int32, device=device))
        self.register_buffer("sym_params", tensor(edge + (4,)))
        self._basis_tensors: dict[str, bool] = {}  # basis_<name> -> trainable
        self.reset_parameters()
        if backend == "kernel" and self._plan is None:
            raise RuntimeError(f"no fused kernel for this basis: {self.basis!r}")

    # --- parameters ------------------------------------------------------------

    def _install_basis_state(self, state) -> None:
        """Registers the basis tensors of ``state`` (replacing the previous ones)
        in the dtype and on the device of ``coef``."""
        for name in self._basis_tensors:
            delattr(self, f"basis_{name}")
        like = {"dtype": self.coef.dtype, "device": self.coef.device}
        self._basis_tensors = {}
        for trainable, values in ((True, state.trainable), (False, state.buffers)):
            for name, value in values.items():
                if isinstance(value, torch.Tensor):
                    t = value.detach().to(**like).contiguous()
                else:
                    t = torch.as_tensor(np.ascontiguousarray(value), **like)
                if trainable:
                    self.register_parameter(f"basis_{name}", nn.Parameter(t))
                else:
                    self.register_buffer(f"basis_{name}", t)
                self._basis_tensors[name] = trainable
        self._plan = plan_for(self.basis)

    @torch.no_grad()
    def reset_parameters(self) -> None:
        """Draws the coefficients and base weights of the layer's scheme
        (reference kanforge/torch/layers.py:131-149) and resets the masks,
        symbolic slots and basis state."""
        opt = self.options
        coef_std, base_std = init_stds(self.basis, self.in_features, self.out_features, opt.coef_init,
                                       opt.coef_init_std, self.base_weight is not None)
        if coef_std:
            self.coef.normal_(0.0, coef_std)
        else:
            self.coef.zero_()
        if self.base_weight is not None:
            if base_std is None:
                nn.init.kaiming_uniform_(self.base_weight, a=math.sqrt(5))
            else:
                self.base_weight.normal_(0.0, base_std)
        for t, value in ((self.bias, 0.0), (self.edge_scale, 1.0), (self.edge_mask, 1.0), (self.sym_code, -1),
                         (self.sym_params, 0.0)):
            if t is not None:
                t.fill_(value)
        self._sym_codes = ()
        self._install_basis_state(initial_basis_state(self.basis, self.groups, self.in_features, opt.grid_ranges))

    def basis_params(self) -> dict[str, torch.Tensor]:
        """Every basis tensor with one row per input, (in, *shape): per-group
        trainables repeated over their group's inputs (reference
        kanforge/torch/layers.py:151-160; one group or one per input: as stored)."""
        per_group = self.in_features // self.groups
        expand = self.groups not in (1, self.in_features)
        out = {}
        for name, trainable in self._basis_tensors.items():
            t = getattr(self, f"basis_{name}")
            out[name] = t.repeat_interleave(per_group, dim=0) if (trainable and expand) else t
        return out

    def effective_coef(self) -> torch.Tensor:
        """coef * edge_scale * edge_mask over the basis axis."""
        gate = self.edge_mask if self.edge_scale is None else self.edge_mask * self.edge_scale
        return self.coef * gate.unsqueeze(-1)

    def effective_base_weight(self) -> torch.Tensor | None:
        """base_weight * edge_mask (None without a base branch)."""
        return None if self.base_weight is None else self.edge_mask * self.base_weight

    # --- computation ------------------------------------------------------------

    def _grid(self):
        return getattr(self, "basis_grid", None) if self._plan is not None and self._plan.grid else None

    def _check_supported(self, derivatives: bool = False) -> None:
        if self._plan is None:
            raise RuntimeError(f"no fused kernel for this basis: {self.basis!r}")
        if self._sym_codes:
            raise NotImplementedError("symbolic edges are not part of the kanforge_b200 kernel path")
        if derivatives and self.base_weight is not None and self.base_activation is not F.silu:
            raise NotImplementedError("edge derivatives take the SiLU base branch; other base activations are not supported")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x)
        self._check_supported()
        if self.training and self.edge_dropout > 0:
            raise NotImplementedError("edge_dropout (DropKAN) is not part of the kanforge_b200 kernel path")
        if self.base_weight is None or self.base_activation is F.silu:
            return self._edges(x, self.base_weight)
        # another base activation: the kernels compute the basis part, the base
        # branch act(x) (W * mask)^T is added as a plain linear map
        y = self._edges(x, None)
        return y + F.linear(self.base_activation(x), self.effective_base_weight()).to(y.dtype)

    def _edges(self, x: torch.Tensor, silu_weight: torch.Tensor | None) -> torch.Tensor:
        """sum_i phi_oi(x_i) + bias, plus the SiLU base branch of ``silu_weight``."""
        plan = self._plan
        has_base = silu_weight is not None
        if plan.kind != "rational" and _kernels.fused_ok(plan, x, self.out_features, has_base, self.coef.dtype):
            # coef * edge_scale * edge_mask and base_weight * edge_mask are formed inside the kernels
            return _kernels.kan_linear_fused(x, self.coef, silu_weight, self.bias, self.edge_scale, self.edge_mask,
                                             self._grid(), plan)
        tf32 = plan.kind != "rational" and _kernels.FP32_TENSOR_CORES and _kernels.tf32_ok(
            plan, x, self.out_features, has_base, self.coef.dtype)
        if _kernels.sparse_ok(plan, x, self.out_features, self.coef.dtype, tf32):
            # float32 B-spline, narrow layer: gather the k+1 non-zero coefficients per (token, input)
            return _kernels.kan_linear_sparse(x, self.coef, silu_weight, self.bias, self.edge_scale, self.edge_mask,
                                              self._grid(), plan)
        if tf32:
            # float32: three TF32 products per contraction on the tensor cores
            return _kernels.kan_linear_tf32(x, self.coef, silu_weight, self.bias, self.edge_scale, self.edge_mask,
                                            self._grid(), plan)
        if plan.kind == "bspline" and x.dtype == torch.bfloat16 and self.coef.dtype == torch.bfloat16:
            # bf16 B-spline layers the fused kernels do not take (more than 31
            # features per input, or output counts they do not tile) compute in
            # float32 on the sparse gather kernels
            f = lambda t: None if t is None else t.float()  # noqa: E731
            if _kernels.sparse_ok(plan, x.float(), self.out_features, torch.float32, False):
                y = _kernels.kan_linear_sparse(x.float(), self.coef.float(), f(silu_weight), f(self.bias),
                                               f(self.edge_scale), f(self.edge_mask), self._grid(), plan)
                return y.to(x.dtype)
        if plan.kind == "bump" and x.dtype == torch.bfloat16 and _kernels.FP32_TENSOR_CORES:
            # bf16 bump layers (centres per input) compute in float32 on the three-TF32 GEMM
            f = lambda t: None if t is None else t.float()  # noqa: E731
            if _kernels.tf32_ok(plan, x.float(), self.out_features, has_base, torch.float32):
                y = _kernels.kan_linear_tf32(x.float(), self.coef.float(), f(silu_weight), f(self.bias),
                                             f(self.edge_scale), f(self.edge_mask), self._grid(), plan)
                return y.to(x.dtype)
        coef_eff = self.effective_coef()
        base_eff = None if silu_weight is None else silu_weight * self.edge_mask
        if plan.kind == "rational":
            lead = x.shape[:-1]
            x2 = x.reshape(-1, self.in_features)
            path = None if base_eff is not None else _kernels.grkan_ok(plan, x2, self.in_features, self.out_features,
                                                                      self.groups, self.coef.dtype)
            if path is not None:
                y = _kernels.grkan_linear(x2, self.basis_numerator, self.basis_denominator, coef_eff[..., 0], self.bias, plan,
                                          self.groups, path)
                return y.reshape(*lead, self.out_features)
            r = _kernels.rational_act(x2, self.basis_numerator, self.basis_denominator, plan, self.groups)
            y = F.linear(r.to(coef_eff.dtype), coef_eff[..., 0], self.bias)
            if base_eff is not None:
                y = y + F.linear(F.silu(x2), base_eff)
            return y.reshape(*lead, self.out_features)
        y = _kernels.spline_forward(x, coef_eff, self._grid(), plan)
        if base_eff is not None:
            y = y + F.linear(self.base_activation(x), base_eff)
        if self.bias is not None:
            y = y + self.bias
        return y

    def uses_kernel(self, device: torch.device) -> bool:
        """Whether forward runs the CUDA kernels on ``device`` (layers.py:194-204)."""
        ok = self._plan is not None and _kernels.available(torch.device(device))
        if self.backend == "kernel" and not ok:
            why = "basis" if self._plan is None else f"device {device}"
            raise RuntimeError(f"no fused kernel for this {why}: {self.basis!r}")
        return ok

    def edge_derivative(self, x: torch.Tensor, order: int = 1) -> torch.Tensor:
        """d^order phi_oi / dx_i^order of every edge, (..., out, in) (layers.py:206-226)."""
        if order < 0:
            raise ValueError("order must be >= 0")
        _require_cuda(x)
        self._check_supported(derivatives=True)
        plan = self._plan
        coef_eff = self.effective_coef()
        base_eff = self.effective_base_weight()
        params = None
        if plan.kind == "rational":
            params = {"numerator": self.basis_numerator, "denominator": self.basis_denominator}
        out = _kernels.edge_derivative(x, coef_eff, base_eff, self._grid(), plan, order, params, self.groups)
        return out.to(x.dtype) if x.dtype != torch.float32 else out

    # --- grid tools (reference kanforge/_layer.py:107-183, kanforge/grid.py) ------
    # Adaptive grids, resampled grids and the least-squares refit run on the
    # device (kf_adaptive_grid, kf_resample_grid, kf_refit); the samples stay
    # there.  Samples are taken in float32.  Parameter shapes can change:
    # re-create the optimizer afterwards.

    @staticmethod
    def _refit_plan(basis: Basis):
        plan = plan_for(basis)
        if plan is None or plan.kind == "rational":
            raise NotImplementedError(f"no device refit for {basis!r}: it has no kernel plan with fixed features")
        return plan

    def _grid64(self) -> torch.Tensor | None:
        return self.basis_grid.detach().to(torch.float64) if "grid" in self._basis_tensors else None

    def _sample_columns(self, x) -> torch.Tensor:
        x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x), dtype=torch.float32)
        x = x.detach().to(self.coef.device)
        _require_cuda(x)
        return _kernels.sample_columns(x.reshape(-1, self.in_features))

    def _ranges(self, grid: torch.Tensor) -> torch.Tensor:
        return torch.stack([grid[:, 0], grid[:, -1]], -1).to(torch.float64).contiguous()

    @torch.no_grad()
    def _refit_to(self, new_basis: Basis, new_grid, samples, ridge: float) -> None:
        """Move to new_basis (grid new_grid, float64) keeping the edge functions on
        samples: (xt, None, n) sample columns or (None, ranges, n) evenly spaced
        points (_layer.py:120-137)."""
        old_fb, keep_old = _kernels.fit_basis(self._refit_plan(self.basis), self._grid64(), self.coef.device)
        new_fb, keep_new = _kernels.fit_basis(self._refit_plan(new_basis), new_grid, self.coef.device)
        xt, ranges, n = samples
        coef, scale = _kernels.refit(xt, ranges, n, old_fb, new_fb, self.coef, self.edge_scale, ridge)
        like = {"dtype": self.coef.dtype, "device": self.coef.device}
        self.basis = new_basis
        self.coef = nn.Parameter(coef.to(**like).contiguous())
        if scale is not None:
            self.edge_scale = nn.Parameter(scale.to(**like).contiguous())
        state = initial_basis_state(new_basis, self.groups, self.in_features)
        if new_grid is not None:
            state.buffers["grid"] = new_grid
        self._install_basis_state(state)
        del keep_old, keep_new

    def update_grid(self, x, *, margin: float = 0.0, grid_eps: float = 0.02, ridge: float = 0.0) -> None:
        """Adapt every input's grid to the samples x (pykan's update_grid_from_samples)
        and refit the edge functions on x (_layer.py:148-164).  Like pykan this
        only approximates the old functions on the new grid."""
        if x is None:
            raise ValueError("update_grid needs input samples x")
        if not self.basis.grid_names():
            raise TypeError(f"{type(self.basis).__name__} has no grid")
        xt = self._sample_columns(x)
        grid = _kernels.adaptive_grid(xt, self.basis_grid.shape[-1], margin, grid_eps)
        self._refit_to(self.basis, grid, (xt, None, xt.shape[1]), ridge)

    def refine_grid(self, grid_size: int, x=None, *, ridge: float = 0.0) -> None:
        """The same basis with grid_size intervals (or centres); each grid keeps
        its per-input shape (_layer.py:166-175)."""
        cfg = self.basis.config()
        key = next((k for k in ("grid_size", "count", "num_knots") if k in cfg), None)
        if key is None:
            raise TypeError(f"{type(self.basis).__name__} has no grid size to refine")
        new_basis = make_basis({**cfg, key: grid_size})
        old_grid = self._grid64()
        new_grid = None
        if old_grid is not None and "grid" in new_basis.grid_names():
            n_new = initial_basis_state(new_basis, self.groups, self.in_features).buffers["grid"].shape[-1]
            new_grid = _kernels.resample_grid(old_grid, n_new)
        samples = self._fit_samples(x, old_grid, 8 * new_basis.size + 64)
        self._refit_to(new_basis, new_grid, samples, ridge)

    def change_basis(self, basis, x=None, *, ridge: float = 0.0) -> None:
        """Convert to another basis by least squares (_layer.py:177-183): a new
        grid spans each input's old grid range; without x the fit uses evenly
        spaced points over the old grid (else the new basis' grid)."""
        new_basis = make_basis(basis)
        old_grid = self._grid64()
        ranges = None if old_grid is None else self._ranges(old_grid)
        state = initial_basis_state(new_basis, self.groups, self.in_features,
                                    None if ranges is None else ranges.cpu().numpy())
        new_grid = state.buffers.get("grid")
        if new_grid is not None:
            new_grid = torch.as_tensor(new_grid, dtype=torch.float64, device=self.coef.device)
        src = old_grid if old_grid is not None else new_grid
        samples = self._fit_samples(x, src, 8 * max(new_basis.size, self.basis.size) + 64)
        self._refit_to(new_basis, new_grid, samples, ridge)

    def _fit_samples(self, x, grid, n: int):
        if x is not None:
            xt = self._sample_columns(x)
            return xt, None, xt.shape[1]
        if grid is None:
            raise ValueError(f"{type(self.basis).__name__} has no grid: pass samples x")
        return None, self._ranges(grid), n

    # --- state export / import (.npz layout, layers.py:230-267) -----------------

    @staticmethod
    def _to_numpy(x) -> np.ndarray:
        return x.detach().cpu().double().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)

    def _export_full(self) -> dict:
        own = {**dict(self.named_parameters(recurse=False)), **dict(self.named_buffers(recurse=False))}
        out = {k: self._to_numpy(v) for k, v in own.items()}
        out.update({k: None for k in ("base_weight", "bias", "edge_scale") if getattr(self, k) is None})
        return out

    @torch.no_grad()
    def _import_full(self, state: dict) -> None:
        for name, value in state.items():
            t = getattr(self, name, None)
            if value is None or t is None:
                continue
            if t.shape != value.shape:
                raise ValueError(f"{name}: shape {value.shape} does not fit {tuple(t.shape)}")
            t.copy_(torch.as_tensor(value, dtype=t.dtype, device=t.device))
        self._refresh_symbolic()

    def _refresh_symbolic(self) -> None:
        codes = np.unique(self.sym_code.detach().cpu().numpy().astype(int))
        self._sym_codes = tuple(int(c) for c in codes if c >= 0)

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._refresh_symbolic()

    def extra_repr(self) -> str:
        groups = "" if self.groups == self.in_features else f", groups={self.groups}"
        return f"in_features={self.in_features}, out_features={self.out_features}, basis={self.basis!r}{groups}"


class GRKAN(KANLinear):
    """Group-rational KAN layer of KAT (layers.py:335-363): rational activations
    shared by ``groups`` of inputs, the coefficients act as the linear weight."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        groups: int = 8,
        num_degree: int = 5,
        den_degree: int = 4,
        init: str = "gelu",
        bias: bool = True,
        device=None,
        dtype=None,
    ):
        super().__init__(
            in_features,
            out_features,
            Rational(num_degree, den_degree, init),
            bias=bias,
            base_activation=None,
            groups=groups,
            coef_init="variance",
            device=device,
            dtype=dtype,
        )


class KAN(nn.Sequential):
    """Stack of KANLinear layers, e.g. ``KAN([2, 5, 1], basis="chebyshev")`` (layers.py:366-398)."""

    def __init__(self, widths: Sequence[int], basis: str | dict | Basis = "bspline", grid_ranges=None, **layer_kwargs):
        if len(widths) < 2:
            raise ValueError("widths needs at least input and output size")
        super().__init__(
            *(
                KANLinear(a, b, basis, grid_ranges=grid_ranges if k == 0 else None, **layer_kwargs)
                for k, (a, b) in enumerate(zip(widths[:-1], widths[1:]))
            )
        )
        self.widths = list(widths)

    def edge_derivative(self, x: torch.Tensor, order: int = 1) -> list[torch.Tensor]:
        """Per-layer edge derivatives at the activations each layer receives."""
        return [layer.edge_derivative(h, order) for layer, h in layer_inputs(self, x)]

    @torch.no_grad()
    def update_grid(self, x: torch.Tensor, **kwargs) -> None:
        """Update every layer's grid from the activations it receives, each layer
        after the ones before it (kanforge/torch/layers.py:389-393)."""
        for layer in self:
            layer.update_grid(x, **kwargs)
            x = layer(x)

    def refine_grid(self, grid_size: int, **kwargs) -> None:
        for layer in self:
            layer.refine_grid(grid_size, **kwargs)


def rebuild_kan(layers: Sequence[KANLinear]) -> KAN:
    """A KAN made of existing layers."""
    model = KAN.__new__(KAN)
    nn.Sequential.__init__(model, *layers)
    model.widths = [layers[0].in_features] + [layer.out_features for layer in layers]
    return model


def layer_inputs(model: nn.Module, x: torch.Tensor) -> list[tuple[KANLinear, torch.Tensor]]:
    """(KANLinear, its input) for every KAN layer of ``model`` (layers.py:446-467)."""
    out = []

    def walk(m, h):
        if isinstance(m, KANLinear):
            out.append((m, h))
            return m(h)
        if isinstance(m, nn.Sequential):
            for sub in m:
                h = walk(sub, h)
            return h
        return m(h)

    with torch.no_grad():
        walk(model, x)
    return out
