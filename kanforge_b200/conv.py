"""KAN convolutions, channels-first like ``torch.nn.ConvNd`` (reference kanforge/torch/conv.py).

Each output position is a KANLinear of its receptive field, one KANLinear per
channel group; the receptive field's values are ordered like the weights of
``nn.ConvNd`` (channel, then the kernel offsets), so parameters and state
dicts carry over.  The layer's input is the *implicit* patch matrix of the
image (``include/kanforge_b200.h``: kf_conv_geom): for bf16 layers on the
tensor-core path the kernels gather every receptive field from the image
(``kf_conv_fwd`` / ``kf_conv_features`` / ``kf_conv_dgrad`` / ``kf_conv_wgrad``)
and the patch-matrix gradient is folded back onto the image
(``kf_conv_fold``); other dtypes and layers materialise the patch matrix with
``kf_conv_patches`` and run the ordinary KANLinear.  Padding modes other than
zeros pad the image first (``F.pad``) and use padding 0.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from . import kernels as _k
from .layers import KANLinear, _require_cuda

PADDING_MODES = ("zeros", "reflect", "replicate", "circular")


def _per_dim(v, n: int, what: str) -> tuple[int, ...]:
    out = tuple(int(u) for u in v) if isinstance(v, Sequence) else (int(v),) * n
    if len(out) != n:
        raise ValueError(f"{what} needs {n} values, got {v!r}")
    return out


def _geometry(x: torch.Tensor, layer: "_KANConvNd", group: int, pad) -> _lib.ConvGeom:
    """kf_conv_geom of group `group` over image x (N, C, *L); spatial
    dimensions padded to three with size-1 dimensions in front."""
    n = layer.n_dims
    lead = 3 - n
    g = _lib.ConvGeom()
    g.batch, g.channels = x.shape[0], x.shape[1]
    g.group_channels = layer.in_channels // layer.groups
    g.channel0 = group * g.group_channels
    for d in range(3):
        k = d - lead
        g.size[d] = x.shape[2 + k] if k >= 0 else 1
        g.kernel[d] = layer.kernel_size[k] if k >= 0 else 1
        g.stride[d] = layer.stride[k] if k >= 0 else 1
        g.padding[d] = pad[k] if k >= 0 else 0
        g.dilation[d] = layer.dilation[k] if k >= 0 else 1
    return g


def _out_shape(g: _lib.ConvGeom) -> tuple[int, int, int]:
    return tuple((g.size[d] + 2 * g.padding[d] - g.dilation[d] * (g.kernel[d] - 1) - 1) // g.stride[d] + 1 for d in range(3))


def _rows_cols(g: _lib.ConvGeom) -> tuple[int, int]:
    return g.batch * math.prod(_out_shape(g)), g.group_channels * math.prod(tuple(g.kernel))


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.KF_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.KF_DTYPE_F32
    raise RuntimeError(f"KAN convolutions take float32 or bfloat16 images, not {t.dtype}")


def _patches(img: torch.Tensor, g: _lib.ConvGeom) -> torch.Tensor:
    rows, cols = _rows_cols(g)
    out = torch.empty(rows, cols, device=img.device, dtype=img.dtype)
    _k._launch("kf_conv_patches", _k._ptr(img), ctypes.byref(g), _k._ptr(out), _dtype_code(img), _k._stream(img))
    return out


def _fold(dpatches: torch.Tensor, g: _lib.ConvGeom, like: torch.Tensor) -> torch.Tensor:
    """Image gradient of one group (zero in the other groups' channels)."""
    dimg = torch.zeros_like(like) if g.group_channels != g.channels else torch.empty_like(like)
    _k._launch("kf_conv_fold", _k._ptr(dpatches.contiguous()), ctypes.byref(g), _k._ptr(dimg), _dtype_code(like),
               _k._stream(like))
    return dimg


class _Patches(torch.autograd.Function):
    """The patch matrix (rows, cols) of one group; backward folds onto the image."""

    @staticmethod
    def forward(ctx, img, g):
        ctx.g = g
        ctx.save_for_backward(img)
        return _patches(img.contiguous(), g)

    @staticmethod
    def backward(ctx, dp):
        (img,) = ctx.saved_tensors
        return _FoldPatches.apply(dp, ctx.g, img), None


class _FoldPatches(torch.autograd.Function):
    """The adjoint of _Patches (used by double backward)."""

    @staticmethod
    def forward(ctx, dp, g, like):
        ctx.g = g
        return _fold(dp.to(like.dtype), g, like)

    @staticmethod
    def backward(ctx, dimg):
        return _Patches.apply(dimg, ctx.g), None, None


class _ImplicitConvKAN(torch.autograd.Function):
    """One channel group of a bf16 KAN convolution on the tensor cores, the
    receptive fields gathered from the image by the kernels (the fused
    KANLinear op of kernels.py with x = the implicit patch matrix)."""

    @staticmethod
    def forward(ctx, img, coef, base_weight, bias, edge_scale, edge_mask, grid, plan, g):
        n_out, n_in, _ = coef.shape
        has_base = base_weight is not None
        nt, f_pad = _k.fused_layout(plan, has_base)
        img = img.contiguous()
        rows, cols = _rows_cols(g)
        packed = _k.pack_coef(coef, base_weight, edge_scale, edge_mask, plan, f_pad)
        y = torch.empty(rows, n_out, device=img.device, dtype=torch.bfloat16)
        b = _k._bf16_or_none(bias)
        gr = None if grid is None else grid.detach().float().contiguous()
        tab = None if gr is None else _k.knot_tables(gr, plan)
        desc = plan.desc()
        feat = _conv_features(img, g, tab, nt, f_pad, has_base, desc) if plan.kind in _k.FEATURES_IN_FORWARD else None
        _k._launch("kf_conv_fwd", _k._ptr(img), ctypes.byref(g), _k._ptr(feat), _k._ptr(packed), _k._ptr(b), _k._ptr(tab),
                   _k._ptr(y), n_out, nt, f_pad, int(has_base), ctypes.byref(desc), _k._stream(img))
        ctx.save_for_backward(img, coef, base_weight, edge_scale, edge_mask, gr)
        ctx.packed, ctx.tab, ctx.feat, ctx.plan, ctx.g = packed, tab, feat, plan, g
        ctx.has_bias, ctx.layout = bias is not None, (nt, f_pad)
        return y

    @staticmethod
    def backward(ctx, gy):
        img, coef, base_weight, edge_scale, edge_mask, grid = ctx.saved_tensors
        plan, g, need = ctx.plan, ctx.g, ctx.needs_input_grad
        if torch.is_grad_enabled():
            # double backward: the differentiable primitives on the patch matrix
            ctx.packed = ctx.tab = ctx.feat = None
            p = _Patches.apply(img, g)
            grads = _k._fused_backward_differentiable(p, gy, coef, base_weight, edge_scale, edge_mask, grid, plan,
                                                      (need[0],) + tuple(need[1:6]) + (False, False), ctx.has_bias)
            dimg = _FoldPatches.apply(grads[0], g, img) if need[0] else None
            return (dimg,) + tuple(grads[1:5]) + (None, None, None, None)
        nt, f_pad = ctx.layout
        n_out, n_in, k = coef.shape
        rows, cols = _rows_cols(g)
        gy = gy.to(torch.bfloat16).contiguous()
        desc = plan.desc()
        stream = _k._stream(img)
        dimg = gc = gb = gbias = gs = None
        if need[1] or need[2] or need[4]:
            gc = torch.empty(n_out, n_in, k, device=img.device, dtype=torch.bfloat16)
            gb = torch.empty(n_out, n_in, device=img.device, dtype=torch.bfloat16) if base_weight is not None else None
            gs = torch.empty(n_out, n_in, device=img.device, dtype=torch.bfloat16) if (edge_scale is not None and need[4]) else None
            fold = _k._fold_on(plan, 0, img.device) if (plan.folded and not plan.is_identity_fold()) else None
            cf, sc, mk = _k._bf16_or_none(coef), _k._bf16_or_none(edge_scale), _k._bf16_or_none(edge_mask)
            feat = ctx.feat if ctx.feat is not None else _conv_features(img, g, ctx.tab, nt, f_pad, base_weight is not None,
                                                                         desc)
            _k._launch("kf_conv_wgrad", _k._ptr(img), ctypes.byref(g), _k._ptr(feat), _k._ptr(gy), _k._ptr(ctx.tab),
                       _k._ptr(fold), _k._ptr(cf), _k._ptr(sc), _k._ptr(mk), _k._ptr(gc), _k._ptr(gb), _k._ptr(gs), n_out, k,
                       nt, f_pad, ctypes.byref(desc), stream)
            del feat
            gc = gc.to(coef.dtype) if need[1] else None
            gb = gb.to(base_weight.dtype) if (gb is not None and need[2]) else None
            gs = gs.to(edge_scale.dtype) if gs is not None else None
        if need[0]:
            dp = torch.empty(rows, cols, device=img.device, dtype=torch.bfloat16)
            _k._launch("kf_conv_dgrad", _k._ptr(img), ctypes.byref(g), _k._ptr(gy), _k._ptr(ctx.packed), _k._ptr(ctx.tab),
                       _k._ptr(dp), n_out, nt, f_pad, int(base_weight is not None), ctypes.byref(desc), stream)
            dimg = _fold(dp, g, img)
        if need[3] and ctx.has_bias:
            gbias = gy.sum(0, dtype=torch.float32)
        ctx.packed = ctx.tab = ctx.feat = None
        return dimg, gc, gb, gbias, gs, None, None, None, None


def _conv_features(img, g, tab, nt, f_pad, has_base, desc):
    """The bf16 feature matrix of the implicit patch matrix, or None above the budget."""
    rows, cols = _rows_cols(g)
    if rows * cols * f_pad * 2 > _k.WGRAD_FEATURE_BYTES_MAX:
        return None
    feat = torch.empty(rows, cols * f_pad, device=img.device, dtype=torch.bfloat16)
    _k._launch("kf_conv_features", _k._ptr(img), ctypes.byref(g), _k._ptr(tab), _k._ptr(feat), nt, f_pad, int(has_base),
               ctypes.byref(desc), _k._stream(img))
    return feat


class _KANConvNd(nn.Module):
    n_dims = 0

    def __init__(self, in_channels: int, out_channels: int, kernel_size, stride=1, padding=0, dilation=1, groups: int = 1,
                 basis="bspline", padding_mode: str = "zeros", **kan_kwargs):
        super().__init__()
        n = self.n_dims
        if in_channels % groups or out_channels % groups:
            raise ValueError("in_channels and out_channels must be divisible by groups")
        if padding_mode not in PADDING_MODES:
            raise ValueError(f"unknown padding_mode {padding_mode!r}")
        self.in_channels, self.out_channels, self.groups = in_channels, out_channels, groups
        self.kernel_size = _per_dim(kernel_size, n, "kernel_size")
        self.stride = _per_dim(stride, n, "stride")
        self.padding = _per_dim(padding, n, "padding")
        self.dilation = _per_dim(dilation, n, "dilation")
        self.padding_mode = padding_mode
        fan_in = (in_channels // groups) * math.prod(self.kernel_size)
        self.kans = nn.ModuleList([KANLinear(fan_in, out_channels // groups, basis, **kan_kwargs) for _ in range(groups)])

    def _implicit(self, kan: KANLinear, x: torch.Tensor) -> bool:
        """Whether a group runs on the implicit-patch tensor-core kernels."""
        plan = kan._plan
        if x.dtype != torch.bfloat16 or plan is None or kan._sym_codes or (self.training and kan.edge_dropout > 0):
            return False
        if kan.base_weight is not None and kan.base_activation is not F.silu:
            return False
        probe = x.new_empty(0, kan.in_features)
        return _k.fused_ok(plan, probe, kan.out_features, kan.base_weight is not None, kan.coef.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x)
        n = self.n_dims
        if x.dim() != n + 2 or x.shape[1] != self.in_channels:
            raise ValueError(f"expected input (N, {self.in_channels}, *{n} spatial dims), got {tuple(x.shape)}")
        pad = self.padding
        if self.padding_mode != "zeros" and any(pad):
            x = F.pad(x, [p for d in reversed(range(n)) for p in (pad[d], pad[d])], mode=self.padding_mode)
            pad = (0,) * n
        x = x.contiguous()
        outs = []
        for grp, kan in enumerate(self.kans):
            g = _geometry(x, self, grp, pad)
            if self._implicit(kan, x):
                outs.append(_ImplicitConvKAN.apply(x, kan.coef, kan.base_weight, kan.bias, kan.edge_scale, kan.edge_mask,
                                                   kan._grid(), kan._plan, g))
            else:
                outs.append(kan(_Patches.apply(x, g)))
        g = _geometry(x, self, 0, pad)
        spatial = _out_shape(g)[3 - n:]
        y = torch.cat(outs, -1).reshape(x.shape[0], *spatial, self.out_channels)
        return y.permute(0, n + 1, *range(1, n + 1)).contiguous()

    @classmethod
    def from_conv(cls, conv: nn.Module, activation=None, basis="bspline", **kan_kwargs):
        """The KAN convolution equal to ``conv`` (reference kanforge/torch/conv.py:86-115):
        its weights become the base branch (identity activation unless
        ``activation`` is given) and the spline coefficients start at zero."""
        if not isinstance(conv.padding, tuple) or isinstance(conv.padding, str):
            raise ValueError("only numeric padding converts")
        layer = cls(conv.in_channels, conv.out_channels, conv.kernel_size, conv.stride, conv.padding, conv.dilation,
                    conv.groups, basis, conv.padding_mode, base_activation=activation or nn.Identity(),
                    bias=conv.bias is not None, coef_init="zero", device=conv.weight.device, dtype=conv.weight.dtype,
                    **kan_kwargs)
        per_group = conv.out_channels // conv.groups
        with torch.no_grad():
            for grp, kan in enumerate(layer.kans):
                rows = slice(grp * per_group, (grp + 1) * per_group)
                kan.base_weight.copy_(conv.weight[rows].reshape(per_group, -1))
                if conv.bias is not None:
                    kan.bias.copy_(conv.bias[rows])
        return layer

    def extra_repr(self) -> str:
        return (f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, stride={self.stride}, "
                f"padding={self.padding}, dilation={self.dilation}, groups={self.groups}")


class KANConv1d(_KANConvNd):
    n_dims = 1


class KANConv2d(_KANConvNd):
    n_dims = 2


class KANConv3d(_KANConvNd):
    n_dims = 3
