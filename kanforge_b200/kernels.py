"""Torch side of the sm_100a kernels: launchers and differentiable primitives.

Mirrors the reference module ``kanforge.torch.kernels`` (kanforge/torch/kernels.py):
``available``, ``_raw``, the closed autograd family ``prim_F / prim_G / prim_P``
and ``spline_forward`` keep their names and argument meaning, so code written
against the reference's kernel layer runs unchanged.  Every launch goes
through the C ABI of ``libkanb200`` (include/kanforge_b200.h) on torch's
current CUDA stream; there is no CPU or Triton path.

On top of the reference's primitives this module adds the fused training op
of the layer (``kan_linear_fused``: basis features, SiLU base branch and bias in
one tensor-core contraction per pass), the streaming ``edge_derivative`` and
the KAT rational activation.
"""

from __future__ import annotations

import ctypes
import functools
import math

import torch

from . import _lib
from ._init import silu_derivative_polys
from .plan import KernelPlan

_BF16 = torch.bfloat16

# Optional observer of kernel launches: a callable(name) returning a context
# manager entered around every compute entry point (bench.py records CUDA
# events with it); LAUNCH_COUNT counts library compute launches.
_observer = None
LAUNCH_COUNT = 0


def set_launch_observer(fn) -> None:
    global _observer
    _observer = fn


# Entry points that launch more than one kernel (partial sums + their reduction).
_KERNELS_PER_CALL = {"kf_rational_bwd": 2, "kf_rational_bwd_noalloc": 2, "kf_grkan_dgrad": 2}


def _launch(name: str, *args, kernels: int | None = None, label: str | None = None) -> None:
    """Call entry point `name`; `kernels` overrides how many kernels it launches,
    `label` the name the launch observer records (a variant of another entry)."""
    global LAUNCH_COUNT
    LAUNCH_COUNT += kernels if kernels is not None else _KERNELS_PER_CALL.get(name, 1)
    if _observer is None:
        _lib.call(name, *args)
        return
    with _observer(label or name):
        _lib.call(name, *args)


# Gradient-ready hook of data parallelism: a callable([(param, grad), ...])
# returning waitables, called by the tensor-core backward passes as soon as
# their parameter gradients are written and before the input-gradient kernel,
# so that the all-reduce of those gradients overlaps it (data_parallel.py).
_grad_hook = None


def set_grad_ready_hook(fn) -> None:
    global _grad_hook
    _grad_hook = fn


def _grads_ready(pairs) -> list:
    if _grad_hook is None:
        return []
    return _grad_hook([(p, g) for p, g in pairs if p is not None and g is not None])


def set_reserved_sms(n: int) -> None:
    """SMs the persistent tensor-core kernels leave to kernels on other streams
    (kf_set_reserved_sms); 0 restores every SM to them."""
    _lib.call("kf_set_reserved_sms", int(n))


def available(device: torch.device) -> bool:
    """True on CUDA devices with the library loaded (kanforge/torch/kernels.py:19-28)."""
    if torch.device(device).type != "cuda":
        return False
    _lib.load()
    return True


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _check_cuda(*ts) -> None:
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(f"kanforge_b200 kernels run on CUDA tensors only (got a {t.device} tensor)")


# --- raw launches (no autograd) ---------------------------------------------


def _prep(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().float()


def _raw(op: str, plan: KernelPlan, m: int, x, a, b, grid, n_out: int, nf: int) -> torch.Tensor:
    """op F: (x, w, cT) -> y; G: (x, w, g) -> GT; P: (x, g, cT) -> p (kanforge/torch/kernels.py:39-55)."""
    _check_cuda(x, a, b, grid)
    batch, n_in = x.shape
    code = {"F": _lib.KF_OP_F, "G": _lib.KF_OP_G, "P": _lib.KF_OP_P}[op]
    if op == "F":
        out = torch.empty(batch, n_out, device=x.device, dtype=torch.float32)
    elif op == "G":
        out = torch.empty(n_out, n_in, nf, device=x.device, dtype=torch.float32)
    else:
        out = torch.empty(batch, n_in, device=x.device, dtype=torch.float32)
    desc = plan.desc()
    _launch("kf_prim", code, m, _ptr(x), _ptr(a), _ptr(b), _ptr(grid), _ptr(out), batch, n_in, n_out, nf,
              ctypes.byref(desc), _stream(x))
    return out


@functools.lru_cache(maxsize=256)
def _fold_on(plan: KernelPlan, m: int, device: torch.device, dtype: torch.dtype = torch.float32):
    """R_m as a read-only device tensor, made once per (plan, order, device,
    dtype): building it is a pageable host-to-device copy, which would
    otherwise stall the stream on every call."""
    r = plan.fold(m)
    return None if r is None else torch.tensor(r, dtype=dtype, device=device)


def _fold(plan: KernelPlan, m: int, like: torch.Tensor):
    return _fold_on(plan, m, like.device, like.dtype)


# --- differentiable primitives (kanforge/torch/kernels.py:70-140) -------------


class _F(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, c, w, grid, plan, m):
        ctx.save_for_backward(x, c, w, grid)
        ctx.plan, ctx.m = plan, m
        r = _fold(plan, m, c)
        ct = c if r is None else c @ r
        return _raw("F", plan, plan.native_order(m), _prep(x), _prep(w), _prep(ct), _prep(grid), c.shape[0], ct.shape[-1])

    @staticmethod
    def backward(ctx, gy):
        x, c, w, grid = ctx.saved_tensors
        plan, m = ctx.plan, ctx.m
        need = ctx.needs_input_grad
        gx = w * prim_P(x, gy, c, grid, plan, m + 1) if need[0] else None
        gc = prim_G(x, gy, w, grid, plan, m) if need[1] else None
        gw = prim_P(x, gy, c, grid, plan, m) if need[2] else None
        return gx, gc, gw, None, None, None


class _G(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g, w, grid, plan, m):
        ctx.save_for_backward(x, g, w, grid)
        ctx.plan, ctx.m = plan, m
        nf = plan.n_features(m)
        gt = _raw("G", plan, plan.native_order(m), _prep(x), _prep(w), _prep(g), _prep(grid), g.shape[1], nf)
        r = _fold(plan, m, gt)
        return gt if r is None else gt @ r.T

    @staticmethod
    def backward(ctx, gg_out):
        x, g, w, grid = ctx.saved_tensors
        plan, m = ctx.plan, ctx.m
        need = ctx.needs_input_grad
        gx = w * prim_P(x, g, gg_out, grid, plan, m + 1) if need[0] else None
        gg = prim_F(x, gg_out, w, grid, plan, m) if need[1] else None
        gw = prim_P(x, g, gg_out, grid, plan, m) if need[2] else None
        return gx, gg, gw, None, None, None


class _P(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g, c, grid, plan, m):
        ctx.save_for_backward(x, g, c, grid)
        ctx.plan, ctx.m = plan, m
        r = _fold(plan, m, c)
        ct = c if r is None else c @ r
        return _raw("P", plan, plan.native_order(m), _prep(x), _prep(g), _prep(ct), _prep(grid), c.shape[0], ct.shape[-1])

    @staticmethod
    def backward(ctx, gp):
        x, g, c, grid = ctx.saved_tensors
        plan, m = ctx.plan, ctx.m
        need = ctx.needs_input_grad
        gx = gp * prim_P(x, g, c, grid, plan, m + 1) if need[0] else None
        gg = prim_F(x, c, gp, grid, plan, m) if need[1] else None
        gc = prim_G(x, g, gp, grid, plan, m) if need[2] else None
        return gx, gg, gc, None, None, None


def prim_F(x, c, w, grid, plan, m=0):
    return _F.apply(x, c, w, grid, plan, m)


def prim_G(x, g, w, grid, plan, m=0):
    return _G.apply(x, g, w, grid, plan, m)


def prim_P(x, g, c, grid, plan, m=0):
    return _P.apply(x, g, c, grid, plan, m)


def spline_forward(x: torch.Tensor, coef: torch.Tensor, grid: torch.Tensor | None, plan: KernelPlan) -> torch.Tensor:
    """sum_{i,k} coef[o,i,k] phi_k(x[..., i]) through the float32 primitive (kernels.py:143-150)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if grid is None:
        grid = x2.new_zeros(1, dtype=torch.float32)
    y = prim_F(x2.float(), coef.float(), torch.ones_like(x2, dtype=torch.float32), grid.float(), plan, 0)
    return y.to(x.dtype).reshape(*lead, coef.shape[0])


# --- fused layer op (tcgen05) ------------------------------------------------


def knot_tables(grid: torch.Tensor, plan: KernelPlan) -> torch.Tensor:
    """(I, order + 1, 64) knot / reciprocal-difference tables of the per-input grids."""
    g = grid.detach().float().contiguous()
    n_in = g.shape[0]
    grid_size, order = plan.consts
    tab = torch.empty(n_in, order + 1, 64, device=g.device, dtype=torch.float32)
    _launch("kf_knot_tables", _ptr(g), _ptr(tab), n_in, grid_size, order, _stream(g))
    return tab


def fused_layout(plan: KernelPlan, has_base: bool) -> tuple[int, int]:
    """(nt, f_pad): basis feature columns per input and the padded width (16 or
    32); the last padded column carries the SiLU base branch."""
    nt = plan.n_features(0)
    return nt, (16 if nt + 1 <= 16 else 32)


def fused_ok(plan: KernelPlan | None, x: torch.Tensor, n_out: int, has_base: bool, coef_dtype=None) -> bool:
    """Whether the tensor-core path serves this call: bf16 inputs and parameters,
    CUDA, a B-spline or Chebyshev-feature plan with <= 31 feature columns,
    outputs a multiple of 8."""
    if plan is None or plan.kind not in ("cheb", "bspline", "fourier") or x.dtype != _BF16 or x.device.type != "cuda":
        return False
    if coef_dtype is not None and coef_dtype != _BF16:
        return False
    nt, _ = fused_layout(plan, has_base)
    if nt + 1 > 32 or n_out % 8:
        return False
    return plan.supported(_lib.KF_QUERY_FUSED, _lib.KF_DTYPE_BF16)


def _bf16_or_none(t):
    return None if t is None else _aligned16(t.detach().to(_BF16).contiguous())


def _aligned16(t: torch.Tensor) -> torch.Tensor:
    """t, or a copy of it when its data does not start on a 16-byte boundary
    (a view into a larger tensor): the kernels read it in 16-byte vectors."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def pack_coef(coef, base, edge_scale, edge_mask, plan: KernelPlan, f_pad: int) -> torch.Tensor:
    """The bf16 tensor-core operand (O, I * f_pad): coef * edge_scale * edge_mask
    folded into Chebyshev features, and the masked base weight in the last column."""
    n_out, n_in, k = coef.shape
    nt = plan.n_features(0)
    coef = coef.detach().contiguous()
    dt = _lib.KF_DTYPE_BF16 if coef.dtype == _BF16 else _lib.KF_DTYPE_F32
    if dt == _lib.KF_DTYPE_F32:
        coef = coef.float()
    like = coef.dtype
    conv = lambda t: None if t is None else t.detach().to(like).contiguous()  # noqa: E731
    base, scale, mask = conv(base), conv(edge_scale), conv(edge_mask)
    fold = None
    if plan.folded and not plan.is_identity_fold():
        fold = _fold_on(plan, 0, coef.device)
    packed = torch.empty(n_out, n_in * f_pad, device=coef.device, dtype=_BF16)
    _launch("kf_pack_coef", _ptr(coef), _ptr(base), _ptr(scale), _ptr(mask), _ptr(fold), _ptr(packed), n_out, n_in, k,
            nt, f_pad, dt, _stream(coef))
    return packed


# The coefficient gradient reads the basis features from a (B, I * f_pad) bf16
# matrix made by kf_features when it fits in this budget (2.1 GB at 16384
# tokens x 4096 inputs); above it, or if the allocation fails, the kernel
# evaluates the features itself (slower, no extra memory).  For B-spline plans,
# whose features are costly to evaluate inside the forward's producer warps,
# the matrix is made in the forward, read there by TMA too, and kept until the
# backward (activation memory traded for one evaluation instead of one per
# output tile); Chebyshev-feature and Fourier plans have the forward kernel
# write it (FEATURES_EMITTED_BY_FORWARD below), or make it in the backward.
WGRAD_FEATURE_BYTES_MAX = 16 << 30

# Plan kinds whose bf16 forward makes the feature matrix and reads it by TMA
# (kept for the coefficient gradient) instead of evaluating the features in
# the forward kernel's producer warps.
FEATURES_IN_FORWARD = ("bspline",)

# Plan kinds whose forward producer warps, which evaluate every feature row,
# also write the feature matrix (kf_fwd_emit_features) when the coefficient
# gradient will need it and it fits this budget: the backward then skips
# kf_features.  The matrix is held from the forward to the backward, like an
# activation (2.1 GB at 16384 tokens x 4096 inputs).
FEATURES_EMITTED_BY_FORWARD = ("cheb", "fourier")
FORWARD_FEATURE_BYTES_MAX = 4 << 30


def _emitted_features(x, f_pad):
    """An empty (B, I * f_pad) bf16 matrix for the forward to fill, or None."""
    if x.shape[0] * x.shape[1] * f_pad * 2 > FORWARD_FEATURE_BYTES_MAX:
        return None
    try:
        return torch.empty(x.shape[0], x.shape[1] * f_pad, device=x.device, dtype=_BF16)
    except torch.cuda.OutOfMemoryError:
        return None


def wgrad_features(x, knot_tab, nt, f_pad, has_base, desc, stream):
    """The feature matrix of x for kf_wgrad, or None for its self-evaluating path."""
    nbytes = x.shape[0] * x.shape[1] * f_pad * 2
    if nbytes > WGRAD_FEATURE_BYTES_MAX:
        return None
    try:
        feat = torch.empty(x.shape[0], x.shape[1] * f_pad, device=x.device, dtype=_BF16)
    except torch.cuda.OutOfMemoryError:
        return None
    _launch("kf_features", _ptr(x), _ptr(knot_tab), _ptr(feat), x.shape[0], x.shape[1], nt, f_pad, int(has_base),
            ctypes.byref(desc), stream)
    return feat


class _FusedKANLinear(torch.autograd.Function):
    """y = sum_{i,j} feat_j(x_i) C_eff[o,i,j] + silu(x_i) W_eff[o,i] + b_o in one
    tcgen05 contraction per pass (forward, input gradient, coefficient gradient),
    with C_eff = coef * edge_scale * edge_mask and W_eff = base_weight * edge_mask
    (kanforge/torch/layers.py:162-191) formed inside the kernels.

    When the backward itself is differentiated (create_graph), the gradients are
    built from the closed float32 primitives instead, so every order works as in
    the reference (kanforge/torch/kernels.py:79-87)."""

    @staticmethod
    def forward(ctx, x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
        n_out, n_in, _ = coef.shape
        has_base = base_weight is not None
        nt, f_pad = fused_layout(plan, has_base)
        x = x.contiguous()
        packed = pack_coef(coef, base_weight, edge_scale, edge_mask, plan, f_pad)
        y = torch.empty(x.shape[0], n_out, device=x.device, dtype=_BF16)
        b = _bf16_or_none(bias)
        g = None if grid is None else grid.detach().float().contiguous()
        tab = None if grid is None else knot_tables(g, plan)
        desc = plan.desc()
        need = ctx.needs_input_grad
        feat = None
        if plan.kind in FEATURES_IN_FORWARD:
            feat = wgrad_features(x, tab, nt, f_pad, has_base, desc, _stream(x))
        elif plan.kind in FEATURES_EMITTED_BY_FORWARD and (need[1] or need[2] or need[4]):
            feat = _emitted_features(x, f_pad)
        if feat is not None and plan.kind in FEATURES_EMITTED_BY_FORWARD:
            _launch("kf_fwd_emit_features", _ptr(x), _ptr(packed), _ptr(b), _ptr(tab), _ptr(y), _ptr(feat), x.shape[0],
                    n_in, n_out, nt, f_pad, int(has_base), ctypes.byref(desc), _stream(x), label="kf_fwd")
        else:
            _launch("kf_fwd", _ptr(x), _ptr(feat), _ptr(packed), _ptr(b), _ptr(tab), _ptr(y), x.shape[0], n_in, n_out, nt,
                    f_pad, int(has_base), ctypes.byref(desc), _stream(x))
        ctx.save_for_backward(x, coef, base_weight, edge_scale, edge_mask, g)
        ctx.packed, ctx.knot_tab, ctx.plan, ctx.has_bias = packed, tab, plan, bias is not None
        ctx.feat = feat
        ctx.layout = (nt, f_pad)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, coef, base_weight, edge_scale, edge_mask, grid = ctx.saved_tensors
        plan = ctx.plan
        need = ctx.needs_input_grad
        if torch.is_grad_enabled():
            ctx.packed = ctx.knot_tab = ctx.feat = None
            return _fused_backward_differentiable(x, gy, coef, base_weight, edge_scale, edge_mask, grid, plan, need,
                                                  ctx.has_bias)
        nt, f_pad = ctx.layout
        n_out, n_in, k = coef.shape
        gy = gy.to(_BF16).contiguous()
        desc = plan.desc()
        stream = _stream(x)
        gx = gc = gb = gbias = gs = None
        if need[1] or need[2] or need[4]:
            gc = torch.empty(n_out, n_in, k, device=x.device, dtype=_BF16)
            gb = torch.empty(n_out, n_in, device=x.device, dtype=_BF16) if base_weight is not None else None
            gs = torch.empty(n_out, n_in, device=x.device, dtype=_BF16) if (edge_scale is not None and need[4]) else None
            fold = None
            if plan.folded and not plan.is_identity_fold():
                fold = _fold_on(plan, 0, x.device)
            cf, sc, mk = _bf16_or_none(coef), _bf16_or_none(edge_scale), _bf16_or_none(edge_mask)
            feat = ctx.feat if ctx.feat is not None else wgrad_features(x, ctx.knot_tab, nt, f_pad,
                                                                         base_weight is not None, desc, stream)
            _launch("kf_wgrad", _ptr(x), _ptr(feat), _ptr(gy), _ptr(ctx.knot_tab), _ptr(fold), _ptr(cf), _ptr(sc), _ptr(mk),
                    _ptr(gc), _ptr(gb), _ptr(gs), x.shape[0], n_in, n_out, k, nt, f_pad, ctypes.byref(desc), stream)
            del feat
            gc = gc.to(coef.dtype) if need[1] else None
            gb = gb.to(base_weight.dtype) if (gb is not None and need[2]) else None
            gs = gs.to(edge_scale.dtype) if gs is not None else None
        # the parameter gradients are complete: a registered hook (data
        # parallelism) can start their all-reduce now, beside the input gradient
        pending = _grads_ready([(coef, gc), (base_weight, gb), (edge_scale, gs)])
        if need[0]:
            gx = torch.empty_like(x)
            _launch("kf_dgrad", _ptr(x), _ptr(gy), _ptr(ctx.packed), _ptr(ctx.knot_tab), _ptr(gx), x.shape[0], n_in, n_out,
                    nt, f_pad, int(base_weight is not None), ctypes.byref(desc), stream)
        if need[3]:
            gbias = gy.sum(0, dtype=torch.float32)
        for work in pending:
            work.wait()
        ctx.packed = ctx.knot_tab = ctx.feat = None
        return gx, gc, gb, gbias, gs, None, None, None


def _fused_backward_differentiable(x, gy, coef, base_weight, edge_scale, edge_mask, grid, plan, need, has_bias):
    """Gradients of the fused op as a graph of float32 primitives (create_graph=True)."""
    xf = x.float()
    gyf = gy.float()
    ones = torch.ones_like(xf)
    g = grid if grid is not None else xf.new_zeros(1)
    mask = edge_mask.float() if edge_mask is not None else torch.ones(coef.shape[:2], device=x.device)
    sm = mask if edge_scale is None else edge_scale.float() * mask
    ce = coef.float() * sm[..., None]
    gx = gc = gb = gbias = gs = None
    if need[0]:
        gx = prim_P(xf, gyf, ce, g, plan, 1)
        if base_weight is not None:
            s = torch.sigmoid(xf)
            gx = gx + (gyf @ (base_weight.float() * mask)) * (s * (1 + xf * (1 - s)))
        gx = gx.to(x.dtype)
    if need[1] or need[4]:
        gce = prim_G(xf, gyf, ones, g, plan, 0)
        if need[1]:
            gc = (gce * sm[..., None]).to(coef.dtype)
        if need[4] and edge_scale is not None:
            gs = ((gce * coef.float()).sum(-1) * mask).to(edge_scale.dtype)
    if need[2] and base_weight is not None:
        gb = ((gyf.T @ torch.nn.functional.silu(xf)) * mask).to(base_weight.dtype)
    if need[3] and has_bias:
        gbias = gyf.sum(0)
    return gx, gc, gb, gbias, gs, None, None, None


def kan_linear_fused(x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
    """Fused KANLinear on (..., I) bf16 inputs; see ``_FusedKANLinear``."""
    lead = x.shape[:-1]
    y = _FusedKANLinear.apply(x.reshape(-1, x.shape[-1]), coef, base_weight, bias, edge_scale, edge_mask, grid, plan)
    return y.reshape(*lead, coef.shape[0])


# --- float32 layers on the tensor cores (three TF32 products) ------------------

# Float32 layers run their contractions on the tensor cores (kf_gemm_tf32x3);
# False routes them through the closed float32 CUDA-core primitives instead.
FP32_TENSOR_CORES = True

# The float32 tensor-core path holds a (B, I * f_pad) float32 feature matrix
# from the forward to the backward and makes a second one (the feature
# gradient) in the backward; above this many bytes for the two, calls take the
# primitives, which need no such buffers.
FP32_FEATURE_BYTES_MAX = 32 << 30


def tf32_ok(plan: KernelPlan | None, x: torch.Tensor, n_out: int, has_base: bool, coef_dtype=None) -> bool:
    """Whether the float32 tensor-core path serves this call: float32 inputs and
    parameters on CUDA, a B-spline or Chebyshev-feature plan with <= 31 feature
    columns, outputs a multiple of 4."""
    if plan is None or plan.kind not in ("cheb", "bspline", "fourier", "bump") or x.dtype != torch.float32 or x.device.type != "cuda":
        return False
    if coef_dtype is not None and coef_dtype != torch.float32:
        return False
    nt, f_pad = fused_layout(plan, has_base)
    if nt + 1 > 32 or n_out % 4:
        return False
    if 2 * 4 * x.numel() * f_pad > FP32_FEATURE_BYTES_MAX:
        return False
    return plan.supported(_lib.KF_OP_F, _lib.KF_DTYPE_F32)


def gemm_tf32x3(a, a_mn: bool, b, b_mn: bool, out, m: int, n: int, k: int, bias=None):
    """out (m, n) = A B^T (+ bias) through kf_gemm_tf32x3; A (m, k) stored K-major
    (a_mn False) or as its (k, m) transpose, B (n, k) likewise."""
    _launch("kf_gemm_tf32x3", _ptr(a), int(a_mn), a.stride(0), _ptr(b), int(b_mn), b.stride(0), _ptr(bias), _ptr(out),
            out.stride(0), m, n, k, _stream(out))
    return out


def packed_f32(coef, base_weight, edge_scale, edge_mask, plan: KernelPlan, f_pad: int) -> torch.Tensor:
    """The float32 operand (O, I * f_pad) of the layout of kf_pack_coef:
    coef * edge_scale * edge_mask (folded into Chebyshev features), zero
    padding, and base_weight * edge_mask in the last column."""
    n_out, n_in, _ = coef.shape
    nt = plan.n_features(0)
    sm = edge_mask.float() if edge_mask is not None else None
    if edge_scale is not None:
        sm = edge_scale.float() if sm is None else edge_scale.float() * sm
    ce = coef.float() if sm is None else coef.float() * sm[..., None]
    if plan.folded and not plan.is_identity_fold():
        ce = ce @ _fold_on(plan, 0, coef.device)
    parts = [ce[..., :nt], ce.new_zeros(n_out, n_in, f_pad - nt - 1)]
    if base_weight is not None:
        bw = base_weight.float() if edge_mask is None else base_weight.float() * edge_mask.float()
        parts.append(bw[..., None])
    else:
        parts.append(ce.new_zeros(n_out, n_in, 1))
    return torch.cat(parts, -1).reshape(n_out, n_in * f_pad).contiguous()


class _Tf32KANLinear(torch.autograd.Function):
    """Float32 KANLinear as three tcgen05 contractions with TF32 hi/lo splits
    (float32 accuracy): y = feat packed^T + b, dfeat = dy packed (then dx by
    the feature derivatives), dpacked = dy^T feat, with the chain rule of
    the packed operand (fold, edge_scale, edge_mask, base column) applied by
    torch on the (O, I, f_pad) gradient.  Double backward falls back to the
    closed float32 primitives, as in the bf16 path."""

    @staticmethod
    def forward(ctx, x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
        n_out, n_in, _ = coef.shape
        has_base = base_weight is not None
        nt, f_pad = fused_layout(plan, has_base)
        x = x.contiguous()
        n_b = x.shape[0]
        det = lambda t: None if t is None else t.detach()  # noqa: E731
        packed = packed_f32(coef.detach(), det(base_weight), det(edge_scale), det(edge_mask), plan, f_pad)
        g = None if grid is None else grid.detach().float().contiguous()
        desc = plan.desc()
        feat = torch.empty(n_b, n_in * f_pad, device=x.device, dtype=torch.float32)
        if plan.kind == "bspline":
            tab = knot_tables(g, plan)
            _launch("kf_features_spline_f32", _ptr(x), _ptr(tab), _ptr(feat), n_b, n_in, nt, f_pad, int(has_base),
                    ctypes.byref(desc), _stream(x))
            del tab
        else:
            _launch("kf_features_f32", _ptr(x), _ptr(g), _ptr(feat), n_b, n_in, nt, f_pad, int(has_base),
                    ctypes.byref(desc), _stream(x))
        y = torch.empty(n_b, n_out, device=x.device, dtype=torch.float32)
        b = None if bias is None else bias.detach().float().contiguous()
        gemm_tf32x3(feat, False, packed, False, y, n_b, n_out, n_in * f_pad, bias=b)
        ctx.save_for_backward(x, coef, base_weight, edge_scale, edge_mask, g)
        ctx.feat, ctx.packed, ctx.plan, ctx.has_bias, ctx.layout = feat, packed, plan, bias is not None, (nt, f_pad)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, coef, base_weight, edge_scale, edge_mask, grid = ctx.saved_tensors
        plan = ctx.plan
        need = ctx.needs_input_grad
        if torch.is_grad_enabled():
            ctx.feat = ctx.packed = None
            return _fused_backward_differentiable(x, gy, coef, base_weight, edge_scale, edge_mask, grid, plan, need,
                                                  ctx.has_bias)
        nt, f_pad = ctx.layout
        n_out, n_in, k = coef.shape
        n_b = x.shape[0]
        gy = gy.float().contiguous()
        desc = plan.desc()
        gx = gc = gb = gbias = gs = None
        if need[0]:
            dfeat = torch.empty(n_b, n_in * f_pad, device=x.device, dtype=torch.float32)
            gemm_tf32x3(gy, False, ctx.packed, True, dfeat, n_b, n_in * f_pad, n_out)
            gx = torch.empty_like(x)
            _launch("kf_features_dot_f32", _ptr(x), _ptr(grid), _ptr(dfeat), _ptr(gx), n_b, n_in, nt, f_pad,
                    int(base_weight is not None), ctypes.byref(desc), _stream(x))
            del dfeat
        if need[1] or need[2] or need[4]:
            dpacked = torch.empty(n_out, n_in * f_pad, device=x.device, dtype=torch.float32)
            gemm_tf32x3(gy, True, ctx.feat, True, dpacked, n_out, n_in * f_pad, n_b)
            dp = dpacked.view(n_out, n_in, f_pad)
            dce = dp[..., :nt]
            if plan.folded and not plan.is_identity_fold():
                dce = dce @ _fold_on(plan, 0, x.device).T
            mask = edge_mask.float() if edge_mask is not None else None
            sm = mask
            if edge_scale is not None:
                sm = edge_scale.float() if sm is None else edge_scale.float() * sm
            if need[1]:
                gc = (dce if sm is None else dce * sm[..., None]).to(coef.dtype)
            if need[4] and edge_scale is not None:
                gsc = (dce * coef.float()).sum(-1)
                gs = (gsc if mask is None else gsc * mask).to(edge_scale.dtype)
            if need[2] and base_weight is not None:
                gbv = dp[..., f_pad - 1]
                gb = (gbv if mask is None else gbv * mask).to(base_weight.dtype)
        if need[3] and ctx.has_bias:
            gbias = gy.sum(0)
        ctx.feat = ctx.packed = None
        return gx, gc, gb, gbias, gs, None, None, None


def kan_linear_tf32(x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
    """Float32 KANLinear on (..., I) inputs through the tensor cores; see ``_Tf32KANLinear``."""
    lead = x.shape[:-1]
    y = _Tf32KANLinear.apply(x.reshape(-1, x.shape[-1]), coef, base_weight, bias, edge_scale, edge_mask, grid, plan)
    return y.reshape(*lead, coef.shape[0])


# --- edge_derivative ---------------------------------------------------------


# --- sparse B-spline (kanforge/bases/base.py:15-16 local / support) ------------

# float32 B-spline layers with at most this many outputs gather the k+1 non-zero
# coefficients per (token, input) on the CUDA cores (kf_sparse_*); wider layers
# run the dense three-TF32 tensor-core contraction (measured crossover between
# 16 and 32 outputs: 65536 x 1024 -> 8 fwd+bwd 7.5 against 9.5 ms, -> 32 15.9
# against 9.6 ms).
SPARSE_MAX_OUT = 16


def sparse_ok(plan: KernelPlan | None, x: torch.Tensor, n_out: int, coef_dtype, has_tf32: bool) -> bool:
    """Whether a float32 B-spline layer takes the sparse kernels: narrow layers,
    and shapes the tensor-core path does not take."""
    if plan is None or plan.kind != "bspline" or not 1 <= plan.consts[1] <= 5:
        return False
    if x.dtype != torch.float32 or coef_dtype != torch.float32 or x.device.type != "cuda":
        return False
    return n_out <= SPARSE_MAX_OUT or not has_tf32


class _SparseKANLinear(torch.autograd.Function):
    """Float32 B-spline KANLinear on the sparse gather kernels: forward, input
    gradient and parameter gradients (fixed-order sums) each one library call.
    Double backward falls back to the closed float32 primitives."""

    @staticmethod
    def forward(ctx, x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
        x = x.contiguous()
        n_b, n_in = x.shape
        n_out = coef.shape[0]
        f = lambda t: None if t is None else t.detach().float().contiguous()  # noqa: E731
        y = torch.empty(n_b, n_out, device=x.device, dtype=torch.float32)
        desc = plan.desc()
        _launch("kf_sparse_fwd", _ptr(x), _ptr(f(coef)), _ptr(f(edge_scale)), _ptr(f(edge_mask)), _ptr(f(base_weight)),
                _ptr(f(bias)), _ptr(f(grid)), _ptr(y), n_b, n_in, n_out, ctypes.byref(desc), _stream(x))
        ctx.save_for_backward(x, coef, base_weight, edge_scale, edge_mask, grid)
        ctx.plan, ctx.has_bias = plan, bias is not None
        return y

    @staticmethod
    def backward(ctx, gy):
        x, coef, base_weight, edge_scale, edge_mask, grid = ctx.saved_tensors
        plan, need = ctx.plan, ctx.needs_input_grad
        if torch.is_grad_enabled():
            return _fused_backward_differentiable(x, gy, coef, base_weight, edge_scale, edge_mask, grid, plan, need,
                                                  ctx.has_bias)
        f = lambda t: None if t is None else t.detach().float().contiguous()  # noqa: E731
        gy = gy.float().contiguous()
        n_b, n_in = x.shape
        n_out = coef.shape[0]
        desc = plan.desc()
        c, s, m, w, g = f(coef), f(edge_scale), f(edge_mask), f(base_weight), f(grid)
        gx = gc = gb = gbias = gs = None
        if need[0]:
            gx = torch.empty_like(x)
            _launch("kf_sparse_dgrad", _ptr(x), _ptr(gy), _ptr(c), _ptr(s), _ptr(m), _ptr(w), _ptr(g), _ptr(gx), n_b,
                    n_in, n_out, ctypes.byref(desc), _stream(x))
        want_c, want_b = need[1], need[2] and base_weight is not None
        want_bias, want_s = need[3] and ctx.has_bias, need[4] and edge_scale is not None
        if want_c or want_b or want_bias or want_s:
            n_ws = _lib.load().kf_sparse_wgrad_workspace(n_b, n_in, n_out, ctypes.byref(desc))
            ws = torch.empty(max(n_ws, 1), device=x.device, dtype=torch.float32)
            gc = torch.empty_like(c) if want_c else None
            gb = torch.empty_like(w) if want_b else None
            gbias = torch.empty(n_out, device=x.device, dtype=torch.float32) if want_bias else None
            gs = torch.empty_like(s) if want_s else None
            _launch("kf_sparse_wgrad", _ptr(x), _ptr(gy), _ptr(c), _ptr(s), _ptr(m), _ptr(g), _ptr(gc), _ptr(gb),
                    _ptr(gs), _ptr(gbias), _ptr(ws), n_b, n_in, n_out, ctypes.byref(desc), _stream(x), kernels=2)
        return gx, gc, gb, gbias, gs, None, None, None


def kan_linear_sparse(x, coef, base_weight, bias, edge_scale, edge_mask, grid, plan):
    """Float32 B-spline KANLinear on (..., I) inputs by the sparse kernels; see ``_SparseKANLinear``."""
    lead = x.shape[:-1]
    y = _SparseKANLinear.apply(x.reshape(-1, x.shape[-1]), coef, base_weight, bias, edge_scale, edge_mask, grid, plan)
    return y.reshape(*lead, coef.shape[0])


def _silu_polys(order: int):
    """(ctypes float array, n): silu^(order) as [h_m, h_{m-1}] polynomials in sigmoid."""
    polys = silu_derivative_polys(order).astype("float32").ravel()
    return (ctypes.c_float * polys.size)(*polys.tolist()), polys.size // 2


def _edge_coef(coef_eff: torch.Tensor, plan: KernelPlan, order: int) -> torch.Tensor:
    """(O, nf, I) float32 coefficients of the order-`order` features: folded
    into the kernel features for Chebyshev / Fourier plans."""
    c = coef_eff.detach().float()
    if plan.folded:
        c = c @ _fold_on(plan, order, c.device)
    return c.permute(0, 2, 1).contiguous()


class _EdgeDerivative(torch.autograd.Function):
    """out[b,o,i] = d^m/dx^m (phi_oi(x_i) + W_eff[o,i] silu(x_i)) (kanforge/torch/layers.py:206-226),
    differentiable in x, the effective coefficients and the base weight like
    the reference's autograd graph: dx from the order-(m+1) edges contracted
    with the output gradient (kf_edge_derivative_dx), the coefficient and base
    gradients from the order-m features (kf_edge_derivative_dcoef)."""

    @staticmethod
    def forward(ctx, x2, coef_eff, base_eff, num, den, grid, plan, order, groups):
        n_out, n_in, _ = coef_eff.shape
        coef_c = _edge_coef(coef_eff, plan, order)
        base = None if base_eff is None else base_eff.detach().float().contiguous()
        g = None if grid is None else grid.detach().float().contiguous()
        numf = None if num is None else num.detach().float().contiguous()
        denf = None if den is None else den.detach().float().contiguous()
        poly_buf, n_poly = _silu_polys(order)
        out = torch.empty(x2.shape[0], n_out, n_in, device=x2.device, dtype=torch.float32)
        desc = plan.desc(groups)
        _launch("kf_edge_derivative", _ptr(x2), _ptr(coef_c), _ptr(base), _ptr(g), _ptr(numf), _ptr(denf), _ptr(out),
                x2.shape[0], n_in, n_out, coef_c.shape[1], order, ctypes.byref(desc), ctypes.cast(poly_buf, ctypes.c_void_p),
                n_poly, _stream(x2))
        ctx.save_for_backward(x2, coef_eff, base_eff)
        ctx.extra = (numf, denf, g, plan, order, groups)
        return out

    @staticmethod
    def backward(ctx, gout):
        x2, coef_eff, base_eff = ctx.saved_tensors
        numf, denf, g, plan, order, groups = ctx.extra
        need = ctx.needs_input_grad
        if need[3] or need[4]:
            raise NotImplementedError("gradients of edge derivatives into the rational parameters are not available")
        gout = gout.float().contiguous()
        n_b, n_in = x2.shape
        n_out = coef_eff.shape[0]
        desc = plan.desc(groups)
        stream = _stream(x2)
        dx = dcoef = dbase = None
        if need[0]:
            coef1 = _edge_coef(coef_eff, plan, order + 1)
            base = None if base_eff is None else base_eff.detach().float().contiguous()
            poly_buf, n_poly = _silu_polys(order + 1)
            dx = torch.empty_like(x2)
            _launch("kf_edge_derivative_dx", _ptr(x2), _ptr(gout), _ptr(coef1), _ptr(base), _ptr(g), _ptr(numf), _ptr(denf),
                    _ptr(dx), n_b, n_in, n_out, coef1.shape[1], order + 1, ctypes.byref(desc),
                    ctypes.cast(poly_buf, ctypes.c_void_p), n_poly, stream)
        if need[1] or need[2]:
            nf = plan.n_features(order) if plan.kind != "rational" else 1
            dct = torch.empty(n_out, nf, n_in, device=x2.device, dtype=torch.float32)
            db = torch.empty(n_out, n_in, device=x2.device, dtype=torch.float32) if (need[2] and base_eff is not None) else None
            ws_n = int(_lib.load().kf_edge_derivative_workspace(n_b, n_in, n_out, nf))
            ws = torch.empty(max(ws_n, 1), device=x2.device, dtype=torch.float32)
            poly_buf, n_poly = _silu_polys(order)
            _launch("kf_edge_derivative_dcoef", _ptr(x2), _ptr(gout), _ptr(g), _ptr(numf), _ptr(denf), _ptr(dct), _ptr(db),
                    _ptr(ws), n_b, n_in, n_out, nf, order, ctypes.byref(desc), ctypes.cast(poly_buf, ctypes.c_void_p),
                    n_poly, stream, kernels=2)
            if need[1]:
                d = dct.permute(0, 2, 1)  # (O, I, nf)
                if plan.folded:
                    d = d @ _fold_on(plan, order, x2.device).T  # features -> basis functions
                dcoef = d.to(coef_eff.dtype)
            if db is not None:
                dbase = db.to(base_eff.dtype)
        return dx, dcoef, dbase, None, None, None, None, None, None


def edge_derivative(x, coef_eff, base_eff, grid, plan: KernelPlan, order: int, basis_params: dict | None = None,
                    groups: int = 1) -> torch.Tensor:
    """(..., O, I) d^m phi_oi / dx_i^m + silu^(m) W_eff, float32 (kanforge/torch/layers.py:206-226);
    differentiable in x, coef_eff and base_eff."""
    _check_cuda(x)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).float().contiguous()
    num = den = None
    if plan.kind == "rational":
        num, den = basis_params["numerator"], basis_params["denominator"]
    out = _EdgeDerivative.apply(x2, coef_eff, base_eff, num, den, grid, plan, order, groups)
    return out.reshape(*lead, coef_eff.shape[0], coef_eff.shape[1])


# --- KAT rational ------------------------------------------------------------


def _rat_dtype(t: torch.Tensor) -> int:
    if t.dtype == _BF16:
        return _lib.KF_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.KF_DTYPE_F32
    raise RuntimeError(f"rational kernels take float32 or bfloat16, not {t.dtype}")


class _RationalAct(torch.autograd.Function):
    """R_g^(m)(x) of the group rational; d/dx is R^(m+1) (closed in x), the
    parameter gradient of order 0 comes from the fused backward kernel."""

    @staticmethod
    def forward(ctx, x, num, den, plan, groups, m):
        _check_cuda(x)
        x = x.contiguous()
        if x.dtype not in (torch.float32, _BF16):
            x = x.float()
        numf, denf = num.detach().float().contiguous(), den.detach().float().contiguous()
        out = torch.empty_like(x)
        desc = plan.desc(groups)
        _launch("kf_rational_act", _ptr(x), _ptr(numf), _ptr(denf), _ptr(out), x.shape[0], x.shape[1], m,
                  ctypes.byref(desc), _rat_dtype(x), _stream(x))
        ctx.save_for_backward(x, num, den)
        ctx.plan, ctx.groups, ctx.m = plan, groups, m
        return out

    @staticmethod
    def backward(ctx, g):
        x, num, den = ctx.saved_tensors
        plan, groups, m = ctx.plan, ctx.groups, ctx.m
        need = ctx.needs_input_grad
        if m == 0 and not torch.is_grad_enabled():
            g = g.to(x.dtype).contiguous()
            dx = torch.empty_like(x)
            dnum = torch.empty(num.shape, device=x.device, dtype=torch.float32)
            dden = torch.empty(den.shape, device=x.device, dtype=torch.float32)
            desc = plan.desc(groups)
            ws_n = _lib.load().kf_rational_workspace(x.shape[0], x.shape[1], ctypes.byref(desc))
            ws = torch.empty(max(int(ws_n), 1), device=x.device, dtype=torch.float32)
            # keep the float32 copies alive until the launch is enqueued
            numf, denf = num.detach().float().contiguous(), den.detach().float().contiguous()
            _launch("kf_rational_bwd", _ptr(x), _ptr(g), _ptr(numf), _ptr(denf), _ptr(dx), _ptr(dnum), _ptr(dden),
                    _ptr(ws), x.shape[0], x.shape[1], ctypes.byref(desc), _rat_dtype(x), _stream(x))
            return (dx if need[0] else None, dnum.to(num.dtype) if need[1] else None,
                    dden.to(den.dtype) if need[2] else None, None, None, None)
        if need[1] or need[2]:
            raise NotImplementedError(
                "gradients of higher derivatives of the rational activation into its parameters are not available"
            )
        dx = g * _RationalAct.apply(x, num, den, plan, groups, m + 1) if need[0] else None
        return dx, None, None, None, None, None


def rational_act(x2, num, den, plan, groups, m=0):
    return _RationalAct.apply(x2, num, den, plan, groups, m)


# --- GR-KAN layers: the rational activation and the linear map on our GEMMs ---


def grkan_ok(plan: KernelPlan | None, x: torch.Tensor, n_in: int, n_out: int, groups: int, coef_dtype) -> str | None:
    """Which GEMM path serves a GR-KAN layer call: "bf16" (the tcgen05
    contractions with the rational backward fused into the input gradient;
    degrees (5, 4), inputs per group a multiple of 32, outputs a multiple of
    8), "f32" (the rational kernels around three-TF32-product GEMMs; inputs and
    outputs multiples of 4), or None."""
    if plan is None or plan.kind != "rational" or x.device.type != "cuda" or coef_dtype != x.dtype:
        return None
    if n_in % groups:
        return None
    if x.dtype == _BF16:
        num_deg, den_deg = plan.consts
        if (num_deg, den_deg) == (5, 4) and (n_in // groups) % 32 == 0 and n_out % 8 == 0:
            return "bf16"
        return None
    if x.dtype == torch.float32 and n_in % 4 == 0 and n_out % 4 == 0 and FP32_TENSOR_CORES:
        return "f32"
    return None


def _grkan_reference_grads(x, num, den, w, bias, plan, groups, gy, need):
    """Gradients of the GR-KAN layer as a differentiable graph (create_graph)."""
    with torch.enable_grad():
        leaves = [t.detach().requires_grad_(n) if t is not None else None for t, n in zip((x, num, den, w, bias), need)]
        r = rational_act(leaves[0], leaves[1], leaves[2], plan, groups)
        y = torch.nn.functional.linear(r.to(leaves[3].dtype), leaves[3], leaves[4])
        want = [t for t, n in zip(leaves, need) if n and t is not None]
        got = iter(torch.autograd.grad(y, want, gy, create_graph=True))
    return tuple(next(got) if (n and t is not None) else None for t, n in zip(leaves, need))


class _GRKANLinear(torch.autograd.Function):
    """y = R(x) w^T + b for a GR-KAN layer (kanforge/torch/layers.py:335-363):
    R = P / (1 + |Q|) per group (kf_rational_act), then the contraction on our
    kernels.  bf16: kf_grkan_fwd / kf_grkan_dgrad (dR = dy w on the tensor
    cores, dx = dR R'(x) and the rational parameter gradients in its epilogue)
    / kf_grkan_wgrad.  float32: kf_gemm_tf32x3 for the three contractions and
    kf_rational_bwd for dx and the parameter gradients.  Double backward builds
    the gradients from differentiable pieces."""

    @staticmethod
    def forward(ctx, x, num, den, w, bias, plan, groups, path):
        n_b, n_in = x.shape
        n_out = w.shape[0]
        x = x.contiguous()
        w_c = w.detach().contiguous()
        numf, denf = num.detach().float().contiguous(), den.detach().float().contiguous()
        desc = plan.desc(groups)
        r = torch.empty_like(x)
        _launch("kf_rational_act", _ptr(x), _ptr(numf), _ptr(denf), _ptr(r), n_b, n_in, 0, ctypes.byref(desc),
                _rat_dtype(x), _stream(x))
        y = torch.empty(n_b, n_out, device=x.device, dtype=x.dtype)
        b = None if bias is None else _aligned16(bias.detach().to(x.dtype).contiguous())
        if path == "bf16":
            _launch("kf_grkan_fwd", _ptr(r), _ptr(w_c), _ptr(b), _ptr(y), n_b, n_in, n_out, _stream(x))
        else:
            gemm_tf32x3(r, False, w_c, False, y, n_b, n_out, n_in, bias=b)
        ctx.save_for_backward(x, num, den, w, bias)
        ctx.r, ctx.w_c, ctx.numf, ctx.denf = r, w_c, numf, denf
        ctx.plan, ctx.groups, ctx.path = plan, groups, path
        return y

    @staticmethod
    def backward(ctx, gy):
        x, num, den, w, bias = ctx.saved_tensors
        plan, groups, path = ctx.plan, ctx.groups, ctx.path
        need = ctx.needs_input_grad
        r, w_c, numf, denf = ctx.r, ctx.w_c, ctx.numf, ctx.denf
        ctx.r = ctx.w_c = ctx.numf = ctx.denf = None
        if torch.is_grad_enabled():
            grads = _grkan_reference_grads(x, num, den, w, bias, plan, groups, gy, need[:5])
            return grads + (None, None, None)
        n_b, n_in = x.shape
        n_out = w.shape[0]
        gy = gy.to(x.dtype).contiguous()
        desc = plan.desc(groups)
        stream = _stream(x)
        dx = dnum = dden = dw = dbias = None
        if need[0] or need[1] or need[2]:
            dx = torch.empty_like(x)
            dnum = torch.empty(num.shape, device=x.device, dtype=torch.float32)
            dden = torch.empty(den.shape, device=x.device, dtype=torch.float32)
            if path == "bf16":
                ws_n = _lib.load().kf_grkan_workspace(n_b, n_in, ctypes.byref(desc))
                ws = torch.empty(max(int(ws_n), 1), device=x.device, dtype=torch.float32)
                _launch("kf_grkan_dgrad", _ptr(x), _ptr(gy), _ptr(w_c), _ptr(numf), _ptr(denf), _ptr(dx), _ptr(dnum),
                        _ptr(dden), _ptr(ws), n_b, n_in, n_out, ctypes.byref(desc), stream)
            else:
                dr = torch.empty_like(x)
                gemm_tf32x3(gy, False, w_c, True, dr, n_b, n_in, n_out)
                ws_n = _lib.load().kf_rational_workspace(n_b, n_in, ctypes.byref(desc))
                ws = torch.empty(max(int(ws_n), 1), device=x.device, dtype=torch.float32)
                _launch("kf_rational_bwd", _ptr(x), _ptr(dr), _ptr(numf), _ptr(denf), _ptr(dx), _ptr(dnum), _ptr(dden),
                        _ptr(ws), n_b, n_in, ctypes.byref(desc), _rat_dtype(x), stream)
        if need[3]:
            dw = torch.empty(n_out, n_in, device=x.device, dtype=x.dtype)
            if path == "bf16":
                ws_n = int(_lib.load().kf_grkan_wgrad_workspace(n_b, n_in, n_out))
                ws = torch.empty(ws_n, device=x.device, dtype=torch.float32) if ws_n else None
                _launch("kf_grkan_wgrad", _ptr(r), _ptr(gy), _ptr(dw), _ptr(ws), n_b, n_in, n_out, stream,
                        kernels=2 if ws_n else 1)  # split K: the partial sums' reduction
            else:
                gemm_tf32x3(gy, True, r, True, dw, n_out, n_in, n_b)
        if need[4] and bias is not None:
            dbias = gy.sum(0, dtype=torch.float32).to(bias.dtype)
        return (dx if need[0] else None, dnum.to(num.dtype) if (need[1] and dnum is not None) else None,
                dden.to(den.dtype) if (need[2] and dden is not None) else None, dw.to(w.dtype) if dw is not None else None,
                dbias, None, None, None)


def grkan_linear(x2, num, den, w, bias, plan, groups, path):
    """GR-KAN layer on (B, I) inputs; see ``_GRKANLinear``."""
    return _GRKANLinear.apply(x2, num, den, w, bias, plan, groups, path)


# --- grid tools (kanforge/grid.py, kanforge/_layer.py:107-183) ----------------


def sample_columns(x2: torch.Tensor) -> torch.Tensor:
    """Samples (n, I) -> (I, n) float32, one column per input (kf_samples_transpose)."""
    _check_cuda(x2)
    x2 = x2.contiguous()
    if x2.dtype not in (torch.float32, _BF16):
        x2 = x2.float()
    n, n_in = x2.shape
    xt = torch.empty(n_in, n, device=x2.device, dtype=torch.float32)
    _launch("kf_samples_transpose", _ptr(x2), _rat_dtype(x2), n, n_in, _ptr(xt), _stream(x2))
    return xt


def _bytes(n: int, device) -> torch.Tensor:
    return torch.empty(max(int(n), 16), dtype=torch.uint8, device=device)


def adaptive_grid(xt: torch.Tensor, n_points: int, margin: float = 0.0, grid_eps: float = 0.02) -> torch.Tensor:
    """Per-input adaptive grids (I, n_points) float64 from sample columns xt (I, n)
    (kanforge/grid.py:19-31), equal to the reference's float64 grid."""
    if not 0 < grid_eps <= 1:
        raise ValueError("grid_eps must be in (0, 1]: some uniform part keeps the grid increasing")
    n_in, n = xt.shape
    if n < 1:
        raise ValueError("adaptive_grid needs at least one sample")
    if not 2 <= n_points <= _lib.KF_GRID_MAX_POINTS:
        raise ValueError(f"grids of {n_points} points are outside [2, {_lib.KF_GRID_MAX_POINTS}]")
    ws = _bytes(_lib.load().kf_grid_workspace(n, n_in, n_points), xt.device)
    grid = torch.empty(n_in, n_points, dtype=torch.float64, device=xt.device)
    _launch("kf_adaptive_grid", _ptr(xt), n, n_in, n_points, float(margin), float(grid_eps), _ptr(grid), _ptr(ws),
            _stream(xt), kernels=8)
    return grid


def resample_grid(grid: torch.Tensor, n_points: int) -> torch.Tensor:
    """Rows of grid (I, n) linearly interpolated to n_points (kanforge/grid.py:34-38), float64."""
    _check_cuda(grid)
    g = grid.detach().to(torch.float64).contiguous()
    out = torch.empty(g.shape[0], n_points, dtype=torch.float64, device=g.device)
    _launch("kf_resample_grid", _ptr(g), g.shape[0], g.shape[1], n_points, _ptr(out), _stream(g))
    return out


def fit_basis(plan: KernelPlan, grid: torch.Tensor | None, device) -> tuple[_lib.FitBasis, list]:
    """The ``kf_fit_basis`` of a plan (float64 constants) and the tensors it points to."""
    b = _lib.FitBasis()
    keep = []
    b.size = plan.size
    if plan.size > _lib.KF_FIT_MAX_SIZE:
        raise ValueError(f"refit handles bases of up to {_lib.KF_FIT_MAX_SIZE} functions per edge, not {plan.size}")
    if plan.kind in ("bspline", "bump"):
        g = grid.detach().to(torch.float64).contiguous()
        keep.append(g)
        b.grid = g.data_ptr()
        b.n_grid = g.shape[-1]
    if plan.kind == "bspline":
        b.kind = _lib.KF_BASIS_BSPLINE
        b.order = plan.consts[1]
    elif plan.kind == "cheb":
        b.kind = _lib.KF_BASIS_CHEB
        b.degree = plan.consts[0]
        b.input_map = _lib.KF_MAP_TANH if plan.consts[1] == "tanh" else _lib.KF_MAP_IDENTITY
        fold = torch.tensor(plan.fold(0), dtype=torch.float64, device=device)
        keep.append(fold)
        b.fold = fold.data_ptr()
    elif plan.kind == "fourier":
        b.kind = _lib.KF_BASIS_FOURIER
        n, period = plan.consts
        b.degree = n
        b.freq = 2 * math.pi / period
    elif plan.kind == "bump":
        b.kind = _lib.KF_BASIS_BUMP
        mode, _count, u_scale, norm, _p = plan.consts
        b.bump_mode = _lib.KF_BUMP_GAUSS if mode == "gauss" else _lib.KF_BUMP_TANH
        b.u_scale, b.norm = float(u_scale), float(norm)
        poly = [float(v) for v in plan.bump_poly(0)]
        b.n_poly = len(poly)
        for j, v in enumerate(poly):
            b.poly[j] = v
    else:
        raise NotImplementedError(f"no refit for {plan.kind} bases")
    return b, keep


def refit(xt, ranges, n: int, old: _lib.FitBasis, new: _lib.FitBasis, coef: torch.Tensor, edge_scale, ridge: float):
    """(coef_out (O, I, new size), scale_out (O, I) or None), float64: the refit of
    kanforge/grid.py:55-85 and the edge_scale handling of kanforge/_layer.py:120-137.
    Samples are the columns xt (I, n), or n points per input over ranges (I, 2)."""
    coef = coef.detach().contiguous()
    if coef.dtype not in (torch.float32, _BF16):
        coef = coef.float()
    scale = None if edge_scale is None else edge_scale.detach().to(coef.dtype).contiguous()
    n_out, n_in, k_old = coef.shape
    if k_old != old.size:
        raise ValueError(f"coef has {k_old} basis functions, the old basis {old.size}")
    ws = _bytes(_lib.load().kf_refit_workspace(n, n_in, old.size, new.size), coef.device)
    out = torch.empty(n_out, n_in, new.size, dtype=torch.float64, device=coef.device)
    scale_out = None if scale is None else torch.empty(n_out, n_in, dtype=torch.float64, device=coef.device)
    _launch("kf_refit", _ptr(xt), _ptr(ranges), n, n_in, n_out, ctypes.byref(old), ctypes.byref(new), _ptr(coef),
            _ptr(scale), _rat_dtype(coef), float(ridge), _ptr(out), _ptr(scale_out), _ptr(ws), _stream(coef),
            kernels=3)
    return out, scale_out


def check_device_errors() -> None:
    """Raise if a kernel recorded a bounded wait that ran out (synchronises)."""
    flags = _lib.device_status()
    if flags:
        raise RuntimeError(f"a kanforge_b200 kernel reported device error flags {flags:#x}")
