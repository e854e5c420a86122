"""ctypes binding of libkanb200.so (the C ABI declared in include/kanforge_b200.h).

The library is built in-tree by ``kanforge_b200.build``.  Loading fails loudly
when it is missing: this package has no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkanb200.so"

KF_OK = 0
KF_BASIS_BSPLINE, KF_BASIS_CHEB, KF_BASIS_RATIONAL, KF_BASIS_FOURIER, KF_BASIS_BUMP = 1, 2, 3, 4, 5
KF_BUMP_GAUSS, KF_BUMP_TANH = 0, 1
KF_BUMP_MAX_ORDER = 5
KF_MAP_TANH, KF_MAP_IDENTITY = 0, 1
KF_DTYPE_F32, KF_DTYPE_BF16 = 0, 1
KF_OP_F, KF_OP_G, KF_OP_P = 0, 1, 2
KF_QUERY_FUSED, KF_QUERY_EDGE = 16, 17

_c_i32, _c_i64, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class BasisDesc(ctypes.Structure):
    """``kf_basis_desc`` (include/kanforge_b200.h)."""

    _fields_ = [
        ("kind", _c_i32),
        ("size", _c_i32),
        ("grid_size", _c_i32),
        ("order", _c_i32),
        ("degree", _c_i32),
        ("den_degree", _c_i32),
        ("input_map", _c_i32),
        ("groups", _c_i32),
        ("period", ctypes.c_float),
        ("bump_mode", _c_i32),
        ("u_scale", ctypes.c_float),
        ("norm", ctypes.c_float),
        ("bump_poly", (ctypes.c_float * 8) * (KF_BUMP_MAX_ORDER + 1)),
    ]


class ConvGeom(ctypes.Structure):
    """``kf_conv_geom`` (include/kanforge_b200.h): the implicit patch matrix of a KAN convolution."""

    _fields_ = [
        ("batch", _c_i32),
        ("channels", _c_i32),
        ("group_channels", _c_i32),
        ("channel0", _c_i32),
        ("size", _c_i32 * 3),
        ("kernel", _c_i32 * 3),
        ("stride", _c_i32 * 3),
        ("padding", _c_i32 * 3),
        ("dilation", _c_i32 * 3),
    ]


class FitBasis(ctypes.Structure):
    """``kf_fit_basis`` (include/kanforge_b200.h): a basis as the refit evaluates it."""

    _fields_ = [
        ("kind", _c_i32),
        ("size", _c_i32),
        ("order", _c_i32),
        ("degree", _c_i32),
        ("input_map", _c_i32),
        ("bump_mode", _c_i32),
        ("n_grid", _c_i32),
        ("n_poly", _c_i32),
        ("grid", _vp),
        ("fold", _vp),
        ("freq", ctypes.c_double),
        ("u_scale", ctypes.c_double),
        ("norm", ctypes.c_double),
        ("poly", ctypes.c_double * 8),
    ]


KF_GRID_MAX_POINTS, KF_FIT_MAX_SIZE = 192, 256

_GEOM = ctypes.POINTER(ConvGeom)
_FIT = ctypes.POINTER(FitBasis)
_f64 = ctypes.c_double

# name -> (restype, argtypes)
PROTOTYPES = {
    "kf_conv_patches": (ctypes.c_int, [_vp, _GEOM, _vp, ctypes.c_int, _vp]),
    "kf_conv_fold": (ctypes.c_int, [_vp, _GEOM, _vp, ctypes.c_int, _vp]),
    "kf_conv_fwd": (
        ctypes.c_int,
        [_vp, _GEOM, _vp, _vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_conv_features": (ctypes.c_int, [_vp, _GEOM, _vp, _vp, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp]),
    "kf_conv_dgrad": (
        ctypes.c_int,
        [_vp, _GEOM, _vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_conv_wgrad": (
        ctypes.c_int,
        [_vp, _GEOM, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32,
         ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_version": (ctypes.c_int, []),
    "kf_set_reserved_sms": (ctypes.c_int, [_c_i32]),
    "kf_last_error": (ctypes.c_char_p, []),
    "kf_query": (ctypes.c_int, [ctypes.POINTER(BasisDesc), ctypes.c_int, ctypes.c_int]),
    "kf_device_status": (ctypes.c_int, [ctypes.POINTER(_c_i32)]),
    "kf_prim": (
        ctypes.c_int,
        [ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_knot_tables": (ctypes.c_int, [_vp, _vp, _c_i32, _c_i32, _c_i32, _vp]),
    "kf_pack_coef": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.c_int, _vp]),
    "kf_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_fwd_emit_features": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_dgrad": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_features": (
        ctypes.c_int,
        [_vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_wgrad": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
         ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_edge_derivative": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp, _c_i32, _vp],
    ),
    "kf_edge_derivative_dx": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp,
         _c_i32, _vp],
    ),
    "kf_edge_derivative_dcoef": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp,
         _c_i32, _vp],
    ),
    "kf_edge_derivative_workspace": (_c_i64, [_c_i64, _c_i32, _c_i32, _c_i32]),
    "kf_gemm_tf32x3": (
        ctypes.c_int,
        [_vp, _c_i32, _c_i64, _vp, _c_i32, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp],
    ),
    "kf_features_f32": (
        ctypes.c_int,
        [_vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_features_spline_f32": (
        ctypes.c_int,
        [_vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_features_dot_f32": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_rational_act": (ctypes.c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), ctypes.c_int, _vp]),
    "kf_rational_bwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, ctypes.POINTER(BasisDesc), ctypes.c_int, _vp],
    ),
    "kf_rational_workspace": (_c_i64, [_c_i64, _c_i32, ctypes.POINTER(BasisDesc)]),
    "kf_grkan_fwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _vp]),
    "kf_grkan_dgrad": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_grkan_workspace": (_c_i64, [_c_i64, _c_i32, ctypes.POINTER(BasisDesc)]),
    "kf_grkan_wgrad_workspace": (_c_i64, [_c_i64, _c_i32, _c_i32]),
    "kf_grkan_wgrad": (ctypes.c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, _vp]),
    "kf_samples_transpose": (ctypes.c_int, [_vp, ctypes.c_int, _c_i64, _c_i32, _vp, _vp]),
    "kf_grid_workspace": (_c_i64, [_c_i64, _c_i32, _c_i32]),
    "kf_adaptive_grid": (ctypes.c_int, [_vp, _c_i64, _c_i32, _c_i32, _f64, _f64, _vp, _vp, _vp]),
    "kf_resample_grid": (ctypes.c_int, [_vp, _c_i32, _c_i32, _c_i32, _vp, _vp]),
    "kf_refit_workspace": (_c_i64, [_c_i64, _c_i32, _c_i32, _c_i32]),
    "kf_refit": (
        ctypes.c_int,
        [_vp, _vp, _c_i64, _c_i32, _c_i32, _FIT, _FIT, _vp, _vp, ctypes.c_int, _f64, _vp, _vp, _vp, _vp],
    ),
    "kf_sparse_fwd": (
        ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_sparse_dgrad": (
        ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_sparse_wgrad_workspace": (_c_i64, [_c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc)]),
    "kf_sparse_wgrad": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, _c_i32, ctypes.POINTER(BasisDesc), _vp],
    ),
    "kf_rational_bwd_noalloc": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i32, ctypes.POINTER(BasisDesc), ctypes.c_int, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library (RuntimeError if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build the sm_100a kernels first (python -m kanforge_b200.build); "
                    "kanforge_b200 has no CPU fallback"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().kf_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Call an entry point; a non-zero status becomes RuntimeError with the library's message."""
    rc = getattr(load(), name)(*args)
    if rc != KF_OK:
        raise RuntimeError(f"{name} failed (status {rc}): {last_error()}")


def device_status() -> int:
    """Reads and clears the device error word (synchronises the device)."""
    flags = _c_i32(0)
    call("kf_device_status", ctypes.byref(flags))
    return int(flags.value)
