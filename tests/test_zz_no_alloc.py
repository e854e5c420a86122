"""kf_rational_bwd_noalloc: the rational backward for callers that cannot
allocate device memory (allocator callbacks, frameworks that own all device
memory, runtimes that forbid allocation after start-up).  Its partial sums live
in the library's fixed device array, so it must match kf_rational_bwd, which
takes a caller workspace, call after call.

Collected last (file name) so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import kanforge_b200 as kb
from kanforge_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(n_b, n_in, groups, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(n_b, n_in, generator=g) * 1.5).to("cuda", dtype)
    dr = torch.randn(n_b, n_in, generator=g).to("cuda", dtype)
    a, b = kb.fit_rational("gelu", 5, 4)
    num = torch.as_tensor(np.tile(a, (groups, 1)), dtype=torch.float32) + 0.05 * torch.randn(groups, 6, generator=g)
    den = torch.as_tensor(np.tile(b, (groups, 1)), dtype=torch.float32) + 0.05 * torch.randn(groups, 4, generator=g)
    return x, dr, num.cuda(), den.cuda()


def _desc(groups):
    return kb.plan_for(kb.Rational(5, 4)).desc(groups)


def _with_workspace(x, dr, num, den, groups):
    n_b, n_in = x.shape
    d = _desc(groups)
    dx = torch.empty_like(x)
    dnum, dden = torch.empty_like(num), torch.empty_like(den)
    ws = torch.empty(int(_lib.load().kf_rational_workspace(n_b, n_in, ctypes.byref(d))), device="cuda")
    dt = _lib.KF_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.KF_DTYPE_F32
    _lib.call("kf_rational_bwd", _ptr(x), _ptr(dr), _ptr(num), _ptr(den), _ptr(dx), _ptr(dnum), _ptr(dden), _ptr(ws),
              n_b, n_in, ctypes.byref(d), dt, _stream())
    return dx, dnum, dden


def _no_alloc(x, dr, num, den, groups):
    n_b, n_in = x.shape
    d = _desc(groups)
    dx = torch.empty_like(x)
    dnum, dden = torch.empty_like(num), torch.empty_like(den)
    dt = _lib.KF_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.KF_DTYPE_F32
    _lib.call("kf_rational_bwd_noalloc", _ptr(x), _ptr(dr), _ptr(num), _ptr(den), _ptr(dx), _ptr(dnum), _ptr(dden),
              n_b, n_in, ctypes.byref(d), dt, _stream())
    return dx, dnum, dden


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return (a - b).abs().max().item() / max(1.0, b.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n_b,n_in,groups", [(513, 64, 8), (4096, 768, 8), (2048, 3072, 8)])
def test_no_alloc_matches_workspace_entry_point_twice(n_b, n_in, groups, dtype):
    # two calls in a row with different inputs: the shared array carries no stale state
    for seed in (1, 2):
        args = _inputs(n_b, n_in, groups, dtype, seed)
        want = _with_workspace(*args, groups)
        got = _no_alloc(*args, groups)
        torch.cuda.synchronize()
        for g_, w_, what in zip(got, want, ("dx", "dnum", "dden")):
            err = _rel(g_, w_)
            assert err <= TOL[dtype], f"{what} (call {seed}): rel err {err:.3e}"


def test_no_alloc_rejects_sizes_beyond_the_fixed_array():
    n_in = (_lib_max() // 10) + 8  # I * (6 + 4) floats of partial sums per CTA exceed the array
    n_in -= n_in % 8
    x = torch.zeros(4, n_in, device="cuda")
    num, den = torch.zeros(8, 6, device="cuda"), torch.zeros(8, 4, device="cuda")
    d = _desc(8)
    rc = _lib.load().kf_rational_bwd_noalloc(_ptr(x), _ptr(x), _ptr(num), _ptr(den), _ptr(x), _ptr(num), _ptr(den), 4,
                                             n_in, ctypes.byref(d), _lib.KF_DTYPE_F32, _stream())
    assert rc == 1 and "fixed scratch" in _lib.last_error()


def _lib_max() -> int:
    header = (kb.__path__[0] + "/../include/kanforge_b200.h")
    for line in open(header):
        if line.startswith("#define KF_RATIONAL_NOALLOC_MAX_FLOATS"):
            return eval(line.split(None, 2)[2])  # "(1 << 20)"
    raise AssertionError("KF_RATIONAL_NOALLOC_MAX_FLOATS not declared")
