// Feature evaluators shared by the float32 kernels (primitives, edge
// derivatives).  BK selects the basis at compile time: 0 = Chebyshev features,
// 1..5 = B-spline of that order.
#pragma once

#include "basis.cuh"

namespace kf {

#define KF_NK_MAX 64   // extended knots per input held in shared memory
#define KF_NF_MAX 32   // features per input in the float32 kernels

struct FeatArgs {
  int m;        // derivative order (B-splines: native; Chebyshev: folded by the caller)
  int nf;       // features per input
  int map;      // KF_MAP_* (Chebyshev)
  int G;        // B-spline grid intervals
  int nk;       // B-spline extended knots = G + 2 order + 1
  const float* grid;  // (I, G+1)
};

// Extended knots of input i into t[0..nk).
template <int BK>
__device__ __forceinline__ void load_knots(const FeatArgs& fa, int i, float* t, int lane, int nlanes) {
  if constexpr (BK > 0) {
    const float* g = fa.grid + (size_t)i * (fa.G + 1);
    for (int r = lane; r < fa.nk; r += nlanes) t[r] = extended_knot(g, fa.G, BK, r);
  }
}

// dst[j * stride] = scale * phi_j(x) for j < nf.  t: knots of this input.
template <int BK>
__device__ __forceinline__ void eval_features(const FeatArgs& fa, float x, float scale, const float* t, float* dst,
                                              int stride) {
  if constexpr (BK == 0) {
    const float z = fa.map == KF_MAP_TANH ? tanhf(x) : x;
    float tm2 = 1.0f, tm1 = z;
    dst[0] = scale;
    if (fa.nf > 1) dst[stride] = scale * z;
    for (int j = 2; j < fa.nf; ++j) {
      const float tj = 2.0f * z * tm1 - tm2;
      dst[j * stride] = scale * tj;
      tm2 = tm1;
      tm1 = tj;
    }
  } else {
    for (int j = 0; j < fa.nf; ++j) dst[j * stride] = 0.0f;
    if (fa.m > BK) return;
    const int j0 = knot_interval(x, t, fa.nk);
    if (j0 < 0) return;
    float v[BK + 1];
    bspline_local<BK>(x, t, fa.nk, j0, fa.m, v);
#pragma unroll
    for (int rp = 0; rp <= BK; ++rp) {
      const int r = j0 - BK + rp;
      if (r >= 0 && r < fa.nf) dst[r * stride] = scale * v[rp];
    }
  }
}

// sum_j h[j * stride] phi_j(x): a dot product with the feature vector
// without materialising it.
template <int BK>
__device__ __forceinline__ float dot_features(const FeatArgs& fa, float x, const float* t, const float* h, int stride) {
  if constexpr (BK == 0) {
    const float z = fa.map == KF_MAP_TANH ? tanhf(x) : x;
    float acc = h[0];
    if (fa.nf > 1) acc += z * h[stride];
    float tm2 = 1.0f, tm1 = z;
    for (int j = 2; j < fa.nf; ++j) {
      const float tj = 2.0f * z * tm1 - tm2;
      acc += tj * h[j * stride];
      tm2 = tm1;
      tm1 = tj;
    }
    return acc;
  } else {
    if (fa.m > BK) return 0.0f;
    const int j0 = knot_interval(x, t, fa.nk);
    if (j0 < 0) return 0.0f;
    float v[BK + 1];
    bspline_local<BK>(x, t, fa.nk, j0, fa.m, v);
    float acc = 0.0f;
#pragma unroll
    for (int rp = 0; rp <= BK; ++rp) {
      const int r = j0 - BK + rp;
      if (r >= 0 && r < fa.nf) acc += v[rp] * h[r * stride];
    }
    return acc;
  }
}

// Dispatch a templated launcher on the basis: fn.template operator()<BK>().
template <typename Fn>
int dispatch_bk(const kf_basis_desc* d, Fn&& fn) {
  if (d->kind == KF_BASIS_CHEB) return fn.template operator()<0>();
  if (d->kind == KF_BASIS_BSPLINE) {
    switch (d->order) {
      case 1: return fn.template operator()<1>();
      case 2: return fn.template operator()<2>();
      case 3: return fn.template operator()<3>();
      case 4: return fn.template operator()<4>();
      case 5: return fn.template operator()<5>();
      default: break;
    }
  }
  set_error("no float32 kernel for basis kind %d order %d", d->kind, d->order);
  return KF_ERR_UNSUPPORTED;
}

}  // namespace kf
