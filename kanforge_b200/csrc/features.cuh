// Feature evaluators shared by the float32 kernels (primitives, edge
// derivatives).  BK selects the basis at compile time: 0 = Chebyshev features,
// 1..5 = B-spline of that order, kFourierBK = Fourier features (folded like
// Chebyshev), kBumpBK = bumps on a per-input grid of centres (native order).
#pragma once

#include "basis.cuh"

namespace kf {

#define KF_NK_MAX 64   // extended knots per input held in shared memory
#define KF_NF_MAX 32   // features per input in the float32 kernels

constexpr int kFourierBK = -2;
constexpr int kBumpBK = -3;

struct FeatArgs {
  int m;        // derivative order (B-splines, bumps: native; Chebyshev, Fourier: folded by the caller)
  int nf;       // features per input
  int map;      // KF_MAP_* (Chebyshev)
  int G;        // B-spline grid intervals
  int nk;       // B-spline extended knots = G + 2 order + 1; bumps: centres per input
  const float* grid;  // B-spline (I, G+1); bumps (I, count)
  float w1;     // Fourier: 2 pi / period
  int bump_mode;      // KF_BUMP_*
  float u_scale, norm;
  float poly[8];      // bumps: P_m of order m, lowest first
};

// Extended knots (B-splines) or centres (bumps) of input i into t[0..nk).
template <int BK>
__device__ __forceinline__ void load_knots(const FeatArgs& fa, int i, float* t, int lane, int nlanes) {
  if constexpr (BK > 0) {
    const float* g = fa.grid + (size_t)i * (fa.G + 1);
    for (int r = lane; r < fa.nk; r += nlanes) t[r] = extended_knot(g, fa.G, BK, r);
  } else if constexpr (BK == kBumpBK) {
    const float* g = fa.grid + (size_t)i * fa.nk;
    for (int r = lane; r < fa.nk; r += nlanes) t[r] = g[r];
  }
}

// Fourier features of order 0: cos(j w1 x) for j = 1..n, then sin(j w1 x),
// n = nf / 2 (kanforge/bases/fourier.py:36-44); the harmonics by the angle
// addition recurrence from one accurate sincos.
__device__ __forceinline__ void fourier_features(const FeatArgs& fa, float x, float scale, float* dst, int stride) {
  const int n = fa.nf / 2;
  float s1, c1;
  sincosf(fa.w1 * x, &s1, &c1);
  float c = c1, s = s1;
  for (int j = 0; j < n; ++j) {
    dst[j * stride] = scale * c;
    dst[(n + j) * stride] = scale * s;
    const float cn = c * c1 - s * s1;
    s = s * c1 + c * s1;
    c = cn;
  }
}

// Bump j of input i at derivative order fa.m: gauss norm P_m(u) exp(-u^2/2) k^m,
// u = (x - c_j) k; tanh P_m(t) / h^m, t = tanh((x - c_j) / h)
// (kanforge/bases/radial.py:61-73, 137-143).  t: the input's centres.
__device__ __forceinline__ void bump_features(const FeatArgs& fa, float x, float scale, const float* t, float* dst,
                                              int stride) {
  const int n = fa.nk;
  const float span = t[n - 1] - t[0];
  float km = 1.0f;
  if (fa.bump_mode == KF_BUMP_GAUSS) {
    const float k = fa.u_scale * (float)(n - 1) / span;
    for (int q = 0; q < fa.m; ++q) km *= k;
    for (int j = 0; j < n; ++j) {
      const float u = (x - t[j]) * k;
      float p = fa.poly[7];
#pragma unroll
      for (int e = 6; e >= 0; --e) p = fmaf(p, u, fa.poly[e]);
      dst[j * stride] = scale * fa.norm * p * expf(-0.5f * u * u) * km;
    }
  } else {
    const float h = span / (float)(n - 1);
    for (int q = 0; q < fa.m; ++q) km /= h;
    for (int j = 0; j < n; ++j) {
      const float th = tanhf((x - t[j]) / h);
      float p = fa.poly[7];
#pragma unroll
      for (int e = 6; e >= 0; --e) p = fmaf(p, th, fa.poly[e]);
      dst[j * stride] = scale * p * km;
    }
  }
}

// dst[j * stride] = scale * phi_j(x) for j < nf.  t: knots of this input.
template <int BK>
__device__ __forceinline__ void eval_features(const FeatArgs& fa, float x, float scale, const float* t, float* dst,
                                              int stride) {
  if constexpr (BK == kFourierBK) {
    fourier_features(fa, x, scale, dst, stride);
  } else if constexpr (BK == kBumpBK) {
    bump_features(fa, x, scale, t, dst, stride);
  } else if constexpr (BK == 0) {
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
  if constexpr (BK == kFourierBK || BK == kBumpBK) {
    float f[KF_NF_MAX];
    eval_features<BK>(fa, x, 1.0f, t, f, 1);
    float acc = 0.0f;
    for (int j = 0; j < fa.nf; ++j) acc = fmaf(f[j], h[j * stride], acc);
    return acc;
  } else if constexpr (BK == 0) {
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

// Fourier / bump fields of fa from the descriptor, order m.  Returns false
// (with the error set) when the descriptor does not describe a usable basis.
inline bool fill_closed_family(const kf_basis_desc* d, const float* grid, int m, FeatArgs& fa) {
  if (d->kind == KF_BASIS_FOURIER) {
    if (!(d->period > 0.0f) || d->size % 2 != 0 || d->size < 2) {
      set_error("Fourier basis needs period > 0 and an even size");
      return false;
    }
    fa.w1 = 6.283185307179586f / d->period;
    return true;
  }
  if (d->kind == KF_BASIS_BUMP) {
    if (grid == nullptr || d->size < 2 || d->size > KF_NK_MAX || m > KF_BUMP_MAX_ORDER ||
        (d->bump_mode != KF_BUMP_GAUSS && d->bump_mode != KF_BUMP_TANH)) {
      set_error("bump basis needs its grid, 2..%d centres, mode gauss or tanh and order <= %d", KF_NK_MAX,
                KF_BUMP_MAX_ORDER);
      return false;
    }
    fa.grid = grid;
    fa.nk = d->size;
    fa.bump_mode = d->bump_mode;
    fa.u_scale = d->u_scale;
    fa.norm = d->norm;
    for (int e = 0; e < 8; ++e) fa.poly[e] = d->bump_poly[m][e];
    return true;
  }
  return true;
}

// Dispatch a templated launcher on the basis: fn.template operator()<BK>().
template <typename Fn>
int dispatch_bk(const kf_basis_desc* d, Fn&& fn) {
  if (d->kind == KF_BASIS_CHEB) return fn.template operator()<0>();
  if (d->kind == KF_BASIS_FOURIER) return fn.template operator()<kFourierBK>();
  if (d->kind == KF_BASIS_BUMP) return fn.template operator()<kBumpBK>();
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
