// Device evaluation of the KAN edge bases and their x-derivatives.
//
// B-splines follow Cox-de Boor on half-open intervals with the knot vector
// extended by `order` mean steps per side, then derivative steps
// (reference kanforge/bases/spline.py:22-30, 74-92).  Only the order+1 splines
// that are non-zero on the interval holding x are evaluated (local support);
// the arithmetic of each surviving term is the reference's.
//
// Polynomial families are evaluated as Chebyshev features T_j(g(x)) with
// g = tanh or identity (kanforge/bases/polynomial.py:66-106); the family
// matrix and the derivative orders are folded into the coefficients on the
// host (kanforge/kernels/plan.py:75-101).  The forward-derivative kernels also
// use d/dx T_j(g(x)) = j U_{j-1}(g) g'(x) directly.
//
// The KAT rational is P(x) / (1 + |Q(x)|) with derivatives from the quotient
// rule (kanforge/bases/rational.py:84-101, kanforge/_calculus.py:79-87).
#pragma once

#include "common.cuh"

namespace kf {

// tanh(x) = sign(x) (1 - e^{-2|x|}) / (1 + e^{-2|x|}); the formula of the
// reference Triton kernels (kanforge/kernels/triton_kernels.py:116-120).  Its
// absolute error is ~1e-7, which is below bf16 resolution; float32 paths use
// tanhf instead.
__device__ __forceinline__ float tanh_exp(float x) {
  float t = __expf(-2.0f * fabsf(x));
  float r = __fdividef(1.0f - t, 1.0f + t);
  return copysignf(r, x);
}

__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_acc(float x) { return x / (1.0f + expf(-x)); }

// d/dx silu = s + x s (1 - s), s = sigmoid(x), with the fast exponential and
// division: relative error ~1e-6, below bf16 resolution (bf16 kernels only).
__device__ __forceinline__ float dsilu_fast(float x) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-x));
  return s + x * s * (1.0f - s);
}

// d/dx silu = s + x s (1 - s), s = sigmoid(x).
__device__ __forceinline__ float dsilu_acc(float x) {
  float s = 1.0f / (1.0f + expf(-x));
  return s + x * s * (1.0f - s);
}

// silu^(m)(x) = x h_m(s) + m h_{m-1}(s), with h_m, h_{m-1} given as
// polynomials in s = sigmoid(x) of n coefficients each
// (kanforge/_calculus.py:90-96).  m = 0 gives silu.
__device__ __forceinline__ float silu_deriv(float x, int m, const float* poly, int n) {
  if (m == 0) return silu_acc(x);
  float s = 1.0f / (1.0f + expf(-x));
  float hm = poly[n - 1], hm1 = poly[2 * n - 1];
  for (int j = n - 2; j >= 0; --j) {
    hm = hm * s + poly[j];
    hm1 = hm1 * s + poly[n + j];
  }
  return x * hm + (float)m * hm1;
}

// ---------------------------------------------------------------------------
// B-splines
// ---------------------------------------------------------------------------

// Extended knot r of input row `g` (G+1 grid points): `order` points with the
// mean step on each side (kanforge/bases/spline.py:22-30).
__device__ __forceinline__ float extended_knot(const float* g, int G, int order, int r) {
  float g0 = g[0], gl = g[G];
  float h = (gl - g0) / (float)G;
  if (r < order) return g0 - h * (float)(order - r);
  if (r <= order + G) return g[r - order];
  return gl + h * (float)(r - order - G);
}

// Index j of the interval [t_j, t_{j+1}) holding x, or -1 outside [t_0, t_{nk-1}).
__device__ __forceinline__ int knot_interval(float x, const float* t, int nk) {
  if (!(x >= t[0]) || !(x < t[nk - 1])) return -1;
  int lo = 0, hi = nk - 1;  // invariant t[lo] <= x < t[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (t[mid] <= x) lo = mid; else hi = mid;
  }
  return lo;
}

// m-th derivative of the order-K B-splines that are non-zero on interval j.
// v[r'] belongs to basis index j - K + r' (r' = 0..K); indices outside
// [0, nk-2-K] are zero.  t: the nk extended knots.  Levels 1..K-m are
// Cox-de Boor steps, the remaining m levels derivative steps; a level-q spline
// r exists for 0 <= r <= nk-2-q exactly as in the reference's arrays.
template <int K>
__device__ __forceinline__ void bspline_local(float x, const float* t, int nk, int j, int m, float (&v)[K + 1]) {
#pragma unroll
  for (int r = 0; r <= K; ++r) v[r] = 0.0f;
  v[0] = 1.0f;  // level 0: window holds B_{0,j}
#pragma unroll
  for (int q = 1; q <= K; ++q) {
    float nv[K + 1];
    const bool deriv = q > K - m;
#pragma unroll
    for (int rp = 0; rp <= q; ++rp) {
      const int r = j - q + rp;
      const float left = rp >= 1 ? v[rp - 1] : 0.0f;   // B_{q-1, r}
      const float right = rp <= q - 1 ? v[rp] : 0.0f;  // B_{q-1, r+1}
      float out = 0.0f;
      if (r >= 0 && r <= nk - 2 - q) {
        const float d1 = t[r + q] - t[r];
        const float d2 = t[r + q + 1] - t[r + 1];
        if (deriv) {
          out = (float)q * (left / d1 - right / d2);
        } else {
          out = (x - t[r]) / d1 * left + (t[r + q + 1] - x) / d2 * right;
        }
      }
      nv[rp] = out;
    }
#pragma unroll
    for (int rp = 0; rp <= K; ++rp) v[rp] = rp <= q ? nv[rp] : 0.0f;
  }
}

// Row stride (floats) of the per-input knot tables: row 0 the extended knots,
// row q the reciprocals 1 / (t_{r+q} - t_r).
constexpr int kKnotTableStride = 64;

// Cox-de Boor / derivative levels of bspline_local (basis.cuh) with the
// reciprocal knot differences read from the table.
template <int K, int ES = 1>
__device__ __forceinline__ void bspline_local_tab(float x, const float* tab, int nk, int j, int m, float (&v)[K + 1],
                                                  int ts = kKnotTableStride) {
  const float* t = tab;
#pragma unroll
  for (int r = 0; r <= K; ++r) v[r] = 0.0f;
  v[0] = 1.0f;
#pragma unroll
  for (int q = 1; q <= K; ++q) {
    float nv[K + 1];
    const bool deriv = q > K - m;
    const float* inv = tab + q * ts;
#pragma unroll
    for (int rp = 0; rp <= q; ++rp) {
      const int r = j - q + rp;
      const float left = rp >= 1 ? v[rp - 1] : 0.0f;
      const float right = rp <= q - 1 ? v[rp] : 0.0f;
      float out = 0.0f;
      if (r >= 0 && r <= nk - 2 - q) {
        const float i1 = inv[r * ES], i2 = inv[(r + 1) * ES];
        out = deriv ? (float)q * (left * i1 - right * i2) : (x - t[r * ES]) * i1 * left + (t[(r + q + 1) * ES] - x) * i2 * right;
      }
      nv[rp] = out;
    }
#pragma unroll
    for (int rp = 0; rp <= K; ++rp) v[rp] = rp <= q ? nv[rp] : 0.0f;
  }
}

// Dense B-spline feature vector: f[0..size) = m-th derivatives of every basis
// function at x (zero where not supported).  t: extended knots (nk of them).
template <int K>
__device__ __forceinline__ void bspline_dense(float x, const float* t, int nk, int m, float* f, int size) {
  for (int r = 0; r < size; ++r) f[r] = 0.0f;
  if (m > K) return;
  const int j = knot_interval(x, t, nk);
  if (j < 0) return;
  float v[K + 1];
  bspline_local<K>(x, t, nk, j, m, v);
#pragma unroll
  for (int rp = 0; rp <= K; ++rp) {
    const int r = j - K + rp;
    if (r >= 0 && r < size) f[r] = v[rp];
  }
}

// ---------------------------------------------------------------------------
// Chebyshev features
// ---------------------------------------------------------------------------

// T_0..T_{n-1}(z) by the three-term recurrence (polynomial.py:91-96).
__device__ __forceinline__ void cheb_features(float z, int n, float* f) {
  f[0] = 1.0f;
  if (n > 1) f[1] = z;
  for (int j = 2; j < n; ++j) f[j] = 2.0f * z * f[j - 1] - f[j - 2];
}

// ---------------------------------------------------------------------------
// KAT rational P(x) / (1 + |Q(x)|)
// ---------------------------------------------------------------------------

#define KF_RAT_MAX_NUM 12
#define KF_RAT_MAX_DEN 12
#define KF_RAT_MAX_ORDER 6

// k-th derivative of sum_{j >= first} c[j - first] x^j, c of length n
// (kanforge/bases/rational.py:90-97).
__device__ __forceinline__ float poly_derivative(const float* c, int n, int first, int k, float x) {
  const int last = first + n - 1;
  float y = 0.0f;
  for (int e = last - k; e >= 0; --e) {
    const int j = e + k;
    float coef = 0.0f;
    if (j >= first) {
      float ff = 1.0f;
      for (int u = 0; u < k; ++u) ff *= (float)(j - u);
      coef = ff * c[j - first];
    }
    y = y * x + coef;
  }
  return y;
}

// R^(m)(x) by the general quotient rule (kanforge/_calculus.py:79-87).
__device__ __forceinline__ float rational_deriv(float x, const float* a, int na, const float* b, int nb, int m) {
  float P[KF_RAT_MAX_ORDER + 1], D[KF_RAT_MAX_ORDER + 1], out[KF_RAT_MAX_ORDER + 1];
  const float q0 = poly_derivative(b, nb, 1, 0, x);
  const float sg = q0 > 0.0f ? 1.0f : (q0 < 0.0f ? -1.0f : 0.0f);
  for (int k = 0; k <= m; ++k) {
    P[k] = poly_derivative(a, na, 0, k, x);
    D[k] = k == 0 ? 1.0f + fabsf(q0) : sg * poly_derivative(b, nb, 1, k, x);
  }
  out[0] = P[0] / D[0];
  for (int n = 1; n <= m; ++n) {
    float acc = P[n];
    float binom = 1.0f;
    for (int k = 1; k <= n; ++k) {
      binom = binom * (float)(n - k + 1) / (float)k;
      acc -= binom * D[k] * out[n - k];
    }
    out[n] = acc / D[0];
  }
  return out[m];
}

// Two elements of the rational backward in float2 lanes (two fp32 operations
// per instruction: __ffma2_rn / __fmul2_rn / __fadd2_rn), degrees fixed: returns
// dx = g R'(x) and adds g dR/da_j, g dR/db_j to the accumulators.  With
// D = 1 + |Q|, Q = x Qs(x):
//   R' = (P' - sign(Q) Q' R) / D,  dR/da_j = x^j / D,  dR/db_j = -R sign(Q) x^(j+1) / D.
// 1 / D uses __fdividef (2 ulp; D >= 1 is far inside its range).  Used by the
// rational kernels and the GR-KAN input-gradient epilogue.
__device__ __forceinline__ float rat_sign(float q) { return q > 0.0f ? 1.0f : (q < 0.0f ? -1.0f : 0.0f); }
__device__ __forceinline__ float2 dup2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 neg2(float2 v) { return make_float2(-v.x, -v.y); }

template <int NA, int NB>
__device__ __forceinline__ float2 rat_bwd_pair(float2 x, float2 g, const float2 (&a)[NA], const float2 (&bq)[NB],
                                               float2 (&acc_a)[NA], float2 (&acc_b)[NB]) {
  float2 P = a[NA - 1], dP = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int j = NA - 2; j >= 0; --j) {
    dP = __ffma2_rn(dP, x, P);
    P = __ffma2_rn(P, x, a[j]);
  }
  float2 Qs = bq[NB - 1], dQs = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int j = NB - 2; j >= 0; --j) {
    dQs = __ffma2_rn(dQs, x, Qs);
    Qs = __ffma2_rn(Qs, x, bq[j]);
  }
  const float2 Q = __fmul2_rn(x, Qs);
  const float2 dQ = __ffma2_rn(x, dQs, Qs);
  const float2 sg = make_float2(rat_sign(Q.x), rat_sign(Q.y));
  const float2 rD = make_float2(__fdividef(1.0f, 1.0f + fabsf(Q.x)), __fdividef(1.0f, 1.0f + fabsf(Q.y)));
  const float2 R = __fmul2_rn(P, rD);
  const float2 u = __fmul2_rn(g, rD);
  acc_a[0] = __fadd2_rn(acc_a[0], u);
  float2 xp = x;
#pragma unroll
  for (int j = 1; j < NA; ++j) {
    acc_a[j] = __ffma2_rn(u, xp, acc_a[j]);
    xp = __fmul2_rn(xp, x);
  }
  const float2 v = __fmul2_rn(__fmul2_rn(neg2(u), R), sg);
  xp = x;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    acc_b[j] = __ffma2_rn(v, xp, acc_b[j]);
    xp = __fmul2_rn(xp, x);
  }
  return __fmul2_rn(g, __fmul2_rn(__ffma2_rn(neg2(__fmul2_rn(sg, dQ)), R, dP), rD));
}

}  // namespace kf
