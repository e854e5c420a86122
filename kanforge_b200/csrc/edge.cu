// edge_derivative: out[b,o,i] = sum_j phi_j^(m)(x[b,i]) coefT[o,j,i] + s_m(x[b,i]) base[o,i]
// (reference kanforge/torch/layers.py:206-226).
//
// The output (B, O, I) is the whole cost (4.3 GB at the PINN configuration),
// so the kernel is organised around writing it once at HBM speed: every thread
// owns 4 consecutive inputs of NB rows, evaluates their features once into
// registers, then streams over all outputs o with one 16-byte streaming store
// per (row, o).  Coefficients are read in the transposed layout (O, nf, I) so
// that the 4 inputs of a thread are one 16-byte load per feature; they stay in
// L1/L2 (O*nf*I floats, 147 KB at the PINN configuration).
#include "features.cuh"

namespace kf {

namespace {

constexpr int kEdgeLanesI = 16;  // float4 lanes along i: 64 inputs per CTA
constexpr int kEdgeLanesB = 8;   // row lanes

struct EdgeArgs {
  const float* x;
  const float* coefT;  // (O, nf, I)
  const float* base;   // (O, I) or null
  const float* num;    // rational: (groups, na)
  const float* den;    // rational: (groups, nb)
  float* out;
  int64_t B;
  int I, O, nf, m;
  int na, nb, in_per_group;
  float poly[2 * 8];   // h_m, h_{m-1} in sigmoid (silu derivatives)
  int n_poly;
  FeatArgs fa;
};

// Feature j of order m at x for input i (rational: j == 0 only).
template <int BK>
__device__ __forceinline__ void edge_features(const EdgeArgs& A, int i, float x, const float* t, float* f) {
  if constexpr (BK < 0) {
    const int g = i / A.in_per_group;
    f[0] = rational_deriv(x, A.num + (size_t)g * A.na, A.na, A.den + (size_t)g * A.nb, A.nb, A.m);
  } else {
    eval_features<BK>(A.fa, x, 1.0f, t, f, 1);
  }
}

template <int BK, int NFM, int NB>
__global__ void __launch_bounds__(kEdgeLanesI * kEdgeLanesB) edge_vec_kernel(EdgeArgs A) {
  __shared__ float Ts[64 * KF_NK_MAX];
  const int li = threadIdx.x % kEdgeLanesI;
  const int lb = threadIdx.x / kEdgeLanesI;
  const int i_base = blockIdx.y * 64;
  const int i4 = i_base + li * 4;
  const int64_t b_base = (int64_t)blockIdx.x * (kEdgeLanesB * NB) + lb * NB;
  if constexpr (BK > 0) {
    for (int e = threadIdx.x; e < 64 * A.fa.nk; e += blockDim.x) {
      const int ii = e / A.fa.nk, r = e % A.fa.nk;
      if (i_base + ii < A.I) Ts[ii * KF_NK_MAX + r] = extended_knot(A.fa.grid + (size_t)(i_base + ii) * (A.fa.G + 1), A.fa.G, BK, r);
    }
    __syncthreads();
  }
  if (i4 >= A.I) return;
  float feat[NB][4][NFM];
  float sb[NB][4];
  bool row_ok[NB];
#pragma unroll
  for (int r = 0; r < NB; ++r) {
    const int64_t b = b_base + r;
    row_ok[r] = b < A.B;
    const float4 xv = row_ok[r] ? *reinterpret_cast<const float4*>(A.x + b * A.I + i4) : make_float4(0, 0, 0, 0);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float tmp[KF_NF_MAX];
      edge_features<BK>(A, i4 + c, xs[c], Ts + (li * 4 + c) * KF_NK_MAX, tmp);
#pragma unroll
      for (int j = 0; j < NFM; ++j) feat[r][c][j] = j < A.nf ? tmp[j] : 0.0f;
      sb[r][c] = A.base ? silu_deriv(xs[c], A.m, A.poly, A.n_poly) : 0.0f;
    }
  }
  for (int o = 0; o < A.O; ++o) {
    float4 cf[NFM];
    const float* crow = A.coefT + (size_t)o * A.nf * A.I + i4;
#pragma unroll
    for (int j = 0; j < NFM; ++j) cf[j] = j < A.nf ? __ldg(reinterpret_cast<const float4*>(crow + (size_t)j * A.I)) : make_float4(0, 0, 0, 0);
    const float4 bw = A.base ? __ldg(reinterpret_cast<const float4*>(A.base + (size_t)o * A.I + i4)) : make_float4(0, 0, 0, 0);
#pragma unroll
    for (int r = 0; r < NB; ++r) {
      if (!row_ok[r]) continue;
      float acc[4] = {sb[r][0] * bw.x, sb[r][1] * bw.y, sb[r][2] * bw.z, sb[r][3] * bw.w};
#pragma unroll
      for (int j = 0; j < NFM; ++j) {
        acc[0] = fmaf(feat[r][0][j], cf[j].x, acc[0]);
        acc[1] = fmaf(feat[r][1][j], cf[j].y, acc[1]);
        acc[2] = fmaf(feat[r][2][j], cf[j].z, acc[2]);
        acc[3] = fmaf(feat[r][3][j], cf[j].w, acc[3]);
      }
      __stcs(reinterpret_cast<float4*>(A.out + ((b_base + r) * A.O + o) * A.I + i4), make_float4(acc[0], acc[1], acc[2], acc[3]));
    }
  }
}

// Any I and nf <= KF_NF_MAX: one thread per (b, i), looping over o.
template <int BK>
__global__ void __launch_bounds__(256) edge_scalar_kernel(EdgeArgs A) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= A.B * A.I) return;
  const int64_t b = e / A.I;
  const int i = (int)(e % A.I);
  float t[KF_NK_MAX];
  if constexpr (BK > 0) load_knots<BK>(A.fa, i, t, 0, 1);
  const float x = A.x[e];
  float f[KF_NF_MAX];
  edge_features<BK>(A, i, x, t, f);
  const float sb = A.base ? silu_deriv(x, A.m, A.poly, A.n_poly) : 0.0f;
  for (int o = 0; o < A.O; ++o) {
    float acc = A.base ? sb * A.base[(size_t)o * A.I + i] : 0.0f;
    for (int j = 0; j < A.nf; ++j) acc = fmaf(f[j], A.coefT[((size_t)o * A.nf + j) * A.I + i], acc);
    A.out[(b * A.O + o) * A.I + i] = acc;
  }
}

struct EdgeLaunch {
  EdgeArgs A;
  cudaStream_t stream;
  bool vec;

  template <int BK>
  int operator()() const {
    if (vec && A.nf <= 10) {
      constexpr int NB = 2;
      dim3 grid((unsigned)cdiv(A.B, kEdgeLanesB * NB), (unsigned)cdiv(A.I, 64));
      edge_vec_kernel<BK, 10, NB><<<grid, kEdgeLanesI * kEdgeLanesB, 0, stream>>>(A);
    } else if (vec && A.nf <= 16) {
      dim3 grid((unsigned)cdiv(A.B, kEdgeLanesB), (unsigned)cdiv(A.I, 64));
      edge_vec_kernel<BK, 16, 1><<<grid, kEdgeLanesI * kEdgeLanesB, 0, stream>>>(A);
    } else {
      edge_scalar_kernel<BK><<<(unsigned)cdiv(A.B * A.I, 256), 256, 0, stream>>>(A);
    }
    return check_launch("kf_edge_derivative");
  }
};

}  // namespace

}  // namespace kf

extern "C" int kf_edge_derivative(const float* x, const float* coef, const float* base_eff, const float* grid,
                                  const float* basis_num, const float* basis_den, float* out, int64_t B, int32_t I,
                                  int32_t O, int32_t nf, int32_t order, const kf_basis_desc* basis,
                                  const float* silu_poly, int32_t n_poly, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(basis != nullptr, "kf_edge_derivative: basis is null");
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1 && nf >= 1 && order >= 0, "kf_edge_derivative: bad sizes");
  KF_CHECK_ARG(nf <= KF_NF_MAX, "kf_edge_derivative: %d features exceed the limit %d", nf, KF_NF_MAX);
  KF_CHECK_ARG(x && coef && out, "kf_edge_derivative: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(base_eff == nullptr || (silu_poly != nullptr && n_poly >= 1 && n_poly <= 8),
               "kf_edge_derivative: the base term needs 1..8 SiLU polynomial coefficients");
  EdgeArgs A{};
  A.x = x;
  A.coefT = coef;
  A.base = base_eff;
  A.out = out;
  A.B = B;
  A.I = I;
  A.O = O;
  A.nf = nf;
  A.m = order;
  A.n_poly = base_eff ? n_poly : 0;
  for (int e = 0; e < 2 * A.n_poly; ++e) A.poly[e] = silu_poly[e];
  A.fa.m = order;
  A.fa.nf = nf;
  A.fa.map = basis->input_map;
  if (B == 0) return KF_OK;
  const bool vec = (I % 4 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)coef % 16 == 0) && ((uintptr_t)out % 16 == 0) &&
                   (base_eff == nullptr || (uintptr_t)base_eff % 16 == 0);
  EdgeLaunch L{A, (cudaStream_t)stream, vec};
  if (basis->kind == KF_BASIS_RATIONAL) {
    KF_CHECK_ARG(basis_num && basis_den, "kf_edge_derivative: rational needs its parameters");
    KF_CHECK_ARG(nf == 1, "kf_edge_derivative: rational has one feature");
    KF_CHECK_ARG(basis->groups >= 1 && I % basis->groups == 0, "kf_edge_derivative: groups must divide I");
    KF_CHECK_ARG(basis->degree + 1 <= KF_RAT_MAX_NUM && basis->den_degree <= KF_RAT_MAX_DEN && order <= KF_RAT_MAX_ORDER,
                 "kf_edge_derivative: rational degree/order beyond the kernel limits");
    L.A.num = basis_num;
    L.A.den = basis_den;
    L.A.na = basis->degree + 1;
    L.A.nb = basis->den_degree;
    L.A.in_per_group = I / basis->groups;
    return L.template operator()<-1>();
  }
  if (basis->kind == KF_BASIS_BSPLINE) {
    KF_CHECK_ARG(grid != nullptr, "kf_edge_derivative: B-spline needs its grid");
    L.A.fa.G = basis->grid_size;
    L.A.fa.nk = basis->grid_size + 2 * basis->order + 1;
    L.A.fa.grid = grid;
    KF_CHECK_ARG(L.A.fa.nk <= KF_NK_MAX, "kf_edge_derivative: too many knots");
  }
  return dispatch_bk(basis, L);
}
