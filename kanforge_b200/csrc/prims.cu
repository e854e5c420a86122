// Float32 CUDA-core kernels of the closed primitive family
// (reference kanforge/kernels/__init__.py:5-13, triton_kernels.py:128-191):
//
//   F_m(x, w, c)[b,o]   = sum_{i,j} w[b,i] c[o,i,j] phi_j^(m)(x[b,i])
//   G_m(x, w, g)[o,i,j] = sum_b     w[b,i] g[b,o]   phi_j^(m)(x[b,i])
//   P_m(x, g, c)[b,i]   = sum_{o,j} g[b,o] c[o,i,j] phi_j^(m)(x[b,i])
//
// They serve every derivative order (the higher-order autograd closure) and
// float32 layers.  Each is a register-blocked shared-memory GEMM whose basis
// operand is evaluated on the fly, never materialised in HBM.  Unlike the
// reference (one input per step, a grid of only ceil(B/32) x ceil(O/32) CTAs
// for F), tiles cover 4 inputs per step and 64x64 outputs.
#include "features.cuh"

namespace kf {

namespace {

constexpr int kThreads = 256;
constexpr int kTile = 64;   // rows (b) and columns (o) per CTA
constexpr int kChunk = 4;   // inputs per main-loop step

// ---------------------------------------------------------------------------
// F: out (B, O)
// ---------------------------------------------------------------------------
template <int BK>
__global__ void __launch_bounds__(kThreads) prim_f_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ c, float* __restrict__ out,
                                                          int64_t B, int I, int O, FeatArgs fa) {
  extern __shared__ float smem[];
  const int nf = fa.nf;
  float* As = smem;                           // [kChunk][nf][kTile]
  float* Bs = As + kChunk * nf * kTile;       // [kChunk][nf][kTile]
  float* Ts = Bs + kChunk * nf * kTile;       // [kChunk][KF_NK_MAX]
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t b0 = (int64_t)blockIdx.x * kTile;
  const int o0 = blockIdx.y * kTile;
  float acc[4][4] = {};

  for (int i0 = 0; i0 < I; i0 += kChunk) {
    if constexpr (BK > 0 || BK == kBumpBK) {
      for (int ii = 0; ii < kChunk; ++ii)
        if (i0 + ii < I) load_knots<BK>(fa, i0 + ii, Ts + ii * KF_NK_MAX, tid, kThreads);
      __syncthreads();
    }
    {  // features of (b, i): one thread each
      const int ii = tid / kTile, bm = tid % kTile;
      const int64_t b = b0 + bm;
      const int i = i0 + ii;
      float* dst = As + (ii * nf) * kTile + bm;
      if (b < B && i < I) {
        eval_features<BK>(fa, x[b * I + i], w[b * I + i], Ts + ii * KF_NK_MAX, dst, kTile);
      } else {
        for (int j = 0; j < nf; ++j) dst[j * kTile] = 0.0f;
      }
    }
    {  // coefficients c[o, i0..i0+3, :]: contiguous per output row
      const int per_row = kChunk * nf;
      for (int e = tid; e < kTile * per_row; e += kThreads) {
        const int bn = e / per_row, rem = e % per_row;
        const int ii = rem / nf, j = rem % nf;
        const int o = o0 + bn, i = i0 + ii;
        Bs[(ii * nf + j) * kTile + bn] = (o < O && i < I) ? c[((int64_t)o * I + i) * nf + j] : 0.0f;
      }
    }
    __syncthreads();
    const int kk = kChunk * nf;
    for (int k = 0; k < kk; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(As + k * kTile + ty * 4);
      const float4 bb = *reinterpret_cast<const float4*>(Bs + k * kTile + tx * 4);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s = 0; s < 4; ++s) acc[r][s] = fmaf(av[r], bv[s], acc[r][s]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t b = b0 + ty * 4 + r;
    if (b >= B) continue;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int o = o0 + tx * 4 + s;
      if (o < O) out[b * O + o] = acc[r][s];
    }
  }
}

// ---------------------------------------------------------------------------
// G: out (O, I, nf)
// ---------------------------------------------------------------------------
constexpr int kBatchStep = 32;
constexpr int kNPerThread = 8;  // columns n = (ii, j) per thread: 4 * nf <= 128

template <int BK>
__global__ void __launch_bounds__(kThreads) prim_g_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ g, float* __restrict__ out,
                                                          int64_t B, int I, int O, FeatArgs fa) {
  extern __shared__ float smem[];
  const int nf = fa.nf;
  const int nn = kChunk * nf;
  float* As = smem;                       // [kBatchStep][nn]
  float* Gs = As + kBatchStep * nn;       // [kBatchStep][kTile]
  float* Ts = Gs + kBatchStep * kTile;    // [kChunk][KF_NK_MAX]
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int i0 = blockIdx.x * kChunk;
  const int o0 = blockIdx.y * kTile;
  if constexpr (BK > 0 || BK == kBumpBK) {
    for (int ii = 0; ii < kChunk; ++ii)
      if (i0 + ii < I) load_knots<BK>(fa, i0 + ii, Ts + ii * KF_NK_MAX, tid, kThreads);
    __syncthreads();
  }
  float acc[4][kNPerThread] = {};
  for (int64_t bs = 0; bs < B; bs += kBatchStep) {
    if (tid < kBatchStep * kChunk) {
      const int bl = tid % kBatchStep, ii = tid / kBatchStep;
      const int64_t b = bs + bl;
      const int i = i0 + ii;
      float* dst = As + bl * nn + ii * nf;
      if (b < B && i < I) {
        eval_features<BK>(fa, x[b * I + i], w[b * I + i], Ts + ii * KF_NK_MAX, dst, 1);
      } else {
        for (int j = 0; j < nf; ++j) dst[j] = 0.0f;
      }
    }
    for (int e = tid; e < kBatchStep * kTile; e += kThreads) {
      const int bl = e / kTile, ol = e % kTile;
      const int64_t b = bs + bl;
      const int o = o0 + ol;
      Gs[e] = (b < B && o < O) ? g[b * O + o] : 0.0f;
    }
    __syncthreads();
    for (int bl = 0; bl < kBatchStep; ++bl) {
      const float4 gv = *reinterpret_cast<const float4*>(Gs + bl * kTile + ty * 4);
      const float ga[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int u = 0; u < kNPerThread; ++u) {
        const int n = tx + 16 * u;
        const float a = n < nn ? As[bl * nn + n] : 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r][u] = fmaf(ga[r], a, acc[r][u]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int o = o0 + ty * 4 + r;
    if (o >= O) continue;
#pragma unroll
    for (int u = 0; u < kNPerThread; ++u) {
      const int n = tx + 16 * u;
      if (n >= nn) continue;
      const int ii = n / nf, j = n % nf;
      if (i0 + ii < I) out[((int64_t)o * I + i0 + ii) * nf + j] = acc[r][u];
    }
  }
}

// ---------------------------------------------------------------------------
// P: out (B, I)
// ---------------------------------------------------------------------------
constexpr int kOutStep = 32;

template <int BK>
__global__ void __launch_bounds__(kThreads) prim_p_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                                          const float* __restrict__ c, float* __restrict__ out,
                                                          int64_t B, int I, int O, FeatArgs fa) {
  extern __shared__ float smem[];
  const int nf = fa.nf;
  const int nn = kChunk * nf;
  float* Gs = smem;                         // [kOutStep][kTile]   (o-major: g[b, o] transposed)
  float* Cs = Gs + kOutStep * kTile;        // [kOutStep][nn]
  float* Hs = Cs + kOutStep * nn;           // [kTile][nn]
  float* Ts = Hs + kTile * nn;              // [kChunk][KF_NK_MAX]
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t b0 = (int64_t)blockIdx.x * kTile;
  const int i0 = blockIdx.y * kChunk;
  float acc[4][kNPerThread] = {};
  for (int os = 0; os < O; os += kOutStep) {
    for (int e = tid; e < kOutStep * kTile; e += kThreads) {
      const int bl = e / kOutStep, ol = e % kOutStep;  // coalesced over o
      const int64_t b = b0 + bl;
      const int o = os + ol;
      Gs[ol * kTile + bl] = (b < B && o < O) ? g[b * O + o] : 0.0f;
    }
    for (int e = tid; e < kOutStep * nn; e += kThreads) {
      const int ol = e / nn, n = e % nn;
      const int ii = n / nf, j = n % nf;
      const int o = os + ol, i = i0 + ii;
      Cs[e] = (o < O && i < I) ? c[((int64_t)o * I + i) * nf + j] : 0.0f;
    }
    __syncthreads();
    for (int ol = 0; ol < kOutStep; ++ol) {
      const float4 gv = *reinterpret_cast<const float4*>(Gs + ol * kTile + ty * 4);
      const float ga[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int u = 0; u < kNPerThread; ++u) {
        const int n = tx + 16 * u;
        const float cv = n < nn ? Cs[ol * nn + n] : 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r][u] = fmaf(ga[r], cv, acc[r][u]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int u = 0; u < kNPerThread; ++u) {
      const int n = tx + 16 * u;
      if (n < nn) Hs[(ty * 4 + r) * nn + n] = acc[r][u];
    }
  if constexpr (BK > 0 || BK == kBumpBK) {
    for (int ii = 0; ii < kChunk; ++ii)
      if (i0 + ii < I) load_knots<BK>(fa, i0 + ii, Ts + ii * KF_NK_MAX, tid, kThreads);
  }
  __syncthreads();
  {
    const int bm = tid % kTile, ii = tid / kTile;
    const int64_t b = b0 + bm;
    const int i = i0 + ii;
    if (b < B && i < I) out[b * I + i] = dot_features<BK>(fa, x[b * I + i], Ts + ii * KF_NK_MAX, Hs + bm * nn + ii * nf, 1);
  }
}

}  // namespace

struct PrimLaunch {
  int op;
  const float *x, *a, *b;
  float* out;
  int64_t B;
  int I, O;
  FeatArgs fa;
  cudaStream_t stream;

  template <int BK>
  int operator()() const {
    const int nf = fa.nf;
    size_t smem = 0;
    dim3 grid;
    if (op == KF_OP_F) {
      smem = sizeof(float) * (2 * kChunk * nf * kTile + kChunk * KF_NK_MAX);
      grid = dim3((unsigned)cdiv(B, kTile), (unsigned)cdiv(O, kTile));
      KF_CUDA_RET(cudaFuncSetAttribute(prim_f_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      prim_f_kernel<BK><<<grid, kThreads, smem, stream>>>(x, a, b, out, B, I, O, fa);
    } else if (op == KF_OP_G) {
      const int nn = kChunk * nf;
      smem = sizeof(float) * (kBatchStep * nn + kBatchStep * kTile + kChunk * KF_NK_MAX);
      grid = dim3((unsigned)cdiv(I, kChunk), (unsigned)cdiv(O, kTile));
      KF_CUDA_RET(cudaFuncSetAttribute(prim_g_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      prim_g_kernel<BK><<<grid, kThreads, smem, stream>>>(x, a, b, out, B, I, O, fa);
    } else {
      const int nn = kChunk * nf;
      smem = sizeof(float) * (kOutStep * kTile + kOutStep * nn + kTile * nn + kChunk * KF_NK_MAX);
      grid = dim3((unsigned)cdiv(B, kTile), (unsigned)cdiv(I, kChunk));
      KF_CUDA_RET(cudaFuncSetAttribute(prim_p_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      prim_p_kernel<BK><<<grid, kThreads, smem, stream>>>(x, a, b, out, B, I, O, fa);
    }
    return check_launch("kf_prim");
  }
};

// ---------------------------------------------------------------------------
// Float32 feature matrix and its input-gradient contraction, for the float32
// tensor-core path (kf_gemm_tf32x3).  Column layout of input i: i * F + j,
// phi_j(x) for j < nf, zero up to F - 2, silu(x) at F - 1 when the base branch
// is fused (the layout of kf_pack_coef).  Threads run along the inputs (one
// input's knots computed once per thread), CTAs along row blocks.
// ---------------------------------------------------------------------------
constexpr int kFeatRows = 64;      // rows per CTA row block
constexpr int64_t kMaxGridY = 65535;  // gridDim.y limit: larger B strides over the row blocks

template <int BK, int F>
__global__ void __launch_bounds__(kThreads) feature_f32_kernel(const float* __restrict__ x, float* __restrict__ feat,
                                                               int64_t B, int I, int has_base, FeatArgs fa) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= I) return;
  float t[KF_NK_MAX];
  load_knots<BK>(fa, i, t, 0, 1);
  // row blocks of kFeatRows, strided by gridDim.y (capped at 65535 by the launch)
  for (int64_t b0 = (int64_t)blockIdx.y * kFeatRows; b0 < B; b0 += (int64_t)gridDim.y * kFeatRows)
  for (int64_t b = b0, b1 = min(B, b0 + kFeatRows); b < b1; ++b) {
    const float xv = x[b * I + i];
    float f[F];  // the row, written out as float4s
    eval_features<BK>(fa, xv, 1.0f, t, f, 1);
    for (int j = fa.nf; j < F - 1; ++j) f[j] = 0.0f;
    f[F - 1] = has_base ? silu_acc(xv) : 0.0f;
    float4* dst = reinterpret_cast<float4*>(feat + (b * I + i) * F);
#pragma unroll
    for (int c = 0; c < F / 4; ++c) dst[c] = make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
  }
}

// dx[b, i] = sum_j dfeat[b, i * F + j] d phi_j / dx + dfeat[b, i * F + F - 1] silu'(x).
// B-splines: the native first-derivative window; Chebyshev features T_j(z):
// dT_j/dz = j U_{j-1}(z) (U_0 = 1, U_1 = 2 z, U_j = 2 z U_{j-1} - U_{j-2}),
// times dz/dx = 1 - z^2 under the tanh map.
template <int BK, int F>
__global__ void __launch_bounds__(kThreads) feature_dot_f32_kernel(const float* __restrict__ x, const float* __restrict__ dfeat,
                                                                   float* __restrict__ dx, int64_t B, int I, int has_base,
                                                                   FeatArgs fa) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= I) return;
  float t[KF_NK_MAX];
  load_knots<BK>(fa, i, t, 0, 1);
  // row blocks of kFeatRows, strided by gridDim.y (capped at 65535 by the launch)
  for (int64_t b0 = (int64_t)blockIdx.y * kFeatRows; b0 < B; b0 += (int64_t)gridDim.y * kFeatRows)
  for (int64_t b = b0, b1 = min(B, b0 + kFeatRows); b < b1; ++b) {
    const float xv = x[b * I + i];
    const float* h = dfeat + (b * I + i) * F;
    float acc;
    if constexpr (BK == kFourierBK) {
      // d/dx cos(j w1 x) = -j w1 sin(j w1 x), d/dx sin(j w1 x) = j w1 cos(j w1 x)
      const int n = fa.nf / 2;
      float s1, c1;
      sincosf(fa.w1 * xv, &s1, &c1);
      float c = c1, sn = s1;
      acc = 0.0f;
      for (int j = 0; j < n; ++j) {
        const float w = (float)(j + 1) * fa.w1;
        acc = fmaf(w, fmaf(h[n + j], c, -h[j] * sn), acc);
        const float cn = c * c1 - sn * s1;
        sn = sn * c1 + c * s1;
        c = cn;
      }
    } else if constexpr (BK == 0) {
      const bool tanh_map = fa.map == KF_MAP_TANH;
      const float z = tanh_map ? tanhf(xv) : xv;
      float um2 = 0.0f, um1 = 1.0f;  // U_{j-2}, U_{j-1} for j = 1
      acc = 0.0f;
      for (int j = 1; j < fa.nf; ++j) {
        acc = fmaf(h[j] * (float)j, um1, acc);
        const float uj = j == 1 ? 2.0f * z : 2.0f * z * um1 - um2;
        um2 = um1;
        um1 = uj;
      }
      if (tanh_map) acc *= 1.0f - z * z;
    } else {
      acc = dot_features<BK>(fa, xv, t, h, 1);
    }
    if (has_base) acc = fmaf(h[F - 1], dsilu_acc(xv), acc);
    dx[b * I + i] = acc;
  }
}

struct FeatureF32Launch {
  bool dot;
  const float *x, *dfeat;
  float* out;
  int64_t B;
  int I, F, has_base;
  FeatArgs fa;
  cudaStream_t stream;
  template <int BK>
  int operator()() const {
    const dim3 grid((unsigned)cdiv((int64_t)I, (int64_t)kThreads),
                    (unsigned)std::min<int64_t>(cdiv(B, (int64_t)kFeatRows), kMaxGridY));
    if (dot) {
      if (F == 16) feature_dot_f32_kernel<BK, 16><<<grid, kThreads, 0, stream>>>(x, dfeat, out, B, I, has_base, fa);
      else feature_dot_f32_kernel<BK, 32><<<grid, kThreads, 0, stream>>>(x, dfeat, out, B, I, has_base, fa);
    } else {
      if (F == 16) feature_f32_kernel<BK, 16><<<grid, kThreads, 0, stream>>>(x, out, B, I, has_base, fa);
      else feature_f32_kernel<BK, 32><<<grid, kThreads, 0, stream>>>(x, out, B, I, has_base, fa);
    }
    return check_launch(dot ? "kf_features_dot_f32" : "kf_features_f32");
  }
};

int feature_args(const kf_basis_desc* basis, const float* grid, int nf, int F, int m, FeatArgs& fa) {
  KF_CHECK_ARG(basis != nullptr, "basis is null");
  KF_CHECK_ARG(F == 16 || F == 32, "F must be 16 or 32 (got %d)", F);
  KF_CHECK_ARG(nf >= 1 && nf + 1 <= F, "nf %d (+ the SiLU column) exceeds F %d", nf, F);
  fa.m = m;
  fa.nf = nf;
  fa.map = basis->input_map;
  if (basis->kind == KF_BASIS_BSPLINE) {
    KF_CHECK_ARG(grid != nullptr, "B-spline needs its grid");
    fa.G = basis->grid_size;
    fa.nk = basis->grid_size + 2 * basis->order + 1;
    fa.grid = grid;
    KF_CHECK_ARG(fa.nk <= KF_NK_MAX, "%d knots exceed the limit %d", fa.nk, KF_NK_MAX);
    KF_CHECK_ARG(nf == basis->size, "B-spline nf %d != size %d", nf, basis->size);
  } else if (basis->kind == KF_BASIS_FOURIER || basis->kind == KF_BASIS_BUMP) {
    KF_CHECK_ARG(nf == basis->size, "nf %d != basis size %d", nf, basis->size);
    if (!fill_closed_family(basis, grid, m, fa)) return KF_ERR_ARG;
  } else if (basis->kind != KF_BASIS_CHEB) {
    set_error("basis kind %d has no float32 feature kernel", basis->kind);
    return KF_ERR_UNSUPPORTED;
  }
  return KF_OK;
}

}  // namespace kf

extern "C" int kf_prim(int op, int m, const float* x, const float* a, const float* b, const float* grid, float* out,
                       int64_t B, int32_t I, int32_t O, int32_t nf, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(basis != nullptr, "kf_prim: basis is null");
  KF_CHECK_ARG(op == KF_OP_F || op == KF_OP_G || op == KF_OP_P, "kf_prim: bad op %d", op);
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1 && nf >= 1 && m >= 0, "kf_prim: bad sizes B=%lld I=%d O=%d nf=%d m=%d",
               (long long)B, I, O, nf, m);
  KF_CHECK_ARG(nf <= KF_NF_MAX, "kf_prim: %d features exceed the limit %d", nf, KF_NF_MAX);
  KF_CHECK_ARG(x && a && b && out, "kf_prim: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  FeatArgs fa{};
  fa.m = m;
  fa.nf = nf;
  fa.map = basis->input_map;
  if (basis->kind == KF_BASIS_BSPLINE) {
    KF_CHECK_ARG(grid != nullptr, "kf_prim: B-spline needs its grid");
    fa.G = basis->grid_size;
    fa.nk = basis->grid_size + 2 * basis->order + 1;
    fa.grid = grid;
    KF_CHECK_ARG(fa.nk <= KF_NK_MAX, "kf_prim: %d knots exceed the limit %d", fa.nk, KF_NK_MAX);
    KF_CHECK_ARG(nf == basis->size, "kf_prim: B-spline nf %d != size %d", nf, basis->size);
  } else if (basis->kind == KF_BASIS_FOURIER || basis->kind == KF_BASIS_BUMP) {
    KF_CHECK_ARG(nf == basis->size, "kf_prim: nf %d != basis size %d", nf, basis->size);
    if (!fill_closed_family(basis, grid, m, fa)) return KF_ERR_ARG;
  } else if (basis->kind != KF_BASIS_CHEB) {
    set_error("kf_prim: basis kind %d has no primitive kernel", basis->kind);
    return KF_ERR_UNSUPPORTED;
  }
  if (B == 0) {
    if (op == KF_OP_G) KF_CUDA_RET(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)O * I * nf, (cudaStream_t)stream));
    return KF_OK;
  }
  PrimLaunch L{op, x, a, b, out, B, I, O, fa, (cudaStream_t)stream};
  return dispatch_bk(basis, L);
}

extern "C" int kf_features_f32(const float* x, const float* grid, float* feat, int64_t B, int32_t I, int32_t nf, int32_t F,
                               int32_t has_base, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && feat && B >= 0 && I >= 1, "kf_features_f32: bad arguments");
  KF_CHECK_ARG(((uintptr_t)feat % 16) == 0, "kf_features_f32: feat must be 16-byte aligned");
  FeatArgs fa{};
  if (int rc = feature_args(basis, grid, nf, F, 0, fa)) return rc;
  if (int rc = bind_device(x)) return rc;
  if (B == 0) return KF_OK;
  FeatureF32Launch L{false, x, nullptr, feat, B, I, F, has_base, fa, (cudaStream_t)stream};
  return dispatch_bk(basis, L);
}

extern "C" int kf_features_dot_f32(const float* x, const float* grid, const float* dfeat, float* dx, int64_t B, int32_t I,
                                   int32_t nf, int32_t F, int32_t has_base, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && dfeat && dx && B >= 0 && I >= 1, "kf_features_dot_f32: bad arguments");
  KF_CHECK_ARG(((uintptr_t)dfeat % 16) == 0, "kf_features_dot_f32: dfeat must be 16-byte aligned");
  FeatArgs fa{};
  if (int rc = feature_args(basis, grid, nf, F, 1, fa)) return rc;
  if (int rc = bind_device(x)) return rc;
  if (B == 0) return KF_OK;
  FeatureF32Launch L{true, x, dfeat, dx, B, I, F, has_base, fa, (cudaStream_t)stream};
  return dispatch_bk(basis, L);
}
