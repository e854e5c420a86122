// edge_derivative: out[b,o,i] = sum_j phi_j^(m)(x[b,i]) coefT[o,j,i] + s_m(x[b,i]) base[o,i]
// (reference kanforge/torch/layers.py:206-226).
//
// The output (B, O, I) is the whole cost (4.3 GB at the PINN configuration),
// so the kernel is organised around writing it once at HBM speed: the
// features of a (row, input) pair are evaluated once and kept in registers
// while all outputs o stream past, and the coefficients (O*nf*I floats, read
// in the (O, nf, I) layout so that a warp's load is one 128-byte line) stay in
// L1/L2 and are reused over many rows per thread.
#include <algorithm>

#include "features.cuh"

namespace kf {

namespace {

constexpr int kEdgeThreads = 256;
constexpr int kEdgeMaxNF = 16;  // features per input of the streaming kernel
constexpr int kEdgeFeatRegs = 168;   // feature registers per thread of the streaming kernel
constexpr int kEdgeBlocksPerSM = 1;  // resident CTAs per SM the streaming kernel is built for

struct EdgeArgs {
  const float* x;
  const float* coef;   // (O, nf, I)
  const float* base;   // (O, I) or null
  const float* num;    // rational: (groups, na)
  const float* den;    // rational: (groups, nb)
  float* out;
  const float* g;      // backward: the output gradient (B, O, I)
  int64_t B;
  int I, O, nf, m;
  int kind, order;     // KF_BASIS_*, B-spline order
  int na, nb, in_per_group;
  float poly[2 * 8];   // h_m, h_{m-1} in sigmoid (silu derivatives)
  int n_poly;
  FeatArgs fa;
};

// Features j < nf of order m at x for input i; t: knots of input i (B-splines).
__device__ __forceinline__ void edge_features_rt(const EdgeArgs& A, int i, float x, const float* t, float* f,
                                                 int stride = 1) {
  const int sel = A.kind == KF_BASIS_BSPLINE ? A.order
                  : A.kind == KF_BASIS_RATIONAL ? -1
                  : A.kind == KF_BASIS_FOURIER ? kFourierBK
                  : A.kind == KF_BASIS_BUMP    ? kBumpBK
                                               : 0;
  switch (sel) {
    case kFourierBK: eval_features<kFourierBK>(A.fa, x, 1.0f, t, f, stride); break;
    case kBumpBK: eval_features<kBumpBK>(A.fa, x, 1.0f, t, f, stride); break;
    case -1: {
      const int g = i / A.in_per_group;
      f[0] = rational_deriv(x, A.num + (size_t)g * A.na, A.na, A.den + (size_t)g * A.nb, A.nb, A.m);
      break;
    }
    case 0: eval_features<0>(A.fa, x, 1.0f, t, f, stride); break;
    case 1: eval_features<1>(A.fa, x, 1.0f, t, f, stride); break;
    case 2: eval_features<2>(A.fa, x, 1.0f, t, f, stride); break;
    case 3: eval_features<3>(A.fa, x, 1.0f, t, f, stride); break;
    case 4: eval_features<4>(A.fa, x, 1.0f, t, f, stride); break;
    default: eval_features<5>(A.fa, x, 1.0f, t, f, stride); break;
  }
}

__device__ __forceinline__ void load_knots_rt(const EdgeArgs& A, int i, float* t) {
  if (A.kind == KF_BASIS_BUMP) {
    for (int r = 0; r < A.fa.nk; ++r) t[r] = A.fa.grid[(size_t)i * A.fa.nk + r];
    return;
  }
  if (A.kind != KF_BASIS_BSPLINE) return;
  const float* g = A.fa.grid + (size_t)i * (A.fa.G + 1);
  for (int r = 0; r < A.fa.nk; ++r) t[r] = extended_knot(g, A.fa.G, A.order, r);
}

// 4-byte asynchronous global -> shared copy (zero-filled when !valid).
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  const int n = valid ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Rows whose features are staged in shared memory at once (the basis code is
// inlined NB / CH times).
__host__ __device__ constexpr int edge_chunk(int nb) { return nb % 4 == 0 ? 4 : 2; }

// Rows per thread of the streaming kernel for NF features: an even number
// that keeps NB x (NF + 1) feature registers near 170, so that the
// coefficients of one output (NF + 1 loads) serve NB outputs.
__host__ __device__ constexpr int edge_rows(int nf) {
  return (kEdgeFeatRegs / (nf + 1) < 2 ? 2 : (kEdgeFeatRegs / (nf + 1) > 16 ? 16 : kEdgeFeatRegs / (nf + 1))) & ~1;
}

// One lane per input; a warp covers il consecutive inputs (il = 32, or the
// power of two covering I when I < 32) times 32 / il consecutive outputs, so
// each of its stores is one contiguous 128-byte run of the (B, O, I) output.
// A warp owns NB rows at a time.  Their x values arrive in the thread's
// shared-memory column by cp.async, issued while the previous group streams.
// The features (the silu term as feature NF) are evaluated CH rows at a time
// into shared memory and moved into registers paired by rows; then the warp
// streams over the outputs o: NF + 1 coalesced coefficient loads feed NB
// outputs, two rows per packed f32x2 FMA.  Warps take row groups
// independently (persistent, no barrier after the knot table), so one warp's
// feature prologue overlaps the others' stores.
template <int NF, int NB>
__global__ void __launch_bounds__(kEdgeThreads, kEdgeBlocksPerSM) edge_vec_kernel(const __grid_constant__ EdgeArgs A, int il_log2) {
  constexpr int NJ = NF + 1, NP = NB / 2, CH = edge_chunk(NB);
  static_assert(NB % 2 == 0 && NB % CH == 0, "rows are processed in pairs and chunks");
  extern __shared__ float smem[];
  float* Fs = smem;                            // [CH][NJ][kEdgeThreads]: features of CH rows
  float* Xs = Fs + CH * NJ * kEdgeThreads;     // [NB][kEdgeThreads]: x of the group's rows
  float* Ts = Xs + NB * kEdgeThreads;          // [il][KF_NK_MAX] (B-splines)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int il = 1 << il_log2, ol = 32 / il;
  const int i = blockIdx.y * il + (lane & (il - 1));
  const int lo = lane >> il_log2;
  const int i_base = blockIdx.y * il;
  if (A.kind == KF_BASIS_BSPLINE || A.kind == KF_BASIS_BUMP) {
    const int n_in = min(il, A.I - i_base);
    for (int e = threadIdx.x; e < n_in * A.fa.nk; e += blockDim.x) {
      const int ii = e / A.fa.nk, r = e % A.fa.nk;
      Ts[ii * KF_NK_MAX + r] = A.kind == KF_BASIS_BUMP
                                   ? A.fa.grid[(size_t)(i_base + ii) * A.fa.nk + r]
                                   : extended_knot(A.fa.grid + (size_t)(i_base + ii) * (A.fa.G + 1), A.fa.G, A.order, r);
    }
    __syncthreads();
  }
  if (i >= A.I) return;
  const float* ti = Ts + (i - i_base) * KF_NK_MAX;
  float* fs = Fs + threadIdx.x;
  float* xs = Xs + threadIdx.x;
  const int64_t n_groups = (A.B + NB - 1) / NB;
  const int64_t g_step = (int64_t)gridDim.x * (kEdgeThreads / 32);
  const size_t c_step = (size_t)ol * NF * A.I, o_step = (size_t)ol * A.I, row_step = (size_t)A.O * A.I;
  auto fetch_x = [&](int64_t grp) {
#pragma unroll
    for (int r = 0; r < NB; ++r) {
      const int64_t b = grp * NB + r;
      cp_async4(xs + r * kEdgeThreads, A.x + (b < A.B ? b : 0) * A.I + i, b < A.B);
    }
    cp_async_commit();
  };
  int64_t grp = (int64_t)blockIdx.x * (kEdgeThreads / 32) + warp;
  if (grp < n_groups) fetch_x(grp);
  for (; grp < n_groups; grp += g_step) {
    const int64_t b0 = grp * NB;
    const int nrows = (int)min((int64_t)NB, A.B - b0);
    cp_async_wait();
    float2 feat[NP][NJ];
#pragma unroll
    for (int c = 0; c < NB / CH; ++c) {
#pragma unroll 1
      for (int rr = 0; rr < CH; ++rr) {
        const float x = xs[(c * CH + rr) * kEdgeThreads];
        float* f = fs + rr * NJ * kEdgeThreads;
        edge_features_rt(A, i, x, ti, f, kEdgeThreads);
        f[NF * kEdgeThreads] = A.base ? silu_deriv(x, A.m, A.poly, A.n_poly) : 0.0f;
      }
#pragma unroll
      for (int rr = 0; rr < CH; ++rr) {
        const int r = c * CH + rr;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const float v = fs[(rr * NJ + j) * kEdgeThreads];
          if (r % 2 == 0)
            feat[r / 2][j].x = v;
          else
            feat[r / 2][j].y = v;
        }
      }
    }
    if (grp + g_step < n_groups) fetch_x(grp + g_step);

    const float* cp = A.coef + (size_t)lo * NF * A.I + i;  // (O, NF, I)
    const float* bp = A.base ? A.base + (size_t)lo * A.I + i : nullptr;
    float* op = A.out + (b0 * A.O + lo) * A.I + i;
    // The coefficients of output o + ol are loaded while output o is computed.
    float q[NJ];
    if (lo < A.O) {
#pragma unroll
      for (int j = 0; j < NF; ++j) q[j] = __ldg(cp + (size_t)j * A.I);
      q[NF] = bp ? __ldg(bp) : 0.0f;
    }
    for (int o = lo; o < A.O; o += ol) {
      float qn[NJ];
      if (o + ol < A.O) {
#pragma unroll
        for (int j = 0; j < NF; ++j) qn[j] = __ldg(cp + c_step + (size_t)j * A.I);
        qn[NF] = bp ? __ldg(bp + o_step) : 0.0f;
      }
      float2 acc[NP];
      {
        const float2 qq = make_float2(q[NF], q[NF]);
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[p] = __fmul2_rn(feat[p][NF], qq);
      }
#pragma unroll
      for (int j = 0; j < NF; ++j) {
        const float2 qq = make_float2(q[j], q[j]);
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[p] = __ffma2_rn(feat[p][j], qq, acc[p]);
      }
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        if (2 * p < nrows) __stcs(op + (2 * p) * row_step, acc[p].x);
        if (2 * p + 1 < nrows) __stcs(op + (2 * p + 1) * row_step, acc[p].y);
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) q[j] = qn[j];
      cp += c_step;
      if (bp) bp += o_step;
      op += o_step;
    }
  }
  cp_async_wait();
}

// Any I and nf <= KF_NF_MAX: one thread per (b, i), looping over o.
__global__ void __launch_bounds__(256) edge_scalar_kernel(EdgeArgs A) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= A.B * A.I) return;
  const int64_t b = e / A.I;
  const int i = (int)(e % A.I);
  float t[KF_NK_MAX];
  load_knots_rt(A, i, t);
  const float x = A.x[e];
  float f[KF_NF_MAX];
  edge_features_rt(A, i, x, t, f);
  const float sb = A.base ? silu_deriv(x, A.m, A.poly, A.n_poly) : 0.0f;
  for (int o = 0; o < A.O; ++o) {
    float acc = A.base ? sb * A.base[(size_t)o * A.I + i] : 0.0f;
    const float* c = A.coef + (size_t)o * A.nf * A.I + i;
    for (int j = 0; j < A.nf; ++j) acc = fmaf(f[j], c[(size_t)j * A.I], acc);
    A.out[(b * A.O + o) * A.I + i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Backward of edge_derivative (the reference's is an autograd graph,
// kanforge/torch/layers.py:206-226): with g = dL/dout (B, O, I),
//   dx[b,i]       = sum_o g[b,o,i] (sum_j phi_j^(m+1)(x) coefT1[o,j,i] + s_(m+1)(x) base[o,i])
//   dcoefT[o,j,i] = sum_b g[b,o,i] phi_j^(m)(x[b,i]),   dbase[o,i] = sum_b g[b,o,i] s_m(x[b,i]).
// Both read g once, lanes along i (a warp's load is one 128-byte line).
// ---------------------------------------------------------------------------

// dx: one thread per (b, i); A holds the order-(m+1) features, coefficients
// and SiLU polynomials, A.out = dx (B, I).
__global__ void __launch_bounds__(256) edge_dx_kernel(EdgeArgs A) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= A.B * A.I) return;
  const int64_t b = e / A.I;
  const int i = (int)(e % A.I);
  float t[KF_NK_MAX];
  load_knots_rt(A, i, t);
  const float x = A.x[e];
  float f[KF_NF_MAX];
  edge_features_rt(A, i, x, t, f);
  const float sb = A.base ? silu_deriv(x, A.m, A.poly, A.n_poly) : 0.0f;
  float dx = 0.0f;
  const float* gp = A.g + b * A.O * A.I + i;
  for (int o = 0; o < A.O; ++o) {
    float v = A.base ? sb * A.base[(size_t)o * A.I + i] : 0.0f;
    const float* c = A.coef + (size_t)o * A.nf * A.I + i;
    for (int j = 0; j < A.nf; ++j) v = fmaf(f[j], c[(size_t)j * A.I], v);
    dx = fmaf(__ldcs(gp + (size_t)o * A.I), v, dx);
  }
  A.out[e] = dx;
}

// dcoefT / dbase partial sums: block (32 inputs) x (OC outputs) x (one of
// gridDim.z row splits); warp w takes the split's rows w, w + 8, ...; each
// thread keeps OC x NJ sums (NJ >= nf + 1: the features and the SiLU term),
// the 8 warps add theirs in shared memory in a fixed order, and the block
// writes ws[split][o][j][i] (j = nf: the base term).
template <int NJ, int OC>
__global__ void __launch_bounds__(256) edge_dcoef_kernel(EdgeArgs A, float* __restrict__ ws, int64_t rows_per_split) {
  __shared__ float red[8][NJ][32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int i = blockIdx.x * 32 + lane;
  const int o0 = blockIdx.y * OC;
  const int nj = A.nf + 1;
  float acc[OC][NJ];
#pragma unroll
  for (int q = 0; q < OC; ++q)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[q][j] = 0.0f;
  float t[KF_NK_MAX];
  if (i < A.I) load_knots_rt(A, i, t);
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_split;
  const int64_t r1 = min(A.B, r0 + rows_per_split);
  if (i < A.I) {
    for (int64_t b = r0 + warp; b < r1; b += 8) {
      const float x = A.x[b * A.I + i];
      float f[NJ];
      edge_features_rt(A, i, x, t, f);
      const float sterm = A.n_poly ? silu_deriv(x, A.m, A.poly, A.n_poly) : 0.0f;
      const float* gp = A.g + (b * A.O + o0) * A.I + i;
#pragma unroll
      for (int q = 0; q < OC; ++q) {
        if (o0 + q < A.O) {
          const float gv = __ldcs(gp + (size_t)q * A.I);
#pragma unroll
          for (int j = 0; j < NJ; ++j)
            if (j < nj) acc[q][j] = fmaf(gv, j < A.nf ? f[j] : sterm, acc[q][j]);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < OC; ++q) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) red[warp][j][lane] = acc[q][j];
    __syncthreads();
    for (int e = threadIdx.x; e < NJ * 32; e += 256) {
      const int l = e % 32, j = e / 32;
      const int ii = blockIdx.x * 32 + l;
      if (ii < A.I && o0 + q < A.O && j < nj) {
        float sum = 0.0f;
        for (int w = 0; w < 8; ++w) sum += red[w][j][l];
        ws[(((size_t)blockIdx.z * A.O + o0 + q) * nj + j) * A.I + ii] = sum;
      }
    }
    __syncthreads();
  }
}

// Sum of the splits in order: dcoefT[o,j,i] (j < nf) and dbase[o,i] (j = nf).
__global__ void __launch_bounds__(256) edge_dcoef_reduce_kernel(const float* __restrict__ ws, float* __restrict__ dcoefT,
                                                                float* __restrict__ dbase, int splits, int O, int nf, int I) {
  const int nj = nf + 1;
  const int64_t n = (int64_t)O * nj * I;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    float sum = 0.0f;
    for (int z = 0; z < splits; ++z) sum += ws[(size_t)z * n + e];
    const int i = (int)(e % I);
    const int64_t oj = e / I;
    const int j = (int)(oj % nj);
    const int64_t o = oj / nj;
    if (j < nf) dcoefT[(o * nf + j) * I + i] = sum;
    else if (dbase) dbase[o * I + i] = sum;
  }
}

template <int NF>
int launch_vec(const EdgeArgs& A, cudaStream_t stream) {
  constexpr int NB = edge_rows(NF);
  int il_log2 = 5;
  while (il_log2 > 0 && (1 << (il_log2 - 1)) >= A.I) --il_log2;
  const size_t smem = ((size_t)(edge_chunk(NB) * (NF + 1) + NB) * kEdgeThreads +
                       ((A.kind == KF_BASIS_BSPLINE || A.kind == KF_BASIS_BUMP) ? (32 * KF_NK_MAX) : 0)) * sizeof(float);
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  // The coefficients are read through L1: keep the shared-memory carve-out small.
  cudaError_t e = cudaFuncSetAttribute(edge_vec_kernel<NF, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(edge_vec_kernel<NF, NB>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxL1);
  if (e != cudaSuccess) {
    set_error("kf_edge_derivative: shared memory attribute: %s", cudaGetErrorString(e));
    return KF_ERR_CUDA;
  }
  const unsigned gy = (unsigned)cdiv(A.I, 1 << il_log2);
  const int64_t n_groups = cdiv(A.B, (int64_t)NB);
  const int64_t gx_need = cdiv(n_groups, (int64_t)(kEdgeThreads / 32));
  const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>(gx_need, std::max(1, kEdgeBlocksPerSM * n_sm / (int)std::min<unsigned>(gy, kEdgeBlocksPerSM * n_sm))));
  edge_vec_kernel<NF, NB><<<dim3(gx, gy), kEdgeThreads, smem, stream>>>(A, il_log2);
  return check_launch("kf_edge_derivative");
}

int launch_edge(const EdgeArgs& A, bool vec, cudaStream_t stream) {
  if (vec) {
    switch (A.nf) {
      case 1: return launch_vec<1>(A, stream);
      case 2: return launch_vec<2>(A, stream);
      case 3: return launch_vec<3>(A, stream);
      case 4: return launch_vec<4>(A, stream);
      case 5: return launch_vec<5>(A, stream);
      case 6: return launch_vec<6>(A, stream);
      case 7: return launch_vec<7>(A, stream);
      case 8: return launch_vec<8>(A, stream);
      case 9: return launch_vec<9>(A, stream);
      case 10: return launch_vec<10>(A, stream);
      case 11: return launch_vec<11>(A, stream);
      case 12: return launch_vec<12>(A, stream);
      case 13: return launch_vec<13>(A, stream);
      case 14: return launch_vec<14>(A, stream);
      case 15: return launch_vec<15>(A, stream);
      case kEdgeMaxNF: return launch_vec<kEdgeMaxNF>(A, stream);
      default: break;
    }
  }
  edge_scalar_kernel<<<(unsigned)cdiv(A.B * A.I, 256), 256, 0, stream>>>(A);
  return check_launch("kf_edge_derivative");
}

}  // namespace

}  // namespace kf

namespace kf {
namespace {
// EdgeArgs of an edge-derivative launch (shared by the forward and backward
// entry points); coefT may be null where the launch reads no coefficients.
int fill_edge_args(EdgeArgs& A, const float* x, const float* coefT, const float* base_eff, const float* grid,
                   const float* basis_num, const float* basis_den, float* out, int64_t B, int32_t I, int32_t O,
                   int32_t nf, int32_t order, const kf_basis_desc* basis, const float* silu_poly, int32_t n_poly,
                   bool need_coef) {
  KF_CHECK_ARG(basis != nullptr, "kf_edge_derivative: basis is null");
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1 && nf >= 1 && order >= 0, "kf_edge_derivative: bad sizes");
  KF_CHECK_ARG(nf <= KF_NF_MAX, "kf_edge_derivative: %d features exceed the limit %d", nf, KF_NF_MAX);
  KF_CHECK_ARG(x && out && (coefT || !need_coef), "kf_edge_derivative: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(base_eff == nullptr || (silu_poly != nullptr && n_poly >= 1 && n_poly <= 8),
               "kf_edge_derivative: the base term needs 1..8 SiLU polynomial coefficients");
  A = EdgeArgs{};
  A.x = x;
  A.coef = coefT;
  A.base = base_eff;
  A.out = out;
  A.B = B;
  A.I = I;
  A.O = O;
  A.nf = nf;
  A.m = order;
  A.kind = basis->kind;
  A.order = basis->order;
  A.n_poly = base_eff ? n_poly : 0;
  for (int e = 0; e < 2 * A.n_poly; ++e) A.poly[e] = silu_poly[e];
  A.fa.m = order;
  A.fa.nf = nf;
  A.fa.map = basis->input_map;
  if (basis->kind == KF_BASIS_RATIONAL) {
    KF_CHECK_ARG(basis_num && basis_den, "kf_edge_derivative: rational needs its parameters");
    KF_CHECK_ARG(nf == 1, "kf_edge_derivative: rational has one feature");
    KF_CHECK_ARG(basis->groups >= 1 && I % basis->groups == 0, "kf_edge_derivative: groups must divide I");
    KF_CHECK_ARG(basis->degree + 1 <= KF_RAT_MAX_NUM && basis->den_degree <= KF_RAT_MAX_DEN && order <= KF_RAT_MAX_ORDER,
                 "kf_edge_derivative: rational degree/order beyond the kernel limits");
    A.num = basis_num;
    A.den = basis_den;
    A.na = basis->degree + 1;
    A.nb = basis->den_degree;
    A.in_per_group = I / basis->groups;
  } else if (basis->kind == KF_BASIS_BSPLINE) {
    KF_CHECK_ARG(grid != nullptr, "kf_edge_derivative: B-spline needs its grid");
    KF_CHECK_ARG(basis->order >= 1 && basis->order <= 5, "kf_edge_derivative: B-spline order %d unsupported", basis->order);
    A.fa.G = basis->grid_size;
    A.fa.nk = basis->grid_size + 2 * basis->order + 1;
    A.fa.grid = grid;
    KF_CHECK_ARG(A.fa.nk <= KF_NK_MAX, "kf_edge_derivative: too many knots");
  } else if (basis->kind == KF_BASIS_FOURIER || basis->kind == KF_BASIS_BUMP) {
    KF_CHECK_ARG(nf == basis->size, "kf_edge_derivative: nf %d != basis size %d", nf, basis->size);
    if (!fill_closed_family(basis, grid, basis->kind == KF_BASIS_BUMP ? order : 0, A.fa)) return KF_ERR_ARG;
  } else if (basis->kind != KF_BASIS_CHEB) {
    set_error("kf_edge_derivative: basis kind %d unsupported", basis->kind);
    return KF_ERR_UNSUPPORTED;
  }
  return KF_OK;
}
}  // namespace
}  // namespace kf

extern "C" int kf_edge_derivative(const float* x, const float* coefT, const float* base_eff, const float* grid,
                                  const float* basis_num, const float* basis_den, float* out, int64_t B, int32_t I,
                                  int32_t O, int32_t nf, int32_t order, const kf_basis_desc* basis,
                                  const float* silu_poly, int32_t n_poly, void* stream) {
  using namespace kf;
  clear_error();
  EdgeArgs A;
  if (int rc = fill_edge_args(A, x, coefT, base_eff, grid, basis_num, basis_den, out, B, I, O, nf, order, basis, silu_poly,
                              n_poly, true))
    return rc;
  if (B == 0) return KF_OK;
  const bool vec = nf <= kEdgeMaxNF;
  return launch_edge(A, vec, (cudaStream_t)stream);
}

namespace kf {
namespace {
// Row splits of the coefficient-gradient kernel: about four CTAs per SM.
int edge_splits(int64_t B, int I, int O, int oc) {
  const int64_t blocks = cdiv((int64_t)I, (int64_t)32) * cdiv((int64_t)O, (int64_t)oc);
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv((int64_t)148 * 4, blocks), cdiv(B, (int64_t)64)));
}
int edge_oc(int nf) { return nf + 1 <= 10 ? 8 : (nf + 1 <= 17 ? 4 : 2); }
}  // namespace
}  // namespace kf

extern "C" int64_t kf_edge_derivative_workspace(int64_t B, int32_t I, int32_t O, int32_t nf) {
  if (B <= 0 || I <= 0 || O <= 0 || nf <= 0) return 0;
  const int oc = kf::edge_oc(nf);
  return (int64_t)kf::edge_splits(B, I, O, oc) * O * (nf + 1) * I;
}

extern "C" int kf_edge_derivative_dx(const float* x, const float* g, const float* coefT, const float* base_eff,
                                     const float* grid, const float* basis_num, const float* basis_den, float* dx,
                                     int64_t B, int32_t I, int32_t O, int32_t nf, int32_t order,
                                     const kf_basis_desc* basis, const float* silu_poly, int32_t n_poly, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(g != nullptr, "kf_edge_derivative_dx: null gradient");
  EdgeArgs A;
  if (int rc = fill_edge_args(A, x, coefT, base_eff, grid, basis_num, basis_den, dx, B, I, O, nf, order, basis, silu_poly,
                              n_poly, true))
    return rc;
  if (B == 0) return KF_OK;
  A.g = g;
  const int64_t n = B * (int64_t)I;
  edge_dx_kernel<<<(unsigned)cdiv(n, (int64_t)256), 256, 0, (cudaStream_t)stream>>>(A);
  return check_launch("kf_edge_derivative_dx");
}

extern "C" int kf_edge_derivative_dcoef(const float* x, const float* g, const float* grid, const float* basis_num,
                                        const float* basis_den, float* dcoefT, float* dbase, float* workspace, int64_t B,
                                        int32_t I, int32_t O, int32_t nf, int32_t order, const kf_basis_desc* basis,
                                        const float* silu_poly, int32_t n_poly, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(g && dcoefT, "kf_edge_derivative_dcoef: null tensor pointer");
  KF_CHECK_ARG(dbase == nullptr || (silu_poly != nullptr && n_poly >= 1 && n_poly <= 8),
               "kf_edge_derivative_dcoef: the base gradient needs 1..8 SiLU polynomial coefficients");
  EdgeArgs A;
  if (int rc = fill_edge_args(A, x, nullptr, nullptr, grid, basis_num, basis_den, dcoefT, B, I, O, nf, order, basis,
                              nullptr, 0, false))
    return rc;
  A.g = g;
  A.n_poly = dbase ? n_poly : 0;
  for (int e = 0; e < 2 * A.n_poly; ++e) A.poly[e] = silu_poly[e];
  cudaStream_t s = (cudaStream_t)stream;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dcoefT, 0, sizeof(float) * (size_t)O * nf * I, s));
    if (dbase) KF_CUDA_RET(cudaMemsetAsync(dbase, 0, sizeof(float) * (size_t)O * I, s));
    return KF_OK;
  }
  KF_CHECK_ARG(workspace != nullptr, "kf_edge_derivative_dcoef: null workspace (kf_edge_derivative_workspace floats)");
  const int oc = edge_oc(nf);
  const int splits = edge_splits(B, I, O, oc);
  const int64_t rows = cdiv(B, (int64_t)splits);
  const dim3 grid3((unsigned)cdiv((int64_t)I, (int64_t)32), (unsigned)cdiv((int64_t)O, (int64_t)oc), (unsigned)splits);
  if (nf + 1 <= 10) edge_dcoef_kernel<10, 8><<<grid3, 256, 0, s>>>(A, workspace, rows);
  else if (nf + 1 <= 17) edge_dcoef_kernel<17, 4><<<grid3, 256, 0, s>>>(A, workspace, rows);
  else edge_dcoef_kernel<KF_NF_MAX + 1, 2><<<grid3, 256, 0, s>>>(A, workspace, rows);
  if (int rc = check_launch("kf_edge_derivative_dcoef")) return rc;
  const int64_t n = (int64_t)O * (nf + 1) * I;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, (int64_t)256), 148 * 8));
  edge_dcoef_reduce_kernel<<<blocks, 256, 0, s>>>(workspace, dcoefT, dbase, splits, O, nf, I);
  return check_launch("kf_edge_derivative_dcoef");
}
