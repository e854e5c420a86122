// Sparse B-spline KANLinear, float32 on the CUDA cores (kanforge/bases/base.py:15-16
// `local` / `support`: a B-spline of order k has at most k+1 non-zero functions at
// any input, so a layer needs k+1 coefficients per (token, input), not G+k).
//
//   kf_sparse_fwd    y[b,o] = sum_i sum_q B_q(x_bi) ce[o,i,j_bi+q] + sum_i we[o,i] silu(x_bi) + bias[o]
//   kf_sparse_dgrad  dx[b,i] = sum_o dy[b,o] (sum_q B'_q(x_bi) ce[o,i,j_bi+q] + we[o,i] silu'(x_bi))
//   kf_sparse_wgrad  dcoef[o,i,j] = sum_b dy[b,o] B_j(x_bi) s m,  dbase[o,i] = sum_b dy[b,o] silu(x_bi) m,
//                    dscale[o,i] = sum_j coef[o,i,j] sum_b dy[b,o] B_j(x_bi) m,  dbias[o] = sum_b dy[b,o]
//
// with ce = coef * edge_scale * edge_mask and we = base * edge_mask (s, m: the scale and
// mask of the edge).  j_bi = the knot interval of x_bi minus k.  Each CTA evaluates the
// k+1 non-zero splines of its (token, input) pairs once into shared memory and gathers
// the matching coefficient rows from a shared-memory slab of its inputs x outputs, so
// the work is (k+2) FMAs per (token, input, output) instead of the dense G+k+1.  This
// is the path for narrow layers (few outputs), where a tensor-core tile would be
// mostly idle; wide layers use the dense tensor-core contractions.  Reductions over
// tokens run in a fixed order (per-split partial sums, then an ordered sum).

#include "basis.cuh"
#include "common.cuh"

namespace kf {
namespace {

constexpr int kSpThreads = 256;
constexpr int kSpRows = 64;  // tokens per CTA tile

struct SparseArgs {
  const float* x;      // (B, I)
  const float* coef;   // (O, I, S)
  const float* scale;  // (O, I) or null
  const float* mask;   // (O, I) or null
  const float* base;   // (O, I) or null
  const float* bias;   // (O) or null
  const float* grid;   // (I, G+1)
  const float* dy;     // (B, O) (backward)
  float* out;          // y (B, O) / dx (B, I)
  int64_t B;
  int I, O, G, S, nk;  // S = G + k basis functions, nk = G + 2k + 1 knots
  int ic;              // inputs per shared-memory slab
  int ts;              // row stride of the knot tables (nk rounded up to odd)
};

// Shared memory of one CTA, for an output tile of TO (TOP = TO + 1 floats per
// row, so that rows of a slab start on different banks).
struct SpSmem {
  float* tab;    // [ic][(k+1) * ts]  knots, then 1 / (t_{r+q} - t_r) for q = 1..k
  float* coefT;  // [ic][S][TOP]      effective coefficients, outputs fastest
  float* baseT;  // [ic][TOP]
  float* val;    // [kSpRows][ic][k+2] spline values (or derivatives), silu (or silu') last
  int* idx;      // [kSpRows][ic]      first basis index of the window, clamped into [0, S-k-1]
  float* extra;  // kernel-specific
};

__host__ __device__ inline size_t sp_smem_floats(int ic, int S, int ts, int k, int top) {
  return (size_t)ic * (k + 1) * ts + (size_t)ic * S * top + (size_t)ic * top + (size_t)kSpRows * ic * (k + 2) +
         (size_t)kSpRows * ic;
}

__device__ __forceinline__ SpSmem sp_carve(float* smem, const SparseArgs& a, int k, int top) {
  SpSmem s;
  s.tab = smem;
  s.coefT = s.tab + a.ic * (k + 1) * a.ts;
  s.baseT = s.coefT + a.ic * a.S * top;
  s.val = s.baseT + a.ic * top;
  s.idx = reinterpret_cast<int*>(s.val + kSpRows * a.ic * (k + 2));
  s.extra = reinterpret_cast<float*>(s.idx + kSpRows * a.ic);
  return s;
}

// Knot tables of inputs i0.. (two passes: knots, then reciprocal differences).
template <int K>
__device__ void sp_stage_tables(const SparseArgs& a, const SpSmem& s, int i0) {
  const int ni = min(a.ic, a.I - i0);
  for (int e = threadIdx.x; e < ni * a.ts; e += blockDim.x) {
    const int il = e / a.ts, r = e % a.ts;
    s.tab[il * (K + 1) * a.ts + r] = r < a.nk ? extended_knot(a.grid + (int64_t)(i0 + il) * (a.G + 1), a.G, K, r) : 0.0f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ni * K * a.ts; e += blockDim.x) {
    const int il = e / (K * a.ts), rem = e % (K * a.ts), q = rem / a.ts + 1, r = rem % a.ts;
    const float* t = s.tab + il * (K + 1) * a.ts;
    s.tab[il * (K + 1) * a.ts + q * a.ts + r] = r <= a.nk - 1 - q ? 1.0f / (t[r + q] - t[r]) : 0.0f;
  }
}

// Effective coefficients and base weights of inputs i0.. and outputs o0..o0+TO-1
// (rows past O are zero).  A coefficient row of one output is contiguous over
// (input, j), so reads run along it.
template <int TO>
__device__ void sp_stage_coef(const SparseArgs& a, const SpSmem& s, int i0, int o0) {
  constexpr int TOP = TO + 1;
  const int ni = min(a.ic, a.I - i0);
  const int row = ni * a.S;
  for (int e = threadIdx.x; e < TO * row; e += blockDim.x) {
    const int ol = e / row, rem = e % row, il = rem / a.S, j = rem % a.S;
    const int o = o0 + ol;
    float v = 0.0f;
    if (o < a.O) {
      const int64_t oi = (int64_t)o * a.I + i0 + il;
      v = a.coef[oi * a.S + j];
      if (a.scale) v *= a.scale[oi];
      if (a.mask) v *= a.mask[oi];
    }
    s.coefT[(il * a.S + j) * TOP + ol] = v;
  }
  for (int e = threadIdx.x; e < TO * ni; e += blockDim.x) {
    const int ol = e / ni, il = e % ni, o = o0 + ol;
    float v = 0.0f;
    if (o < a.O && a.base) {
      const int64_t oi = (int64_t)o * a.I + i0 + il;
      v = a.base[oi];
      if (a.mask) v *= a.mask[oi];
    }
    s.baseT[il * TOP + ol] = v;
  }
}

// Spline values (m = 0) or first derivatives (m = 1) of the (token, input) pairs
// of the tile, and silu or silu' in the last slot.
template <int K>
__device__ void sp_stage_basis(const SparseArgs& a, const SpSmem& s, int64_t b0, int i0, int m) {
  const int ni = min(a.ic, a.I - i0);
  for (int e = threadIdx.x; e < kSpRows * a.ic; e += blockDim.x) {
    const int r = e / a.ic, il = e % a.ic;
    const int64_t b = b0 + r;
    float* v = s.val + (r * a.ic + il) * (K + 2);
    float vals[K + 1];
#pragma unroll
    for (int q = 0; q <= K; ++q) vals[q] = 0.0f;
    int first = 0;
    float act = 0.0f;
    if (b < a.B && il < ni) {
      const float xv = a.x[b * a.I + i0 + il];
      const float* tab = s.tab + il * (K + 1) * a.ts;
      const int j = knot_interval(xv, tab, a.nk);
      if (j >= 0) {
        bspline_local_tab<K>(xv, tab, a.nk, j, m, vals, a.ts);
        first = j - K;
      }
      act = m == 0 ? silu_acc(xv) : dsilu_acc(xv);
    }
    // indices outside [0, S) carry value 0: shift the window into range
    if (first < 0) {
#pragma unroll
      for (int q = 0; q <= K; ++q) vals[q] = q - first <= K ? vals[q - first] : 0.0f;
      first = 0;
    } else if (first > a.S - 1 - K) {
      const int sh = first - (a.S - 1 - K);
#pragma unroll
      for (int q = K; q >= 0; --q) vals[q] = q - sh >= 0 ? vals[q - sh] : 0.0f;
      first = a.S - 1 - K;
    }
#pragma unroll
    for (int q = 0; q <= K; ++q) v[q] = vals[q];
    v[K + 1] = act;
    s.idx[r * a.ic + il] = first;
  }
}

// Forward: CTA = 64 tokens x TO outputs; each thread owns 64 * TO / 256 of the
// (token, output) pairs (consecutive lanes: consecutive outputs).
template <int K, int TO>
__global__ void __launch_bounds__(kSpThreads) sparse_fwd_kernel(SparseArgs a) {
  constexpr int TOP = TO + 1, PPT = kSpRows * TO / kSpThreads;
  extern __shared__ float smem[];
  const SpSmem s = sp_carve(smem, a, K, TOP);
  const int64_t b0 = (int64_t)blockIdx.x * kSpRows;
  const int o0 = blockIdx.y * TO;
  float acc[PPT];
#pragma unroll
  for (int p = 0; p < PPT; ++p) acc[p] = 0.0f;
  for (int i0 = 0; i0 < a.I; i0 += a.ic) {
    const int ni = min(a.ic, a.I - i0);
    sp_stage_tables<K>(a, s, i0);
    sp_stage_coef<TO>(a, s, i0, o0);
    __syncthreads();
    sp_stage_basis<K>(a, s, b0, i0, 0);
    __syncthreads();
#pragma unroll
    for (int p = 0; p < PPT; ++p) {
      const int e = threadIdx.x + p * kSpThreads;
      const int r = e / TO, ol = e % TO;
      float t = 0.0f;
      for (int il = 0; il < ni; ++il) {
        const float* v = s.val + (r * a.ic + il) * (K + 2);
        const float* c = s.coefT + (il * a.S + s.idx[r * a.ic + il]) * TOP + ol;
        t = fmaf(v[K + 1], s.baseT[il * TOP + ol], t);
#pragma unroll
        for (int q = 0; q <= K; ++q) t = fmaf(v[q], c[q * TOP], t);
      }
      acc[p] += t;
    }
    __syncthreads();
  }
#pragma unroll
  for (int p = 0; p < PPT; ++p) {
    const int e = threadIdx.x + p * kSpThreads;
    const int64_t b = b0 + e / TO;
    const int o = o0 + e % TO;
    if (b < a.B && o < a.O) a.out[b * a.O + o] = acc[p] + (a.bias ? a.bias[o] : 0.0f);
  }
}

// dx: CTA tile = 64 tokens x ic inputs, looping over TO-output slabs; every
// thread owns (token, input) pairs and sums over the outputs of each slab.
template <int K, int TO>
__global__ void __launch_bounds__(kSpThreads) sparse_dgrad_kernel(SparseArgs a) {
  constexpr int TOP = TO + 1;
  extern __shared__ float smem[];
  const SpSmem s = sp_carve(smem, a, K, TOP);
  float* gy = s.extra;  // [kSpRows][TOP]
  const int64_t b0 = (int64_t)blockIdx.x * kSpRows;
  const int i0 = blockIdx.y * a.ic;
  const int ni = min(a.ic, a.I - i0);
  constexpr int kMaxPairs = 2;  // pairs per thread: kSpRows * ic <= 2 * kSpThreads
  float acc[kMaxPairs];
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) acc[p] = 0.0f;
  sp_stage_tables<K>(a, s, i0);
  __syncthreads();
  sp_stage_basis<K>(a, s, b0, i0, 1);  // derivatives of the splines and silu'
  for (int o0 = 0; o0 < a.O; o0 += TO) {
    sp_stage_coef<TO>(a, s, i0, o0);
    for (int e = threadIdx.x; e < kSpRows * TO; e += blockDim.x) {
      const int r = e / TO, ol = e % TO;
      const int64_t b = b0 + r;
      gy[r * TOP + ol] = (b < a.B && o0 + ol < a.O) ? a.dy[b * a.O + o0 + ol] : 0.0f;
    }
    __syncthreads();
    const int n_o = min(TO, a.O - o0);
#pragma unroll
    for (int p = 0; p < kMaxPairs; ++p) {
      const int e = threadIdx.x + p * kSpThreads;
      if (e >= kSpRows * a.ic) break;
      const int r = e / a.ic, il = e % a.ic;
      if (il >= ni) continue;
      const float* v = s.val + (r * a.ic + il) * (K + 2);
      const float* c = s.coefT + (il * a.S + s.idx[r * a.ic + il]) * TOP;
      const float* g = gy + r * TOP;
      const float* w = s.baseT + il * TOP;
      float vq[K + 1];
#pragma unroll
      for (int q = 0; q <= K; ++q) vq[q] = v[q];
      float sc = 0.0f, sb = 0.0f;
      for (int ol = 0; ol < n_o; ++ol) {
        float t = 0.0f;
#pragma unroll
        for (int q = 0; q <= K; ++q) t = fmaf(vq[q], c[q * TOP + ol], t);
        sc = fmaf(g[ol], t, sc);
        sb = fmaf(g[ol], w[ol], sb);
      }
      acc[p] += fmaf(sb, v[K + 1], sc);
    }
    __syncthreads();
  }
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) {
    const int e = threadIdx.x + p * kSpThreads;
    if (e >= kSpRows * a.ic) break;
    const int r = e / a.ic, il = e % a.ic;
    const int64_t b = b0 + r;
    if (b < a.B && il < ni) a.out[b * a.I + i0 + il] = acc[p];
  }
}

// Coefficient gradients, first pass: CTA = (ic inputs, TO outputs, token split);
// each thread owns (input, output) pairs and accumulates the S spline columns and
// the silu column of its pairs in private shared-memory columns, tokens in order.
// part (splits, O, I, S+1) and, from the CTAs of input tile 0, pbias (splits, O).
template <int K, int TO>
__global__ void __launch_bounds__(kSpThreads) sparse_wgrad_kernel(SparseArgs a, int64_t rows_per_split, float* part,
                                                                  float* pbias) {
  constexpr int TOP = TO + 1;
  extern __shared__ float smem[];
  const SpSmem s = sp_carve(smem, a, K, TOP);
  const int n_pairs = a.ic * TO;
  float* acc = s.extra;                    // [S+1][n_pairs]
  float* gy = acc + (a.S + 1) * n_pairs;   // [kSpRows][TOP]
  const int i0 = blockIdx.x * a.ic, o0 = blockIdx.y * TO, split = blockIdx.z;
  const int ni = min(a.ic, a.I - i0);
  for (int e = threadIdx.x; e < (a.S + 1) * n_pairs; e += blockDim.x) acc[e] = 0.0f;
  sp_stage_tables<K>(a, s, i0);
  float bias_acc = 0.0f;  // threads < TO of input tile 0: sum of dy over tokens for output o0 + tid
  const int64_t t_begin = (int64_t)split * rows_per_split;
  const int64_t t_end = min(a.B, t_begin + rows_per_split);
  for (int64_t b0 = t_begin; b0 < t_end; b0 += kSpRows) {
    __syncthreads();
    sp_stage_basis<K>(a, s, b0, i0, 0);
    for (int e = threadIdx.x; e < kSpRows * TO; e += blockDim.x) {
      const int r = e / TO, ol = e % TO;
      const int64_t b = b0 + r;
      gy[r * TOP + ol] = (b < t_end && o0 + ol < a.O) ? a.dy[b * a.O + o0 + ol] : 0.0f;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x) {
      const int il = p / TO, ol = p % TO;
      if (il >= ni) continue;
      for (int r = 0; r < kSpRows; ++r) {
        const float g = gy[r * TOP + ol];
        const float* v = s.val + (r * a.ic + il) * (K + 2);
        float* col = acc + s.idx[r * a.ic + il] * n_pairs + p;
#pragma unroll
        for (int q = 0; q <= K; ++q) col[q * n_pairs] = fmaf(g, v[q], col[q * n_pairs]);
        acc[a.S * n_pairs + p] = fmaf(g, v[K + 1], acc[a.S * n_pairs + p]);
      }
    }
    if (blockIdx.x == 0 && threadIdx.x < TO)
      for (int r = 0; r < kSpRows; ++r) bias_acc += gy[r * TOP + threadIdx.x];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < (a.S + 1) * n_pairs; e += blockDim.x) {
    const int col = e / n_pairs, p = e % n_pairs;
    const int il = p / TO, ol = p % TO, o = o0 + ol;
    if (il >= ni || o >= a.O) continue;
    part[(((int64_t)split * a.O + o) * a.I + i0 + il) * (a.S + 1) + col] = acc[e];
  }
  if (blockIdx.x == 0 && threadIdx.x < TO && o0 + threadIdx.x < a.O)
    pbias[(int64_t)split * a.O + o0 + threadIdx.x] = bias_acc;
}

// Second pass: ordered sum over the splits and the chain rule of the effective
// coefficients (one thread per edge).
__global__ void __launch_bounds__(256) sparse_wgrad_finish_kernel(SparseArgs a, int n_split, const float* part,
                                                                  const float* pbias, float* dcoef, float* dbase,
                                                                  float* dscale, float* dbias) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t edges = (int64_t)a.O * a.I;
  if (dbias && e < a.O) {
    float v = 0.0f;
    for (int s = 0; s < n_split; ++s) v += pbias[(int64_t)s * a.O + e];
    dbias[e] = v;
  }
  if (e >= edges) return;
  const float m = a.mask ? a.mask[e] : 1.0f;
  const float sm = a.scale ? a.scale[e] * m : m;
  float ds = 0.0f;
  for (int j = 0; j <= a.S; ++j) {
    float v = 0.0f;
    for (int s = 0; s < n_split; ++s) v += part[((int64_t)s * edges + e) * (a.S + 1) + j];
    if (j < a.S) {
      if (dcoef) dcoef[e * a.S + j] = v * sm;
      ds = fmaf(v, a.coef[e * a.S + j], ds);
    } else if (dbase) {
      dbase[e] = v * m;
    }
  }
  if (dscale) dscale[e] = ds * m;
}

// Output tile: the smallest of 8, 16, 32, 64 that holds min(O, 64) outputs.
int out_tile(int O) {
  int to = 8;
  while (to < 64 && to < O) to *= 2;
  return to;
}

constexpr size_t kSpSmemMax = 200 * 1024;

size_t fwd_smem(const SparseArgs& a, int k, int to) { return 4 * sp_smem_floats(a.ic, a.S, a.ts, k, to + 1); }
size_t dgrad_smem(const SparseArgs& a, int k, int to) { return fwd_smem(a, k, to) + 4 * (size_t)kSpRows * (to + 1); }
size_t wgrad_smem(const SparseArgs& a, int k, int to) {
  return fwd_smem(a, k, to) + 4 * ((size_t)(a.S + 1) * a.ic * to + (size_t)kSpRows * (to + 1));
}

int sparse_args(SparseArgs& a, const kf_basis_desc* basis, int64_t B, int32_t I, int32_t O, const char* who) {
  KF_CHECK_ARG(basis && basis->kind == KF_BASIS_BSPLINE, "%s: the sparse path is for B-spline bases", who);
  const int k = basis->order, G = basis->grid_size;
  KF_CHECK_ARG(k >= 1 && k <= 5 && G >= 1 && basis->size == G + k, "%s: B-spline order 1..5 with size G + k", who);
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1 && I <= 65535 * 8, "%s: bad shape", who);
  a.B = B;
  a.I = I;
  a.O = O;
  a.G = G;
  a.S = G + k;
  a.nk = G + 2 * k + 1;
  a.ts = a.nk | 1;
  // inputs per slab: as many as fit (at most 8, the dgrad pairs per thread allow 8)
  const int to = out_tile(O);
  a.ic = 8;
  while (a.ic > 1 && wgrad_smem(a, k, to) > kSpSmemMax) --a.ic;
  KF_CHECK_ARG(wgrad_smem(a, k, to) <= kSpSmemMax, "%s: %d basis functions do not fit the sparse kernels' shared memory",
               who, a.S);
  return KF_OK;
}

template <typename Kern, typename... Args>
int sp_launch(Kern kern, dim3 grid, size_t smem, cudaStream_t st, const char* what, Args... args) {
  if (smem > 48 * 1024) KF_CUDA_RET(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, kSpThreads, smem, st>>>(args...);
  return check_launch(what);
}

// Instantiates CALL for the spline order k and output tile to.
#define KF_SPARSE_DISPATCH(k, to, ...)                                   \
  [&]() -> int {                                                         \
    switch (to) {                                                        \
      case 8: { constexpr int TO = 8; KF_SPARSE_ORDER(k, __VA_ARGS__) }  \
      case 16: { constexpr int TO = 16; KF_SPARSE_ORDER(k, __VA_ARGS__) } \
      case 32: { constexpr int TO = 32; KF_SPARSE_ORDER(k, __VA_ARGS__) } \
      default: { constexpr int TO = 64; KF_SPARSE_ORDER(k, __VA_ARGS__) } \
    }                                                                    \
  }()
#define KF_SPARSE_ORDER(k, ...)                           \
  switch (k) {                                            \
    case 1: { constexpr int K = 1; return __VA_ARGS__; }  \
    case 2: { constexpr int K = 2; return __VA_ARGS__; }  \
    case 3: { constexpr int K = 3; return __VA_ARGS__; }  \
    case 4: { constexpr int K = 4; return __VA_ARGS__; }  \
    default: { constexpr int K = 5; return __VA_ARGS__; } \
  }

int64_t wgrad_splits(int64_t B, int I, int O, int ic, int to) {
  const int64_t tiles = cdiv(I, ic) * cdiv(O, to);
  return std::max<int64_t>(1, std::min<int64_t>(cdiv(592, tiles), cdiv(B, 4 * kSpRows)));
}

}  // namespace
}  // namespace kf

extern "C" int kf_sparse_fwd(const float* x, const float* coef, const float* edge_scale, const float* edge_mask,
                             const float* base, const float* bias, const float* grid, float* y, int64_t B, int32_t I,
                             int32_t O, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  SparseArgs a{};
  if (int rc = sparse_args(a, basis, B, I, O, "kf_sparse_fwd")) return rc;
  KF_CHECK_ARG(x && coef && grid && y, "kf_sparse_fwd: null pointer");
  if (int rc = bind_device(x)) return rc;
  if (B == 0) return KF_OK;
  a.x = x; a.coef = coef; a.scale = edge_scale; a.mask = edge_mask; a.base = base; a.bias = bias; a.grid = grid; a.out = y;
  const int to = out_tile(O), k = basis->order;
  const size_t smem = fwd_smem(a, k, to);
  const dim3 g((unsigned)cdiv(B, kSpRows), (unsigned)cdiv(O, to));
  return KF_SPARSE_DISPATCH(k, to, sp_launch(sparse_fwd_kernel<K, TO>, g, smem, (cudaStream_t)stream, "kf_sparse_fwd", a));
}

extern "C" int kf_sparse_dgrad(const float* x, const float* dy, const float* coef, const float* edge_scale,
                               const float* edge_mask, const float* base, const float* grid, float* dx, int64_t B,
                               int32_t I, int32_t O, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  SparseArgs a{};
  if (int rc = sparse_args(a, basis, B, I, O, "kf_sparse_dgrad")) return rc;
  KF_CHECK_ARG(x && dy && coef && grid && dx, "kf_sparse_dgrad: null pointer");
  if (int rc = bind_device(x)) return rc;
  if (B == 0) return KF_OK;
  a.x = x; a.dy = dy; a.coef = coef; a.scale = edge_scale; a.mask = edge_mask; a.base = base; a.grid = grid; a.out = dx;
  const int to = out_tile(O), k = basis->order;
  const size_t smem = dgrad_smem(a, k, to);
  const dim3 g((unsigned)cdiv(B, kSpRows), (unsigned)cdiv(I, a.ic));
  return KF_SPARSE_DISPATCH(k, to, sp_launch(sparse_dgrad_kernel<K, TO>, g, smem, (cudaStream_t)stream, "kf_sparse_dgrad", a));
}

extern "C" int64_t kf_sparse_wgrad_workspace(int64_t B, int32_t I, int32_t O, const kf_basis_desc* basis) {
  using namespace kf;
  SparseArgs a{};
  if (sparse_args(a, basis, B, I, O, "kf_sparse_wgrad_workspace") != KF_OK) return 0;
  const int64_t splits = wgrad_splits(B, I, O, a.ic, out_tile(O));
  return splits * ((int64_t)O * I * (a.S + 1) + O);
}

extern "C" int kf_sparse_wgrad(const float* x, const float* dy, const float* coef, const float* edge_scale,
                               const float* edge_mask, const float* grid, float* dcoef, float* dbase, float* dscale,
                               float* dbias, float* workspace, int64_t B, int32_t I, int32_t O,
                               const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  SparseArgs a{};
  if (int rc = sparse_args(a, basis, B, I, O, "kf_sparse_wgrad")) return rc;
  KF_CHECK_ARG(x && dy && coef && grid && workspace, "kf_sparse_wgrad: null pointer");
  if (int rc = bind_device(x)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  a.x = x; a.dy = dy; a.coef = coef; a.scale = edge_scale; a.mask = edge_mask; a.grid = grid;
  const int to = out_tile(O), k = basis->order;
  const int64_t splits = wgrad_splits(B, I, O, a.ic, to);
  const int64_t per = cdiv(std::max<int64_t>(B, 1), splits);
  float* part = workspace;
  float* pbias = part + splits * (int64_t)O * I * (a.S + 1);
  const size_t smem = wgrad_smem(a, k, to);
  const dim3 g((unsigned)cdiv(I, a.ic), (unsigned)cdiv(O, to), (unsigned)splits);
  int rc = KF_SPARSE_DISPATCH(k, to, sp_launch(sparse_wgrad_kernel<K, TO>, g, smem, st, "kf_sparse_wgrad", a, per, part, pbias));
  if (rc) return rc;
  const int64_t n = std::max<int64_t>((int64_t)O * I, O);
  sparse_wgrad_finish_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(a, (int)splits, part, pbias, dcoef, dbase, dscale,
                                                                      dbias);
  return check_launch("kf_sparse_wgrad (finish)");
}
