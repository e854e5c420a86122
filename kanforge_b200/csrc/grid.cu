// Grid tools on the GPU (kanforge/grid.py:19-85, kanforge/_layer.py:107-183):
//
//   kf_samples_transpose  samples (n, I) -> one float32 column per input (I, n)
//   kf_adaptive_grid      per-input grid from the sample order statistics at
//                         round(linspace(0, n-1, T)) mixed with the uniform grid
//                         over [min - margin, max + margin] (grid.py:19-31)
//   kf_resample_grid      linear interpolation of each grid row (grid.py:34-38)
//   kf_refit              coefficients in a new basis / on a new grid whose edge
//                         functions match the old ones on the samples, by least
//                         squares per input (grid.py:55-85, _layer.py:120-137)
//
// Order statistics come from a radix select (four 8-bit passes over the
// order-preserving integer keys of the samples) instead of a sort: per pass one
// histogram per input and distinct key prefix, merged across CTAs with global
// atomics, then one CTA per input walks its histograms to the next digit of
// every target rank.  The values are exact sample values, so the grid equals
// the reference's float64 result bit for bit: the final mix is evaluated with
// explicitly rounded double operations in the reference's order.
//
// The refit never forms the (samples x inputs x outputs) targets: for input i
// with new features b(x) (K') and old features a(x) (K) it accumulates in
// float64 the Gram matrix G = sum b b^T and the cross matrix M = sum b a^T over
// the samples, takes the pseudo-inverse of G by a parallel cyclic Jacobi
// eigen-decomposition, and maps every edge's old coefficients c to
// pinv(G) M c.  That is the least-squares solution of the reference
// (np.linalg.lstsq per input), with its minimum-norm choice for basis functions
// that no sample reaches.

#include "common.cuh"

#include <cmath>

namespace kf {
namespace {

constexpr int kGridThreads = 256;      // = the 256 digit values of one radix pass
constexpr int kFitThreads = 256;
constexpr int kJacobiMaxSweeps = 40;
constexpr int kFitSmall = 64;          // both sizes up to this: shared-memory Jacobi solve (exact minimum norm)
constexpr double kEigenCut = 1e-13;    // eigenvalues below kEigenCut * max are dropped

struct GridState {
  uint32_t prefix;  // key bits fixed so far
  uint32_t rank;    // rank of the target among the samples that share the prefix
};

// Order-preserving map float -> uint32; every NaN maps to the largest key
// (np.sort puts NaN last).
__device__ __forceinline__ uint32_t order_key(float v) {
  if (isnan(v)) return 0xFFFFFFFFu;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  if (k == 0xFFFFFFFFu) return __uint_as_float(0x7FC00000u);
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// np.linspace(0, 1, n)[j]: j * (1 / (n - 1)), the last point exactly 1.
__device__ __forceinline__ double unit_linspace(int64_t j, int64_t n) {
  if (n <= 1) return 0.0;
  if (j == n - 1) return 1.0;
  return __dmul_rn((double)j, __ddiv_rn(1.0, (double)(n - 1)));
}

// ---- samples (n, I) -> columns (I, n) ---------------------------------------

template <typename T>
__global__ void samples_transpose_kernel(const T* __restrict__ x, float* __restrict__ xt, int64_t n, int32_t I) {
  __shared__ float tile[32][33];
  const int64_t s0 = (int64_t)blockIdx.x * 32;
  const int i0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int64_t s = s0 + r;
    const int i = i0 + threadIdx.x;
    tile[r][threadIdx.x] = (s < n && i < I) ? to_f32(x[s * I + i]) : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int i = i0 + r;
    const int64_t s = s0 + threadIdx.x;
    if (i < I && s < n) xt[(int64_t)i * n + s] = tile[threadIdx.x][r];
  }
}

// ---- radix select ------------------------------------------------------------

// Pass `pass` (0..3) counts digit (key >> (24 - 8 pass)) & 255 of every sample
// whose higher bits equal the prefix of some target.  Targets are sorted by rank,
// so their prefixes are non-decreasing and the distinct ones form `groups`.
__global__ void __launch_bounds__(kGridThreads) grid_hist_kernel(const float* __restrict__ xt, int64_t n, int T,
                                                                  int pass, const GridState* __restrict__ state,
                                                                  uint32_t* __restrict__ ghist, int64_t per_split) {
  extern __shared__ uint32_t sh[];
  uint32_t* hist = sh;             // [T][256]
  uint32_t* group = sh + T * 256;  // [T] distinct prefixes
  __shared__ int n_groups;
  const int i = blockIdx.y;
  const GridState* st = state + (int64_t)i * T;
  if (threadIdx.x == 0) {
    int g = 0;
    if (pass == 0) {
      group[g++] = 0;
    } else {
      for (int t = 0; t < T; ++t) {
        const uint32_t p = st[t].prefix;
        if (g == 0 || group[g - 1] != p) group[g++] = p;
      }
    }
    n_groups = g;
  }
  for (int j = threadIdx.x; j < T * 256; j += blockDim.x) hist[j] = 0;
  __syncthreads();
  const int G = n_groups;
  const int shift_digit = 24 - 8 * pass;
  const int64_t s0 = (int64_t)blockIdx.x * per_split;
  const int64_t s1 = min(n, s0 + per_split);
  const float* col = xt + (int64_t)i * n;
  for (int64_t s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const uint32_t key = order_key(col[s]);
    int g = 0;
    if (pass > 0) {
      const uint32_t p = key >> (32 - 8 * pass);
      int lo = 0, hi = G - 1;
      g = -1;
      while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        const uint32_t v = group[mid];
        if (v == p) {
          g = mid;
          break;
        }
        if (v < p) lo = mid + 1;
        else hi = mid - 1;
      }
      if (g < 0) continue;
    }
    atomicAdd(&hist[g * 256 + ((key >> shift_digit) & 255u)], 1u);
  }
  __syncthreads();
  uint32_t* out = ghist + (int64_t)i * T * 256;
  for (int j = threadIdx.x; j < G * 256; j += blockDim.x)
    if (hist[j]) atomicAdd(&out[j], hist[j]);
}

// Inclusive prefix sum over the 256 threads of the block.
__device__ __forceinline__ uint32_t block_scan_256(uint32_t v, uint32_t* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t u = __shfl_up_sync(0xFFFFFFFFu, v, d);
    if (lane >= d) v += u;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  uint32_t before = 0;
  for (int w = 0; w < warp; ++w) before += warp_tot[w];
  __syncthreads();
  return v + before;
}

// One CTA per input: the digit of every target from this pass's histograms,
// which it clears for the next pass.  Pass 0 first sets the target ranks
// round(linspace(0, n-1, T)) (grid.py:24); after pass 3 every prefix is a whole
// key and the CTA writes the grid (grid.py:25-31).
__global__ void __launch_bounds__(kGridThreads) grid_resolve_kernel(int64_t n, int T, int pass,
                                                                     GridState* __restrict__ state,
                                                                     uint32_t* __restrict__ ghist, double margin,
                                                                     double grid_eps, double* __restrict__ grid) {
  extern __shared__ uint32_t sh[];
  GridState* cur = reinterpret_cast<GridState*>(sh);  // [T]
  GridState* nxt = cur + T;                           // [T]
  int* tgroup = reinterpret_cast<int*>(nxt + T);      // [T]
  __shared__ uint32_t warp_tot[kGridThreads / 32];
  const int i = blockIdx.x;
  GridState* st = state + (int64_t)i * T;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    if (pass == 0) {
      const double step = __ddiv_rn((double)(n - 1), (double)(T - 1));
      double y = (step == 0.0) ? 0.0 : __dmul_rn((double)t, step);
      if (t == T - 1) y = (double)(n - 1);
      cur[t] = GridState{0u, (uint32_t)rint(y)};
    } else {
      cur[t] = st[t];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int g = -1;
    for (int t = 0; t < T; ++t) {
      if (t == 0 || (pass > 0 && cur[t].prefix != cur[t - 1].prefix)) ++g;
      tgroup[t] = g;
    }
  }
  __syncthreads();
  uint32_t* hist = ghist + (int64_t)i * T * 256;
  const uint32_t digit = threadIdx.x;
  for (int t = 0, g = 0; t < T; ++g) {
    int t_end = t;
    while (t_end < T && tgroup[t_end] == g) ++t_end;
    const uint32_t c = hist[g * 256 + digit];
    hist[g * 256 + digit] = 0u;
    const uint32_t inc = block_scan_256(c, warp_tot);
    const uint32_t exc = inc - c;
    for (int u = t; u < t_end; ++u) {
      const uint32_t r = cur[u].rank;
      if (r >= exc && r < inc) nxt[u] = GridState{(cur[u].prefix << 8) | digit, r - exc};
    }
    t = t_end;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) st[t] = nxt[t];
  if (pass != 3) return;
  // grid = eps * uniform + (1 - eps) * quantiles, in the reference's operation order
  double lo = __dsub_rn((double)key_value(nxt[0].prefix), margin);
  double hi = __dadd_rn((double)key_value(nxt[T - 1].prefix), margin);
  const bool flat = __dsub_rn(hi, lo) < 1e-8;
  if (flat) {
    lo = __dsub_rn(lo, 0.5);
    hi = __dadd_rn(hi, 0.5);
  }
  const double keep = __dsub_rn(1.0, grid_eps);
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const double u = __dadd_rn(lo, __dmul_rn(__dsub_rn(hi, lo), unit_linspace(t, T)));
    const double q = flat ? u : (double)key_value(nxt[t].prefix);
    grid[(int64_t)i * T + t] = __dadd_rn(__dmul_rn(grid_eps, u), __dmul_rn(keep, q));
  }
}

// ---- resampling ------------------------------------------------------------

// out[i, j] = np.interp(linspace(0,1,n_new)[j], linspace(0,1,n_old), grid[i])
// with NumPy's arithmetic: slope (y1 - y0) / (x1 - x0), then slope (x - x0) + y0.
__global__ void resample_grid_kernel(const double* __restrict__ grid, int32_t I, int32_t n_old, int32_t n_new,
                                     double* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)I * n_new) return;
  const int i = (int)(idx / n_new), j = (int)(idx % n_new);
  const double* y = grid + (int64_t)i * n_old;
  const double x = unit_linspace(j, n_new);
  double res;
  if (n_old == 1 || x >= 1.0) {
    res = y[n_old - 1];
  } else {
    int k = 0;  // largest k with xp[k] <= x
    int lo = 0, hi = n_old - 1;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      if (unit_linspace(mid, n_old) <= x) {
        k = mid;
        lo = mid + 1;
      } else {
        hi = mid - 1;
      }
    }
    const double x0 = unit_linspace(k, n_old), x1 = unit_linspace(k + 1, n_old);
    if (x0 == x) {
      res = y[k];
    } else {
      const double slope = __ddiv_rn(__dsub_rn(y[k + 1], y[k]), __dsub_rn(x1, x0));
      res = __dadd_rn(__dmul_rn(slope, __dsub_rn(x, x0)), y[k]);
    }
  }
  out[idx] = res;
}

// ---- refit: float64 basis functions of one sample ---------------------------

// Per-input tables of a basis in shared memory: B-splines the extended knots
// (kanforge/bases/spline.py:22-30) t[0..nt) followed by, for q = 1..k, the
// reciprocals 1 / (t[j+q] - t[j]) (j < nt - q) in rows of nt; bumps the centres.
__host__ __device__ inline int fit_table_len(const kf_fit_basis& b) {
  if (b.kind == KF_BASIS_BSPLINE) return (b.n_grid + 2 * b.order) * (b.order + 1);
  if (b.kind == KF_BASIS_BUMP) return b.n_grid;
  return 0;
}

__device__ void stage_table(const kf_fit_basis& b, int i, double* out) {
  if (b.kind != KF_BASIS_BSPLINE && b.kind != KF_BASIS_BUMP) return;
  const double* g = b.grid + (int64_t)i * b.n_grid;
  if (b.kind == KF_BASIS_BUMP) {
    for (int j = threadIdx.x; j < b.n_grid; j += blockDim.x) out[j] = g[j];
    return;
  }
  const int k = b.order, ng = b.n_grid, nt = ng + 2 * k;
  const double g0 = g[0], gl = g[ng - 1];
  const double h = __ddiv_rn(__dsub_rn(gl, g0), (double)(ng - 1));
  for (int j = threadIdx.x; j < nt; j += blockDim.x) {
    double t;
    if (j < k) t = __dsub_rn(g0, __dmul_rn(h, (double)(k - j)));
    else if (j < k + ng) t = g[j - k];
    else t = __dadd_rn(gl, __dmul_rn(h, (double)(j - k - ng + 1)));
    out[j] = t;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < k * nt; e += blockDim.x) {
    const int q = e / nt + 1, j = e % nt;
    out[q * nt + j] = j + q < nt ? 1.0 / (out[j + q] - out[j]) : 0.0;
  }
}

// B-splines of order k at x: Cox-de Boor on the half-open knot interval that
// holds x, evaluating only its k+1 non-zero functions (the products and sums of
// the full recursion of kanforge/bases/spline.py:74-85, with the knot-difference
// divisions as products with the staged reciprocals).
__device__ void fit_bspline(const double* tab, int nt, int k, int size, double x, double* out) {
  const double* t = tab;
  for (int j = 0; j < size; ++j) out[j] = 0.0;
  if (!(x >= t[0] && x < t[nt - 1])) return;
  int lo = 0, hi = nt - 2, m = 0;  // largest m with t[m] <= x
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (t[mid] <= x) {
      m = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  double nv[6] = {1.0, 0.0, 0.0, 0.0, 0.0, 0.0};  // nv[r] = B_{m-q+r, q}
  for (int q = 1; q <= k; ++q) {
    const double* rq = tab + q * nt;        // 1 / (t[j+q] - t[j])
    const double* rq1 = tab + q * nt + 1;   // 1 / (t[j+q+1] - t[j+1])
    double nw[6];
    for (int r = 0; r <= q; ++r) {
      const int j = m - q + r;
      if (j < 0 || j > nt - 2 - q) {  // no such function at degree q
        nw[r] = 0.0;
        continue;
      }
      double v = 0.0;
      if (r >= 1) v = (x - t[j]) * rq[j] * nv[r - 1];                 // left term, from B_{j, q-1}
      if (r <= q - 1) v = fma((t[j + q + 1] - x) * rq1[j], nv[r], v);  // right term, from B_{j+1, q-1}
      nw[r] = v;
    }
    for (int r = 0; r <= q; ++r) nv[r] = nw[r];
  }
  for (int r = 0; r <= k; ++r) {
    const int j = m - k + r;
    if (j >= 0 && j < size) out[j] = nv[r];
  }
}

__device__ __forceinline__ double fit_polyval(const double* c, int n, double x) {
  double y = c[n - 1];
  for (int j = n - 2; j >= 0; --j) y = fma(y, x, c[j]);
  return y;
}

// Order-0 basis functions of input sample x (kanforge/bases/*.py _eval, m = 0);
// MAXT bounds the Chebyshev features held per thread.
template <int MAXT>
__device__ void fit_eval(const kf_fit_basis& b, const double* tab, double x, double* out) {
  switch (b.kind) {
    case KF_BASIS_BSPLINE:
      fit_bspline(tab, b.n_grid + 2 * b.order, b.order, b.size, x, out);
      return;
    case KF_BASIS_CHEB: {
      // T_j(g(x)) by the three-term recurrence into out[], then phi_k = sum_j fold[k, j] T_j
      const double u = b.input_map == KF_MAP_TANH ? tanh(x) : x;
      const int nt = b.degree + 1;
      double tv[MAXT];
      tv[0] = 1.0;
      if (nt > 1) tv[1] = u;
      for (int j = 2; j < nt; ++j) tv[j] = fma(2.0 * u, tv[j - 1], -tv[j - 2]);
      for (int k = 0; k < b.size; ++k) {
        const double* f = b.fold + (int64_t)k * nt;
        double acc = 0.0;
        for (int j = 0; j < nt; ++j) acc = fma(f[j], tv[j], acc);
        out[k] = acc;
      }
      return;
    }
    case KF_BASIS_FOURIER: {
      const int nfreq = b.degree;
      for (int j = 0; j < nfreq; ++j) {
        double sn, cs;
        sincos(x * (b.freq * (double)(j + 1)), &sn, &cs);
        out[j] = cs;
        out[nfreq + j] = sn;
      }
      return;
    }
    case KF_BASIS_BUMP: {
      const int n = b.n_grid;
      const double span = tab[n - 1] - tab[0];
      if (b.bump_mode == KF_BUMP_GAUSS) {
        const double kk = b.u_scale * (double)(n - 1) / span;
        for (int j = 0; j < n; ++j) {
          const double u = (x - tab[j]) * kk;
          out[j] = b.norm * fit_polyval(b.poly, b.n_poly, u) * exp(-0.5 * u * u);
        }
      } else {
        const double inv_h = (double)(n - 1) / span;
        for (int j = 0; j < n; ++j) out[j] = fit_polyval(b.poly, b.n_poly, tanh((x - tab[j]) * inv_h));
      }
      return;
    }
    default:
      for (int j = 0; j < b.size; ++j) out[j] = 0.0;
  }
}

// ---- refit: Gram and cross matrices -----------------------------------------

constexpr int kFitTileGroup = 2 * kFitThreads;  // 4x4 result tiles per CTA when they are many (two per thread)

struct FitShape {
  int kn, ko, kt, ld;      // new size, old size, kn + ko, feature row stride (multiple of 4)
  int tab_new, tab_old;    // table lengths (doubles) of the two bases
  int n_tiles, n_groups;   // 4x4 result tiles; sample groups (threads per tile)
  int chunk;               // samples per feature tile (128, or 32 for wide feature rows)
  int tile_groups;         // CTAs that share one (split, input)'s result tiles
  bool small;              // both sizes <= kFitSmall
};

__host__ inline FitShape fit_shape(const kf_fit_basis& nb, const kf_fit_basis& ob) {
  FitShape s;
  s.kn = nb.size;
  s.ko = ob.size;
  s.kt = s.kn + s.ko;
  s.ld = (s.kt + 3) & ~3;
  s.tab_new = fit_table_len(nb);
  s.tab_old = fit_table_len(ob);
  s.n_tiles = ((s.kn + 3) / 4) * (s.ld / 4);
  s.n_groups = std::max(1, kFitThreads / s.n_tiles);
  s.chunk = s.ld <= 128 ? 128 : 32;
  s.tile_groups = s.n_tiles <= kFitThreads ? 1 : (s.n_tiles + kFitTileGroup - 1) / kFitTileGroup;
  s.small = s.kn <= kFitSmall && s.ko <= kFitSmall;
  return s;
}

__host__ inline size_t fit_gram_smem(const FitShape& s) {
  const size_t red = s.n_tiles <= kFitThreads ? (size_t)s.n_groups * s.n_tiles * 16 : 0;
  return sizeof(double) * ((size_t)s.chunk * s.ld + s.tab_new + s.tab_old + red);
}

// One CTA per (sample split, input, tile group): part[i, split] = sum over its
// samples of b (b, a)^T, b the new and a the old basis functions, float64.  Each
// feature tile of CHUNK samples is evaluated by 2 CHUNK threads (one sample and
// basis each); the (kn x kt) result is cut into 4x4 register tiles.  With at
// most 256 tiles each is owned by n_groups threads that take every n_groups-th
// sample, reduced in a fixed order at the end; with more, each thread owns two
// tiles of its CTA's tile group and all samples.
template <int CHUNK, int MAXT>
__global__ void __launch_bounds__(kFitThreads) refit_gram_kernel(const float* __restrict__ xt,
                                                                  const double* __restrict__ ranges, int64_t n,
                                                                  kf_fit_basis nb, kf_fit_basis ob, FitShape fs,
                                                                  int n_split, int64_t per_split,
                                                                  double* __restrict__ part) {
  extern __shared__ double fsm[];
  double* feat = fsm;                        // [CHUNK][ld]
  double* tab_new = feat + CHUNK * fs.ld;    // [tab_new]
  double* tab_old = tab_new + fs.tab_new;    // [tab_old]
  double* red = tab_old + fs.tab_old;        // [n_groups][n_tiles][16]
  const int i = blockIdx.y, split = blockIdx.x, tid = threadIdx.x;
  stage_table(nb, i, tab_new);
  stage_table(ob, i, tab_old);
  for (int j = tid; j < CHUNK * fs.ld; j += blockDim.x) feat[j] = 0.0;
  const bool wide = fs.n_tiles > kFitThreads;
  const int tile0 = blockIdx.z * kFitTileGroup;
  const int tq = fs.ld / 4;
  const int grp = wide ? 0 : tid / fs.n_tiles;
  const int my_tile = wide ? tile0 + tid : tid % fs.n_tiles;
  const bool active = wide || grp < fs.n_groups;
  const int step = wide ? 1 : fs.n_groups;
  double acc[2][4][4];
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[u][r][c] = 0.0;
  double lo = 0.0, span = 0.0;
  if (!xt) {
    lo = ranges[2 * i];
    span = __dsub_rn(ranges[2 * i + 1], lo);
  }
  const int64_t s_begin = (int64_t)split * per_split;
  const int64_t s_end = min(n, s_begin + per_split);
  __syncthreads();
  for (int64_t c0 = s_begin; c0 < s_end; c0 += CHUNK) {
    if (tid < 2 * CHUNK) {
      const int row = tid % CHUNK;
      const bool is_new = tid < CHUNK;
      const int64_t s = c0 + row;
      double* dst = feat + row * fs.ld + (is_new ? 0 : fs.kn);
      if (s < s_end) {
        const double x = xt ? (double)xt[(int64_t)i * n + s] : __dadd_rn(lo, __dmul_rn(unit_linspace(s, n), span));
        if (is_new) fit_eval<MAXT>(nb, tab_new, x, dst);
        else fit_eval<MAXT>(ob, tab_old, x, dst);
      } else {
        const int size = is_new ? fs.kn : fs.ko;
        for (int j = 0; j < size; ++j) dst[j] = 0.0;
      }
    }
    __syncthreads();
    if (active) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int tile = my_tile + u * kFitThreads;
        if ((u == 1 && !wide) || tile >= fs.n_tiles || (wide && tile >= tile0 + kFitTileGroup)) continue;
        const int p0 = (tile / tq) * 4, q0 = (tile % tq) * 4;
        for (int c = grp; c < CHUNK; c += step) {
          const double* row = feat + c * fs.ld;
          const double2 a01 = *reinterpret_cast<const double2*>(row + p0);
          const double2 a23 = *reinterpret_cast<const double2*>(row + p0 + 2);
          const double2 b01 = *reinterpret_cast<const double2*>(row + q0);
          const double2 b23 = *reinterpret_cast<const double2*>(row + q0 + 2);
          const double av[4] = {a01.x, a01.y, a23.x, a23.y};
          const double bv[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
          for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) acc[u][r][cc] = fma(av[r], bv[cc], acc[u][r][cc]);
        }
      }
    }
    __syncthreads();
  }
  double* out = part + ((int64_t)i * n_split + split) * fs.kn * fs.kt;
  if (wide) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int tile = my_tile + u * kFitThreads;
      if (tile >= fs.n_tiles || tile >= tile0 + kFitTileGroup) continue;
      const int p0 = (tile / tq) * 4, q0 = (tile % tq) * 4;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (p0 + r < fs.kn && q0 + c < fs.kt) out[(p0 + r) * fs.kt + q0 + c] = acc[u][r][c];
    }
    return;
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) red[((int64_t)grp * fs.n_tiles + my_tile) * 16 + r * 4 + c] = acc[0][r][c];
  }
  __syncthreads();
  for (int e = tid; e < fs.n_tiles * 16; e += blockDim.x) {  // sample groups summed in order
    const int tile = e / 16, r = (e % 16) / 4, c = e % 4;
    double v = 0.0;
    for (int g = 0; g < fs.n_groups; ++g) v += red[((int64_t)g * fs.n_tiles + tile) * 16 + r * 4 + c];
    const int p = (tile / tq) * 4 + r, q = (tile % tq) * 4 + c;
    if (p < fs.kn && q < fs.kt) out[p * fs.kt + q] = v;
  }
}

// ---- refit: pseudo-inverse and the coefficient map ---------------------------

// Round-robin pairing of indices 0..ne-1 (ne even) in round r: slot 0 stays,
// the others rotate; over ne-1 rounds every pair meets once.
__device__ __forceinline__ void jacobi_pair(int k, int r, int ne, int& p, int& q) {
  auto at = [&](int pos) { return pos == 0 ? 0 : ((pos - 1 + r) % (ne - 1)) + 1; };
  const int a = at(k), b = at(ne - 1 - k);
  p = min(a, b);
  q = max(a, b);
}

// One CTA per input: G = sum of the split partials (+ ridge), its eigen-
// decomposition V diag(l) V^T by parallel cyclic Jacobi, and
// X = V diag(1/l) V^T M (dropped eigenvalues contribute 0), written to xmap.
__global__ void __launch_bounds__(kFitThreads) refit_solve_kernel(const double* __restrict__ part, int n_split,
                                                                   int64_t n, FitShape fs, double ridge,
                                                                   double* __restrict__ xmap) {
  extern __shared__ double ssm[];
  const int kn = fs.kn, ko = fs.ko, kt = fs.kt, la = kn + 1;
  double* A = ssm;             // [kn][la]
  double* V = A + kn * la;     // [kn][la]
  double* M = V + kn * la;     // [kn][ko]
  double* W = M + kn * ko;     // [kn][ko]
  __shared__ double rot_c[kFitSmall / 2], rot_s[kFitSmall / 2], red[kFitThreads / 32];
  __shared__ int stop;
  const int i = blockIdx.x, tid = threadIdx.x;
  const double* src = part + (int64_t)i * n_split * kn * kt;
  for (int e = tid; e < kn * kt; e += blockDim.x) {
    double v = 0.0;
    for (int s = 0; s < n_split; ++s) v += src[(int64_t)s * kn * kt + e];
    const int p = e / kt, q = e % kt;
    if (q < kn) A[p * la + q] = v;
    else M[p * ko + (q - kn)] = v;
  }
  for (int e = tid; e < kn * kn; e += blockDim.x) V[(e / kn) * la + e % kn] = (e / kn == e % kn) ? 1.0 : 0.0;
  __syncthreads();
  if (ridge > 0.0 && tid == 0) {
    double tr = 0.0;
    for (int p = 0; p < kn; ++p) tr += A[p * la + p];
    const double lam = sqrt(ridge * (tr / ((double)n * kn)) * (double)n);
    for (int p = 0; p < kn; ++p) A[p * la + p] += lam * lam;
  }
  __syncthreads();
  const int ne = kn + (kn & 1);
  const int lane = tid & 31, warp = tid >> 5;
  for (int sweep = 0; sweep < kJacobiMaxSweeps; ++sweep) {
    // convergence: off-diagonal mass against the diagonal
    double off = 0.0, dia = 0.0;
    for (int e = tid; e < kn * kn; e += blockDim.x) {
      const int p = e / kn, q = e % kn;
      const double v = A[p * la + q];
      if (p == q) dia += v * v;
      else off += v * v;
    }
    for (int d = 16; d > 0; d >>= 1) {
      off += __shfl_xor_sync(0xFFFFFFFFu, off, d);
      dia += __shfl_xor_sync(0xFFFFFFFFu, dia, d);
    }
    if (lane == 0) red[warp] = off;
    __syncthreads();
    if (tid == 0) {
      double o = 0.0;
      for (int w = 0; w < kFitThreads / 32; ++w) o += red[w];
      red[0] = o;
    }
    __syncthreads();
    off = red[0];
    __syncthreads();
    if (lane == 0) red[warp] = dia;
    __syncthreads();
    if (tid == 0) {
      double d2 = 0.0;
      for (int w = 0; w < kFitThreads / 32; ++w) d2 += red[w];
      stop = !(off > 1e-30 * d2);
    }
    __syncthreads();
    if (stop) break;
    for (int r = 0; r < ne - 1; ++r) {
      if (tid < ne / 2) {
        int p, q;
        jacobi_pair(tid, r, ne, p, q);
        double c = 1.0, s = 0.0;
        if (q < kn) {
          const double apq = A[p * la + q];
          if (fabs(apq) > 1e-300) {
            const double tau = (A[q * la + q] - A[p * la + p]) / (2.0 * apq);
            const double t = (tau >= 0.0 ? 1.0 : -1.0) / (fabs(tau) + sqrt(1.0 + tau * tau));
            c = 1.0 / sqrt(1.0 + t * t);
            s = t * c;
          }
        }
        rot_c[tid] = c;
        rot_s[tid] = s;
      }
      __syncthreads();
      for (int e = tid; e < (ne / 2) * kn; e += blockDim.x) {  // A <- A J, V <- V J
        const int k = e / kn, row = e % kn;
        int p, q;
        jacobi_pair(k, r, ne, p, q);
        if (q >= kn) continue;
        const double c = rot_c[k], s = rot_s[k];
        const double ap = A[row * la + p], aq = A[row * la + q];
        A[row * la + p] = c * ap - s * aq;
        A[row * la + q] = s * ap + c * aq;
        const double vp = V[row * la + p], vq = V[row * la + q];
        V[row * la + p] = c * vp - s * vq;
        V[row * la + q] = s * vp + c * vq;
      }
      __syncthreads();
      for (int e = tid; e < (ne / 2) * kn; e += blockDim.x) {  // A <- J^T A
        const int k = e / kn, col = e % kn;
        int p, q;
        jacobi_pair(k, r, ne, p, q);
        if (q >= kn) continue;
        const double c = rot_c[k], s = rot_s[k];
        const double ap = A[p * la + col], aq = A[q * la + col];
        A[p * la + col] = c * ap - s * aq;
        A[q * la + col] = s * ap + c * aq;
      }
      __syncthreads();
    }
  }
  // eigenvalues on the diagonal of A; W = diag(1/l) V^T M
  double lmax = 0.0;
  for (int j = 0; j < kn; ++j) lmax = fmax(lmax, A[j * la + j]);
  const double cut = kEigenCut * lmax;
  for (int e = tid; e < kn * ko; e += blockDim.x) {
    const int j = e / ko, k = e % ko;
    const double l = A[j * la + j];
    double v = 0.0;
    if (l > cut && l > 0.0) {
      for (int p = 0; p < kn; ++p) v = fma(V[p * la + j], M[p * ko + k], v);
      v /= l;
    }
    W[j * ko + k] = v;
  }
  __syncthreads();
  double* X = xmap + (int64_t)i * kn * ko;
  for (int e = tid; e < kn * ko; e += blockDim.x) {
    const int p = e / ko, k = e % ko;
    double v = 0.0;
    for (int j = 0; j < kn; ++j) v = fma(V[p * la + j], W[j * ko + k], v);
    X[e] = v;
  }
}

// Sizes above kFitSmall: G = sum of the split partials (+ ridge) factored in
// place as L L^T (one CTA per input, G in the global workspace `gwork`), then
// X = G^-1 M by forward and back substitution, one right-hand side per thread.
// A pivot below kEigenCut of the largest diagonal entry marks a basis function
// the samples do not determine: its row and column are dropped and its row of
// X is zero (for functions no sample reaches, as in the minimum-norm solution).
__global__ void __launch_bounds__(kFitThreads) refit_chol_kernel(const double* __restrict__ part, int n_split,
                                                                  int64_t n, FitShape fs, double ridge,
                                                                  double* __restrict__ gwork,
                                                                  double* __restrict__ xmap) {
  const int kn = fs.kn, ko = fs.ko, kt = fs.kt;
  const int i = blockIdx.x, tid = threadIdx.x;
  double* G = gwork + (int64_t)i * kn * kn;
  double* X = xmap + (int64_t)i * kn * ko;
  __shared__ double diag_max, pivot;
  __shared__ unsigned char dropped[KF_FIT_MAX_SIZE];
  const double* src = part + (int64_t)i * n_split * kn * kt;
  for (int e = tid; e < kn * kt; e += blockDim.x) {
    double v = 0.0;
    for (int sp = 0; sp < n_split; ++sp) v += src[(int64_t)sp * kn * kt + e];
    const int p = e / kt, q = e % kt;
    if (q < kn) G[p * kn + q] = v;
    else X[p * ko + (q - kn)] = v;
  }
  __syncthreads();
  if (tid == 0) {
    double tr = 0.0, mx = 0.0;
    for (int p = 0; p < kn; ++p) {
      tr += G[p * kn + p];
      mx = fmax(mx, G[p * kn + p]);
    }
    double lam2 = 0.0;
    if (ridge > 0.0) {
      const double lam = sqrt(ridge * (tr / ((double)n * kn)) * (double)n);
      lam2 = lam * lam;
      for (int p = 0; p < kn; ++p) G[p * kn + p] += lam2;
    }
    diag_max = mx + lam2;
  }
  __syncthreads();
  const double cut = kEigenCut * diag_max;
  for (int j = 0; j < kn; ++j) {
    if (tid == 0) {
      const double d = G[j * kn + j];
      const bool drop = !(d > cut);
      dropped[j] = drop;
      pivot = drop ? 0.0 : sqrt(d);
      G[j * kn + j] = pivot;
    }
    __syncthreads();
    const double piv = pivot;
    for (int r = j + 1 + tid; r < kn; r += blockDim.x) G[r * kn + j] = piv > 0.0 ? G[r * kn + j] / piv : 0.0;
    __syncthreads();
    // trailing update of the lower triangle: G[r][c] -= L[r][j] L[c][j], j < c <= r
    const int m = kn - j - 1;
    for (int e = tid; e < m * (m + 1) / 2; e += blockDim.x) {
      int r = (int)((sqrt(8.0 * e + 1.0) - 1.0) * 0.5);
      while ((r + 1) * (r + 2) / 2 <= e) ++r;
      while (r * (r + 1) / 2 > e) --r;
      const int c = e - r * (r + 1) / 2;
      const int rr = j + 1 + r, cc = j + 1 + c;
      G[rr * kn + cc] -= G[rr * kn + j] * G[cc * kn + j];
    }
    __syncthreads();
  }
  // forward substitution L y = m, then back substitution L^T x = y, per column
  for (int c = tid; c < ko; c += blockDim.x) {
    for (int r = 0; r < kn; ++r) {
      double v = X[r * ko + c];
      for (int q = 0; q < r; ++q) v -= G[r * kn + q] * X[q * ko + c];
      X[r * ko + c] = dropped[r] ? 0.0 : v / G[r * kn + r];
    }
    for (int r = kn - 1; r >= 0; --r) {
      double v = X[r * ko + c];
      for (int q = r + 1; q < kn; ++q) v -= G[q * kn + r] * X[q * ko + c];
      X[r * ko + c] = dropped[r] ? 0.0 : v / G[r * kn + r];
    }
  }
}

// coef_out[o, i, :] = X_i (coef[o, i, :] s) / safe(s), scale_out[o, i] = safe(s)
// (kanforge/_layer.py:122-137).  One CTA per (32 outputs, input); X_i staged in
// shared memory when it fits (XSMEM), else read through the caches.
template <typename T, bool XSMEM>
__global__ void __launch_bounds__(kFitThreads) refit_apply_kernel(const double* __restrict__ xmap,
                                                                   const T* __restrict__ coef,
                                                                   const T* __restrict__ scale, int32_t O, int32_t I,
                                                                   int kn, int ko, double* __restrict__ coef_out,
                                                                   double* __restrict__ scale_out) {
  extern __shared__ double asm_[];
  double* ce = asm_;                          // [32][ko]
  double* Xs = ce + 32 * ko;                  // [kn][ko] (XSMEM)
  __shared__ double safe[32];
  const int i = blockIdx.y, o0 = blockIdx.x * 32, tid = threadIdx.x;
  const double* X = XSMEM ? Xs : xmap + (int64_t)i * kn * ko;
  if (XSMEM)
    for (int e = tid; e < kn * ko; e += blockDim.x) Xs[e] = xmap[(int64_t)i * kn * ko + e];
  if (tid < 32) {
    const int o = o0 + tid;
    double s = 1.0;
    if (scale && o < O) s = (double)to_f32(scale[(int64_t)o * I + i]);
    safe[tid] = fabs(s) > 1e-12 ? s : 1.0;
    if (scale_out && o < O) scale_out[(int64_t)o * I + i] = safe[tid];
  }
  for (int e = tid; e < 32 * ko; e += blockDim.x) {
    const int ol = e / ko, k = e % ko, o = o0 + ol;
    double v = 0.0;
    if (o < O) {
      v = (double)to_f32(coef[((int64_t)o * I + i) * ko + k]);
      if (scale) v = __dmul_rn(v, (double)to_f32(scale[(int64_t)o * I + i]));
    }
    ce[e] = v;
  }
  __syncthreads();
  for (int e = tid; e < 32 * kn; e += blockDim.x) {
    const int ol = e / kn, p = e % kn, o = o0 + ol;
    if (o >= O) continue;
    double v = 0.0;
    for (int k = 0; k < ko; ++k) v = fma(X[p * ko + k], ce[ol * ko + k], v);
    coef_out[((int64_t)o * I + i) * kn + p] = __ddiv_rn(v, safe[ol]);
  }
}

}  // namespace
}  // namespace kf

// ---- entry points ------------------------------------------------------------

namespace kf {
namespace {

int64_t hist_splits(int64_t n, int32_t I) { return std::max<int64_t>(1, std::min<int64_t>(cdiv(1184, I), cdiv(n, 4096))); }

int64_t fit_splits(int64_t n, int32_t I) {
  return std::max<int64_t>(1, std::min<int64_t>({cdiv(592, I), cdiv(n, 1024), (int64_t)256}));
}

int check_fit_basis(const kf_fit_basis* b, const char* which) {
  KF_CHECK_ARG(b, "kf_refit: %s basis is null", which);
  KF_CHECK_ARG(b->size >= 1 && b->size <= KF_FIT_MAX_SIZE, "kf_refit: %s basis size %d outside [1, %d]", which,
               b->size, KF_FIT_MAX_SIZE);
  switch (b->kind) {
    case KF_BASIS_BSPLINE:
      KF_CHECK_ARG(b->grid && b->order >= 0 && b->order <= 5 && b->n_grid >= 2 && b->n_grid <= KF_GRID_MAX_POINTS &&
                       b->size == b->n_grid - 1 + b->order,
                   "kf_refit: %s B-spline needs a grid of 2..%d points, order <= 5, size = points - 1 + order", which,
                   KF_GRID_MAX_POINTS);
      return KF_OK;
    case KF_BASIS_CHEB:
      KF_CHECK_ARG(b->fold && b->degree >= 0 && b->degree + 1 <= KF_FIT_MAX_SIZE &&
                       (b->input_map == KF_MAP_TANH || b->input_map == KF_MAP_IDENTITY),
                   "kf_refit: %s polynomial basis needs a fold matrix, degree < %d and a tanh / identity map", which,
                   KF_FIT_MAX_SIZE);
      return KF_OK;
    case KF_BASIS_FOURIER:
      KF_CHECK_ARG(b->degree >= 1 && b->size == 2 * b->degree, "kf_refit: %s Fourier basis needs size = 2 frequencies",
                   which);
      return KF_OK;
    case KF_BASIS_BUMP:
      KF_CHECK_ARG(b->grid && b->n_grid >= 2 && b->size == b->n_grid && b->n_poly >= 1 && b->n_poly <= 8 &&
                       (b->bump_mode == KF_BUMP_GAUSS || b->bump_mode == KF_BUMP_TANH),
                   "kf_refit: %s bump basis needs a grid of size >= 2 centres and a 1..8 term polynomial", which);
      return KF_OK;
    default:
      set_error("kf_refit: %s basis kind %d has no refit", which, b->kind);
      return KF_ERR_UNSUPPORTED;
  }
}

int set_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return KF_OK;
  KF_CUDA_RET(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return KF_OK;
}

}  // namespace
}  // namespace kf

extern "C" int kf_samples_transpose(const void* x, int dtype, int64_t n, int32_t I, float* xt, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && xt && n >= 0 && I >= 1 && I <= 65535 * 32, "kf_samples_transpose: bad arguments");
  if (int rc = bind_device(x)) return rc;
  if (n == 0) return KF_OK;
  KF_CHECK_ARG(cdiv(n, 32) <= 0x7FFFFFFF, "kf_samples_transpose: too many samples");
  const dim3 grid((unsigned)cdiv(n, 32), (unsigned)cdiv(I, 32)), block(32, 8);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32) {
    samples_transpose_kernel<float><<<grid, block, 0, s>>>((const float*)x, xt, n, I);
  } else if (dtype == KF_DTYPE_BF16) {
    samples_transpose_kernel<__nv_bfloat16><<<grid, block, 0, s>>>((const __nv_bfloat16*)x, xt, n, I);
  } else {
    set_error("kf_samples_transpose: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  return check_launch("kf_samples_transpose");
}

extern "C" int64_t kf_grid_workspace(int64_t n, int32_t I, int32_t n_points) {
  if (n < 1 || I < 1 || n_points < 2 || n_points > KF_GRID_MAX_POINTS) return 0;
  return (int64_t)I * n_points * (int64_t)(sizeof(kf::GridState) + 256 * sizeof(uint32_t));
}

extern "C" int kf_adaptive_grid(const float* xt, int64_t n, int32_t I, int32_t n_points, double margin,
                                double grid_eps, double* grid, void* workspace, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(xt && grid && workspace && I >= 1 && I <= 65535, "kf_adaptive_grid: bad arguments");
  KF_CHECK_ARG(n >= 1 && n <= 0x7FFFFFFF, "kf_adaptive_grid: needs 1 <= n < 2^31 samples (got %lld)", (long long)n);
  KF_CHECK_ARG(n_points >= 2 && n_points <= KF_GRID_MAX_POINTS, "kf_adaptive_grid: n_points %d outside [2, %d]",
               n_points, KF_GRID_MAX_POINTS);
  KF_CHECK_ARG(grid_eps > 0.0 && grid_eps <= 1.0,
               "kf_adaptive_grid: grid_eps must be in (0, 1]: some uniform part keeps the grid increasing");
  if (int rc = bind_device(xt)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int T = n_points;
  GridState* state = (GridState*)workspace;
  uint32_t* hist = (uint32_t*)(state + (int64_t)I * T);
  KF_CUDA_RET(cudaMemsetAsync(hist, 0, sizeof(uint32_t) * 256 * (size_t)I * T, s));
  const int64_t splits = hist_splits(n, I);
  const int64_t per_split = cdiv(n, splits);
  const size_t hist_smem = sizeof(uint32_t) * (size_t)T * 257;
  const size_t res_smem = (2 * sizeof(GridState) + sizeof(int)) * (size_t)T;
  if (int rc = set_smem((const void*)grid_hist_kernel, hist_smem)) return rc;
  for (int pass = 0; pass < 4; ++pass) {
    grid_hist_kernel<<<dim3((unsigned)splits, (unsigned)I), kGridThreads, hist_smem, s>>>(xt, n, T, pass, state, hist,
                                                                                           per_split);
    if (int rc = check_launch("kf_adaptive_grid (histogram)")) return rc;
    grid_resolve_kernel<<<(unsigned)I, kGridThreads, res_smem, s>>>(n, T, pass, state, hist, margin, grid_eps, grid);
    if (int rc = check_launch("kf_adaptive_grid (select)")) return rc;
  }
  return KF_OK;
}

extern "C" int kf_resample_grid(const double* grid, int32_t I, int32_t n_old, int32_t n_new, double* out,
                                void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(grid && out && I >= 0 && n_old >= 1 && n_new >= 1, "kf_resample_grid: bad arguments");
  if (int rc = bind_device(grid)) return rc;
  const int64_t total = (int64_t)I * n_new;
  if (total == 0) return KF_OK;
  resample_grid_kernel<<<(unsigned)cdiv(total, 256), 256, 0, (cudaStream_t)stream>>>(grid, I, n_old, n_new, out);
  return check_launch("kf_resample_grid");
}

extern "C" int64_t kf_refit_workspace(int64_t n, int32_t I, int32_t k_old, int32_t k_new) {
  if (n < 1 || I < 1 || k_old < 1 || k_new < 1) return 0;
  const int64_t splits = kf::fit_splits(n, I);
  const bool small = k_old <= kf::kFitSmall && k_new <= kf::kFitSmall;
  return (int64_t)sizeof(double) * I *
         ((int64_t)splits * k_new * (k_new + k_old) + (int64_t)k_new * k_old + (small ? 0 : (int64_t)k_new * k_new));
}

namespace kf {
namespace {

template <typename T>
int launch_apply(const FitShape& fs, const double* xmap, const void* coef, const void* scale, int32_t O, int32_t I,
                 double* coef_out, double* scale_out, cudaStream_t s) {
  const size_t ce = sizeof(double) * 32 * (size_t)fs.ko;
  const size_t with_x = ce + sizeof(double) * (size_t)fs.kn * fs.ko;
  const dim3 agrid((unsigned)cdiv(O, 32), (unsigned)I);
  if (with_x <= 200 * 1024) {
    if (int rc = set_smem((const void*)refit_apply_kernel<T, true>, with_x)) return rc;
    refit_apply_kernel<T, true><<<agrid, kFitThreads, with_x, s>>>(xmap, (const T*)coef, (const T*)scale, O, I, fs.kn,
                                                                    fs.ko, coef_out, scale_out);
  } else {
    if (int rc = set_smem((const void*)refit_apply_kernel<T, false>, ce)) return rc;
    refit_apply_kernel<T, false><<<agrid, kFitThreads, ce, s>>>(xmap, (const T*)coef, (const T*)scale, O, I, fs.kn,
                                                                 fs.ko, coef_out, scale_out);
  }
  return check_launch("kf_refit (apply)");
}

template <int CHUNK, int MAXT>
int launch_gram(const FitShape& fs, dim3 grid, cudaStream_t s, const float* xt, const double* ranges, int64_t n,
                const kf_fit_basis& nb, const kf_fit_basis& ob, int splits, int64_t per_split, double* part) {
  const size_t smem = fit_gram_smem(fs);
  if (int rc = set_smem((const void*)refit_gram_kernel<CHUNK, MAXT>, smem)) return rc;
  refit_gram_kernel<CHUNK, MAXT><<<grid, kFitThreads, smem, s>>>(xt, ranges, n, nb, ob, fs, splits, per_split, part);
  return check_launch("kf_refit (gram)");
}

}  // namespace
}  // namespace kf

extern "C" int kf_refit(const float* xt, const double* ranges, int64_t n, int32_t I, int32_t O,
                        const kf_fit_basis* old_basis, const kf_fit_basis* new_basis, const void* coef,
                        const void* edge_scale, int dtype, double ridge, double* coef_out, double* scale_out,
                        void* workspace, void* stream) {
  using namespace kf;
  clear_error();
  if (int rc = check_fit_basis(old_basis, "old")) return rc;
  if (int rc = check_fit_basis(new_basis, "new")) return rc;
  KF_CHECK_ARG((xt || ranges) && coef && coef_out && workspace && I >= 1 && I <= 65535 && O >= 0 && ridge >= 0.0,
               "kf_refit: bad arguments");
  KF_CHECK_ARG(!edge_scale || scale_out, "kf_refit: edge_scale needs scale_out");
  KF_CHECK_ARG(n >= 1 && n <= 0x7FFFFFFF, "kf_refit: needs 1 <= n < 2^31 samples (got %lld)", (long long)n);
  KF_CHECK_ARG(dtype == KF_DTYPE_F32 || dtype == KF_DTYPE_BF16, "kf_refit: dtype %d unsupported", dtype);
  if (int rc = bind_device(coef)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const FitShape fs = fit_shape(*new_basis, *old_basis);
  KF_CHECK_ARG(fit_gram_smem(fs) <= 200 * 1024, "kf_refit: basis tables too large for shared memory");
  const int64_t splits = fit_splits(n, I);
  const int64_t per_split = cdiv(n, splits);
  double* part = (double*)workspace;
  double* xmap = part + (int64_t)I * splits * fs.kn * fs.kt;
  double* gwork = xmap + (int64_t)I * fs.kn * fs.ko;
  const dim3 ggrid((unsigned)splits, (unsigned)I, (unsigned)fs.tile_groups);
  int rc;
  if (fs.small) rc = launch_gram<128, kFitSmall>(fs, ggrid, s, xt, ranges, n, *new_basis, *old_basis, (int)splits, per_split, part);
  else if (fs.chunk == 128) rc = launch_gram<128, KF_FIT_MAX_SIZE>(fs, ggrid, s, xt, ranges, n, *new_basis, *old_basis, (int)splits, per_split, part);
  else rc = launch_gram<32, KF_FIT_MAX_SIZE>(fs, ggrid, s, xt, ranges, n, *new_basis, *old_basis, (int)splits, per_split, part);
  if (rc) return rc;
  if (fs.small) {
    const size_t solve_smem = sizeof(double) * (2 * (size_t)fs.kn * (fs.kn + 1) + 2 * (size_t)fs.kn * fs.ko);
    if (int r2 = set_smem((const void*)refit_solve_kernel, solve_smem)) return r2;
    refit_solve_kernel<<<(unsigned)I, kFitThreads, solve_smem, s>>>(part, (int)splits, n, fs, ridge, xmap);
  } else {
    refit_chol_kernel<<<(unsigned)I, kFitThreads, 0, s>>>(part, (int)splits, n, fs, ridge, gwork, xmap);
  }
  if (int r2 = check_launch("kf_refit (solve)")) return r2;
  if (O == 0) return KF_OK;
  if (dtype == KF_DTYPE_F32) return launch_apply<float>(fs, xmap, coef, edge_scale, O, I, coef_out, scale_out, s);
  return launch_apply<__nv_bfloat16>(fs, xmap, coef, edge_scale, O, I, coef_out, scale_out, s);
}
