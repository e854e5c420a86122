// KAT group-rational activation R(x) = P(x) / (1 + |Q(x)|) of GR-KAN layers
// (reference kanforge/bases/rational.py:84-101; layer layout
// kanforge/torch/layers.py:335-363, parameters shared by I/groups consecutive
// inputs, kanforge/torch/layers.py:151-160).
//
//   kf_rational_act : out = R^(m)(x) elementwise (the GEMM operand, or PINN derivatives)
//   kf_rational_bwd : dx = dr * R'(x) and the per-group parameter gradients
//                     dR/da_j = x^j / D,  dR/db_j = -R sign(Q) x^j / D.
// The parameter gradients are reduced deterministically: each CTA writes
// per-(CTA, input) partial sums into the caller's workspace, a second kernel
// sums them in a fixed order.
#include <atomic>
#include <mutex>

#include "basis.cuh"

namespace kf {

namespace {

constexpr int kRatThreads = 256;
constexpr int kRatVecThreads = 128;  // vector backward: two adjacent inputs per thread, 256 per CTA
constexpr int kRatRows = 8;          // rows whose loads one thread of the vector backward has in flight
constexpr int kRatWave = 148 * 8;    // CTA cap of the forward grid (148 SMs x 8)
constexpr int kRatBwdWave = 148 * 6; // CTAs of one wave of the vector backward (148 SMs x 6 resident)

struct RatParams {
  int na, nb;          // numerator coefficients (p+1), denominator coefficients (q)
  int groups, in_per_group;
};

// Two adjacent elements of T, and their float32 values.
template <typename T>
struct Pair;
template <>
struct Pair<float> {
  using type = float2;
};
template <>
struct Pair<__nv_bfloat16> {
  using type = __nv_bfloat162;
};
__device__ __forceinline__ float2 pair_f32(float2 v) { return v; }
__device__ __forceinline__ float2 pair_f32(__nv_bfloat162 v) { return __bfloat1622float2(v); }
template <typename T>
__device__ __forceinline__ typename Pair<T>::type pair_from(float a, float b);
template <>
__device__ __forceinline__ float2 pair_from<float>(float a, float b) { return make_float2(a, b); }
template <>
__device__ __forceinline__ __nv_bfloat162 pair_from<__nv_bfloat16>(float a, float b) { return __floats2bfloat162_rn(a, b); }

// Coefficient table of all groups in shared memory: sp[g][na + nb].
__device__ __forceinline__ void load_rat_table(float* sp, const float* num, const float* den, const RatParams& p) {
  const int w = p.na + p.nb;
  for (int e = threadIdx.x; e < p.groups * w; e += blockDim.x) {
    const int g = e / w, c = e % w;
    sp[e] = c < p.na ? num[g * p.na + c] : den[g * p.nb + (c - p.na)];
  }
  __syncthreads();
}

// The elementwise arithmetic below comes in two forms with the same sequence
// of IEEE operations, so they give the same bits: one element (degrees up to
// MA / MB, the steps at or beyond na / nb skipped) and a pair of elements in
// float2 lanes (degrees fixed), two fp32 operations per instruction
// (__ffma2_rn / __fmul2_rn / __fadd2_rn).  1 / D uses __fdividef (2 ulp;
// D = 1 + |Q| >= 1 is far inside its range).

// R(x) = P(x) / (1 + |x Qs(x)|) by Horner.
template <int MA, int MB>
__device__ __forceinline__ float rat_value(float xv, const float* a, const float* bq, int na, int nb) {
  float P = a[na - 1], Qs = bq[nb - 1];
#pragma unroll
  for (int j = MA - 2; j >= 0; --j)
    if (j < na - 1) P = fmaf(P, xv, a[j]);
#pragma unroll
  for (int j = MB - 2; j >= 0; --j)
    if (j < nb - 1) Qs = fmaf(Qs, xv, bq[j]);
  return __fdividef(P, 1.0f + fabsf(xv * Qs));
}

template <int NA, int NB>
__device__ __forceinline__ float2 rat_value2(float2 x, const float2 (&a)[NA], const float2 (&bq)[NB]) {
  float2 P = a[NA - 1], Qs = bq[NB - 1];
#pragma unroll
  for (int j = NA - 2; j >= 0; --j) P = __ffma2_rn(P, x, a[j]);
#pragma unroll
  for (int j = NB - 2; j >= 0; --j) Qs = __ffma2_rn(Qs, x, bq[j]);
  const float2 Q = __fmul2_rn(x, Qs);
  return make_float2(__fdividef(P.x, 1.0f + fabsf(Q.x)), __fdividef(P.y, 1.0f + fabsf(Q.y)));
}

// One element of the backward: returns dx = g R'(x) and adds g dR/da_j,
// g dR/db_j to the accumulators.  With D = 1 + |Q|, Q = x Qs(x):
//   R' = (P' - sign(Q) Q' R) / D,  dR/da_j = x^j / D,  dR/db_j = -R sign(Q) x^(j+1) / D.
template <int MA, int MB>
__device__ __forceinline__ float rat_bwd_elem(float xv, float g, const float* a, const float* bq, int na, int nb,
                                              float (&acc_a)[MA], float (&acc_b)[MB]) {
  float P = a[na - 1], dP = 0.0f;
#pragma unroll
  for (int j = MA - 2; j >= 0; --j) {
    if (j < na - 1) {
      dP = fmaf(dP, xv, P);
      P = fmaf(P, xv, a[j]);
    }
  }
  float Qs = bq[nb - 1], dQs = 0.0f;
#pragma unroll
  for (int j = MB - 2; j >= 0; --j) {
    if (j < nb - 1) {
      dQs = fmaf(dQs, xv, Qs);
      Qs = fmaf(Qs, xv, bq[j]);
    }
  }
  const float Q = xv * Qs;
  const float dQ = fmaf(xv, dQs, Qs);
  const float sg = rat_sign(Q);
  const float rD = __fdividef(1.0f, 1.0f + fabsf(Q));
  const float R = P * rD;
  const float u = g * rD;
  acc_a[0] += u;
  float xp = xv;
#pragma unroll
  for (int j = 1; j < MA; ++j) {
    if (j < na) acc_a[j] = fmaf(u, xp, acc_a[j]);
    xp *= xv;
  }
  const float v = (-u * R) * sg;
  xp = xv;
#pragma unroll
  for (int j = 0; j < MB; ++j) {
    if (j < nb) acc_b[j] = fmaf(v, xp, acc_b[j]);
    xp *= xv;
  }
  return g * (fmaf(-(sg * dQ), R, dP) * rD);
}

// Forward (and PINN derivatives): one element per thread, any layout.
template <typename T>
__global__ void __launch_bounds__(kRatThreads) rational_act_kernel(const T* __restrict__ x, const float* __restrict__ num,
                                                                   const float* __restrict__ den, T* __restrict__ out,
                                                                   int64_t n, int I, int m, RatParams p) {
  extern __shared__ float sp[];  // [groups][na + nb]
  load_rat_table(sp, num, den, p);
  const int w = p.na + p.nb;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e % I);
    const float* th = sp + (i / p.in_per_group) * w;
    const float xv = to_f32(x[e]);
    if (m == 0)
      out[e] = from_f32<T>(rat_value<KF_RAT_MAX_NUM, KF_RAT_MAX_DEN>(xv, th, th + p.na, p.na, p.nb));
    else
      out[e] = from_f32<T>(rational_deriv(xv, th, p.na, th + p.na, p.nb, m));
  }
}

// Forward R(x) on 16-byte vectors (8 bf16 / 4 float32 elements of one group):
// nvec vectors, ivec per row, vpg per group, four vectors per thread in flight.
// NA = NB = 0: degrees from p (up to the kernel limits).
template <typename T, int NA, int NB>
__global__ void __launch_bounds__(kRatThreads) rational_act_vec_kernel(const T* __restrict__ x, const float* __restrict__ num,
                                                                       const float* __restrict__ den, T* __restrict__ out,
                                                                       uint32_t nvec, uint32_t ivec, uint32_t vpg,
                                                                       RatParams p) {
  constexpr int V = 16 / sizeof(T);
  struct __align__(16) Vec {
    T e[V];
  };
  extern __shared__ float sp[];
  load_rat_table(sp, num, den, p);
  const int w = p.na + p.nb;
  const Vec* xv = reinterpret_cast<const Vec*>(x);
  Vec* ov = reinterpret_cast<Vec*>(out);
  auto eval = [&](const Vec& in, uint32_t v) {
    const float* th = sp + ((v % ivec) / vpg) * w;
    Vec r;
    if constexpr (NA > 0) {  // pairs of elements in float2 lanes
      float2 ca[NA], cb[NB];
#pragma unroll
      for (int j = 0; j < NA; ++j) ca[j] = dup2(th[j]);
#pragma unroll
      for (int j = 0; j < NB; ++j) cb[j] = dup2(th[NA + j]);
#pragma unroll
      for (int k = 0; k < V; k += 2) {
        const float2 y = rat_value2(make_float2(to_f32(in.e[k]), to_f32(in.e[k + 1])), ca, cb);
        r.e[k] = from_f32<T>(y.x);
        r.e[k + 1] = from_f32<T>(y.y);
      }
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k)
        r.e[k] = from_f32<T>(rat_value<KF_RAT_MAX_NUM, KF_RAT_MAX_DEN>(to_f32(in.e[k]), th, th + p.na, p.na, p.nb));
    }
    ov[v] = r;
  };
  constexpr int kIn = 4;  // vectors per thread in flight
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += kIn * stride) {
    Vec in[kIn];
#pragma unroll
    for (int k = 0; k < kIn; ++k)
      if (v + k * stride < nvec) in[k] = xv[v + k * stride];
#pragma unroll
    for (int k = 0; k < kIn; ++k)
      if (v + k * stride < nvec) eval(in[k], v + k * stride);
  }
}

// Backward partial sums per (row block, input), workspace layout
// ws[blk][c][i] (c < na: numerator, then denominator).  Grid (row blocks,
// 256-input chunks); each thread walks its block's rows in order, so the
// partial sums of both kernels below are the same.
//
// Any layout: one input per thread, degrees up to the kernel limits.
template <typename T>
__global__ void __launch_bounds__(kRatThreads) rational_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dr,
                                                                   const float* __restrict__ num, const float* __restrict__ den,
                                                                   T* __restrict__ dx, float* __restrict__ ws, int64_t B, int I,
                                                                   int64_t rows_per_blk, RatParams p) {
  extern __shared__ float sp[];
  load_rat_table(sp, num, den, p);
  const int i = blockIdx.y * kRatThreads + threadIdx.x;
  if (i >= I) return;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_blk;
  const int64_t r1 = min(B, r0 + rows_per_blk);
  const int w = p.na + p.nb;
  const float* a = sp + (i / p.in_per_group) * w;
  float acc_a[KF_RAT_MAX_NUM], acc_b[KF_RAT_MAX_DEN];
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_NUM; ++j) acc_a[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_DEN; ++j) acc_b[j] = 0.0f;
  for (int64_t b = r0; b < r1; ++b) {
    const int64_t e = b * I + i;
    dx[e] = from_f32<T>(rat_bwd_elem(to_f32(x[e]), to_f32(dr[e]), a, a + p.na, p.na, p.nb, acc_a, acc_b));
  }
  float* dst = ws + (size_t)blockIdx.x * w * I + i;
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_NUM; ++j)
    if (j < p.na) dst[(size_t)j * I] = acc_a[j];
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_DEN; ++j)
    if (j < p.nb) dst[(size_t)(p.na + j) * I] = acc_b[j];
}

// Pairs of inputs (in_per_group even, x / dr / dx aligned to two elements, ws
// to two floats):
// one bf16x2 / float2 load of x and of dr per row, loaded kRatRows rows at a
// time one group ahead of the arithmetic, the degrees fixed at compile time (the
// accumulators of both inputs and the coefficients stay in registers).
template <typename T, int NA, int NB>
__global__ void __launch_bounds__(kRatVecThreads, 6) rational_bwd_vec_kernel(
    const T* __restrict__ x, const T* __restrict__ dr, const float* __restrict__ num, const float* __restrict__ den,
    T* __restrict__ dx, float* __restrict__ ws, int64_t B, int I, int64_t rows_per_blk, RatParams p) {
  static_assert(NA > 0 && NB > 0, "the vector backward fixes the degrees");
  constexpr int MA = NA, MB = NB;
  using P2 = typename Pair<T>::type;
  extern __shared__ float sp[];
  load_rat_table(sp, num, den, p);
  const int i0 = blockIdx.y * (2 * kRatVecThreads) + 2 * threadIdx.x;
  if (i0 >= I) return;
  const int w = p.na + p.nb;
  const float* th = sp + (i0 / p.in_per_group) * w;
  // coefficients duplicated into both lanes; accumulators (input i0, i0 + 1)
  float2 ca[MA], cb[MB], acc_a[MA], acc_b[MB];
#pragma unroll
  for (int j = 0; j < MA; ++j) {
    ca[j] = dup2(th[j]);
    acc_a[j] = make_float2(0.0f, 0.0f);
  }
#pragma unroll
  for (int j = 0; j < MB; ++j) {
    cb[j] = dup2(th[MA + j]);
    acc_b[j] = make_float2(0.0f, 0.0f);
  }
  const int64_t ih = I / 2;
  const P2* xp = reinterpret_cast<const P2*>(x) + i0 / 2;
  const P2* gp = reinterpret_cast<const P2*>(dr) + i0 / 2;
  P2* dp = reinterpret_cast<P2*>(dx) + i0 / 2;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_blk;
  const int64_t r1 = min(B, r0 + rows_per_blk);
  auto row = [&](int64_t b, P2 xv2, P2 gv2) {
    const float2 d = rat_bwd_pair(pair_f32(xv2), pair_f32(gv2), ca, cb, acc_a, acc_b);
    dp[b * ih] = pair_from<T>(d.x, d.y);
  };
  int64_t b = r0;
  for (; b + kRatRows <= r1; b += kRatRows) {
    P2 xv[kRatRows], gv[kRatRows];
#pragma unroll
    for (int r = 0; r < kRatRows; ++r) {
      xv[r] = xp[(b + r) * ih];
      gv[r] = gp[(b + r) * ih];
    }
#pragma unroll
    for (int r = 0; r < kRatRows; ++r) row(b + r, xv[r], gv[r]);
  }
  for (; b < r1; ++b) row(b, xp[b * ih], gp[b * ih]);
  float* dst = ws + (size_t)blockIdx.x * w * I + i0;
#pragma unroll
  for (int j = 0; j < MA; ++j) *reinterpret_cast<float2*>(dst + (size_t)j * I) = acc_a[j];
#pragma unroll
  for (int j = 0; j < MB; ++j) *reinterpret_cast<float2*>(dst + (size_t)(MA + j) * I) = acc_b[j];
}

// dnum[g, j], dden[g, j] = sum over row blocks and the inputs of group g, in a
// fixed order (row block major, then input), so the result is deterministic.
__global__ void __launch_bounds__(kRatThreads) rational_reduce_kernel(const float* __restrict__ ws, float* __restrict__ dnum,
                                                                      float* __restrict__ dden, int nblk, int I, RatParams p) {
  __shared__ float red[kRatThreads];
  const int w = p.na + p.nb;
  const int g = blockIdx.x / w, c = blockIdx.x % w;
  const int n = nblk * p.in_per_group;
  float acc = 0.0f;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int blk = e / p.in_per_group, ii = e % p.in_per_group;
    acc += ws[((size_t)blk * w + c) * I + g * p.in_per_group + ii];
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (c < p.na) dnum[g * p.na + c] = red[0];
    else dden[g * p.nb + (c - p.na)] = red[0];
  }
}

bool aligned_to(const void* q, size_t n) { return ((uintptr_t)q % n) == 0; }

// The backward kernel for one dtype: pairs of inputs for the degrees of the
// GR-KAN default (5, 4) where the layout allows, else one input per thread.
template <typename T>
void launch_rational_bwd(int64_t used, int I, size_t smem, cudaStream_t s, const T* x, const T* dr, const float* num,
                         const float* den, T* dx, float* ws, int64_t B, int64_t rows, const RatParams& p) {
  const dim3 grid((unsigned)used, (unsigned)cdiv((int64_t)I, (int64_t)kRatThreads));
  const size_t two = 2 * sizeof(T);
  if (p.na == 6 && p.nb == 4 && p.in_per_group % 2 == 0 && aligned_to(x, two) && aligned_to(dr, two) &&
      aligned_to(dx, two) && aligned_to(ws, 2 * sizeof(float))) {
    rational_bwd_vec_kernel<T, 6, 4><<<grid, kRatVecThreads, smem, s>>>(x, dr, num, den, dx, ws, B, I, rows, p);
  } else {
    rational_bwd_kernel<T><<<grid, kRatThreads, smem, s>>>(x, dr, num, den, dx, ws, B, I, rows, p);
  }
}

// CTAs of Kern that fit the GPU at once (queried once per kernel).
template <auto Kern>
int64_t resident_ctas(int threads, size_t smem, int64_t fallback) {
  static std::atomic<int64_t> cached{0};
  int64_t n = cached.load();
  if (n > 0) return n;
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, Kern, threads, smem) != cudaSuccess || sms * per_sm <= 0) {
    (void)cudaGetLastError();
    return fallback;
  }
  n = (int64_t)sms * per_sm;
  cached.store(n);
  return n;
}

// The forward for one dtype: 16-byte vectors where the layout allows, one
// wave of CTAs striding over the vectors.
template <typename T>
void launch_rational_act(int64_t B, int I, int m, size_t smem, cudaStream_t s, const T* x, const float* num,
                         const float* den, T* out, const RatParams& p) {
  constexpr int V = 16 / sizeof(T);
  const int64_t n = B * I;
  const int64_t nvec = n / V;
  if (m == 0 && p.in_per_group % V == 0 && nvec < (int64_t(1) << 29) && aligned_to(x, 16) && aligned_to(out, 16)) {
    const bool fixed = p.na == 6 && p.nb == 4;
    auto kern = fixed ? rational_act_vec_kernel<T, 6, 4> : rational_act_vec_kernel<T, 0, 0>;
    const int64_t wave = fixed ? resident_ctas<rational_act_vec_kernel<T, 6, 4>>(kRatThreads, smem, kRatWave)
                               : resident_ctas<rational_act_vec_kernel<T, 0, 0>>(kRatThreads, smem, kRatWave);
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(nvec, (int64_t)kRatThreads), wave);
    kern<<<grid, kRatThreads, smem, s>>>(x, num, den, out, (uint32_t)nvec, (uint32_t)(I / V), (uint32_t)(p.in_per_group / V),
                                         p);
  } else {
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n, (int64_t)kRatThreads), kRatWave);
    rational_act_kernel<T><<<grid, kRatThreads, smem, s>>>(x, num, den, out, n, I, m, p);
  }
}

int rat_params(const kf_basis_desc* d, int I, RatParams& p) {
  KF_CHECK_ARG(d != nullptr && d->kind == KF_BASIS_RATIONAL, "rational kernel needs a rational basis");
  KF_CHECK_ARG(d->groups >= 1 && I % d->groups == 0, "rational: groups %d must divide I %d", d->groups, I);
  KF_CHECK_ARG(d->degree >= 0 && d->degree + 1 <= KF_RAT_MAX_NUM && d->den_degree >= 1 && d->den_degree <= KF_RAT_MAX_DEN,
               "rational: degrees (%d, %d) beyond the kernel limits", d->degree, d->den_degree);
  p.na = d->degree + 1;
  p.nb = d->den_degree;
  p.groups = d->groups;
  p.in_per_group = I / d->groups;
  return KF_OK;
}

// Row blocks of the backward: the grid (row blocks x 256-input chunks) is one
// wave of the vector backward, each thread walking its block's rows.
int64_t rat_blocks(int64_t B, int I) {
  const int64_t chunks = cdiv((int64_t)I, (int64_t)kRatThreads);
  const int64_t target = std::max<int64_t>(1, kRatBwdWave / chunks);
  return B <= 0 ? 1 : std::min<int64_t>(target, B);
}

// ---------------------------------------------------------------------------
// Scratch for kf_rational_bwd_noalloc: a fixed array in device memory, one per
// GPU that loads this library, held until the process exits.  Host code must
// not pass the symbol itself to a kernel (on the host it is only a stand-in);
// the device address comes from cudaGetSymbolAddress, once per device.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_rational_scratch[KF_RATIONAL_NOALLOC_MAX_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_rational_scratch on the current device (resolved on the
// first call per device).
int rational_scratch(float** out) {
  int dev = -1;
  KF_CUDA_RET(cudaGetDevice(&dev));
  KF_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "kf_rational_bwd_noalloc: device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_rational_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("kf_rational_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(err));
      return KF_ERR_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return KF_OK;
}

}  // namespace

}  // namespace kf

extern "C" int64_t kf_rational_workspace(int64_t B, int32_t I, const kf_basis_desc* basis) {
  if (!basis || basis->kind != KF_BASIS_RATIONAL) return 0;
  return kf::rat_blocks(B, I) * (int64_t)I * (basis->degree + 1 + basis->den_degree);
}

extern "C" int kf_rational_act(const void* x, const float* num, const float* den, void* out, int64_t B, int32_t I,
                               int32_t m, const kf_basis_desc* basis, int dtype, void* stream) {
  using namespace kf;
  clear_error();
  RatParams p{};
  if (int rc = rat_params(basis, I, p)) return rc;
  KF_CHECK_ARG(x && num && den && out && B >= 0 && m >= 0 && m <= KF_RAT_MAX_ORDER, "kf_rational_act: bad arguments");
  if (int rc = bind_device(x)) return rc;
  if (B == 0) return KF_OK;
  const size_t smem = sizeof(float) * p.groups * (p.na + p.nb);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32) {
    launch_rational_act<float>(B, I, m, smem, s, (const float*)x, num, den, (float*)out, p);
  } else if (dtype == KF_DTYPE_BF16) {
    launch_rational_act<__nv_bfloat16>(B, I, m, smem, s, (const __nv_bfloat16*)x, num, den, (__nv_bfloat16*)out, p);
  } else {
    set_error("kf_rational_act: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  return check_launch("kf_rational_act");
}

extern "C" int kf_rational_bwd(const void* x, const void* dr, const float* num, const float* den, void* dx, float* dnum,
                               float* dden, float* workspace, int64_t B, int32_t I, const kf_basis_desc* basis, int dtype,
                               void* stream) {
  using namespace kf;
  clear_error();
  RatParams p{};
  if (int rc = rat_params(basis, I, p)) return rc;
  KF_CHECK_ARG(x && dr && num && den && dx && dnum && dden && workspace && B >= 0, "kf_rational_bwd: bad arguments");
  if (int rc = bind_device(x)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dnum, 0, sizeof(float) * p.groups * p.na, s));
    KF_CUDA_RET(cudaMemsetAsync(dden, 0, sizeof(float) * p.groups * p.nb, s));
    return KF_OK;
  }
  const int64_t nblk = rat_blocks(B, I);
  const int64_t rows = cdiv(B, nblk);
  const int64_t used = cdiv(B, rows);
  const size_t smem = sizeof(float) * p.groups * (p.na + p.nb);
  if (dtype == KF_DTYPE_F32) {
    launch_rational_bwd<float>(used, I, smem, s, (const float*)x, (const float*)dr, num, den, (float*)dx, workspace, B,
                               rows, p);
  } else if (dtype == KF_DTYPE_BF16) {
    launch_rational_bwd<__nv_bfloat16>(used, I, smem, s, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dr, num, den,
                                       (__nv_bfloat16*)dx, workspace, B, rows, p);
  } else {
    set_error("kf_rational_bwd: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  if (int rc = check_launch("kf_rational_bwd")) return rc;
  rational_reduce_kernel<<<(unsigned)(p.groups * (p.na + p.nb)), kRatThreads, 0, s>>>(workspace, dnum, dden, (int)used, I, p);
  return check_launch("kf_rational_bwd (reduce)");
}

// Same computation as kf_rational_bwd, with the per-CTA partial sums in the
// library's fixed device array instead of a caller workspace.  The number of
// partial rows is lowered until they fit the array (the final sums then run in
// a different order than kf_rational_bwd, equal up to float32 rounding).
// Every element the reduction reads is written by the same call first, so
// nothing needs to start at zero; calls that overlap on the GPU share the array
// and race.
extern "C" int kf_rational_bwd_noalloc(const void* x, const void* dr, const float* num, const float* den, void* dx,
                                       float* dnum, float* dden, int64_t B, int32_t I, const kf_basis_desc* basis,
                                       int dtype, void* stream) {
  using namespace kf;
  clear_error();
  RatParams p{};
  if (int rc = rat_params(basis, I, p)) return rc;
  KF_CHECK_ARG(x && dr && num && den && dx && dnum && dden && B >= 0, "kf_rational_bwd_noalloc: bad arguments");
  const int64_t row = (int64_t)I * (p.na + p.nb);  // partial sums of one CTA
  KF_CHECK_ARG(row <= KF_RATIONAL_NOALLOC_MAX_FLOATS,
               "kf_rational_bwd_noalloc: I * (p + 1 + q) = %lld exceeds the fixed scratch of %d floats",
               (long long)row, KF_RATIONAL_NOALLOC_MAX_FLOATS);
  if (int rc = bind_device(x)) return rc;
  float* ws = nullptr;
  if (int rc = rational_scratch(&ws)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dnum, 0, sizeof(float) * p.groups * p.na, s));
    KF_CUDA_RET(cudaMemsetAsync(dden, 0, sizeof(float) * p.groups * p.nb, s));
    return KF_OK;
  }
  const int64_t cap = std::max<int64_t>(1, KF_RATIONAL_NOALLOC_MAX_FLOATS / row);
  const int64_t nblk = std::min<int64_t>(rat_blocks(B, I), cap);
  const int64_t rows = cdiv(B, nblk);
  const int64_t used = cdiv(B, rows);
  const size_t smem = sizeof(float) * p.groups * (p.na + p.nb);
  if (dtype == KF_DTYPE_F32) {
    launch_rational_bwd<float>(used, I, smem, s, (const float*)x, (const float*)dr, num, den, (float*)dx, ws, B,
                               rows, p);
  } else if (dtype == KF_DTYPE_BF16) {
    launch_rational_bwd<__nv_bfloat16>(used, I, smem, s, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dr, num, den,
                                       (__nv_bfloat16*)dx, ws, B, rows, p);
  } else {
    set_error("kf_rational_bwd_noalloc: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  if (int rc = check_launch("kf_rational_bwd_noalloc")) return rc;
  rational_reduce_kernel<<<(unsigned)(p.groups * (p.na + p.nb)), kRatThreads, 0, s>>>(ws, dnum, dden, (int)used, I, p);
  return check_launch("kf_rational_bwd_noalloc (reduce)");
}
