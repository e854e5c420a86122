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
#include <mutex>

#include "basis.cuh"

namespace kf {

namespace {

constexpr int kRatThreads = 256;
constexpr int kRatMaxBlocks = 128;

struct RatParams {
  int na, nb;          // numerator coefficients (p+1), denominator coefficients (q)
  int groups, in_per_group;
};

template <typename T>
__global__ void __launch_bounds__(kRatThreads) rational_act_kernel(const T* __restrict__ x, const float* __restrict__ num,
                                                                   const float* __restrict__ den, T* __restrict__ out,
                                                                   int64_t n, int I, int m, RatParams p) {
  extern __shared__ float sp[];  // [groups][na + nb]
  const int w = p.na + p.nb;
  for (int e = threadIdx.x; e < p.groups * w; e += blockDim.x) {
    const int g = e / w, c = e % w;
    sp[e] = c < p.na ? num[g * p.na + c] : den[g * p.nb + (c - p.na)];
  }
  __syncthreads();
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e % I);
    const float* th = sp + (i / p.in_per_group) * w;
    const float xv = to_f32(x[e]);
    if (m == 0) {  // R = P / (1 + |x Qs(x)|), Horner unrolled to the kernel limits (registers only)
      float P = 0.0f, Qs = 0.0f;
#pragma unroll
      for (int j = KF_RAT_MAX_NUM - 1; j >= 0; --j)
        if (j < p.na) P = P * xv + th[j];
#pragma unroll
      for (int j = KF_RAT_MAX_DEN - 1; j >= 0; --j)
        if (j < p.nb) Qs = Qs * xv + th[p.na + j];
      out[e] = from_f32<T>(P / (1.0f + fabsf(xv * Qs)));
    } else {
      out[e] = from_f32<T>(rational_deriv(xv, th, p.na, th + p.na, p.nb, m));
    }
  }
}

// Partial sums per (row block, input): workspace[blk][i][na + nb].  Grid
// (row blocks, 256-input chunks), one thread per input of the chunk walking the
// block's rows; the accumulators and polynomial steps are unrolled to the
// kernel limits with predicates, so they stay in registers.
template <typename T>
__global__ void __launch_bounds__(kRatThreads) rational_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dr,
                                                                   const float* __restrict__ num, const float* __restrict__ den,
                                                                   T* __restrict__ dx, float* __restrict__ ws, int64_t B, int I,
                                                                   int64_t rows_per_blk, RatParams p) {
  extern __shared__ float sp[];
  const int w = p.na + p.nb;
  for (int e = threadIdx.x; e < p.groups * w; e += blockDim.x) {
    const int g = e / w, c = e % w;
    sp[e] = c < p.na ? num[g * p.na + c] : den[g * p.nb + (c - p.na)];
  }
  __syncthreads();
  const int i = blockIdx.y * kRatThreads + threadIdx.x;
  if (i >= I) return;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_blk;
  const int64_t r1 = min(B, r0 + rows_per_blk);
  const float* a = sp + (i / p.in_per_group) * w;
  const float* bq = a + p.na;
  float acc_a[KF_RAT_MAX_NUM], acc_b[KF_RAT_MAX_DEN];
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_NUM; ++j) acc_a[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_DEN; ++j) acc_b[j] = 0.0f;
  for (int64_t b = r0; b < r1; ++b) {
    const int64_t e = b * I + i;
    const float xv = to_f32(x[e]);
    const float g = to_f32(dr[e]);
    // P, P', Q, Q' by Horner (Q = x * Qs(x))
    float P = 0.0f, dP = 0.0f;
#pragma unroll
    for (int j = KF_RAT_MAX_NUM - 1; j >= 0; --j) {
      if (j < p.na) {
        dP = dP * xv + P;
        P = P * xv + a[j];
      }
    }
    float Qs = 0.0f, dQs = 0.0f;
#pragma unroll
    for (int j = KF_RAT_MAX_DEN - 1; j >= 0; --j) {
      if (j < p.nb) {
        dQs = dQs * xv + Qs;
        Qs = Qs * xv + bq[j];
      }
    }
    const float Q = xv * Qs;
    const float dQ = Qs + xv * dQs;
    const float sg = Q > 0.0f ? 1.0f : (Q < 0.0f ? -1.0f : 0.0f);
    const float D = 1.0f + fabsf(Q);
    const float R = P / D;
    const float dR = (dP - sg * dQ * R) / D;
    dx[e] = from_f32<T>(g * dR);
    const float u = g / D;
    float xp = 1.0f;
#pragma unroll
    for (int j = 0; j < KF_RAT_MAX_NUM; ++j) {
      if (j < p.na) acc_a[j] = fmaf(u, xp, acc_a[j]);
      xp *= xv;
    }
    const float v = -u * R * sg;
    xp = xv;
#pragma unroll
    for (int j = 0; j < KF_RAT_MAX_DEN; ++j) {
      if (j < p.nb) acc_b[j] = fmaf(v, xp, acc_b[j]);
      xp *= xv;
    }
  }
  float* dst = ws + ((size_t)blockIdx.x * I + i) * w;
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_NUM; ++j)
    if (j < p.na) dst[j] = acc_a[j];
#pragma unroll
  for (int j = 0; j < KF_RAT_MAX_DEN; ++j)
    if (j < p.nb) dst[p.na + j] = acc_b[j];
}

// dnum[g, j], dden[g, j] = sum over CTAs and the inputs of group g, in a fixed order.
__global__ void __launch_bounds__(kRatThreads) rational_reduce_kernel(const float* __restrict__ ws, float* __restrict__ dnum,
                                                                      float* __restrict__ dden, int nblk, int I, RatParams p) {
  __shared__ float red[kRatThreads];
  const int w = p.na + p.nb;
  const int g = blockIdx.x / w, c = blockIdx.x % w;
  const int n = nblk * p.in_per_group;
  float acc = 0.0f;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int blk = e / p.in_per_group, ii = e % p.in_per_group;
    acc += ws[((size_t)blk * I + g * p.in_per_group + ii) * w + c];
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

// Row blocks of the backward: at least kRatMaxBlocks, more when I has few
// 256-input chunks, so that the grid (row blocks x chunks) fills the GPU.
int64_t rat_blocks(int64_t B, int I) {
  const int64_t chunks = cdiv((int64_t)I, (int64_t)kRatThreads);
  const int64_t target = std::max<int64_t>(kRatMaxBlocks, (148 * 8) / chunks);
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
  const int64_t n = B * I;
  const size_t smem = sizeof(float) * p.groups * (p.na + p.nb);
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n, kRatThreads), 148 * 8);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32) {
    rational_act_kernel<float><<<grid, kRatThreads, smem, s>>>((const float*)x, num, den, (float*)out, n, I, m, p);
  } else if (dtype == KF_DTYPE_BF16) {
    rational_act_kernel<__nv_bfloat16><<<grid, kRatThreads, smem, s>>>((const __nv_bfloat16*)x, num, den,
                                                                        (__nv_bfloat16*)out, n, I, m, p);
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
    rational_bwd_kernel<float><<<dim3((unsigned)used, (unsigned)cdiv(I, kRatThreads)), kRatThreads, smem, s>>>((const float*)x, (const float*)dr, num, den,
                                                                         (float*)dx, workspace, B, I, rows, p);
  } else if (dtype == KF_DTYPE_BF16) {
    rational_bwd_kernel<__nv_bfloat16><<<dim3((unsigned)used, (unsigned)cdiv(I, kRatThreads)), kRatThreads, smem, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)dr, num, den, (__nv_bfloat16*)dx, workspace, B, I, rows, p);
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
    rational_bwd_kernel<float><<<dim3((unsigned)used, (unsigned)cdiv(I, kRatThreads)), kRatThreads, smem, s>>>((const float*)x, (const float*)dr, num, den,
                                                                         (float*)dx, ws, B, I, rows, p);
  } else if (dtype == KF_DTYPE_BF16) {
    rational_bwd_kernel<__nv_bfloat16><<<dim3((unsigned)used, (unsigned)cdiv(I, kRatThreads)), kRatThreads, smem, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)dr, num, den, (__nv_bfloat16*)dx, ws, B, I, rows, p);
  } else {
    set_error("kf_rational_bwd_noalloc: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  if (int rc = check_launch("kf_rational_bwd_noalloc")) return rc;
  rational_reduce_kernel<<<(unsigned)(p.groups * (p.na + p.nb)), kRatThreads, 0, s>>>(ws, dnum, dden, (int)used, I, p);
  return check_launch("kf_rational_bwd_noalloc (reduce)");
}
