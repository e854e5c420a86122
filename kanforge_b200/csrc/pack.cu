// Builds the bf16 coefficient operand of the fused tensor-core kernels.
//
//   coef_eff = coef * edge_scale * edge_mask, base_eff = base * edge_mask
//   packed[o, i, j]  = sum_k coef_eff[o,i,k] fold[k,j]   j < nt   (fold null: j = k)
//   packed[o, i, f_pad-1] = base_eff[o,i]                (SiLU column, the last one)
//   packed[o, i, j]  = 0                                 elsewhere
//
// For folded plans this is the reference's `ct = c @ R` (kanforge/torch/kernels.py:75-77,
// kanforge/kernels/plan.py:75-101) with the base branch of
// kanforge/torch/layers.py:185-186 appended as one more feature column, so the
// layer forward becomes a single contraction over I * f_pad.
#include "common.cuh"

namespace kf {

namespace {

constexpr int kPackThreads = 256;
constexpr int kMaxFold = 64;

// One thread per edge.  KM (16, 32 or 64) bounds K at compile time so the
// scaled coefficients live in registers (loops unrolled with predicates).
template <typename T, int KM>
__global__ void __launch_bounds__(kPackThreads) pack_kernel(const T* __restrict__ coef, const T* __restrict__ base,
                                                            const T* __restrict__ scale, const T* __restrict__ mask,
                                                            const float* __restrict__ fold, __nv_bfloat16* __restrict__ packed,
                                                            int64_t n_edges, int K, int nt, int f_pad, int has_fold) {
  __shared__ float R[KM * KM];
  if (has_fold)
    for (int e = threadIdx.x; e < K * nt; e += blockDim.x) R[e] = fold[e];
  __syncthreads();
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_edges; e += (int64_t)gridDim.x * blockDim.x) {
    const T* c = coef + e * K;
    // effective coefficients coef * edge_scale * edge_mask (kanforge/torch/layers.py:162-167)
    const float mk = mask ? to_f32(mask[e]) : 1.0f;
    const float sm = mk * (scale ? to_f32(scale[e]) : 1.0f);
    const float bv = base != nullptr ? to_f32(base[e]) * mk : 0.0f;
    float cv[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) cv[k] = k < K ? to_f32(c[k]) * sm : 0.0f;
    __nv_bfloat16* dst = packed + e * f_pad;
    for (int j0 = 0; j0 < f_pad; j0 += 8) {
      __align__(16) __nv_bfloat16 tmp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        float v = 0.0f;
        if (j < nt) {
          if (has_fold) {
#pragma unroll
            for (int k = 0; k < KM; ++k)
              if (k < K) v = fmaf(cv[k], R[k * nt + j], v);
          } else {
            // no fold: column j is coefficient j (nt <= K)
#pragma unroll
            for (int k = 0; k < KM; ++k)
              if (k == j) v = cv[k];
          }
        } else if (j == f_pad - 1) {
          v = bv;  // the SiLU column (zero without a base branch)
        }
        tmp[u] = __float2bfloat16_rn(v);
      }
      *reinterpret_cast<uint4*>(dst + j0) = *reinterpret_cast<const uint4*>(tmp);
    }
  }
}

template <typename T>
void launch_pack(unsigned grid, cudaStream_t s, const T* coef, const T* base, const T* scale, const T* mask, const float* fold,
                 __nv_bfloat16* packed, int64_t n, int K, int nt, int f_pad) {
  const int km = std::max(K, nt);
  if (km <= 16)
    pack_kernel<T, 16><<<grid, kPackThreads, 0, s>>>(coef, base, scale, mask, fold, packed, n, K, nt, f_pad, fold != nullptr);
  else if (km <= 32)
    pack_kernel<T, 32><<<grid, kPackThreads, 0, s>>>(coef, base, scale, mask, fold, packed, n, K, nt, f_pad, fold != nullptr);
  else
    pack_kernel<T, 64><<<grid, kPackThreads, 0, s>>>(coef, base, scale, mask, fold, packed, n, K, nt, f_pad, fold != nullptr);
}

}  // namespace

}  // namespace kf

extern "C" int kf_pack_coef(const void* coef_eff, const void* base_eff, const void* edge_scale, const void* edge_mask,
                            const float* fold, void* packed, int32_t O, int32_t I, int32_t K, int32_t nt, int32_t f_pad,
                            int dtype, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(coef_eff && packed, "kf_pack_coef: null pointer");
  if (int rc = bind_device(packed)) return rc;
  KF_CHECK_ARG(O >= 1 && I >= 1 && K >= 1 && nt >= 1 && K <= kMaxFold && nt <= kMaxFold, "kf_pack_coef: bad sizes");
  KF_CHECK_ARG(f_pad % 8 == 0 && f_pad >= nt + 1, "kf_pack_coef: f_pad %d too small", f_pad);
  KF_CHECK_ARG(fold != nullptr || nt <= K, "kf_pack_coef: without a fold nt must be <= K");
  KF_CHECK_ARG(((uintptr_t)packed % 16) == 0, "kf_pack_coef: packed must be 16-byte aligned");
  const int64_t n = (int64_t)O * I;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n, kPackThreads), 148 * 16);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32) {
    launch_pack<float>(grid, s, (const float*)coef_eff, (const float*)base_eff, (const float*)edge_scale,
                       (const float*)edge_mask, fold, (__nv_bfloat16*)packed, n, K, nt, f_pad);
  } else if (dtype == KF_DTYPE_BF16) {
    launch_pack<__nv_bfloat16>(grid, s, (const __nv_bfloat16*)coef_eff, (const __nv_bfloat16*)base_eff,
                               (const __nv_bfloat16*)edge_scale, (const __nv_bfloat16*)edge_mask, fold,
                               (__nv_bfloat16*)packed, n, K, nt, f_pad);
  } else {
    set_error("kf_pack_coef: dtype %d unsupported", dtype);
    return KF_ERR_UNSUPPORTED;
  }
  return check_launch("kf_pack_coef");
}
