// Float32 GEMM on the 5th-generation tensor cores with three TF32 products
// (the float32 KANLinear path: feature matrix x packed coefficients, the
// input-gradient features and the coefficient gradient, i.e. the reference's
// F/G/P contractions of kanforge/kernels/__init__.py:5-13 at m = 0, w = 1):
//
//   C[m, n] = sum_k A[m, k] B[n, k]  (+ bias[n]),  all float32,
//
// A and B each stored K-major (row m / n contiguous in k) or MN-major (row k
// contiguous in m / n).  tcgen05.mma kind::tf32 reads the upper 19 bits of
// each 32-bit operand (the low 13 mantissa bits are dropped), so the tile as
// loaded is hi = trunc(v); a second tile in shared memory holds lo = v - hi
// (exact in float32), and the accumulator takes hi*hi + hi*lo + lo*hi
// (float32 accumulation in tensor memory): the dropped lo*lo term and the
// truncation of lo leave a relative error near 2^-21 per product, float32
// accuracy for these sums (the tests hold every case to 1e-5 of float64).
//
// The tensor core's float32 accumulation loses precision with the number of
// MMAs accumulated into one tensor-memory accumulator (measured: the error
// grows linearly with K, about 40x round-to-nearest at K = 3000), so each
// tile's K loop runs in segments of kGSeg stages (256 floats of K, 96 MMAs):
// every segment starts a fresh accumulator, and the epilogue adds the segment
// sums in float32 registers (round to nearest).
//
// Persistent CTA pairs (clusters of 2, tcgen05 cta_group::2): a pair tile is
// 256 x 128 outputs, CTA r holding A rows 128 r .. 128 r + 127 and B rows
// 64 r .. 64 r + 63 (half of B per CTA, so that a stage of A, B and their lo
// halves is 48 KB and 4 stages fit; each stage's loads, split and MMAs form a
// latency chain, and more stages in flight raise its throughput).  K steps of
// 32 floats (128-byte rows).  K-major tiles use the 128-byte swizzle (16-byte
// chunks XOR row % 8); MN-major tiles of 32-bit elements must use the
// 128-byte swizzle with 32-byte atoms (32-byte chunks XOR row % 4, descriptor
// layout type 1), the only MN-major layout the tensor core takes for TF32.
// Warp roles in each CTA: w0 TMA (its own halves, local barriers), w1 MMA
// issue (CTA 0), w4-7 split (lo into a second buffer of the same layout,
// fenced into the async proxy, then an arrive on CTA 0's barrier),
// w8-15 epilogue in two column halves (two 128-column accumulators in tensor
// memory, so a segment's drain overlaps the next segment's MMAs).
#include "umma.cuh"

namespace kf {

namespace {

using namespace umma;

constexpr int kGM = 128, kGN = 128, kGK = 32;  // rows per CTA, pair tile columns, K floats per stage
constexpr int kGPairM = 2 * kGM;               // pair tile rows
constexpr int kGStages = 4;
constexpr int kGSeg = 8;  // stages per accumulation segment
constexpr int kGTile = kGM * kGK * 4;          // 16 KB: A tile of a stage (this CTA's 128 rows)
constexpr int kGBHalf = (kGN / 2) * kGK * 4;   // 8 KB: this CTA's 64 rows of B
constexpr int kGStage = 2 * (kGTile + kGBHalf);  // 48 KB: A, B, A_lo, B_lo
constexpr int kGThreads = 512;
constexpr int kGEpiWarps = 8;

struct GemmCtl {
  uint64_t full[kGStages];   // TMA landed (expect_tx)
  uint64_t split[kGStages];  // hi / lo written (4 split warps of each CTA; used in CTA 0)
  uint64_t empty[kGStages];  // MMAs of the stage done (tcgen05.commit)
  uint64_t acc_full[2];
  uint64_t acc_empty[2];     // 8 epilogue warps of each CTA (used in CTA 0)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kGSmem = 1024 + (size_t)kGStages * kGStage + sizeof(GemmCtl);

struct GemmParams {
  const float* bias;  // (N) or null
  float* C;           // (M, ldc)
  int64_t M, N, K, ldc;
  int a_mn, b_mn;     // operand stored MN-major
  int m_fast;         // tile order: M fastest (else N fastest)
  int m_tiles, n_tiles, k_steps;
};

// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T, issued by one thread of CTA 0.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0, mask4 = 0, mask5 = 0, mask6 = 0, mask7 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3), "r"(mask4),
      "r"(mask5), "r"(mask6), "r"(mask7)
      : "memory");
}

// Instruction descriptor of kind::tf32 with f32 accumulation.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                          // D format: f32
         | (2u << 7)                        // A format: tf32
         | (2u << 10)                       // B format: tf32
         | ((a_mn_major ? 1u : 0u) << 15)   // A major
         | ((b_mn_major ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Shared-memory descriptor, layout type 1: 128-byte swizzle with 32-byte
// atoms (MN-major 32-bit operands).  128-byte MN chunks `lbo` apart, 4-row K
// groups `sbo` apart.
__device__ __forceinline__ uint64_t smem_desc_sw128_b32(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)1 << 61;  // SWIZZLE_128B_BASE32B
  return d;
}

// The value the tensor core reads from a 32-bit operand: its upper 19 bits.
__device__ __forceinline__ float tf32_trunc(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// Descriptor of k-step j (8 floats) of a 128-row operand tile.  K-major: rows
// of 128 B, 8-row groups 1 KB apart, a k-step is 32 B along the row.
// MN-major: blocks of 32 MN-elements x 32 k-rows (4 KB apart), 4-row K groups
// 512 B apart, a k-step is 8 rows = 1 KB.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, bool mn_major, int j) {
  return mn_major ? smem_desc_sw128_b32(base + 1024u * j, 4096, 512) : smem_desc_sw128(base + 32u * j, 16, 1024);
}

__global__ void __launch_bounds__(kGThreads, 1) gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                                   const __grid_constant__ CUtensorMap tmap_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: A (16 KB), B half (8 KB) -- TMA, then hi in place -- A_lo, B_lo
  auto a_tile = [&](int s, bool lo) { return base + (size_t)s * kGStage + (lo ? kGTile + kGBHalf : 0); };
  auto b_tile = [&](int s, bool lo) { return base + (size_t)s * kGStage + kGTile + (lo ? kGTile + kGBHalf : 0); };
  GemmCtl* ctl = reinterpret_cast<GemmCtl*>(base + (size_t)kGStages * kGStage);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2, n_pairs = gridDim.x / 2;
  volatile int* abort = &ctl->abort;
  const int n_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->split[s], 8);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 2 * kGEpiWarps);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, 256);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  auto tile_mn = [&](int t, int& m, int& n) {
    if (p.m_fast) {
      m = t % p.m_tiles;
      n = t / p.m_tiles;
    } else {
      n = t % p.n_tiles;
      m = t / p.n_tiles;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs) {
        int m, n;
        tile_mn(t, m, n);
        const int a_row = m * kGPairM + (int)rank * kGM;      // this CTA's A rows
        const int b_row = n * kGN + (int)rank * (kGN / 2);    // this CTA's B rows
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = it % kGStages;
          if (!mbar_wait(&ctl->empty[s], ((it / kGStages) & 1) ^ 1, abort)) break;
          mbar_arrive_expect_tx(&ctl->full[s], kGTile + kGBHalf);
          const int k0 = k * kGK;
          if (p.a_mn) {
#pragma unroll
            for (int c = 0; c < kGM / 32; ++c) tma_load_2d(a_tile(s, false) + c * 4096, &tmap_a, &ctl->full[s], a_row + 32 * c, k0);
          } else {
            tma_load_2d(a_tile(s, false), &tmap_a, &ctl->full[s], k0, a_row);
          }
          if (p.b_mn) {
#pragma unroll
            for (int c = 0; c < kGN / 64; ++c) tma_load_2d(b_tile(s, false) + c * 4096, &tmap_b, &ctl->full[s], b_row + 32 * c, k0);
          } else {
            tma_load_2d(b_tile(s, false), &tmap_b, &ctl->full[s], k0, b_row);
          }
        }
      }
      if (*abort) {  // the loads issued on every stage land before the CTA exits
        for (int s = 0; s < kGStages; ++s) {
          const int last = it - 1 - ((it - 1 - s) % kGStages + kGStages) % kGStages;
          if (it > 0 && last >= 0) mbar_drain(&ctl->full[s], (last / kGStages) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_tf32_f32(kGPairM, kGN, p.a_mn != 0, p.b_mn != 0);
      int it = 0, sc = 0;  // stages and segments issued
      bool ok = true;
      for (int t = pair; t < n_tiles && ok && !*abort; t += n_pairs) {
        for (int k0 = 0; k0 < p.k_steps && ok; k0 += kGSeg, ++sc) {
          const int acc = sc & 1;
          if (!mbar_wait_cluster(&ctl->acc_empty[acc], ((sc >> 1) & 1) ^ 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + acc * kGN;
          const int k1 = min(p.k_steps, k0 + kGSeg);
          for (int k = k0; k < k1; ++k, ++it) {
            const int s = it % kGStages;
            if (!mbar_wait_cluster(&ctl->split[s], (it / kGStages) & 1, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(a_tile(s, false)), b_hi = smem_u32(b_tile(s, false));
            const uint32_t a_lo = smem_u32(a_tile(s, true)), b_lo = smem_u32(b_tile(s, true));
#pragma unroll
            for (int j = 0; j < kGK / 8; ++j) {
              const uint64_t ah = operand_desc(a_hi, p.a_mn, j), al = operand_desc(a_lo, p.a_mn, j);
              const uint64_t bh = operand_desc(b_hi, p.b_mn, j), bl = operand_desc(b_lo, p.b_mn, j);
              mma_tf32_pair(d, ah, bh, idesc, (k > k0 || j > 0) ? 1u : 0u);
              mma_tf32_pair(d, ah, bl, idesc, 1u);
              mma_tf32_pair(d, al, bh, idesc, 1u);
            }
            mma_commit_pair(&ctl->empty[s], 0x3);
          }
          if (!ok) break;
          mma_commit_pair(&ctl->acc_full[acc], 0x3);
        }
      }
      // every MMA issued above has completed once the drain barrier flips
      mma_commit_pair(&ctl->drain, 0x1);
      mbar_drain(&ctl->drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // split: lo = v - trunc(v) at the same offset of the lo tile (hi is the tile as loaded)
    const int st = (warp - 4) * 32 + lane;  // 0 .. 127
    int it = 0;
    for (int t = pair; t < n_tiles; t += n_pairs) {
      bool ok = true;
      for (int k = 0; k < p.k_steps; ++k, ++it) {
        const int s = it % kGStages;
        if (!mbar_wait_warp(&ctl->full[s], (it / kGStages) & 1, abort)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const float4* hi = reinterpret_cast<const float4*>(w ? b_tile(s, false) : a_tile(s, false));
          float4* lo = reinterpret_cast<float4*>(w ? b_tile(s, true) : a_tile(s, true));
          const int n4 = (w ? kGBHalf : kGTile) / 16;
#pragma unroll 4
          for (int e = st; e < n4; e += 128) {
            const float4 v = hi[e];
            lo[e] = make_float4(v.x - tf32_trunc(v.x), v.y - tf32_trunc(v.y), v.z - tf32_trunc(v.z), v.w - tf32_trunc(v.w));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(&ctl->split[s]);
          else mbar_arrive_peer(&ctl->split[s], 0);
        }
      }
      if (!ok) break;
    }
  } else if (warp >= 8) {
    // half e of the columns (64 of them), lane quarter q of this CTA's rows:
    // each thread sums its row's 64 columns over the tile's segments in registers
    const int q = warp % 4, e = (warp - 8) / 4;
    int sc = 0;
    for (int t = pair; t < n_tiles; t += n_pairs) {
      int m, n;
      tile_mn(t, m, n);
      float r[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) r[j] = 0.0f;
      bool ok = true;
      for (int k0 = 0; k0 < p.k_steps; k0 += kGSeg, ++sc) {
        const int acc = sc & 1;
        if (!mbar_wait_warp(&ctl->acc_full[acc], (sc >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kGN + e * 64, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] += v[j];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kGN + e * 64 + 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) r[32 + j] += v[j];
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
      }
      if (!ok) break;
      const int64_t row = (int64_t)m * kGPairM + (int64_t)rank * kGM + q * 32 + lane;
      const int64_t n0 = (int64_t)n * kGN + e * 64;
      if (row < p.M) {
        float* crow = p.C + row * p.ldc;
        if (p.bias) {
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (n0 + j < p.N) r[j] += __ldg(p.bias + n0 + j);
        }
        if (n0 + 64 <= p.N && (p.ldc % 4) == 0 && ((uintptr_t)p.C % 16) == 0) {
#pragma unroll
          for (int j = 0; j < 64; j += 4)
            *reinterpret_cast<float4*>(crow + n0 + j) = make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (n0 + j < p.N) crow[n0 + j] = r[j];
        }
      }
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or MMA of the pair is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 256);
  }
}

// ---- host ------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D float32 tensor map, rows x cols (cols contiguous, row pitch ld floats),
// box 32 columns (128 B) x box_rows rows; the 128-byte swizzle with 16-byte
// chunks (K-major tiles) or 32-byte atoms (MN-major tiles).
int make_tmap_f32(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, bool atom32) {
  auto enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return KF_ERR_CUDA;
  }
  KF_CHECK_ARG(((uintptr_t)ptr % 16) == 0, "kf_gemm_tf32x3: operands must be 16-byte aligned");
  KF_CHECK_ARG(ld % 4 == 0 && ld >= cols, "kf_gemm_tf32x3: row pitch %lld must be a multiple of 4 floats and >= %lld",
               (long long)ld, (long long)cols);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for %lldx%lld", (int)r, (long long)rows, (long long)cols);
    return KF_ERR_CUDA;
  }
  return KF_OK;
}

}  // namespace

}  // namespace kf

extern "C" int kf_gemm_tf32x3(const float* a, int32_t a_mn_major, int64_t lda, const float* b, int32_t b_mn_major,
                              int64_t ldb, const float* bias, float* c, int64_t ldc, int64_t M, int64_t N, int64_t K,
                              void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(a && b && c, "kf_gemm_tf32x3: null operand");
  KF_CHECK_ARG(M >= 0 && N >= 0 && K >= 1 && ldc >= N, "kf_gemm_tf32x3: bad sizes (M %lld, N %lld, K %lld, ldc %lld)",
               (long long)M, (long long)N, (long long)K, (long long)ldc);
  // tile counts and TMA coordinates are 32-bit
  KF_CHECK_ARG(M < (int64_t)kGPairM * 65536 && N < (int64_t)kGN * 65536 && K <= (int64_t)INT32_MAX - kGK,
               "kf_gemm_tf32x3: sizes beyond the kernel limits (M %lld, N %lld, K %lld)", (long long)M, (long long)N,
               (long long)K);
  if (int rc = bind_device(a)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (M == 0 || N == 0) return KF_OK;
  CUtensorMap ta, tb;
  // A: K-major (M rows of K) or MN-major (K rows of M); B likewise with N.
  if (int rc = a_mn_major ? make_tmap_f32(&ta, a, K, M, lda, 32, true) : make_tmap_f32(&ta, a, M, K, lda, kGM, false))
    return rc;
  if (int rc = b_mn_major ? make_tmap_f32(&tb, b, K, N, ldb, 32, true) : make_tmap_f32(&tb, b, N, K, ldb, kGN / 2, false))
    return rc;
  GemmParams p{};
  p.bias = bias;
  p.C = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.a_mn = a_mn_major ? 1 : 0;
  p.b_mn = b_mn_major ? 1 : 0;
  p.m_tiles = (int)cdiv(M, (int64_t)kGPairM);
  p.n_tiles = (int)cdiv(N, (int64_t)kGN);
  p.k_steps = (int)cdiv(K, (int64_t)kGK);
  // Tiles in flight together share the operand that is not streamed: along
  // the larger of M and N that is the other operand (the coefficients of the
  // forward and input gradient, the features of the coefficient gradient).
  p.m_fast = M <= N ? 1 : 0;
  static bool attr_set[64] = {};
  int dev = 0;
  KF_CUDA_RET(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    KF_CUDA_RET(cudaFuncSetAttribute(gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    attr_set[dev] = true;
  }
  int sms = 0;
  KF_CUDA_RET(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = kGSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(2 * (unsigned)((sms > 0 ? sms : 148) / 2));
  static int pair_cache[64] = {0};  // clusters of 2 that fit at once, per device
  if (dev >= 0 && dev < 64 && pair_cache[dev] <= 0) {
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, gemm_tf32x3_kernel, &cfg) != cudaSuccess || nc <= 0) {
      (void)cudaGetLastError();
      nc = (sms > 0 ? sms : 148) / 2;
    }
    pair_cache[dev] = nc;
  }
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  const int pairs = (int)std::min<int64_t>(tiles, dev >= 0 && dev < 64 ? pair_cache[dev] : 1);
  cfg.gridDim = dim3(2 * (unsigned)pairs);
  KF_CUDA_RET(cudaLaunchKernelEx(&cfg, gemm_tf32x3_kernel, ta, tb, p));
  return check_launch("kf_gemm_tf32x3");
}
