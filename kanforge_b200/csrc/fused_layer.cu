// Fused KANLinear forward / input-gradient / coefficient-gradient kernels on
// the 5th-generation tensor cores (tcgen05, sm_100a).
//
// A KANLinear of basis size K with the SiLU base branch is one contraction
// over I * F features, F = f_pad >= nt + 1 (kanforge/torch/layers.py:184-186
// folded together):
//
//   FWD   y[b,o]       = sum_{i,j} feat_j(x[b,i]) packed[o,i,j]         M=B    N=O    K=I*F
//   DGRAD dx[b,i]      = sum_j dfeat_j(x[b,i]) sum_o dy[b,o] packed[o,i,j]  M=B  N=I*F  K=O
//   WGRAD dpacked[o,i,j] = sum_b feat_j(x[b,i]) dy[b,o]                  M=I*F  N=O    K=B
//
// (reference F/G/P closure, kanforge/kernels/__init__.py:5-13, at m = 0 with
// w = 1; dx is P_1, the coefficient gradient G_0 followed by the fold
// transpose of kanforge/torch/kernels.py:97-98).
//
// All three run on persistent 2-CTA clusters (one CTA per SM): one thread of
// CTA 0 issues tcgen05.mma.cta_group::2 with M = 256 (rows 0-127 of A and of
// the accumulator in CTA 0, rows 128-255 in CTA 1, B split by N between the
// CTAs) into 256-column f32 accumulators in tensor memory while the epilogue
// warps of both CTAs drain the accumulator of the previous tile.  The basis
// operand is evaluated by producer warps from x into shared memory in the
// canonical 128-byte swizzled layout the tensor core reads (fenced into the
// async proxy, signalled on an mbarrier), or, for the coefficient gradient,
// read by TMA from the feature matrix of kf_features; coefficients and dy
// arrive by TMA (no multicast).  A CTA-1 stage completes on CTA 0's barriers
// (remote arrives and cta_group::2 TMA), MMA completions are multicast to
// both CTAs.
//
// Tiles: pair M = 256 rows, N = 256 columns per accumulator (the forward uses
// two: 512 outputs), K steps of 64 bf16 (128 B), 4 stages.
#include <atomic>

#include "basis.cuh"
#include "conv.cuh"
#include "features.cuh"
#include "umma.cuh"

namespace kf {

namespace {

using namespace umma;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // bf16 elements per stage row = 128 bytes
constexpr int kStages = 4;     // pipeline depth of the kernels with producer warps
constexpr int kMaxStages = 6;  // deepest pipeline (TMA-fed kernels, where shared memory allows)
constexpr int kATile = kBM * 128;  // 16 KB
constexpr int kTabStride = kKnotTableStride;  // floats per knot/inverse-difference row
constexpr int kMaxOrder = 5;

struct TileMap {
  int m_tiles, n_tiles, gm;
  __device__ __forceinline__ void get(int t, int& m, int& n) const {
    const int per_super = gm * n_tiles;
    const int sup = t / per_super, local = t % per_super;
    const int rows = min(gm, m_tiles - sup * gm);
    m = sup * gm + local % rows;
    n = local / rows;
  }
  __device__ __forceinline__ int count() const { return m_tiles * n_tiles; }
};

// Template values of BK: 1..5 B-spline order; 0 Chebyshev features;
// kFourierBK Fourier features (closed-form rows like Chebyshev: no per-input
// data); kRationalBK the GR-KAN rational (input-gradient kernel only).
constexpr bool is_closed(int bk) { return bk == 0 || bk == kFourierBK; }

struct BasisDev {
  float w1;      // Fourier: 2 pi / period
  int nfreq;     // Fourier: frequencies (nt = 2 nfreq)
  int map;       // KF_MAP_* (Chebyshev)
  int nt;        // basis feature columns (Chebyshev: T_0..T_{nt-1}; B-spline: size)
  int has_base;  // SiLU column at index F - 1 (the last padded column)
  int G, nk;     // B-spline grid intervals and extended knots
  const float* tab;  // B-spline knot tables (I, order + 1, 64), see kf_knot_tables
};

struct Ctl {
  uint64_t full_a[kMaxStages];
  uint64_t full_b[kMaxStages];
  uint64_t tab_full[kMaxStages];   // CTA pairs: this CTA's knot tables of the stage landed
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Ctl) % 16 == 0, "the shared memory after Ctl must stay 16-byte aligned");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 16-byte asynchronous global -> shared copy (zero-filled when !valid) and
// the wait for all of this thread's copies.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Largest power of two <= n (n >= 1): the first step of the fixed-step knot search.
__device__ __forceinline__ int pow2_floor(int n) { return 1 << (31 - __clz(n)); }

// Knot table of one input (kTabStride floats per row): row 0 = extended knots
// t_r (r < nk), row q = 1 / (t_{r+q} - t_r) for r <= nk - 1 - q; zero elsewhere.
template <int BK>
__global__ void __launch_bounds__(256) knot_table_kernel(const float* __restrict__ grid, float* __restrict__ tab, int I, int G) {
  const int nk = G + 2 * BK + 1;
  const int per_in = (BK + 1) * kTabStride;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)I * per_in; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / per_in), rem = (int)(e % per_in);
    const int q = rem / kTabStride, r = rem % kTabStride;
    const float* g = grid + (size_t)i * (G + 1);
    float v = 0.0f;
    if (q == 0) {
      if (r < nk) v = extended_knot(g, G, BK, r);
    } else if (r <= nk - 1 - q) {
      v = 1.0f / (extended_knot(g, G, BK, r + q) - extended_knot(g, G, BK, r));
    }
    tab[e] = v;
  }
}

// Abort path of the TMA thread: wait for the last load issued on every stage
// (iterations < `issued`) so that no bulk copy targets shared memory after exit.
template <int NS>
__device__ __forceinline__ void drain_tma(Ctl* ctl, int issued) {
  for (int s = 0; s < NS; ++s) {
    int last = issued - 1 - ((issued - 1 - s) % NS + NS) % NS;
    if (issued <= 0 || last < 0) continue;
    mbar_drain(&ctl->full_b[s], (last / NS) & 1);
  }
}

// Chebyshev feature row of one input: T_0..T_{F-2}(g(x)) and silu(x) in the
// last column.  Columns nt..F-2 meet zero coefficients (kf_pack_coef), so for
// the tanh map (|T_j| <= 1) they need no masking; the identity map masks them
// so that large |x| cannot produce inf * 0.
template <int F>
__device__ __forceinline__ void cheb_row(float x, const BasisDev& bd, float (&f)[F]) {
  const bool tanh_map = bd.map == KF_MAP_TANH;
  const float z = tanh_map ? tanh_exp(x) : x;
  const float z2 = 2.0f * z;
  f[0] = 1.0f;
  f[1] = z;
#pragma unroll
  for (int j = 2; j < F - 1; ++j) f[j] = fmaf(z2, f[j - 1], -f[j - 2]);
  if (!tanh_map) {
#pragma unroll
    for (int j = 1; j < F - 1; ++j) f[j] = j < bd.nt ? f[j] : 0.0f;
  }
  f[F - 1] = bd.has_base ? silu_fast(x) : 0.0f;
}

// d/dx of the Chebyshev feature row: j U_{j-1}(z) g'(x), and silu' in the last column.
template <int F>
__device__ __forceinline__ void cheb_drow(float x, const BasisDev& bd, float (&f)[F]) {
  const bool tanh_map = bd.map == KF_MAP_TANH;
  float z, gp;
  if (tanh_map) {
    z = tanhf(x);
    gp = 1.0f - z * z;
  } else {
    z = x;
    gp = 1.0f;
  }
  const float z2 = 2.0f * z;
  float um2 = 0.0f, um1 = 1.0f;  // U_{-1} = 0, U_0 = 1
  f[0] = 0.0f;
#pragma unroll
  for (int j = 1; j < F - 1; ++j) {
    f[j] = (tanh_map || j < bd.nt) ? (float)j * um1 * gp : 0.0f;
    const float u = fmaf(z2, um1, -um2);
    um2 = um1;
    um1 = u;
  }
  f[F - 1] = bd.has_base ? dsilu_fast(x) : 0.0f;
}

// Fourier feature row: cos(j w1 x) in columns 0..n-1, sin(j w1 x) in n..2n-1
// (kanforge/bases/fourier.py:36-44), zero up to F-2, silu(x) in the last column.
template <int F>
__device__ __forceinline__ void fourier_row(float x, const BasisDev& bd, float (&f)[F]) {
  float s1, c1;
  sincosf(bd.w1 * x, &s1, &c1);
  float c = c1, s = s1;
#pragma unroll
  for (int j = 0; j < F; ++j) f[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < (F - 1) / 2; ++j) {
    if (j < bd.nfreq) {
      // columns j and nfreq + j: a compile-time loop over possible positions keeps f in registers
#pragma unroll
      for (int q = 0; q < F - 1; ++q) {
        if (q == j) f[q] = c;
        if (q == bd.nfreq + j) f[q] = s;
      }
    }
    const float cn = c * c1 - s * s1;
    s = s * c1 + c * s1;
    c = cn;
  }
  f[F - 1] = bd.has_base ? silu_fast(x) : 0.0f;
}

// d/dx of the Fourier row: -j w1 sin(j w1 x), j w1 cos(j w1 x), and silu'.
template <int F>
__device__ __forceinline__ void fourier_drow(float x, const BasisDev& bd, float (&f)[F]) {
  float s1, c1;
  sincosf(bd.w1 * x, &s1, &c1);
  float c = c1, s = s1;
#pragma unroll
  for (int j = 0; j < F; ++j) f[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < (F - 1) / 2; ++j) {
    if (j < bd.nfreq) {
      const float w = (float)(j + 1) * bd.w1;
#pragma unroll
      for (int q = 0; q < F - 1; ++q) {
        if (q == j) f[q] = -w * s;
        if (q == bd.nfreq + j) f[q] = w * c;
      }
    }
    const float cn = c * c1 - s * s1;
    s = s * c1 + c * s1;
    c = cn;
  }
  f[F - 1] = bd.has_base ? dsilu_fast(x) : 0.0f;
}

template <int BK, int F>
__device__ __forceinline__ void closed_row(float x, const BasisDev& bd, float (&f)[F]) {
  if constexpr (BK == kFourierBK) fourier_row<F>(x, bd, f);
  else cheb_row<F>(x, bd, f);
}

template <int BK, int F>
__device__ __forceinline__ void closed_drow(float x, const BasisDev& bd, float (&f)[F]) {
  if constexpr (BK == kFourierBK) fourier_drow<F>(x, bd, f);
  else cheb_drow<F>(x, bd, f);
}

// ===========================================================================
// FWD
// ===========================================================================

struct FwdParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  int64_t B;
  int I, O;
  int k_steps;
  int nblk;  // 256-output accumulator blocks per tile: kFwdNB, or 1 when O <= 256
  TileMap tiles;
  BasisDev bd;
  ConvDev conv;  // active: x is an image read through the implicit patch matrix
  // Closed-form plans, optional: for the first output tile of each token tile
  // the producers also store their feature stages here (TMA, by tmap_a),
  // (B, I * F) bf16 row-major, the layout kf_features writes for the
  // coefficient gradient.
  __nv_bfloat16* feat_out;
};

constexpr int kFwdThreads = 768;  // w0 TMA, w1 MMA (CTA 0), w4-7 epilogue, w8-23 producers (4 groups)
constexpr int kFwdGroups = 4;     // producer group g owns the K-steps it with it % 4 == g (stage g)
constexpr int kPairM = 2 * kBM;   // rows of a CTA-pair tile
constexpr int kBHalf = (kBN / 2) * 128;  // 16 KB: the half of a B stage one CTA of the pair holds
constexpr int kFwdNB = 2;                 // forward: 256-column accumulator blocks per tile (all of TMEM)

// The forward runs on CTA pairs: a tile is 256 tokens x 512 outputs, CTA r of
// the pair evaluates the feature rows of tokens 128 r .. 128 r + 127 (its half
// of A) and loads coefficient rows 128 r .. 128 r + 127 of each 256-output
// block of the tile (its half of B), and CTA 0 issues
// tcgen05.mma.cta_group::2 with M = 256 into two 256-column accumulators that
// fill the tensor memory; each CTA's tensor memory holds its own 128 rows.
// One feature stage thus feeds 512 outputs, halving the feature evaluation per
// MMA, at the price of an epilogue that is not overlapped (about 1% of a
// tile's K loop at 4096 inputs).  The stage barriers that the MMA waits on live in CTA 0:
// CTA 1's producers arrive there remotely and its coefficient TMA completes
// there; the MMA completions are multicast to both CTAs' barriers.
//
// A_TMA: the feature rows are not evaluated here but read by TMA from the
// (B, I*F) feature matrix of kf_features (tmap_a, K-major 128 x 64 boxes);
// the kernel then has no producer warps.
constexpr int kFwdTmaThreads = 256;  // A_TMA: w0 TMA, w1 MMA (CTA 0), w4-7 epilogue

template <int BK, int F, bool A_TMA, int NS>
__global__ void __launch_bounds__(A_TMA ? kFwdTmaThreads : kFwdThreads, 1)
    fused_fwd_kernel(const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_a, FwdParams p) {
  constexpr int IPK = kBK / F;  // inputs per K-step
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  const int b_stage = p.nblk * kBHalf;                  // bytes of B per stage (this CTA's halves)
  uint8_t* sa = base;                                   // NS x 16 KB
  uint8_t* sb = sa + NS * kATile;                       // NS x nblk x 16 KB
  Ctl* ctl = reinterpret_cast<Ctl*>(sb + NS * b_stage);
  constexpr int kTabIn = (BK + 1) * kTabStride;          // floats of one input's knot table
  float* tabs = reinterpret_cast<float*>(align1024(reinterpret_cast<uint8_t*>(ctl + 1)));  // B-spline: [stage][IPK][kTabIn]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2, n_pairs = gridDim.x / 2;
  volatile int* abort = &ctl->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctl->full_a[s], 8);    // 4 producer warps of each CTA (used in CTA 0)
      mbar_init(&ctl->full_b[s], 1);    // CTA 0's expect_tx for both halves (used in CTA 0)
      mbar_init(&ctl->tab_full[s], 1);  // this CTA's knot tables
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 8);  // 4 epilogue warps of each CTA (used in CTA 0)
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_c);
    if (A_TMA) prefetch_tmap(&tmap_a);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int n_tiles = p.tiles.count();

  if (warp == 0) {
    // ---------------- TMA producer: this CTA's half of the coefficient tile ----------------
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs) {
        int m, n;
        p.tiles.get(t, m, n);
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!mbar_wait(&ctl->empty[s], ph ^ 1, abort)) break;
          if constexpr (BK > 0 && !A_TMA) {
            // the knot tables of the step's inputs, into this CTA
            const int n_in = min(IPK, p.I - k * IPK);
            const uint32_t tb = (uint32_t)(n_in * kTabIn * sizeof(float));
            mbar_arrive_expect_tx(&ctl->tab_full[s], tb);
            bulk_load(tabs + s * IPK * kTabIn, p.bd.tab + (size_t)k * IPK * kTabIn, tb, &ctl->tab_full[s]);
          }
          uint8_t* sbs = sb + s * b_stage;
          // both CTAs' coefficient halves (and A_TMA: feature rows) complete here
          if (rank == 0) mbar_arrive_expect_tx(&ctl->full_b[s], 2 * p.nblk * kBHalf + (A_TMA ? 2 * kATile : 0));
          if constexpr (A_TMA) {
            const int a_row = m * kPairM + (int)rank * kBM;
            if (rank == 0)
              tma_load_2d(sa + s * kATile, &tmap_a, &ctl->full_b[s], k * kBK, a_row);
            else
              tma_load_2d_pair(sa + s * kATile, &tmap_a, &ctl->full_b[s], 0, k * kBK, a_row);
          }
          for (int nb = 0; nb < p.nblk; ++nb) {
            const int c_row = (n * p.nblk + nb) * kBN + (int)rank * (kBN / 2);
            if (rank == 0)
              tma_load_2d(sbs + nb * kBHalf, &tmap_c, &ctl->full_b[s], k * kBK, c_row);
            else
              tma_load_2d_pair(sbs + nb * kBHalf, &tmap_c, &ctl->full_b[s], 0, k * kBK, c_row);
          }
        }
      }
      // Abort: CTA 0 drains the coefficient loads of both CTAs (they complete
      // on its barriers) before the pair's final cluster barrier.
      if (*abort && rank == 0) drain_tma<NS>(ctl, it);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (CTA 0 of the pair) ----------------
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kPairM, kBN, false, false);
      int it = 0, tc = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs, ++tc) {
        // one 256-column block per tile: the two accumulators alternate, so the
        // epilogue of a tile overlaps the MMAs of the next
        const int acc = p.nblk == 1 ? (tc & 1) : 0;
        const uint32_t par = p.nblk == 1 ? ((tc >> 1) & 1) : (tc & 1);
        if (!mbar_wait_cluster(&ctl->acc_empty[acc], par ^ 1, abort)) break;
        tc_fence_after();
        bool ok = true;
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if ((!A_TMA && !mbar_wait_cluster(&ctl->full_a[s], ph, abort)) || !mbar_wait_cluster(&ctl->full_b[s], ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + s * kATile), b0 = smem_u32(sb + s * b_stage);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            const uint64_t adesc = smem_desc_sw128(a0 + 32 * j, 16, 1024);
            for (int nb = 0; nb < p.nblk; ++nb)
              mma_bf16_pair(tmem + (acc + nb) * kBN, adesc, smem_desc_sw128(b0 + nb * kBHalf + 32 * j, 16, 1024), idesc,
                            (k > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit_pair(&ctl->empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&ctl->acc_full[acc], 0x3);
      }
      // Every MMA of this CTA has completed (and every commit above has
      // arrived) once the drain barrier flips: the pair may then exit.
      mma_commit_pair(&ctl->drain, 0x1);
      mbar_drain(&ctl->drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- epilogue: TMEM -> +bias -> bf16 -> y ----------------
    const int q = warp - 4;
    const int row = q * 32 + lane;
    int tc = 0;
    for (int t = pair; t < n_tiles; t += n_pairs, ++tc) {
      int m, n;
      p.tiles.get(t, m, n);
      const int acc = p.nblk == 1 ? (tc & 1) : 0;
      const uint32_t par = p.nblk == 1 ? ((tc >> 1) & 1) : (tc & 1);
      if (!mbar_wait_warp(&ctl->acc_full[acc], par, abort)) break;
      tc_fence_after();
      const int64_t b = (int64_t)m * kPairM + (int64_t)rank * kBM + row;
      const int o_base = n * (p.nblk * kBN);
      const int n_chunks = p.nblk * kBN / 32;
#pragma unroll 1
      for (int c = 0; c < n_chunks; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kBN + c * 32, v);
        if (c == n_chunks - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
        }
        const int o0 = o_base + c * 32;
        if (b < p.B && o0 < p.O) {
          // O % 8 == 0: the chunk's outputs are whole groups of 8 (one 16-byte
          // vector of y and of the bias each)
          if (p.bias) {
            const uint4* bv = reinterpret_cast<const uint4*>(p.bias + o0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (o0 + 8 * u < p.O) {
                const uint4 w = __ldg(bv + u);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  v[8 * u + 2 * h] += __uint_as_float(ws[h] << 16);
                  v[8 * u + 2 * h + 1] += __uint_as_float(ws[h] & 0xffff0000u);
                }
              }
            }
          }
          __nv_bfloat16* dst = p.y + b * p.O + o0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (o0 + 8 * u < p.O) {
              uint4 pk;
              pk.x = pack_bf16x2(v[8 * u + 0], v[8 * u + 1]);
              pk.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
              pk.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
              pk.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
              *reinterpret_cast<uint4*>(dst + 8 * u) = pk;
            }
          }
        }
      }
    }
  } else if (!A_TMA && warp >= 8) {
    // ---------------- feature producers: x -> basis rows in smem ----------------
    // Group grp owns the K-steps it with it % 4 == grp, i.e. always stage grp;
    // each thread owns one row.  The x values of a thread's next step are
    // loaded one step ahead so global latency overlaps the current step.
    static_assert(A_TMA || NS % kFwdGroups == 0, "each producer group owns whole stages");
    const int grp = (warp - 8) / 4;
    const int row = ((warp - 8) % 4) * 32 + lane;
    const bool group_lead = row == 0;  // issues the group's feature stores (kf_fwd_emit_features)
    bool store_pending = false;        // a store from the group's stage may still be reading it
    int it = 0;
    bool alive = true;
    for (int t = pair; t < n_tiles && alive; t += n_pairs) {  // abort is seen (warp-uniformly) by the waits
      int m, n;
      p.tiles.get(t, m, n);
      const int64_t b = (int64_t)m * kPairM + (int64_t)rank * kBM + row;
      const bool row_ok = b < p.B;
      const unsigned short* xrow = reinterpret_cast<const unsigned short*>(p.x) + (row_ok ? b : 0) * p.I;
      // the token tile's features go to the feature matrix once: from its tile of output block 0
      const bool emit = is_closed(BK) && !A_TMA && p.feat_out != nullptr && n == 0;
      int k = ((grp - it) % kFwdGroups + kFwdGroups) % kFwdGroups;
      unsigned short xa[IPK], xb[IPK];
#pragma unroll
      for (int u = 0; u < IPK; ++u)
        xa[u] = (row_ok && k < p.k_steps && k * IPK + u < p.I)
                    ? (p.conv.active ? x_bits(p.x, p.conv, b, k * IPK + u, p.I) : __ldg(xrow + k * IPK + u)) : 0;
      for (; k < p.k_steps; k += kFwdGroups) {
        const int git = it + k;
        const int s = git % NS;
        const uint32_t ph = (git / NS) & 1;
        const int i0 = k * IPK;
        const int inext = i0 + kFwdGroups * IPK;
#pragma unroll
        for (int u = 0; u < IPK; ++u)
          xb[u] = (row_ok && k + kFwdGroups < p.k_steps && inext + u < p.I)
                      ? (p.conv.active ? x_bits(p.x, p.conv, b, inext + u, p.I) : __ldg(xrow + inext + u)) : 0;
        bool ok = mbar_wait_warp(&ctl->empty[s], ph ^ 1, abort);
        if constexpr (BK > 0) ok = ok && mbar_wait_warp(&ctl->tab_full[s], ph, abort);  // tables landed
        if (emit || store_pending) {
          // the group's last store from this stage has read it; the four warps agree on ok
          if (group_lead) bulk_wait_read_all();
          ok = named_bar_and(2 + grp, 128, ok);
          store_pending = false;
        }
        if (!ok) {
          alive = false;
          break;
        }
        float xv[IPK];
#pragma unroll
        for (int u = 0; u < IPK; ++u) xv[u] = __uint_as_float((uint32_t)xa[u] << 16);
        uint8_t* arow = sa + s * kATile;
        if constexpr (is_closed(BK)) {
#pragma unroll
          for (int u = 0; u < IPK; ++u) {
            float f[F];
            closed_row<BK, F>(xv[u], p.bd, f);
            if (i0 + IPK > p.I && i0 + u >= p.I) {  // tail step only
#pragma unroll
              for (int j = 0; j < F; ++j) f[j] = 0.0f;
            }
#pragma unroll
            for (int c = 0; c < F / 8; ++c) {
              uint4 pk;
              pk.x = pack_bf16x2(f[8 * c + 0], f[8 * c + 1]);
              pk.y = pack_bf16x2(f[8 * c + 2], f[8 * c + 3]);
              pk.z = pack_bf16x2(f[8 * c + 4], f[8 * c + 5]);
              pk.w = pack_bf16x2(f[8 * c + 6], f[8 * c + 7]);
              *reinterpret_cast<uint4*>(arow + sw128_offset(row, u * (F / 8) + c)) = pk;
            }
          }
        } else {
          const float* tab_s = tabs + s * IPK * kTabIn;
#pragma unroll
          for (int u = 0; u < IPK; ++u) {
            // zero the input's F columns, then scatter the BK+1 supported splines and silu
#pragma unroll
            for (int c = 0; c < F / 8; ++c) *reinterpret_cast<uint4*>(arow + sw128_offset(row, u * (F / 8) + c)) = make_uint4(0, 0, 0, 0);
            if (i0 + u >= p.I) continue;
            const float* tu = tab_s + u * kTabIn;
            const int j0 = knot_interval(xv[u], tu, p.bd.nk);
            if (j0 >= 0) {
              float v[BK + 1];
              bspline_local_tab<BK>(xv[u], tu, p.bd.nk, j0, 0, v);
#pragma unroll
              for (int rp = 0; rp <= BK; ++rp) {
                const int r = j0 - BK + rp;
                if (r >= 0 && r < p.bd.nt) {
                  const int col = u * F + r;
                  *reinterpret_cast<__nv_bfloat16*>(arow + sw128_offset(row, col >> 3) + (col & 7) * 2) = __float2bfloat16_rn(v[rp]);
                }
              }
            }
            if (p.bd.has_base) {
              const int col = u * F + F - 1;
              *reinterpret_cast<__nv_bfloat16*>(arow + sw128_offset(row, col >> 3) + (col & 7) * 2) = __float2bfloat16_rn(silu_fast(xv[u]));
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (emit) {
          // the stage as the four warps wrote it (128 rows x 64 columns, 128-byte
          // swizzle, the layout of tmap_a's box); rows past B are not stored
          named_bar(2 + grp, 128);
          if (group_lead) tma_store_2d(&tmap_a, arow, k * kBK, (int)((int64_t)m * kPairM + rank * kBM));
          store_pending = true;
        }
        if (lane == 0) {
          if (rank == 0)
            mbar_arrive(&ctl->full_a[s]);
          else
            mbar_arrive_peer(&ctl->full_a[s], 0);
        }
#pragma unroll
        for (int u = 0; u < IPK; ++u) xa[u] = xb[u];
      }
      it += p.k_steps;
    }
    if (group_lead && p.feat_out != nullptr) bulk_wait_all();  // shared memory stays until the stores are done
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or MMA of the pair is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ===========================================================================
// DGRAD
// ===========================================================================

struct DgradParams {
  const __nv_bfloat16* x;
  __nv_bfloat16* dx;
  int64_t B;
  int I, O;
  int k_steps;
  int tab_ts;  // B-spline: row stride of the staged knot tables (nk rounded up to 4)
  TileMap tiles;
  BasisDev bd;
  // GR-KAN (BK = kRationalBK): R = P / (1 + |Q|) of degrees (5, 4), parameters
  // shared by ipg consecutive inputs (ipg a multiple of 32)
  const float* rnum;  // (groups, 6)
  const float* rden;  // (groups, 4)
  int ipg;
  float* rws;  // parameter-gradient partial sums [10][I / 32][n_rq]
  int n_rq;    // 32-row blocks: 8 per pair tile of 256 rows (those past B hold zeros)
  ConvDev conv;  // active: x is an image read through the implicit patch matrix (dx is still (B, I))
};

// Template value of BK that selects the GR-KAN epilogue of the input-gradient
// kernel: the accumulator holds dR = dy W (one column per input), the
// epilogue writes dx = dR R'(x) and the per-group parameter-gradient partial
// sums of R = P / (1 + |Q|) (kanforge/bases/rational.py:84-101,
// kanforge/torch/layers.py:335-363).
constexpr int kRationalBK = -1;
constexpr int kRatNA = 6, kRatNB = 4;  // the GR-KAN degrees (5, 4)

// Threads of the input-gradient kernel: w0 TMA, w1 MMA (CTA 0), then the
// epilogue warps from w4 on: two sets of four for Chebyshev features, four
// sets of four for B-splines and the GR-KAN rational (whose per-input
// derivative windows / rational backward are the epilogue's main cost).
constexpr int dgrad_threads(int bk) { return (bk > 0 || bk == kRationalBK) ? 640 : 384; }
// Pipeline depth: six stages of 32 KB where the epilogue's shared memory
// leaves room (deeper buffering hides the TMA latency of operands read from
// DRAM); B-spline plans keep four for their knot tables and staging.
constexpr int dgrad_stages(int bk) { return bk > 0 ? kStages : kMaxStages; }

// The input gradient runs on CTA pairs: a tile is 256 tokens x 256 feature
// columns, CTA r loads dy rows 128 r .. 128 r + 127 (its half of A) and
// packed columns 128 r .. 128 r + 127 (its half of B), both completing on CTA
// 0's barrier, and each CTA's epilogue contracts its own 128 accumulator rows
// with the derivative features.
template <int BK, int F>
__global__ void __launch_bounds__(dgrad_threads(BK), 1) fused_dgrad_kernel(const __grid_constant__ CUtensorMap tmap_dy,
                                                                           const __grid_constant__ CUtensorMap tmap_c, DgradParams p) {
  constexpr int NS = dgrad_stages(BK);
  constexpr int IPT = BK == kRationalBK ? kBN : kBN / F;  // inputs per tile
  constexpr int kEpiWarps = dgrad_threads(BK) / 32 - 4;
  constexpr int kEpiThreads = 32 * kEpiWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* sa = base;
  uint8_t* sb = sa + NS * kATile;                  // NS x 16 KB (this CTA's half of B)
  Ctl* ctl = reinterpret_cast<Ctl*>(sb + NS * kBHalf);
  float* xsm = reinterpret_cast<float*>(ctl + 1);       // Chebyshev: x of each row's tile inputs [128][IPT + 1]
  float* tabs = reinterpret_cast<float*>(ctl + 1);      // B-spline: knot tables [2][IPT][BK+1][tab_ts]
  float* stage = tabs + 2 * IPT * (BK + 1) * p.tab_ts;  // B-spline: per epilogue warp [32][F + 1]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2, n_pairs = gridDim.x / 2;
  volatile int* abort = &ctl->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctl->full_b[s], 1);  // CTA 0's expect_tx for both CTAs' A and B halves (used in CTA 0)
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 2 * kEpiWarps);  // the epilogue warps of both CTAs (used in CTA 0)
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_dy);
    prefetch_tmap(&tmap_c);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int n_tiles = p.tiles.count();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs) {
        int m, n;
        p.tiles.get(t, m, n);
        const int a_row = m * kPairM + (int)rank * kBM;
        const int b_col = n * kBN + (int)rank * (kBN / 2);
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!mbar_wait(&ctl->empty[s], ph ^ 1, abort)) break;
          if (rank == 0) {
            mbar_arrive_expect_tx(&ctl->full_b[s], 2 * (kATile + kBHalf));  // both CTAs' loads complete here
            // A: dy rows, K = o (K-major, 128 x 64)
            tma_load_2d(sa + s * kATile, &tmap_dy, &ctl->full_b[s], k * kBK, a_row);
            // B: packed[o, feature columns] as MN-major 64 x 64 boxes
#pragma unroll
            for (int c = 0; c < kBN / 128; ++c)
              tma_load_2d(sb + s * kBHalf + c * 8192, &tmap_c, &ctl->full_b[s], b_col + c * 64, k * kBK);
          } else {
            tma_load_2d_pair(sa + s * kATile, &tmap_dy, &ctl->full_b[s], 0, k * kBK, a_row);
#pragma unroll
            for (int c = 0; c < kBN / 128; ++c)
              tma_load_2d_pair(sb + s * kBHalf + c * 8192, &tmap_c, &ctl->full_b[s], 0, b_col + c * 64, k * kBK);
          }
        }
      }
      // Abort: CTA 0 drains the loads of both CTAs (they complete on its
      // barriers) before the pair's final cluster barrier.
      if (*abort && rank == 0) drain_tma<NS>(ctl, it);
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kPairM, kBN, false, true);
      int it = 0, tc = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs, ++tc) {
        const int acc = tc & 1;
        if (!mbar_wait_cluster(&ctl->acc_empty[acc], ((tc >> 1) & 1) ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kBN;
        bool ok = true;
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!mbar_wait_cluster(&ctl->full_b[s], ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + s * kATile), b0 = smem_u32(sb + s * kBHalf);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            mma_bf16_pair(d_tmem, smem_desc_sw128(a0 + 32 * j, 16, 1024), smem_desc_sw128(b0 + 2048 * j, 8192, 1024), idesc,
                          (k > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit_pair(&ctl->empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&ctl->acc_full[acc], 0x3);
      }
      // Every MMA of the pair has completed (and every commit above has
      // arrived) once the drain barrier flips: the pair may then exit.
      mma_commit_pair(&ctl->drain, 0x1);
      mbar_drain(&ctl->drain, 0);
    }
  } else if (warp >= 4) {
    if constexpr (BK == kRationalBK) {
      // GR-KAN: four sets of four warps; set `set` reads TMEM lane quarter q
      // (rows 32 q ..) of column chunks 2 set and 2 set + 1, each chunk 32
      // inputs of one parameter group, in halves of 16 columns.  Per half a
      // thread loads its row's 16 x values, evaluates the rational backward in
      // float2 lanes and writes dx; per chunk the warp sums the parameter-
      // gradient terms over its 32 rows (a fixed shuffle tree) into rws.
      const int q = (warp - 4) % 4, set = (warp - 4) / 4;
      const int row = q * 32 + lane;
      const int n_chunks = p.I / 32;
      int g_cur = -1;
      float2 ca[kRatNA], cb[kRatNB];
      int tc = 0;
      for (int t = pair; t < n_tiles; t += n_pairs, ++tc) {
        int m, n;
        p.tiles.get(t, m, n);
        const int acc = tc & 1;
        const int64_t b = (int64_t)m * kPairM + (int64_t)rank * kBM + row;
        const bool row_ok = b < p.B;
        const int rq = (m * 2 + (int)rank) * 4 + q;  // this warp's 32-row block
        const uint4* xrow = reinterpret_cast<const uint4*>(p.x + (row_ok ? b : 0) * p.I);
        uint4* dxrow = reinterpret_cast<uint4*>(p.dx + (row_ok ? b : 0) * p.I);
        if (!mbar_wait_warp(&ctl->acc_full[acc], (tc >> 1) & 1, abort)) break;
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * set + cc;
          const int i0 = n * kBN + c * 32;
          const bool chunk_ok = i0 < p.I;  // warp-uniform
          if (chunk_ok && i0 / p.ipg != g_cur) {
            g_cur = i0 / p.ipg;
#pragma unroll
            for (int j = 0; j < kRatNA; ++j) ca[j] = dup2(__ldg(p.rnum + g_cur * kRatNA + j));
#pragma unroll
            for (int j = 0; j < kRatNB; ++j) cb[j] = dup2(__ldg(p.rden + g_cur * kRatNB + j));
          }
          float2 acc_a[kRatNA], acc_b[kRatNB];
#pragma unroll
          for (int j = 0; j < kRatNA; ++j) acc_a[j] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < kRatNB; ++j) acc_b[j] = make_float2(0.0f, 0.0f);
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int ih = i0 + 16 * h;
            uint4 xq[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) xq[k] = (row_ok && chunk_ok) ? __ldg(xrow + ih / 8 + k) : make_uint4(0, 0, 0, 0);
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + acc * kBN + c * 32 + 16 * h, v);
            if (cc == 1 && h == 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
            }
            if (!chunk_ok) continue;
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(xq);
            uint32_t out[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float2 xv = make_float2(__uint_as_float(xw[k] << 16), __uint_as_float(xw[k] & 0xffff0000u));
              const float2 d = rat_bwd_pair(xv, make_float2(v[2 * k], v[2 * k + 1]), ca, cb, acc_a, acc_b);
              out[k] = pack_bf16x2(d.x, d.y);
            }
            if (row_ok) {
              dxrow[ih / 8] = make_uint4(out[0], out[1], out[2], out[3]);
              dxrow[ih / 8 + 1] = make_uint4(out[4], out[5], out[6], out[7]);
            }
          }
          if (!chunk_ok) continue;
          float ps[kRatNA + kRatNB];
#pragma unroll
          for (int j = 0; j < kRatNA; ++j) ps[j] = acc_a[j].x + acc_a[j].y;
#pragma unroll
          for (int j = 0; j < kRatNB; ++j) ps[kRatNA + j] = acc_b[j].x + acc_b[j].y;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
            for (int j = 0; j < kRatNA + kRatNB; ++j) ps[j] += __shfl_xor_sync(0xffffffffu, ps[j], off);
          }
          if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kRatNA + kRatNB; ++j) p.rws[((size_t)j * n_chunks + i0 / 32) * p.n_rq + rq] = ps[j];
          }
        }
      }
    } else if constexpr (is_closed(BK)) {
      // Two sets of four warps: set h2 reads TMEM lane quarter q (rows 32 q ..) of
      // column chunks 4 h2 .. 4 h2 + 3, i.e. the inputs IPT/2 h2 .. of the tile,
      // and writes those inputs' dx.
      constexpr int kHalfIn = IPT / 2;
      const int q = (warp - 4) % 4, h2 = (warp - 4) / 4;
      const int row = q * 32 + lane;
      const int etid = (warp - 4) * 32 + lane;  // 0 .. 255
      float* wst = stage + (warp - 4) * (32 * 33);
      int tc = 0;
      for (int t = pair; t < n_tiles; t += n_pairs, ++tc) {
        int m, n;
        p.tiles.get(t, m, n);
        const int i_base = n * IPT;
        const int acc = tc & 1;
        bool ok = mbar_wait_warp(&ctl->acc_full[acc], (tc >> 1) & 1, abort);
        if constexpr (BK > 0) {
          // all eight warps are past the previous tile (its table readers are done) and agree
          ok = named_bar_and(1, 256, ok);
          if (ok) {
            constexpr int kTab = (BK + 1) * kTabStride;  // knots and reciprocal differences of one input
            for (int e = etid; e < IPT * kTab; e += 256) {
              const int u = e / kTab, r = e % kTab;
              tabs[e] = (i_base + u < p.I) ? __ldg(p.bd.tab + (size_t)(i_base + u) * kTab + r) : 0.0f;
            }
          }
          named_bar(1, 256);
        }
        if (!ok) break;
        tc_fence_after();
        const int64_t b = (int64_t)m * kPairM + (int64_t)rank * kBM + row;
        const bool row_ok = b < p.B;
        // this row's x for this set's inputs, loaded once (4-byte loads when aligned)
        const int u0 = h2 * kHalfIn;
        float* xr = xsm + row * (IPT + 1);
        if (p.conv.active) {
          for (int u = u0; u < u0 + kHalfIn; ++u)
            xr[u] = (row_ok && i_base + u < p.I) ? x_value(p.x, p.conv, b, i_base + u, p.I) : 0.0f;
        } else if (row_ok && i_base + u0 + kHalfIn <= p.I && ((p.I | i_base) % 2) == 0) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(p.x + b * p.I + i_base + u0);
  #pragma unroll
          for (int k2 = 0; k2 < kHalfIn / 2; ++k2) {
            const uint32_t wv = __ldg(src + k2);
            xr[u0 + 2 * k2] = __uint_as_float(wv << 16);
            xr[u0 + 2 * k2 + 1] = __uint_as_float(wv & 0xffff0000u);
          }
        } else {
          for (int u = u0; u < u0 + kHalfIn; ++u)
            xr[u] = (row_ok && i_base + u < p.I) ? __bfloat162float(p.x[b * p.I + i_base + u]) : 0.0f;
        }
        float dxv[kHalfIn];  // this set's inputs u0 .. u0 + kHalfIn - 1 (static indices: the chunk loop unrolls)
  #pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * h2 + cc;
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kBN + c * 32, v);
          if (cc == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
          }
          if constexpr (is_closed(BK)) {
  #pragma unroll
            for (int h = 0; h < 32 / F + (F > 32 ? 1 : 0); ++h) {
              // F == 16: two inputs per chunk; F == 32: one input per chunk
              const int u = (c * 32) / F + h;
              const float xval = xr[u];
              float df[F];
              closed_drow<BK, F>(xval, p.bd, df);
              float s = 0.0f;
  #pragma unroll
              for (int j = 0; j < F; ++j) s = fmaf(v[h * F + j], df[j], s);
              dxv[(cc * 32) / F + h] = s;
            }
          } else {
            // stage the 32 columns of this row, then dot with the local derivative window
  #pragma unroll
            for (int j = 0; j < 32; ++j) wst[lane * 33 + j] = v[j];
            __syncwarp();
  #pragma unroll
            for (int h = 0; h < 32 / F; ++h) {
              const int u = (c * 32) / F + h;
              const int i = i_base + u;
              float s = 0.0f;
              if (row_ok && i < p.I) {
                const float xval = xr[u];
                const float* tu = tabs + u * ((BK + 1) * kTabStride);
                const int j0 = knot_interval(xval, tu, p.bd.nk);
                if (j0 >= 0) {
                  float dv[BK + 1];
                  // derivative step of kanforge/bases/spline.py:86-91 with the reciprocal differences of the table
                  bspline_local_tab<BK>(xval, tu, p.bd.nk, j0, 1, dv);
  #pragma unroll
                  for (int rp = 0; rp <= BK; ++rp) {
                    const int r = j0 - BK + rp;
                    if (r >= 0 && r < p.bd.nt) s = fmaf(wst[lane * 33 + h * F + r], dv[rp], s);
                  }
                }
                if (p.bd.has_base) s = fmaf(wst[lane * 33 + h * F + F - 1], dsilu_fast(xval), s);
              }
              dxv[(cc * 32) / F + h] = s;
            }
            __syncwarp();
          }
        }
        if (row_ok) {
          __nv_bfloat16* dst = p.dx + b * p.I + i_base + u0;
          if (i_base + u0 + kHalfIn <= p.I && ((p.I | i_base) % 2) == 0) {
  #pragma unroll
            for (int k2 = 0; k2 < kHalfIn / 2; ++k2) {
              const float lo = dxv[2 * k2], hi = dxv[2 * k2 + 1];
              reinterpret_cast<uint32_t*>(dst)[k2] = pack_bf16x2(lo, hi);
            }
          } else {
  #pragma unroll
            for (int k = 0; k < kHalfIn; ++k)
              if (i_base + u0 + k < p.I) p.dx[b * p.I + i_base + u0 + k] = __float2bfloat16_rn(dxv[k]);
          }
        }
      }
    } else {
      // B-spline: four sets of four warps; set `set` reads TMEM lane quarter q
      // (rows 32 q ..) of column chunks 2 set, 2 set + 1, i.e. the kSetIn
      // inputs IPT/4 set .. of the tile, and writes those inputs' dx.
      constexpr int kSetIn = IPT / 4;  // inputs per set
      constexpr int kIPC = 32 / F;     // inputs per 32-column chunk
      const int q = (warp - 4) % 4, set = (warp - 4) / 4;
      const int row = q * 32 + lane;
      const int etid = (warp - 4) * 32 + lane;  // 0 .. 511
      float* wst = stage + (warp - 4) * (32 * (F + 1));
      // tile t's knot tables (IPT inputs x (BK + 1) rows x tab_ts floats, zero
      // past I) go to buffer t % 2 by 16-byte cp.async, issued one tile ahead
      // so that the copy overlaps the previous tile's epilogue
      const int ts = p.tab_ts, tab_in = (BK + 1) * p.tab_ts;
      auto stage_tables = [&](int t, int buf) {
        int m2, n2;
        p.tiles.get(t, m2, n2);
        const int ib = n2 * IPT;
        float* dstb = tabs + buf * (IPT * tab_in);
        const int c4 = ts / 4, per_in = (BK + 1) * c4;
        for (int e = etid; e < IPT * per_in; e += kEpiThreads) {
          const int u = e / per_in, rem = e % per_in;
          const int qq = rem / c4, cc = rem % c4;
          const bool in_ok = ib + u < p.I;
          const float* src = p.bd.tab + (size_t)(in_ok ? ib + u : 0) * ((BK + 1) * kTabStride) + qq * kTabStride + cc * 4;
          cp_async16(dstb + u * tab_in + qq * ts + cc * 4, src, in_ok);
        }
        cp_async_commit();
      };
      if (pair < n_tiles) stage_tables(pair, 0);
      int tc = 0;
      for (int t = pair; t < n_tiles; t += n_pairs, ++tc) {
        int m, n;
        p.tiles.get(t, m, n);
        const int i_base = n * IPT;
        const int acc = tc & 1;
        bool ok = mbar_wait_warp(&ctl->acc_full[acc], (tc >> 1) & 1, abort);
        cp_async_wait_all();
        // every warp's table copies for this tile have landed, every warp is
        // past the previous tile (its buffer is free again), and all agree
        ok = named_bar_and(1, kEpiThreads, ok);
        if (ok && t + n_pairs < n_tiles) stage_tables(t + n_pairs, (tc + 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const int64_t b = (int64_t)m * kPairM + (int64_t)rank * kBM + row;
        const bool row_ok = b < p.B;
        const int u0 = set * kSetIn;
        const bool pairs_ok = row_ok && i_base + u0 + kSetIn <= p.I && ((p.I | i_base) % 2) == 0;
        // this row's x for the set's inputs (4-byte loads when aligned)
        float xv[kSetIn];
        if (p.conv.active) {
#pragma unroll
          for (int u = 0; u < kSetIn; ++u)
            xv[u] = (row_ok && i_base + u0 + u < p.I) ? x_value(p.x, p.conv, b, i_base + u0 + u, p.I) : 0.0f;
        } else if (pairs_ok) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(p.x + b * p.I + i_base + u0);
#pragma unroll
          for (int k2 = 0; k2 < kSetIn / 2; ++k2) {
            const uint32_t wv = __ldg(src + k2);
            xv[2 * k2] = __uint_as_float(wv << 16);
            xv[2 * k2 + 1] = __uint_as_float(wv & 0xffff0000u);
          }
        } else {
#pragma unroll
          for (int u = 0; u < kSetIn; ++u)
            xv[u] = (row_ok && i_base + u0 + u < p.I) ? __bfloat162float(p.x[b * p.I + i_base + u0 + u]) : 0.0f;
        }
        // the derivative windows of the set's inputs, side by side: a
        // fixed-step knot search (the largest r <= nk - 2 with t_r <= x) and
        // the derivative step of kanforge/bases/spline.py:86-91 from the staged
        // reciprocal differences
        const float* tb = tabs + (tc & 1) * (IPT * tab_in) + u0 * tab_in;
        const int nk = p.bd.nk;
        int pos[kSetIn];
        bool live[kSetIn], in_ok[kSetIn];
#pragma unroll
        for (int u = 0; u < kSetIn; ++u) {
          const float* tu = tb + u * tab_in;
          in_ok[u] = row_ok && i_base + u0 + u < p.I;
          live[u] = in_ok[u] && xv[u] >= tu[0] && xv[u] < tu[nk - 1];
          pos[u] = 0;
        }
        for (int st = pow2_floor(nk - 2); st > 0; st >>= 1) {
#pragma unroll
          for (int u = 0; u < kSetIn; ++u) {
            const int c = pos[u] + st;
            if (c <= nk - 2 && tb[u * tab_in + c] <= xv[u]) pos[u] = c;
          }
        }
        float dv[kSetIn][BK + 1], dsl[kSetIn];
#pragma unroll
        for (int u = 0; u < kSetIn; ++u) {
          bspline_local_tab<BK>(xv[u], tb + u * tab_in, nk, pos[u], 1, dv[u], ts);
          dsl[u] = (p.bd.has_base && in_ok[u]) ? dsilu_fast(xv[u]) : 0.0f;
        }
        float dxl[kSetIn];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kBN + (2 * set + cc) * 32, v);
          if (cc == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
          }
#pragma unroll
          for (int h = 0; h < kIPC; ++h) {
            const int ul = cc * kIPC + h;
            // stage this input's F columns of the row, then dot with its window
#pragma unroll
            for (int j = 0; j < F; ++j) wst[lane * (F + 1) + j] = v[h * F + j];
            __syncwarp();
            float s = 0.0f;
#pragma unroll
            for (int rp = 0; rp <= BK; ++rp) {
              const int r = pos[ul] - BK + rp;
              if (live[ul] && r >= 0 && r < p.bd.nt) s = fmaf(wst[lane * (F + 1) + r], dv[ul][rp], s);
            }
            if (p.bd.has_base && in_ok[ul]) s = fmaf(wst[lane * (F + 1) + F - 1], dsl[ul], s);
            dxl[ul] = s;
            __syncwarp();
          }
        }
        if (row_ok) {
          __nv_bfloat16* dst = p.dx + b * p.I + i_base + u0;
          if (pairs_ok) {
#pragma unroll
            for (int k2 = 0; k2 < kSetIn / 2; ++k2) reinterpret_cast<uint32_t*>(dst)[k2] = pack_bf16x2(dxl[2 * k2], dxl[2 * k2 + 1]);
          } else {
#pragma unroll
            for (int u = 0; u < kSetIn; ++u)
              if (i_base + u0 + u < p.I) dst[u] = __float2bfloat16_rn(dxl[u]);
          }
        }
      }
      cp_async_wait_all();  // no table copy lands after the loop (abort path)
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or MMA of the pair is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ===========================================================================
// WGRAD
// ===========================================================================

struct WgradParams {
  const __nv_bfloat16* x;
  const float* fold;     // (K, nt) or null
  const __nv_bfloat16* coef;   // (O, I, K): needed for the edge_scale gradient
  const __nv_bfloat16* scale;  // (O, I) edge_scale or null
  const __nv_bfloat16* mask;   // (O, I) edge_mask or null
  __nv_bfloat16* dcoef;  // (O, I, K)
  __nv_bfloat16* dbase;  // (O, I) or null
  __nv_bfloat16* dscale; // (O, I) or null
  int64_t B;
  int I, O, K;
  int k_steps;
  int x_tma;  // x tiles arrive by TMA with the dy tile (row pitch 16-byte aligned)
  int tab_stride;  // B-spline: row stride of the producers' private knot tables (>= nk)
  TileMap tiles;
  BasisDev bd;
  // split K (feature matrix by TMA, no fold / mask / scale / base): tile t of
  // split s = t / tiles.count() sums K steps [s ks, (s + 1) ks) and writes its
  // float32 partial (O, I K) block s of `part`; 1 = no split
  int n_split, ks;
  float* part;
  ConvDev conv;  // active: x is an image read through the implicit patch matrix
};

constexpr int kWgradThreads = 768;     // w0 TMA, w1 MMA (CTA 0), w4-7 epilogue, w8-23 producers (2 groups)
constexpr int kWgradTmaThreads = 256;  // A_TMA: w0 TMA, w1 MMA (CTA 0), w4-7 epilogue
constexpr int kXTile = kBK * 8 * 2;  // x tile per stage: 64 rows x 8 inputs bf16 = 1 KB
// Pipeline depth: five stages when both operands arrive by TMA, four with
// producer warps (their two groups own alternate K steps).
constexpr int wgrad_stages(bool a_tma) { return a_tma ? 5 : kStages; }

// The coefficient gradient runs on CTA pairs like the forward: a tile is 256
// feature rows (CTA r evaluates the features of inputs IPT r .. IPT r + IPT - 1
// of the pair's 2 IPT) x 256 outputs (CTA r loads dy columns 128 r .. 128 r +
// 127 of the tile), CTA 0 issues tcgen05.mma.cta_group::2 with M = 256, and
// each CTA's epilogue folds its own 128 accumulator rows.  The x tile a CTA's
// producers read completes on that CTA's own barrier (tab_full).
//
// A_TMA: the feature operand is not evaluated here but read by TMA from the
// (B, I*F) feature matrix of kf_features (tmap_x then maps that matrix), in the
// same MN-major swizzled layout; the kernel then has no producer warps and is
// a TMA-fed GEMM with the fold / chain-rule epilogue.
template <int BK, int F, bool A_TMA>
__global__ void __launch_bounds__(A_TMA ? kWgradTmaThreads : kWgradThreads, 1)
    fused_wgrad_kernel(const __grid_constant__ CUtensorMap tmap_dy, const __grid_constant__ CUtensorMap tmap_x,
                       WgradParams p) {
  constexpr int NS = wgrad_stages(A_TMA);
  constexpr int IPT = kBM / F;  // inputs per tile (rows of the feature operand)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* sa = base;
  uint8_t* sb = sa + NS * kATile;                           // NS x 16 KB (this CTA's half of dy)
  Ctl* ctl = reinterpret_cast<Ctl*>(sb + NS * kBHalf);
  uint8_t* sx = align1024(reinterpret_cast<uint8_t*>(ctl + 1));  // x tiles [stage][64 rows][8 inputs]
  float* stg = reinterpret_cast<float*>(sx + NS * kXTile);  // epilogue staging [128][33]
  float* tabs = stg + 128 * 33;                                   // B-spline: per producer warp [(BK+1) * ts]
  float* sfold = tabs + (BK > 0 ? 16 * (BK + 1) * p.tab_stride : 0);  // fold matrix [K][F], zero past nt
  __nv_bfloat16* sout = reinterpret_cast<__nv_bfloat16*>(sfold + 32 * 32);  // dcoef of a chunk [32][IPT * K]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2, n_pairs = gridDim.x / 2;
  volatile int* abort = &ctl->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctl->full_a[s], 16);   // the 8 warps of the owning producer group, in each CTA (used in CTA 0)
      mbar_init(&ctl->full_b[s], 1);    // CTA 0's expect_tx for both dy halves (and A_TMA: feature halves)
      mbar_init(&ctl->tab_full[s], 1);  // this CTA's x tile
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 8);  // 4 epilogue warps of each CTA (used in CTA 0)
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_dy);
    if (A_TMA || p.x_tma) prefetch_tmap(&tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int n_mn = p.tiles.count();
  const int n_tiles = n_mn * p.n_split;
  // tile t: output tile (m, n) of split t / n_mn, K steps [k0, k1)
  auto decode = [&](int t, int& m, int& n, int& k0, int& k1) {
    const int sp = t / n_mn;
    p.tiles.get(t - sp * n_mn, m, n);
    k0 = sp * p.ks;
    k1 = min(p.k_steps, k0 + p.ks);
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs) {
        int m, n, k0, k1;
        decode(t, m, n, k0, k1);
        const int x0 = ((m * 2 + (int)rank) * IPT) & ~7;  // TMA x coordinate rounded down to 16 bytes
        const int o0 = n * kBN + (int)rank * (kBN / 2);
        const int f0 = (m * 2 + (int)rank) * kBM;         // A_TMA: first feature column of this CTA
        for (int k = k0; k < k1; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!mbar_wait(&ctl->empty[s], ph ^ 1, abort)) break;
          if (!A_TMA && p.x_tma) {
            mbar_arrive_expect_tx(&ctl->tab_full[s], kXTile);
            tma_load_2d(sx + s * kXTile, &tmap_x, &ctl->tab_full[s], x0, k * kBK);
          }
          if (rank == 0) {
            // both CTAs' dy halves (and feature halves) complete here
            mbar_arrive_expect_tx(&ctl->full_b[s], 2 * kBHalf + (A_TMA ? 2 * kATile : 0));
#pragma unroll
            for (int c = 0; c < kBN / 128; ++c)
              tma_load_2d(sb + s * kBHalf + c * 8192, &tmap_dy, &ctl->full_b[s], o0 + c * 64, k * kBK);
            if constexpr (A_TMA) {
#pragma unroll
              for (int c = 0; c < kBM / 64; ++c)
                tma_load_2d(sa + s * kATile + c * 8192, &tmap_x, &ctl->full_b[s], f0 + c * 64, k * kBK);
            }
          } else {
#pragma unroll
            for (int c = 0; c < kBN / 128; ++c)
              tma_load_2d_pair(sb + s * kBHalf + c * 8192, &tmap_dy, &ctl->full_b[s], 0, o0 + c * 64, k * kBK);
            if constexpr (A_TMA) {
#pragma unroll
              for (int c = 0; c < kBM / 64; ++c)
                tma_load_2d_pair(sa + s * kATile + c * 8192, &tmap_x, &ctl->full_b[s], 0, f0 + c * 64, k * kBK);
            }
          }
        }
      }
      // Abort: CTA 0 drains the dy loads of both CTAs (they complete on its
      // barriers); each CTA drains its own x tiles.
      if (*abort) {
        if (rank == 0) drain_tma<NS>(ctl, it);
        if (p.x_tma) {
          for (int s = 0; s < NS; ++s) {
            const int last = it - 1 - ((it - 1 - s) % NS + NS) % NS;
            if (it > 0 && last >= 0) mbar_drain(&ctl->tab_full[s], (last / NS) & 1);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kPairM, kBN, true, true);  // both operands MN-major
      int it = 0, tc = 0;
      for (int t = pair; t < n_tiles && !*abort; t += n_pairs, ++tc) {
        int m, n, k0, k1;
        decode(t, m, n, k0, k1);
        const int acc = tc & 1;
        if (!mbar_wait_cluster(&ctl->acc_empty[acc], ((tc >> 1) & 1) ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kBN;
        bool ok = true;
        for (int k = k0; k < k1; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if ((!A_TMA && !mbar_wait_cluster(&ctl->full_a[s], ph, abort)) || !mbar_wait_cluster(&ctl->full_b[s], ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + s * kATile), b0 = smem_u32(sb + s * kBHalf);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            mma_bf16_pair(d_tmem, smem_desc_sw128(a0 + 2048 * j, 8192, 1024), smem_desc_sw128(b0 + 2048 * j, 8192, 1024), idesc,
                          (k > k0 || j > 0) ? 1u : 0u);
          }
          mma_commit_pair(&ctl->empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&ctl->acc_full[acc], 0x3);
      }
      // Every MMA of the pair has completed (and every commit above has
      // arrived) once the drain barrier flips: the pair may then exit.
      mma_commit_pair(&ctl->drain, 0x1);
      mbar_drain(&ctl->drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    const int q = warp - 4;
    const int mrow = q * 32 + lane;  // feature row (il, f) of this thread
    const int etid = mrow;
    const int K = p.K;
    for (int e = etid; e < K * F; e += 128) {
      const int kk = e / F, j = e % F;
      sfold[e] = (p.fold != nullptr && j < p.bd.nt) ? __ldg(p.fold + kk * p.bd.nt + j) : 0.0f;
    }
    int tc = 0;
    for (int t = pair; t < n_tiles; t += n_pairs, ++tc) {
      int m, n, k0, k1;
      decode(t, m, n, k0, k1);
      float* part = p.part ? p.part + (size_t)(t / n_mn) * p.O * ((size_t)p.I * p.K) : nullptr;
      const int i_base = (m * 2 + (int)rank) * IPT;
      const int n_u = min(IPT, p.I - i_base);  // inputs of this CTA's rows that exist
      const int row_len = n_u * K;              // bf16 of one output's contiguous dcoef slice
      const int acc = tc & 1;
      bool ok = mbar_wait_warp(&ctl->acc_full[acc], (tc >> 1) & 1, abort);
      if (!named_bar_and(1, 128, ok)) break;  // the four epilogue warps leave together
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * kBN + c * 32, v);
        if (c == kBN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(&ctl->acc_empty[acc], 0);
        }
        named_bar(1, 128);  // staging (stg, sout) free
#pragma unroll
        for (int j = 0; j < 32; ++j) stg[mrow * 33 + j] = v[j];
        named_bar(1, 128);
        // 32 outputs x IPT inputs, 128 threads; the input index runs fastest so
        // that neighbouring threads own neighbouring (o, i) edges.
        for (int pr = etid; pr < 32 * IPT; pr += 128) {
          const int u = pr % IPT, ol = pr / IPT;
          const int o = n * kBN + c * 32 + ol;
          const int i = i_base + u;
          if (o >= p.O || i >= p.I) continue;
          const float* dcol = stg + (u * F) * 33 + ol;  // dpacked[o, i, j] = dcol[j * 33]
          const int64_t e = (int64_t)o * p.I + i;
          if (part) {  // split K: this split's float32 partial, reduced by the caller's kernel
            float* dst = part + e * K;
            for (int kk = 0; kk < K; ++kk) dst[kk] = dcol[kk * 33];
            continue;
          }
          __nv_bfloat16* so = sout + ol * (IPT * K) + u * K;
          // C_eff = coef * scale * mask  =>  dcoef = dC_eff * scale * mask,
          // dscale = sum_k dC_eff * coef * mask; base_eff = base * mask (kanforge/torch/layers.py:162-167)
          const float mk = p.mask ? __bfloat162float(p.mask[e]) : 1.0f;
          const float sm = mk * (p.scale ? __bfloat162float(p.scale[e]) : 1.0f);
          const __nv_bfloat16* ce = p.coef + e * K;
          float dsc = 0.0f;
          if (is_closed(BK) && p.fold) {  // only Chebyshev-feature plans fold
            float d[F - 1];
#pragma unroll
            for (int j = 0; j < F - 1; ++j) d[j] = dcol[j * 33];
            for (int kk = 0; kk < K; ++kk) {
              const float* fr = sfold + kk * F;
              float dce = 0.0f;
#pragma unroll
              for (int j = 0; j < F - 1; ++j) dce = fmaf(d[j], fr[j], dce);
              so[kk] = __float2bfloat16_rn(dce * sm);
              if (p.dscale) dsc = fmaf(dce, __bfloat162float(ce[kk]), dsc);
            }
          } else {
            for (int kk = 0; kk < K; ++kk) {
              const float dce = dcol[kk * 33];
              so[kk] = __float2bfloat16_rn(dce * sm);
              if (p.dscale) dsc = fmaf(dce, __bfloat162float(ce[kk]), dsc);
            }
          }
          if (p.dscale) p.dscale[e] = __float2bfloat16_rn(dsc * mk);
          if (p.dbase) p.dbase[e] = __float2bfloat16_rn(dcol[(F - 1) * 33] * mk);
        }
        named_bar(1, 128);  // sout complete
        if (part) continue;
        // each output's slice (o, i_base .. i_base + n_u - 1, 0 .. K - 1) is
        // contiguous in dcoef: warp q copies rows q, q + 4, ..., lanes along the
        // row, in bf16 pairs when the row starts 4-byte aligned and is even.
        for (int ol = q; ol < 32; ol += 4) {
          const int o = n * kBN + c * 32 + ol;
          if (o >= p.O) break;
          const int64_t g0 = ((int64_t)o * p.I + i_base) * K;
          const __nv_bfloat16* src = sout + ol * (IPT * K);
          if (((g0 | row_len | (IPT * K)) & 1) == 0) {
            uint32_t* dst2 = reinterpret_cast<uint32_t*>(p.dcoef + g0);
            const uint32_t* src2 = reinterpret_cast<const uint32_t*>(src);
            for (int col = lane; col < row_len / 2; col += 32) dst2[col] = src2[col];
          } else {
            for (int col = lane; col < row_len; col += 32) p.dcoef[g0 + col] = src[col];
          }
        }
      }
    }
  } else if (!A_TMA && warp >= 8) {
    // producers: two groups of 8 warps own the K-steps of global parity 0 / 1.
    // F == 16 -> warp pw owns input u = pw of the tile's 8 inputs, each lane two
    // batch columns; F == 32 -> 4 inputs, warps 2u and 2u+1 split the 64 columns.
    const int grp = (warp - 8) / 8;
    const int pw = (warp - 8) % 8;
    const int u = (F == 16) ? pw : pw / 2;
    const int bsub = (F == 16) ? lane * 2 : (pw % 2) * 32 + lane;  // first batch column of this lane
    constexpr int NB = (F == 16) ? 2 : 1;
    const int ts = p.tab_stride;
    float* tab = tabs + (warp - 8) * ((BK + 1) * ts);
    int it = 0;
    bool alive = true;
    for (int t = pair; t < n_tiles && alive; t += n_pairs) {  // abort is seen (warp-uniformly) by the waits
      int m, n;
      p.tiles.get(t, m, n);
      const int i_base = (m * 2 + (int)rank) * IPT;
      const int i = i_base + u;
      const int xoff = i_base - (i_base & ~7) + u;  // column of input i inside the TMA x tile
      if constexpr (BK > 0) {
        __syncwarp();
        for (int e = lane; e < (BK + 1) * ts; e += 32) {
          const int q = e / ts, r = e % ts;
          tab[e] = (i < p.I && r < kTabStride) ? __ldg(p.bd.tab + (size_t)i * ((BK + 1) * kTabStride) + q * kTabStride + r) : 0.0f;
        }
        __syncwarp();
      }
      int k = ((it & 1) == grp) ? 0 : 1;
      for (; k < p.k_steps; k += 2) {
        const int git = it + k;
        const int s = git % NS;
        const uint32_t ph = (git / NS) & 1;
        float xv[2] = {0.0f, 0.0f};
        if (!p.x_tma) {
#pragma unroll
          for (int r = 0; r < NB; ++r) {
            const int64_t b = (int64_t)k * kBK + bsub + r;
            if (b < p.B && i < p.I) xv[r] = x_value(p.x, p.conv, b, i, p.I);
          }
        }
        bool ok = mbar_wait_warp(&ctl->empty[s], ph ^ 1, abort);
        if (p.x_tma) ok = ok && mbar_wait_warp(&ctl->tab_full[s], ph, abort);  // x tile landed
        if (!ok) {
          alive = false;
          break;
        }
        if (p.x_tma) {
          const __nv_bfloat16* xt = reinterpret_cast<const __nv_bfloat16*>(sx + s * kXTile);
#pragma unroll
          for (int r = 0; r < NB; ++r) xv[r] = __bfloat162float(xt[(bsub + r) * 8 + xoff]);
        }
        uint8_t* at = sa + s * kATile;
        float f[2][F];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int64_t b = (int64_t)k * kBK + bsub + r;
          const bool okr = r < NB && b < p.B && i < p.I;
#pragma unroll
          for (int j = 0; j < F; ++j) f[r][j] = 0.0f;
          if (!okr) continue;
          if constexpr (is_closed(BK)) {
            closed_row<BK, F>(xv[r], p.bd, f[r]);
          } else {
            const int j0 = knot_interval(xv[r], tab, p.bd.nk);
            float vv[BK + 1];
#pragma unroll
            for (int rp = 0; rp <= BK; ++rp) vv[rp] = 0.0f;
            if (j0 >= 0) bspline_local_tab<BK>(xv[r], tab, p.bd.nk, j0, 0, vv, ts);
#pragma unroll
            for (int j = 0; j < F; ++j) {
              float val = 0.0f;
#pragma unroll
              for (int rp = 0; rp <= BK; ++rp)
                if (j == j0 - BK + rp) val = vv[rp];
              f[r][j] = j < p.bd.nt ? val : 0.0f;
            }
            if (p.bd.has_base) f[r][F - 1] = silu_fast(xv[r]);
          }
        }
        // A[m = u*F + j][k = token], MN-major: 64-row chunks of m (8 KB apart),
        // each token a 128-byte swizzled row holding 64 consecutive m; the F
        // features of one (token, input) are F / 8 consecutive 16-byte granules.
        {
          const int m0 = u * F;
          uint8_t* chunk = at + (m0 / 64) * 8192;
          const int gr0 = (m0 % 64) / 8;
#pragma unroll
          for (int r = 0; r < NB; ++r) {
            const int kt = bsub + r;
#pragma unroll
            for (int g = 0; g < F / 8; ++g) {
              uint4 pk;
              pk.x = pack_bf16x2(f[r][8 * g + 0], f[r][8 * g + 1]);
              pk.y = pack_bf16x2(f[r][8 * g + 2], f[r][8 * g + 3]);
              pk.z = pack_bf16x2(f[r][8 * g + 4], f[r][8 * g + 5]);
              pk.w = pack_bf16x2(f[r][8 * g + 6], f[r][8 * g + 7]);
              *reinterpret_cast<uint4*>(chunk + sw128_offset(kt, gr0 + g)) = pk;
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0)
            mbar_arrive(&ctl->full_a[s]);
          else
            mbar_arrive_peer(&ctl->full_a[s], 0);
        }
      }
      it += p.k_steps;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or MMA of the pair is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ===========================================================================
// feature matrix for the coefficient gradient
// ===========================================================================

// feat[b, i*F + j] = feature j of x[b,i], bf16: the forward's basis row
// (Chebyshev T_j(g(x)) or the B-spline values, zero past nt) with silu(x) in
// column F - 1.
//
// Chebyshev: one thread per 16-byte chunk (8 features) of the output, so that
// a warp's store is 512 contiguous bytes; the F / 8 threads of one (b, i) each
// evaluate its (cheap) row and keep their own chunk.
template <int BK, int F>
__global__ void __launch_bounds__(256) feature_cheb_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ feat,
                                                           int64_t n, int I, BasisDev bd, ConvDev conv) {
  constexpr int CH = F / 8;
  const int64_t n_chunks = n * CH;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n_chunks; c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = c / CH;
    const int q = (int)(c % CH);
    float f[F];
    closed_row<BK, F>(conv.active ? x_value(x, conv, e / I, (int)(e % I), I) : __bfloat162float(x[e]), bd, f);
    float g[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      g[u] = f[u];
#pragma unroll
      for (int qq = 1; qq < CH; ++qq)
        if (q == qq) g[u] = f[8 * qq + u];
    }
    uint4 pk;
    pk.x = pack_bf16x2(g[0], g[1]);
    pk.y = pack_bf16x2(g[2], g[3]);
    pk.z = pack_bf16x2(g[4], g[5]);
    pk.w = pack_bf16x2(g[6], g[7]);
    reinterpret_cast<uint4*>(feat)[c] = pk;
  }
}

// B-splines: a CTA owns 32 consecutive inputs and stages their knot tables in
// shared memory once (rows of ts >= nk floats), element-major and lane-minor:
// element k of lane L's table at tabs[32 k + L], so each lane reads only its
// own bank whatever index it needs.  Its warps walk the rows, kSplineRows
// rows' x loaded together, each lane evaluating one (row, input) once: the
// kSplineRows knot searches side by side (fixed steps: the largest r <= nk - 2
// with t_r <= x), then Cox-de Boor from the table.  The BK + 1 non-zero values of a row start at feature s = j0 - BK:
// packed as bf16 pairs from an even position, a funnel shift by 16 bits moves
// them to an odd one, and the NW words they touch are placed among the row's
// F / 2 words; silu(x) is the high half of the last word.  Each lane stores
// its own row (F / 8 16-byte chunks).
constexpr int kSplineRows = 4;

__device__ __forceinline__ uint32_t bf16_bits(float v) { return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v)); }

template <int BK, int F>
__global__ void __launch_bounds__(256) feature_spline_kernel(const __nv_bfloat16* __restrict__ x,
                                                             __nv_bfloat16* __restrict__ feat, int64_t B, int I, BasisDev bd,
                                                             int ts, ConvDev conv) {
  constexpr int NW = (BK + 3) / 2;  // words that BK + 1 consecutive bf16 values can touch
  extern __shared__ float tabs[];   // [(BK + 1) * ts][32]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int i0 = blockIdx.y * 32;
  for (int e = threadIdx.x; e < 32 * (BK + 1) * ts; e += blockDim.x) {
    const int u = e / ((BK + 1) * ts), rem = e % ((BK + 1) * ts);
    const int q = rem / ts, r = rem % ts;
    tabs[rem * 32 + u] = (i0 + u < I) ? __ldg(bd.tab + (size_t)(i0 + u) * ((BK + 1) * kTabStride) + q * kTabStride + r) : 0.0f;
  }
  __syncthreads();
  const int i = i0 + lane;
  if (i >= I) return;
  const float* tu = tabs + lane;  // element k at tu[32 k]
  const int nk = bd.nk, top = pow2_floor(nk - 2);
  const float t_lo = tu[0], t_hi = tu[32 * (nk - 1)];
  const int64_t stride = (int64_t)gridDim.x * 8;
  for (int64_t b0 = (int64_t)blockIdx.x * 8 + warp; b0 < B; b0 += kSplineRows * stride) {
    float xs[kSplineRows];
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) {
      const int64_t b = b0 + u * stride;
      xs[u] = b < B ? x_value(x, conv, b, i, I) : 0.0f;
    }
    int pos[kSplineRows];
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) pos[u] = 0;
    for (int st = top; st > 0; st >>= 1) {
#pragma unroll
      for (int u = 0; u < kSplineRows; ++u) {
        const int c = pos[u] + st;
        if (c <= nk - 2 && tu[32 * c] <= xs[u]) pos[u] = c;
      }
    }
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) {
      const int64_t b = b0 + u * stride;
      if (b >= B) break;
      const float xv = xs[u];
      uint32_t wd[F / 2];
#pragma unroll
      for (int k = 0; k < F / 2; ++k) wd[k] = 0u;
      const int j0 = (xv >= t_lo && xv < t_hi) ? pos[u] : -1;
      if (j0 >= 0) {
        float vv[BK + 1];
        bspline_local_tab<BK, 32>(xv, tu, nk, j0, 0, vv, 32 * ts);
        const int s0 = j0 - BK;
        uint32_t h[2 * NW];
#pragma unroll
        for (int rp = 0; rp < 2 * NW; ++rp) {
          const int j = s0 + rp;
          h[rp] = (rp <= BK && j >= 0 && j < bd.nt) ? bf16_bits(vv[rp <= BK ? rp : 0]) : 0u;
        }
        const int par = s0 & 1, a = s0 >> 1;  // word a holds feature 2a (floor for s0 < 0)
        uint32_t w[NW];
#pragma unroll
        for (int m = 0; m < NW; ++m) {
          const uint32_t e = h[2 * m] | (h[2 * m + 1] << 16);
          const uint32_t ep = m > 0 ? (h[2 * m - 2] | (h[2 * m - 1] << 16)) : 0u;
          w[m] = par ? __funnelshift_l(ep, e, 16) : e;
        }
#pragma unroll
        for (int k = 0; k < F / 2; ++k) {
          const int m = k - a;
          uint32_t v = 0u;
#pragma unroll
          for (int mm = 0; mm < NW; ++mm)
            if (m == mm) v = w[mm];
          wd[k] = v;
        }
      }
      if (bd.has_base) wd[F / 2 - 1] |= bf16_bits(silu_fast(xv)) << 16;
      uint4* dst = reinterpret_cast<uint4*>(feat + (b * I + i) * F);
#pragma unroll
      for (int c = 0; c < F / 8; ++c) dst[c] = make_uint4(wd[4 * c], wd[4 * c + 1], wd[4 * c + 2], wd[4 * c + 3]);
    }
  }
}

// Float32 rows of the same B-spline features for the float32 tensor-core
// path: the tables, knot search and Cox-de Boor steps of
// feature_spline_kernel, the values placed among the row's F floats by
// selects, silu(x) (accurate exponential and division) in column F - 1, each
// lane storing its own row as float4s.
template <int BK, int F>
__global__ void __launch_bounds__(256) feature_spline_f32_kernel(const float* __restrict__ x, float* __restrict__ feat,
                                                                 int64_t B, int I, BasisDev bd, int ts) {
  extern __shared__ float tabs[];  // [(BK + 1) * ts][32]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int i0 = blockIdx.y * 32;
  for (int e = threadIdx.x; e < 32 * (BK + 1) * ts; e += blockDim.x) {
    const int u = e / ((BK + 1) * ts), rem = e % ((BK + 1) * ts);
    const int q = rem / ts, r = rem % ts;
    tabs[rem * 32 + u] = (i0 + u < I) ? __ldg(bd.tab + (size_t)(i0 + u) * ((BK + 1) * kTabStride) + q * kTabStride + r) : 0.0f;
  }
  __syncthreads();
  const int i = i0 + lane;
  if (i >= I) return;
  const float* tu = tabs + lane;  // element k at tu[32 k]
  const int nk = bd.nk, top = pow2_floor(nk - 2);
  const float t_lo = tu[0], t_hi = tu[32 * (nk - 1)];
  const int64_t stride = (int64_t)gridDim.x * 8;
  for (int64_t b0 = (int64_t)blockIdx.x * 8 + warp; b0 < B; b0 += kSplineRows * stride) {
    float xs[kSplineRows];
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) {
      const int64_t b = b0 + u * stride;
      xs[u] = b < B ? x[b * I + i] : 0.0f;
    }
    int pos[kSplineRows];
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) pos[u] = 0;
    for (int st = top; st > 0; st >>= 1) {
#pragma unroll
      for (int u = 0; u < kSplineRows; ++u) {
        const int c = pos[u] + st;
        if (c <= nk - 2 && tu[32 * c] <= xs[u]) pos[u] = c;
      }
    }
#pragma unroll
    for (int u = 0; u < kSplineRows; ++u) {
      const int64_t b = b0 + u * stride;
      if (b >= B) break;
      const float xv = xs[u];
      float f[F];
#pragma unroll
      for (int k = 0; k < F; ++k) f[k] = 0.0f;
      const int j0 = (xv >= t_lo && xv < t_hi) ? pos[u] : -1;
      if (j0 >= 0) {
        float vv[BK + 1];
        bspline_local_tab<BK, 32>(xv, tu, nk, j0, 0, vv, 32 * ts);
        const int s0 = j0 - BK;
#pragma unroll
        for (int k = 0; k < F - 1; ++k) {
          const int m = k - s0;
          float v = 0.0f;
#pragma unroll
          for (int mm = 0; mm <= BK; ++mm)
            if (m == mm) v = vv[mm];
          f[k] = k < bd.nt ? v : 0.0f;
        }
      }
      f[F - 1] = bd.has_base ? silu_acc(xv) : 0.0f;
      float4* dst = reinterpret_cast<float4*>(feat + (b * I + i) * F);
#pragma unroll
      for (int c = 0; c < F / 4; ++c) dst[c] = make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
    }
  }
}

// ===========================================================================
// host side
// ===========================================================================

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// 2-D bf16 tensor map: `rows` x `cols` row-major (cols contiguous), box box_cols x box_rows,
// 128-byte swizzle (or none).
int make_tmap_bf16(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows,
                   bool swizzle = true) {
  auto enc = get_encode();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return KF_ERR_CUDA;
  }
  KF_CHECK_ARG(((uintptr_t)ptr % 16) == 0, "TMA operand must be 16-byte aligned");
  KF_CHECK_ARG((cols * 2) % 16 == 0, "TMA operand row pitch (%lld bf16) must be a multiple of 16 bytes", (long long)cols);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for %lldx%lld box %dx%d", (int)r, (long long)rows, (long long)cols,
              box_rows, box_cols);
    return KF_ERR_CUDA;
  }
  return KF_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int fill_basis(const kf_basis_desc* d, const float* knot_tab, int nt, int has_base, int f_pad, BasisDev& bd) {
  KF_CHECK_ARG(d != nullptr, "basis is null");
  KF_CHECK_ARG(f_pad == 16 || f_pad == 32, "f_pad must be 16 or 32 (got %d)", f_pad);
  KF_CHECK_ARG(nt >= 1 && nt + 1 <= f_pad, "nt %d (+ the SiLU column) exceeds f_pad %d", nt, f_pad);
  bd.map = d->input_map;
  bd.nt = nt;
  bd.has_base = has_base;
  bd.tab = knot_tab;
  if (d->kind == KF_BASIS_BSPLINE) {
    KF_CHECK_ARG(knot_tab != nullptr, "B-spline needs its knot tables (kf_knot_tables)");
    KF_CHECK_ARG(((uintptr_t)knot_tab % 16) == 0, "knot tables must be 16-byte aligned");
    KF_CHECK_ARG(d->order >= 1 && d->order <= kMaxOrder, "B-spline order %d unsupported", d->order);
    bd.G = d->grid_size;
    bd.nk = d->grid_size + 2 * d->order + 1;
    KF_CHECK_ARG(bd.nk <= kTabStride, "B-spline with %d knots exceeds %d", bd.nk, kTabStride);
    KF_CHECK_ARG(nt == d->size, "B-spline nt %d must equal the basis size %d", nt, d->size);
  } else if (d->kind == KF_BASIS_FOURIER) {
    KF_CHECK_ARG(d->period > 0.0f && d->size % 2 == 0 && nt == d->size, "Fourier: period > 0 and nt = size (even)");
    bd.w1 = 6.283185307179586f / d->period;
    bd.nfreq = d->size / 2;
  } else if (d->kind != KF_BASIS_CHEB) {
    set_error("fused kernels support B-spline, Chebyshev-feature and Fourier bases");
    return KF_ERR_UNSUPPORTED;
  }
  return KF_OK;
}

template <typename Fn>
int dispatch_fused(const kf_basis_desc* d, int f_pad, Fn&& fn) {
  if (d->kind == KF_BASIS_CHEB) return f_pad == 16 ? fn.template go<0, 16>() : fn.template go<0, 32>();
  if (d->kind == KF_BASIS_FOURIER)
    return f_pad == 16 ? fn.template go<kFourierBK, 16>() : fn.template go<kFourierBK, 32>();
  if (d->kind != KF_BASIS_BSPLINE) {
    set_error("fused kernels: basis kind %d unsupported", d->kind);
    return KF_ERR_UNSUPPORTED;
  }
  switch (d->order) {
    case 1: return f_pad == 16 ? fn.template go<1, 16>() : fn.template go<1, 32>();
    case 2: return f_pad == 16 ? fn.template go<2, 16>() : fn.template go<2, 32>();
    case 3: return f_pad == 16 ? fn.template go<3, 16>() : fn.template go<3, 32>();
    case 4: return f_pad == 16 ? fn.template go<4, 16>() : fn.template go<4, 32>();
    case 5: return f_pad == 16 ? fn.template go<5, 16>() : fn.template go<5, 32>();
    default: break;
  }
  set_error("B-spline order %d unsupported", d->order);
  return KF_ERR_UNSUPPORTED;
}


// Shared memory of the pair kernels with ns stages of A (16 KB) and nb halves of B (16 KB each).
constexpr size_t pair_smem(int ns, int nb) { return 1024 + (size_t)ns * (kATile + nb * kBHalf) + sizeof(Ctl); }

// Largest number of co-resident CTA pairs for a cluster launch of `kern`
// (clusters of 2), cached per device in the caller's `cache`.
std::atomic<int> g_reserved_sms{0};

template <typename K>
int max_pairs(K kern, const cudaLaunchConfig_t& cfg, int (&cache)[64]) {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = (dev >= 0 && dev < 64) ? cache[dev] : 0;
  if (n <= 0) {
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    if (dev >= 0 && dev < 64) cache[dev] = n;
  }
  // SMs left to kernels that run beside the persistent grids (a collective
  // overlapping the backward): kf_set_reserved_sms
  const int reserved = g_reserved_sms.load(std::memory_order_relaxed);
  if (reserved > 0) n = std::max(1, std::min(n, (sm_count() - reserved) / 2));
  return n;
}

struct FwdLaunch {
  const CUtensorMap *tmap, *tmap_a;  // tmap_a maps the feature matrix when a_tma
  FwdParams p;
  bool a_tma;
  cudaStream_t stream;
  template <int BK, int F>
  int go() const {
    return a_tma ? launch<BK, F, true>() : launch<BK, F, false>();
  }
  // Six stages when both operands arrive by TMA into 256-output tiles (the
  // GR-KAN contractions), else four (producer groups own one stage each; a
  // 512-output stage is 48 KB).
  template <int BK, int F, bool A_TMA>
  int launch() const {
    if constexpr (A_TMA && BK == 0 && F == 16) {
      if (p.nblk == 1) return launch_ns<BK, F, A_TMA, kMaxStages>();
    }
    return launch_ns<BK, F, A_TMA, kStages>();
  }
  template <int BK, int F, bool A_TMA, int NS>
  int launch_ns() const {
    constexpr int IPK = kBK / F;
    const size_t smem = pair_smem(NS, p.nblk) + (BK > 0 && !A_TMA ? 1024 + sizeof(float) * NS * IPK * (BK + 1) * kTabStride : 0);
    auto kern = fused_fwd_kernel<BK, F, A_TMA, NS>;
    KF_CUDA_RET(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(A_TMA ? kFwdTmaThreads : kFwdThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (unsigned)(sm_count() / 2));
    static int pair_cache[64] = {0};  // per instantiation
    const int pairs = (int)std::min<int64_t>(p.tiles.m_tiles * (int64_t)p.tiles.n_tiles, max_pairs(kern, cfg, pair_cache));
    cfg.gridDim = dim3(2 * (unsigned)pairs);
    KF_CUDA_RET(cudaLaunchKernelEx(&cfg, kern, *tmap, *tmap_a, p));
    return check_launch("kf_fwd");
  }
};

struct DgradLaunch {
  const CUtensorMap *tmap_dy, *tmap_c;
  DgradParams p;
  cudaStream_t stream;
  template <int BK, int F>
  int go() const {
    constexpr int IPT = kBN / F;
    const size_t smem = pair_smem(dgrad_stages(BK), 1) + sizeof(float) * (BK > 0 ? 2 * IPT * (BK + 1) * p.tab_ts + 16 * 32 * (F + 1)
                                                      : is_closed(BK) ? kBM * (IPT + 1) : 0);
    auto kern = fused_dgrad_kernel<BK, F>;
    KF_CUDA_RET(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(dgrad_threads(BK));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (unsigned)(sm_count() / 2));
    static int pair_cache[64] = {0};  // per instantiation
    const int pairs = (int)std::min<int64_t>(p.tiles.m_tiles * (int64_t)p.tiles.n_tiles, max_pairs(kern, cfg, pair_cache));
    cfg.gridDim = dim3(2 * (unsigned)pairs);
    KF_CUDA_RET(cudaLaunchKernelEx(&cfg, kern, *tmap_dy, *tmap_c, p));
    return check_launch("kf_dgrad");
  }
};

struct WgradLaunch {
  const CUtensorMap *tmap_dy, *tmap_x;  // tmap_x maps the feature matrix when a_tma
  WgradParams p;
  bool a_tma;
  cudaStream_t stream;
  template <int BK, int F>
  int go() const {
    return a_tma ? launch<BK, F, true>() : launch<BK, F, false>();
  }
  template <int BK, int F, bool A_TMA>
  int launch() const {
    const size_t smem = pair_smem(wgrad_stages(A_TMA), 1) + 1024 + wgrad_stages(A_TMA) * kXTile +
                        sizeof(float) * (128 * 33 + (BK > 0 ? 16 * (BK + 1) * p.tab_stride : 0) + 32 * 32) +
                        sizeof(__nv_bfloat16) * 32 * 128;
    if (smem > 232448) {
      set_error("kf_wgrad: B-spline order %d with %d knots needs %zu bytes of shared memory", BK, p.bd.nk, smem);
      return KF_ERR_UNSUPPORTED;
    }
    auto kern = fused_wgrad_kernel<BK, F, A_TMA>;
    KF_CUDA_RET(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(A_TMA ? kWgradTmaThreads : kWgradThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (unsigned)(sm_count() / 2));
    static int pair_cache[64] = {0};  // per instantiation
    const int pairs = (int)std::min<int64_t>(p.tiles.m_tiles * (int64_t)p.tiles.n_tiles * p.n_split,
                                             max_pairs(kern, cfg, pair_cache));
    cfg.gridDim = dim3(2 * (unsigned)pairs);
    KF_CUDA_RET(cudaLaunchKernelEx(&cfg, kern, *tmap_dy, *tmap_x, p));
    return check_launch("kf_wgrad");
  }
};

struct FeatureLaunch {
  const __nv_bfloat16* x;
  __nv_bfloat16* feat;
  int64_t B;
  int I;
  BasisDev bd;
  cudaStream_t stream;
  ConvDev conv;
  template <int BK, int F>
  int go() const {
    if constexpr (is_closed(BK)) {
      const int64_t n = B * (int64_t)I;
      const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n * (F / 8), 256), (int64_t)sm_count() * 16);
      feature_cheb_kernel<BK, F><<<grid, 256, 0, stream>>>(x, feat, n, I, bd, conv);
    } else {
      const unsigned gy = (unsigned)cdiv(I, 32);
      const int64_t want = std::max<int64_t>(1, (int64_t)sm_count() * 8 / gy);
      const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(B, (int64_t)8), want));
      const int ts = (bd.nk + 15) & ~15;  // table row stride in shared memory (>= nk)
      const size_t smem = sizeof(float) * 32 * (BK + 1) * ts;
      KF_CUDA_RET(cudaFuncSetAttribute(feature_spline_kernel<BK, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      feature_spline_kernel<BK, F><<<dim3(gx, gy), 256, smem, stream>>>(x, feat, B, I, bd, ts, conv);
    }
    return check_launch("kf_features");
  }
};

struct FeatureF32SplineLaunch {
  const float* x;
  float* feat;
  int64_t B;
  int I;
  BasisDev bd;
  cudaStream_t stream;
  template <int BK, int F>
  int go() const {
    if constexpr (BK <= 0) {
      set_error("kf_features_f32: the knot-table kernel is for B-splines");
      return KF_ERR_UNSUPPORTED;
    } else {
      const unsigned gy = (unsigned)cdiv(I, 32);
      const int64_t want = std::max<int64_t>(1, (int64_t)sm_count() * 8 / gy);
      const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(B, (int64_t)8), want));
      const int ts = (bd.nk + 15) & ~15;  // table row stride in shared memory (>= nk)
      const size_t smem = sizeof(float) * 32 * (BK + 1) * ts;
      KF_CUDA_RET(cudaFuncSetAttribute(feature_spline_f32_kernel<BK, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
      feature_spline_f32_kernel<BK, F><<<dim3(gx, gy), 256, smem, stream>>>(x, feat, B, I, bd, ts);
      return check_launch("kf_features_f32");
    }
  }
};

// GR-KAN parameter gradients: dnum[g, j] (j < 6) and dden[g, j - 6] = the sum
// of the input-gradient epilogue's partial sums rws[j][chunk][rq] over the 32-row
// blocks rq and the group's 32-input chunks, which are cpg * n_rq consecutive
// floats; one CTA per (group, coefficient), fixed per-thread strides and a fixed
// tree, so the result is deterministic.
__global__ void __launch_bounds__(256) grkan_reduce_kernel(const float* __restrict__ rws, float* __restrict__ dnum,
                                                           float* __restrict__ dden, int n_chunks, int cpg, int n_rq) {
  __shared__ float red[256];
  constexpr int W = kRatNA + kRatNB;
  const int g = blockIdx.x / W, j = blockIdx.x % W;
  const float* src = rws + ((size_t)j * n_chunks + (size_t)g * cpg) * n_rq;
  const int64_t n = (int64_t)cpg * n_rq;
  float acc = 0.0f;
  for (int64_t e = threadIdx.x; e < n; e += 256) acc += src[e];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int st = 128; st > 0; st >>= 1) {
    if (threadIdx.x < st) red[threadIdx.x] += red[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (j < kRatNA) dnum[g * kRatNA + j] = red[0];
    else dden[g * kRatNB + (j - kRatNA)] = red[0];
  }
}

int grkan_check(const kf_basis_desc* d, int64_t B, int I, int O, const char* who) {
  KF_CHECK_ARG(d != nullptr && d->kind == KF_BASIS_RATIONAL, "%s: needs a rational basis", who);
  KF_CHECK_ARG(d->degree == kRatNA - 1 && d->den_degree == kRatNB, "%s: rational degrees (%d, %d), the kernel takes (5, 4)", who,
               d->degree, d->den_degree);
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1, "%s: bad sizes", who);
  KF_CHECK_ARG(d->groups >= 1 && I % d->groups == 0 && (I / d->groups) % 32 == 0,
               "%s: inputs per group (I %d / groups %d) must be a multiple of 32", who, I, d->groups);
  KF_CHECK_ARG(O % 8 == 0, "%s: O (%d) must be a multiple of 8", who, O);
  return KF_OK;
}

}  // namespace


}  // namespace kf

static int kf_fwd_impl(const kf::ConvDev* conv, const void* x, const void* feat, const void* packed, const void* bias, const float* knot_tab, void* y, int64_t B,
                      int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
                      void* stream, void* feat_out = nullptr) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && packed && y, "kf_fwd: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1, "kf_fwd: bad sizes");
  KF_CHECK_ARG(O % 8 == 0, "kf_fwd: O (%d) must be a multiple of 8", O);
  KF_CHECK_ARG(((uintptr_t)y % 16) == 0 && ((uintptr_t)bias % 16) == 0, "kf_fwd: y and bias must be 16-byte aligned");
  FwdParams p{};
  if (int rc = fill_basis(basis, knot_tab, nt, has_base, f_pad, p.bd)) return rc;
  if (B == 0) return KF_OK;
  p.x = (const __nv_bfloat16*)x;
  p.bias = (const __nv_bfloat16*)bias;
  p.y = (__nv_bfloat16*)y;
  p.B = B;
  p.I = I;
  p.O = O;
  const int ipk = kBK / f_pad;
  p.k_steps = (int)cdiv(I, ipk);
  p.tiles.m_tiles = (int)cdiv(B, kPairM);
  p.nblk = O > kBN ? kFwdNB : 1;
  p.tiles.n_tiles = (int)cdiv(O, p.nblk * kBN);
  // Without the feature matrix, M fastest: concurrent pairs share one
  // coefficient column block and nothing else is read.  With it, super-rows of
  // 8 M tiles, so that the pairs in flight share feature and coefficient blocks.
  p.tiles.gm = feat ? std::min(p.tiles.m_tiles, 8) : p.tiles.m_tiles;
  CUtensorMap tmap, tmap_a;
  if (int rc = make_tmap_bf16(&tmap, packed, O, (int64_t)I * f_pad, kBK, kBN / 2)) return rc;
  if (feat) {
    KF_CHECK_ARG(((uintptr_t)feat % 16) == 0, "kf_fwd: feat must be 16-byte aligned");
    if (int rc = make_tmap_bf16(&tmap_a, feat, B, (int64_t)I * f_pad, kBK, kBM)) return rc;
  } else {
    tmap_a = tmap;  // unused
  }
  if (conv) p.conv = *conv;
  if (feat_out) {
    KF_CHECK_ARG(!conv && !feat && (basis->kind == KF_BASIS_CHEB || basis->kind == KF_BASIS_FOURIER),
                 "kf_fwd_emit_features: Chebyshev-feature or Fourier plans of the plain layer only");
    KF_CHECK_ARG(((uintptr_t)feat_out % 16) == 0, "kf_fwd_emit_features: feat_out must be 16-byte aligned");
    p.feat_out = (__nv_bfloat16*)feat_out;
    // the producers store their A stages through this map (the box the TMA-fed forward loads)
    if (int rc = make_tmap_bf16(&tmap_a, feat_out, B, (int64_t)I * f_pad, kBK, kBM)) return rc;
  }
  FwdLaunch L{&tmap, &tmap_a, p, feat != nullptr, (cudaStream_t)stream};
  return dispatch_fused(basis, f_pad, L);
}

static int kf_dgrad_impl(const kf::ConvDev* conv, const void* x, const void* dy, const void* packed, const float* knot_tab, void* dx, int64_t B,
                        int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
                        void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && dy && packed && dx, "kf_dgrad: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1, "kf_dgrad: bad sizes");
  KF_CHECK_ARG(O % 8 == 0, "kf_dgrad: O (%d) must be a multiple of 8", O);
  DgradParams p{};
  if (int rc = fill_basis(basis, knot_tab, nt, has_base, f_pad, p.bd)) return rc;
  if (B == 0) return KF_OK;
  p.x = (const __nv_bfloat16*)x;
  p.dx = (__nv_bfloat16*)dx;
  p.B = B;
  p.I = I;
  p.O = O;
  p.k_steps = (int)cdiv(O, kBK);
  p.tiles.m_tiles = (int)cdiv(B, kPairM);
  p.tiles.n_tiles = (int)cdiv((int64_t)I * f_pad, kBN);
  // Super-rows of 16 pair M tiles: their dy panels (16 x 256 rows x O) stay
  // in L2 while the super-row streams every coefficient block once.  At the
  // 4096 Chebyshev layer (2 MB panels) 16 measured faster than 8, 32 and 64
  // (the L2 serves data shared by both dies at about half its capacity).
  p.tiles.gm = std::min(p.tiles.m_tiles, 16);
  p.tab_ts = (p.bd.nk + 3) & ~3;
  CUtensorMap tdy, tc;
  if (int rc = make_tmap_bf16(&tdy, dy, B, O, kBK, kBM)) return rc;
  if (int rc = make_tmap_bf16(&tc, packed, O, (int64_t)I * f_pad, 64, kBK)) return rc;
  if (conv) p.conv = *conv;
  DgradLaunch L{&tdy, &tc, p, (cudaStream_t)stream};
  return dispatch_fused(basis, f_pad, L);
}

extern "C" int kf_features_spline_f32(const float* x, const float* knot_tab, float* feat, int64_t B, int32_t I, int32_t nt,
                                      int32_t f_pad, int32_t has_base, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && feat, "kf_features_spline_f32: null tensor pointer");
  KF_CHECK_ARG(basis && basis->kind == KF_BASIS_BSPLINE, "kf_features_spline_f32: B-spline bases only");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1, "kf_features_spline_f32: bad sizes");
  KF_CHECK_ARG(((uintptr_t)feat % 16) == 0, "kf_features_spline_f32: feat must be 16-byte aligned");
  BasisDev bd{};
  if (int rc = fill_basis(basis, knot_tab, nt, has_base, f_pad, bd)) return rc;
  if (B == 0) return KF_OK;
  FeatureF32SplineLaunch L{x, feat, B, I, bd, (cudaStream_t)stream};
  return dispatch_fused(basis, f_pad, L);
}

static int kf_features_impl(const kf::ConvDev* conv, const void* x, const float* knot_tab, void* feat, int64_t B, int32_t I, int32_t nt,
                           int32_t f_pad, int32_t has_base, const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && feat, "kf_features: null tensor pointer");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1, "kf_features: bad sizes");
  KF_CHECK_ARG(((uintptr_t)feat % 16) == 0, "kf_features: feat must be 16-byte aligned");
  BasisDev bd{};
  if (int rc = fill_basis(basis, knot_tab, nt, has_base, f_pad, bd)) return rc;
  if (B == 0) return KF_OK;
  FeatureLaunch L{(const __nv_bfloat16*)x, (__nv_bfloat16*)feat, B, I, bd, (cudaStream_t)stream};
  if (conv) L.conv = *conv;
  return dispatch_fused(basis, f_pad, L);
}

static int kf_wgrad_impl(const kf::ConvDev* conv, const void* x, const void* feat, const void* dy, const float* knot_tab, const float* fold, const void* coef,
                        const void* edge_scale, const void* edge_mask, void* dcoef, void* dbase, void* dscale, int64_t B,
                        int32_t I, int32_t O, int32_t K, int32_t nt, int32_t f_pad, const kf_basis_desc* basis,
                        void* stream) {
  using namespace kf;
  clear_error();
  void* dcoef_eff = dcoef;
  KF_CHECK_ARG(x && dy && dcoef, "kf_wgrad: null tensor pointer");
  KF_CHECK_ARG(dscale == nullptr || (coef != nullptr && edge_scale != nullptr), "kf_wgrad: dscale needs coef and edge_scale");
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1 && K >= 1, "kf_wgrad: bad sizes");
  KF_CHECK_ARG(O % 8 == 0, "kf_wgrad: O (%d) must be a multiple of 8", O);
  KF_CHECK_ARG(fold != nullptr || K == nt, "kf_wgrad: without a fold K must equal nt");
  WgradParams p{};
  if (int rc = fill_basis(basis, knot_tab, nt, dbase != nullptr, f_pad, p.bd)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dcoef_eff, 0, sizeof(__nv_bfloat16) * (size_t)O * I * K, s));
    if (dbase) KF_CUDA_RET(cudaMemsetAsync(dbase, 0, sizeof(__nv_bfloat16) * (size_t)O * I, s));
    if (dscale) KF_CUDA_RET(cudaMemsetAsync(dscale, 0, sizeof(__nv_bfloat16) * (size_t)O * I, s));
    return KF_OK;
  }
  p.x = (const __nv_bfloat16*)x;
  p.fold = fold;
  p.coef = (const __nv_bfloat16*)coef;
  p.scale = (const __nv_bfloat16*)edge_scale;
  p.mask = (const __nv_bfloat16*)edge_mask;
  p.dcoef = (__nv_bfloat16*)dcoef_eff;
  p.dbase = (__nv_bfloat16*)dbase;
  p.dscale = (__nv_bfloat16*)dscale;
  p.B = B;
  p.I = I;
  p.O = O;
  p.K = K;
  p.k_steps = (int)cdiv(B, kBK);
  p.n_split = 1;
  p.ks = p.k_steps;
  const int ipt = kBM / f_pad;  // inputs per CTA of a pair tile
  p.tiles.m_tiles = (int)cdiv(I, 2 * ipt);
  p.tiles.n_tiles = (int)cdiv(O, kBN);
  // Without the feature matrix, M fastest: concurrent pairs share the dy column
  // block and nothing else is read.  With it, super-rows of 8 M tiles: the
  // pairs in flight share a few feature blocks and a few dy blocks, so neither
  // the 2 B I f_pad-byte feature matrix nor dy is re-read per output block.
  p.tiles.gm = feat ? std::min(p.tiles.m_tiles, 8) : p.tiles.m_tiles;
  CUtensorMap tdy, tx;
  if (int rc = make_tmap_bf16(&tdy, dy, B, O, 64, kBK)) return rc;
  if (conv) p.conv = *conv;
  p.x_tma = !conv && (I % 8 == 0) && ((uintptr_t)x % 16 == 0);  // an image is gathered, not tiled
  p.tab_stride = basis->kind == KF_BASIS_BSPLINE ? ((p.bd.nk + 15) & ~15) : 16;
  if (feat) {
    KF_CHECK_ARG(((uintptr_t)feat % 16) == 0, "kf_wgrad: feat must be 16-byte aligned");
    if (int rc = make_tmap_bf16(&tx, feat, B, (int64_t)I * f_pad, 64, kBK)) return rc;
  } else if (p.x_tma) {
    if (int rc = make_tmap_bf16(&tx, x, B, I, 8, kBK, false)) return rc;
  } else {
    tx = tdy;  // unused
  }
  WgradLaunch L{&tdy, &tx, p, feat != nullptr, s};
  return dispatch_fused(basis, f_pad, L);
}

extern "C" int kf_knot_tables(const float* grid, float* tab, int32_t I, int32_t grid_size, int32_t order, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(grid && tab && I >= 1 && grid_size >= 1, "kf_knot_tables: bad arguments");
  KF_CHECK_ARG(order >= 1 && order <= kMaxOrder && grid_size + 2 * order + 1 <= kTabStride,
               "kf_knot_tables: order %d / grid %d beyond the kernel limits", order, grid_size);
  if (int rc = bind_device(grid)) return rc;
  const int64_t n = (int64_t)I * (order + 1) * kTabStride;
  const unsigned blocks = (unsigned)std::min<int64_t>(cdiv(n, 256), 148 * 8);
  cudaStream_t s = (cudaStream_t)stream;
  switch (order) {
    case 1: knot_table_kernel<1><<<blocks, 256, 0, s>>>(grid, tab, I, grid_size); break;
    case 2: knot_table_kernel<2><<<blocks, 256, 0, s>>>(grid, tab, I, grid_size); break;
    case 3: knot_table_kernel<3><<<blocks, 256, 0, s>>>(grid, tab, I, grid_size); break;
    case 4: knot_table_kernel<4><<<blocks, 256, 0, s>>>(grid, tab, I, grid_size); break;
    default: knot_table_kernel<5><<<blocks, 256, 0, s>>>(grid, tab, I, grid_size); break;
  }
  return check_launch("kf_knot_tables");
}

// ---------------------------------------------------------------------------
// GR-KAN layers (kanforge/torch/layers.py:335-363): the rational activation R
// (kf_rational_act) followed by the linear map of coef[..., 0] = W (O, I),
// the three contractions on the CTA-pair kernels above.
// ---------------------------------------------------------------------------

extern "C" int64_t kf_grkan_workspace(int64_t B, int32_t I, const kf_basis_desc* basis) {
  (void)basis;
  if (B <= 0 || I <= 0) return 0;
  // one slot per 32-row block of every pair tile (rows past B included, they hold zeros)
  return (int64_t)(kf::kRatNA + kf::kRatNB) * (I / 32) * 8 * kf::cdiv(B, (int64_t)kf::kPairM);
}

extern "C" int kf_grkan_fwd(const void* r, const void* w, const void* bias, void* y, int64_t B, int32_t I, int32_t O,
                            void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(r && w && y, "kf_grkan_fwd: null tensor pointer");
  if (int rc = bind_device(r)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1, "kf_grkan_fwd: bad sizes");
  KF_CHECK_ARG(I % 16 == 0 && O % 8 == 0, "kf_grkan_fwd: I (%d) must be a multiple of 16 and O (%d) of 8", I, O);
  KF_CHECK_ARG(((uintptr_t)r % 16) == 0 && ((uintptr_t)w % 16) == 0 && ((uintptr_t)y % 16) == 0 && ((uintptr_t)bias % 16) == 0,
               "kf_grkan_fwd: r, w, y and bias must be 16-byte aligned");
  if (B == 0) return KF_OK;
  FwdParams p{};
  p.bias = (const __nv_bfloat16*)bias;
  p.y = (__nv_bfloat16*)y;
  p.B = B;
  p.I = I / 16;  // the kernel's K extent is I * F with F = 16
  p.O = O;
  p.k_steps = (int)cdiv(I, kBK);
  p.tiles.m_tiles = (int)cdiv(B, kPairM);
  // 256-output tiles: the two accumulators alternate between tiles, so each
  // tile's epilogue overlaps the next tile's MMAs (the K loops are short)
  p.nblk = 1;
  p.tiles.n_tiles = (int)cdiv(O, p.nblk * kBN);
  p.tiles.gm = std::min(p.tiles.m_tiles, 8);
  CUtensorMap tmap, tmap_a;
  if (int rc = make_tmap_bf16(&tmap, w, O, I, kBK, kBN / 2)) return rc;
  if (int rc = make_tmap_bf16(&tmap_a, r, B, I, kBK, kBM)) return rc;
  FwdLaunch L{&tmap, &tmap_a, p, true, (cudaStream_t)stream};
  return L.launch<0, 16, true>();
}

extern "C" int kf_grkan_dgrad(const void* x, const void* dy, const void* w, const float* num, const float* den, void* dx,
                              float* dnum, float* dden, float* workspace, int64_t B, int32_t I, int32_t O,
                              const kf_basis_desc* basis, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(x && dy && w && num && den && dx && dnum && dden, "kf_grkan_dgrad: null tensor pointer");
  if (int rc = grkan_check(basis, B, I, O, "kf_grkan_dgrad")) return rc;
  if (int rc = bind_device(x)) return rc;
  KF_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)dx % 16) == 0 && ((uintptr_t)dy % 16) == 0 && ((uintptr_t)w % 16) == 0,
               "kf_grkan_dgrad: x, dx, dy and w must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const int groups = basis->groups;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dnum, 0, sizeof(float) * groups * kRatNA, s));
    KF_CUDA_RET(cudaMemsetAsync(dden, 0, sizeof(float) * groups * kRatNB, s));
    return KF_OK;
  }
  KF_CHECK_ARG(workspace != nullptr, "kf_grkan_dgrad: null workspace (kf_grkan_workspace floats)");
  DgradParams p{};
  p.x = (const __nv_bfloat16*)x;
  p.dx = (__nv_bfloat16*)dx;
  p.B = B;
  p.I = I;
  p.O = O;
  p.k_steps = (int)cdiv(O, kBK);
  p.tiles.m_tiles = (int)cdiv(B, kPairM);
  p.tiles.n_tiles = (int)cdiv(I, kBN);
  p.tiles.gm = std::min(p.tiles.m_tiles, 8);
  p.rnum = num;
  p.rden = den;
  p.ipg = I / groups;
  p.rws = workspace;
  p.n_rq = 8 * p.tiles.m_tiles;  // 32-row blocks of all pair tiles, rows past B included
  CUtensorMap tdy, tc;
  if (int rc = make_tmap_bf16(&tdy, dy, B, O, kBK, kBM)) return rc;
  if (int rc = make_tmap_bf16(&tc, w, O, I, 64, kBK)) return rc;
  DgradLaunch L{&tdy, &tc, p, s};
  if (int rc = L.go<kRationalBK, 16>()) return rc;
  grkan_reduce_kernel<<<groups * (kRatNA + kRatNB), 256, 0, s>>>(workspace, dnum, dden, I / 32, p.ipg / 32, p.n_rq);
  return check_launch("kf_grkan_dgrad");
}

namespace kf {
namespace {
// K splits of the GR-KAN weight gradient: enough (pair tile, split) work items
// to give every CTA pair of the GPU one, each split at least 16 K steps.
int grkan_wgrad_splits(int64_t B, int I, int O) {
  const int64_t tiles = cdiv(I, kPairM) * cdiv(O, kBN);
  const int64_t k_steps = cdiv(B, kBK);
  const int64_t pairs = sm_count() / 2;
  const int64_t by_pairs = std::max<int64_t>(1, pairs / std::max<int64_t>(tiles, 1));
  return (int)std::max<int64_t>(1, std::min<int64_t>({by_pairs, k_steps / 16, 16}));
}

// dw[e] = bf16(sum_s part[s][e]) in split order.
__global__ void __launch_bounds__(256) split_sum_kernel(const float* __restrict__ part, __nv_bfloat16* __restrict__ dw, int64_t n,
                                                        int n_split) {
  for (int64_t e2 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; 2 * e2 < n; e2 += (int64_t)gridDim.x * blockDim.x) {
    float2 acc = make_float2(0.0f, 0.0f);
    for (int sp = 0; sp < n_split; ++sp) {
      const float2 v = reinterpret_cast<const float2*>(part + (size_t)sp * n)[e2];
      acc.x += v.x;
      acc.y += v.y;
    }
    reinterpret_cast<uint32_t*>(dw)[e2] = pack_bf16x2(acc.x, acc.y);
  }
}
}  // namespace
}  // namespace kf

extern "C" int64_t kf_grkan_wgrad_workspace(int64_t B, int32_t I, int32_t O) {
  if (B <= 0 || I <= 0 || O <= 0) return 0;
  const int ns = kf::grkan_wgrad_splits(B, I, O);
  return ns > 1 ? (int64_t)ns * O * I : 0;
}

extern "C" int kf_grkan_wgrad(const void* r, const void* dy, void* dw, float* workspace, int64_t B, int32_t I, int32_t O,
                              void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(r && dy && dw, "kf_grkan_wgrad: null tensor pointer");
  if (int rc = bind_device(r)) return rc;
  KF_CHECK_ARG(B >= 0 && I >= 1 && O >= 1, "kf_grkan_wgrad: bad sizes");
  KF_CHECK_ARG(I % 16 == 0 && O % 8 == 0, "kf_grkan_wgrad: I (%d) must be a multiple of 16 and O (%d) of 8", I, O);
  KF_CHECK_ARG(((uintptr_t)r % 16) == 0 && ((uintptr_t)dy % 16) == 0 && ((uintptr_t)dw % 4) == 0,
               "kf_grkan_wgrad: r and dy must be 16-byte aligned, dw 4-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  if (B == 0) {
    KF_CUDA_RET(cudaMemsetAsync(dw, 0, sizeof(__nv_bfloat16) * (size_t)O * I, s));
    return KF_OK;
  }
  // dW = dy^T R as the coefficient-gradient kernel with F = 16 feature columns
  // per "input" (I / 16 of them), K = 16, no fold, mask, scale or base column:
  // its (O, I / 16, 16) output is W's (O, I) layout.
  WgradParams p{};
  p.x = (const __nv_bfloat16*)r;
  p.dcoef = (__nv_bfloat16*)dw;
  p.B = B;
  p.I = I / 16;
  p.O = O;
  p.K = 16;
  p.k_steps = (int)cdiv(B, kBK);
  p.n_split = grkan_wgrad_splits(B, I, O);
  p.ks = (int)cdiv(p.k_steps, p.n_split);
  p.n_split = (int)cdiv(p.k_steps, p.ks);  // no empty split
  if (p.n_split > 1) {
    KF_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace % 16) == 0,
                 "kf_grkan_wgrad: needs a 16-byte aligned workspace of kf_grkan_wgrad_workspace floats");
    p.part = workspace;
  }
  p.x_tma = 0;
  p.tab_stride = 16;
  p.bd.nt = 16;
  p.tiles.m_tiles = (int)cdiv(I, kPairM);
  p.tiles.n_tiles = (int)cdiv(O, kBN);
  p.tiles.gm = std::min(p.tiles.m_tiles, 8);
  CUtensorMap tdy, tx;
  if (int rc = make_tmap_bf16(&tdy, dy, B, O, 64, kBK)) return rc;
  if (int rc = make_tmap_bf16(&tx, r, B, I, 64, kBK)) return rc;
  WgradLaunch L{&tdy, &tx, p, true, s};
  if (int rc = L.launch<0, 16, true>()) return rc;
  if (p.n_split > 1) {
    const int64_t n = (int64_t)O * I;
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n / 2, 256), (int64_t)sm_count() * 8);
    split_sum_kernel<<<grid, 256, 0, s>>>(workspace, (__nv_bfloat16*)dw, n, p.n_split);
    return check_launch("kf_grkan_wgrad");
  }
  return KF_OK;
}

// ---------------------------------------------------------------------------
// Entry points of the plain (rows, I) layer and of the KAN convolution, whose
// x operand is an image read through the implicit patch matrix (conv.cuh).
// ---------------------------------------------------------------------------

extern "C" int kf_fwd(const void* x, const void* feat, const void* packed, const void* bias, const float* knot_tab, void* y,
                      int64_t B, int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
                      void* stream) {
  return kf_fwd_impl(nullptr, x, feat, packed, bias, knot_tab, y, B, I, O, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_fwd_emit_features(const void* x, const void* packed, const void* bias, const float* knot_tab, void* y,
                                    void* feat_out, int64_t B, int32_t I, int32_t O, int32_t nt, int32_t f_pad,
                                    int32_t has_base, const kf_basis_desc* basis, void* stream) {
  kf::clear_error();
  KF_CHECK_ARG(feat_out && basis, "kf_fwd_emit_features: null pointer");
  return kf_fwd_impl(nullptr, x, nullptr, packed, bias, knot_tab, y, B, I, O, nt, f_pad, has_base, basis, stream, feat_out);
}

extern "C" int kf_dgrad(const void* x, const void* dy, const void* packed, const float* knot_tab, void* dx, int64_t B,
                        int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
                        void* stream) {
  return kf_dgrad_impl(nullptr, x, dy, packed, knot_tab, dx, B, I, O, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_features(const void* x, const float* knot_tab, void* feat, int64_t B, int32_t I, int32_t nt,
                           int32_t f_pad, int32_t has_base, const kf_basis_desc* basis, void* stream) {
  return kf_features_impl(nullptr, x, knot_tab, feat, B, I, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_wgrad(const void* x, const void* feat, const void* dy, const float* knot_tab, const float* fold,
                        const void* coef, const void* edge_scale, const void* edge_mask, void* dcoef, void* dbase,
                        void* dscale, int64_t B, int32_t I, int32_t O, int32_t K, int32_t nt, int32_t f_pad,
                        const kf_basis_desc* basis, void* stream) {
  return kf_wgrad_impl(nullptr, x, feat, dy, knot_tab, fold, coef, edge_scale, edge_mask, dcoef, dbase, dscale, B, I, O, K,
                       nt, f_pad, basis, stream);
}

namespace kf {
namespace {

// The implicit patch matrix of `g`: its device description, rows and columns.
int conv_geometry(const kf_conv_geom* g, ConvDev& d, int64_t& rows, int& cols, const char* who) {
  KF_CHECK_ARG(g != nullptr, "%s: null geometry", who);
  KF_CHECK_ARG(g->batch >= 0 && g->channels >= 1 && g->group_channels >= 1 && g->channel0 >= 0 &&
                   g->channel0 + g->group_channels <= g->channels,
               "%s: bad channel layout", who);
  d = ConvDev{};
  d.active = 1;
  d.c0 = g->channel0;
  int64_t per_image = g->channels, out_n = 1, ksz = 1;
  for (int k = 0; k < 3; ++k) {
    KF_CHECK_ARG(g->size[k] >= 1 && g->kernel[k] >= 1 && g->stride[k] >= 1 && g->dilation[k] >= 1 && g->padding[k] >= 0,
                 "%s: bad size / kernel / stride / dilation / padding in dimension %d", who, k);
    const int span = g->dilation[k] * (g->kernel[k] - 1) + 1;
    const int padded = g->size[k] + 2 * g->padding[k];
    KF_CHECK_ARG(padded >= span, "%s: kernel larger than the padded input in dimension %d", who, k);
    d.size[k] = g->size[k];
    d.kernel[k] = g->kernel[k];
    d.stride[k] = g->stride[k];
    d.pad[k] = g->padding[k];
    d.dil[k] = g->dilation[k];
    d.out[k] = (padded - span) / g->stride[k] + 1;
    per_image *= g->size[k];
    out_n *= d.out[k];
    ksz *= g->kernel[k];
  }
  d.img_n_stride = per_image;
  rows = (int64_t)g->batch * out_n;
  KF_CHECK_ARG((int64_t)g->group_channels * ksz < (1 << 30), "%s: too many patch columns", who);
  cols = (int)(g->group_channels * ksz);
  return KF_OK;
}

// out[r, c] = the implicit patch matrix, row-major (rows, cols).
template <typename T>
__global__ void __launch_bounds__(256) conv_patches_kernel(const T* __restrict__ img, T* __restrict__ out, int64_t n, int cols,
                                                           ConvDev g) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t src = conv_index(g, e / cols, (int)(e % cols));
    out[e] = src >= 0 ? img[src] : from_f32<T>(0.0f);
  }
}

// dimg[n, c0 + c, p] = sum over the kernel offsets k of dpatches[(n, o), (c, k)]
// with o_d = (p_d + pad_d - k_d dil_d) / stride_d exact and inside the output:
// the transpose of the patch gather, one thread per image element of the
// group, offsets in a fixed order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) conv_fold_kernel(const T* __restrict__ dp, T* __restrict__ dimg, int64_t n_elem, int cg,
                                                        int cols, ConvDev g) {
  const int64_t plane = (int64_t)g.size[0] * g.size[1] * g.size[2];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_elem; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pix = e % plane;
    const int64_t nc = e / plane;
    const int c = (int)(nc % cg);
    const int64_t n = nc / cg;
    const int p2 = (int)(pix % g.size[2]);
    const int p1 = (int)((pix / g.size[2]) % g.size[1]);
    const int p0 = (int)(pix / ((int64_t)g.size[2] * g.size[1]));
    float acc = 0.0f;
    for (int k0 = 0; k0 < g.kernel[0]; ++k0) {
      const int a0 = p0 + g.pad[0] - k0 * g.dil[0];
      if (a0 < 0 || a0 % g.stride[0] || a0 / g.stride[0] >= g.out[0]) continue;
      for (int k1 = 0; k1 < g.kernel[1]; ++k1) {
        const int a1 = p1 + g.pad[1] - k1 * g.dil[1];
        if (a1 < 0 || a1 % g.stride[1] || a1 / g.stride[1] >= g.out[1]) continue;
        for (int k2 = 0; k2 < g.kernel[2]; ++k2) {
          const int a2 = p2 + g.pad[2] - k2 * g.dil[2];
          if (a2 < 0 || a2 % g.stride[2] || a2 / g.stride[2] >= g.out[2]) continue;
          const int64_t row = ((n * g.out[0] + a0 / g.stride[0]) * g.out[1] + a1 / g.stride[1]) * g.out[2] + a2 / g.stride[2];
          const int col = ((c * g.kernel[0] + k0) * g.kernel[1] + k1) * g.kernel[2] + k2;
          acc += to_f32(dp[row * cols + col]);
        }
      }
    }
    dimg[(n * g.img_n_stride / plane + g.c0 + c) * plane + pix] = from_f32<T>(acc);
  }
}

unsigned elementwise_grid(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 16)); }

}  // namespace
}  // namespace kf

extern "C" int kf_conv_patches(const void* img, const kf_conv_geom* geom, void* patches, int dtype, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(img && patches, "kf_conv_patches: null tensor pointer");
  KF_CHECK_ARG(dtype == KF_DTYPE_F32 || dtype == KF_DTYPE_BF16, "kf_conv_patches: dtype %d", dtype);
  ConvDev g;
  int64_t rows;
  int cols;
  if (int rc = conv_geometry(geom, g, rows, cols, "kf_conv_patches")) return rc;
  if (int rc = bind_device(img)) return rc;
  const int64_t n = rows * cols;
  if (n == 0) return KF_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32)
    conv_patches_kernel<float><<<elementwise_grid(n), 256, 0, s>>>((const float*)img, (float*)patches, n, cols, g);
  else
    conv_patches_kernel<__nv_bfloat16><<<elementwise_grid(n), 256, 0, s>>>((const __nv_bfloat16*)img, (__nv_bfloat16*)patches,
                                                                          n, cols, g);
  return check_launch("kf_conv_patches");
}

extern "C" int kf_conv_fold(const void* dpatches, const kf_conv_geom* geom, void* dimg, int dtype, void* stream) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(dpatches && dimg, "kf_conv_fold: null tensor pointer");
  KF_CHECK_ARG(dtype == KF_DTYPE_F32 || dtype == KF_DTYPE_BF16, "kf_conv_fold: dtype %d", dtype);
  ConvDev g;
  int64_t rows;
  int cols;
  if (int rc = conv_geometry(geom, g, rows, cols, "kf_conv_fold")) return rc;
  if (int rc = bind_device(dimg)) return rc;
  const int64_t n = (int64_t)geom->batch * geom->group_channels * g.size[0] * g.size[1] * g.size[2];
  if (n == 0) return KF_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == KF_DTYPE_F32)
    conv_fold_kernel<float><<<elementwise_grid(n), 256, 0, s>>>((const float*)dpatches, (float*)dimg, n, geom->group_channels,
                                                               cols, g);
  else
    conv_fold_kernel<__nv_bfloat16><<<elementwise_grid(n), 256, 0, s>>>((const __nv_bfloat16*)dpatches, (__nv_bfloat16*)dimg, n,
                                                                       geom->group_channels, cols, g);
  return check_launch("kf_conv_fold");
}

extern "C" int kf_conv_fwd(const void* img, const kf_conv_geom* geom, const void* feat, const void* packed, const void* bias,
                           const float* knot_tab, void* y, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base,
                           const kf_basis_desc* basis, void* stream) {
  kf::ConvDev g;
  int64_t rows;
  int cols;
  kf::clear_error();
  if (int rc = kf::conv_geometry(geom, g, rows, cols, "kf_conv_fwd")) return rc;
  return kf_fwd_impl(&g, img, feat, packed, bias, knot_tab, y, rows, cols, O, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_conv_features(const void* img, const kf_conv_geom* geom, const float* knot_tab, void* feat, int32_t nt,
                                int32_t f_pad, int32_t has_base, const kf_basis_desc* basis, void* stream) {
  kf::ConvDev g;
  int64_t rows;
  int cols;
  kf::clear_error();
  if (int rc = kf::conv_geometry(geom, g, rows, cols, "kf_conv_features")) return rc;
  return kf_features_impl(&g, img, knot_tab, feat, rows, cols, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_conv_dgrad(const void* img, const kf_conv_geom* geom, const void* dy, const void* packed,
                             const float* knot_tab, void* dpatches, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base,
                             const kf_basis_desc* basis, void* stream) {
  kf::ConvDev g;
  int64_t rows;
  int cols;
  kf::clear_error();
  if (int rc = kf::conv_geometry(geom, g, rows, cols, "kf_conv_dgrad")) return rc;
  return kf_dgrad_impl(&g, img, dy, packed, knot_tab, dpatches, rows, cols, O, nt, f_pad, has_base, basis, stream);
}

extern "C" int kf_conv_wgrad(const void* img, const kf_conv_geom* geom, const void* feat, const void* dy, const float* knot_tab,
                             const float* fold, const void* coef, const void* edge_scale, const void* edge_mask, void* dcoef,
                             void* dbase, void* dscale, int32_t O, int32_t K, int32_t nt, int32_t f_pad,
                             const kf_basis_desc* basis, void* stream) {
  kf::ConvDev g;
  int64_t rows;
  int cols;
  kf::clear_error();
  if (int rc = kf::conv_geometry(geom, g, rows, cols, "kf_conv_wgrad")) return rc;
  return kf_wgrad_impl(&g, img, feat, dy, knot_tab, fold, coef, edge_scale, edge_mask, dcoef, dbase, dscale, rows, cols, O, K,
                       nt, f_pad, basis, stream);
}

extern "C" int kf_set_reserved_sms(int32_t n) {
  kf::clear_error();
  KF_CHECK_ARG(n >= 0 && n < kf::sm_count(), "kf_set_reserved_sms: %d out of range", n);
  kf::g_reserved_sms.store(n, std::memory_order_relaxed);
  return KF_OK;
}
