/*
 * kanforge_b200 -- C ABI of the B200 (sm_100a) KAN-layer kernels.
 *
 * Every pointer is a device pointer owned by the caller (torch allocates; the
 * library allocates nothing).  Every compute entry point takes the CUDA stream
 * to launch on (a cudaStream_t passed as void*), is stream-ordered, never
 * synchronises the host and returns KF_OK or an error code; kf_last_error()
 * returns the message of the last failure on the calling thread.  The only
 * process-wide state is per-device initialisation done once.
 *
 * Reference interfaces replaced (fx-xf/kanforge v0.8.0, paths within the project):
 *   kanforge/torch/kernels.py:19-28    available(device)      -> kf_query
 *   kanforge/torch/kernels.py:39-55    _raw(op, plan, m, ...) -> kf_prim
 *   kanforge/kernels/triton_kernels.py:225-242 launch(...)     -> kf_prim
 *   kanforge/torch/kernels.py:143-150  spline_forward + the SiLU/bias epilogue of
 *   kanforge/torch/layers.py:177-191   KANLinear.forward      -> kf_pack_coef + kf_fwd
 *   kanforge/torch/kernels.py:79-87    _F.backward (m = 0)    -> kf_dgrad + kf_wgrad
 *   kanforge/torch/layers.py:206-226   edge_derivative        -> kf_edge_derivative
 *   kanforge/bases/rational.py:84-101  Rational._eval (GRKAN) -> kf_rational_act,
 *                                                               kf_rational_bwd
 *   kanforge/grid.py:19-31             adaptive_grid          -> kf_adaptive_grid
 *   kanforge/grid.py:34-38             resample_grid          -> kf_resample_grid
 *   kanforge/grid.py:55-85             refit                  -> kf_refit
 *   kanforge/bases/base.py:15-16       local / support (sparse gather, the
 *                                      reference's planned kernel) -> kf_sparse_*
 */
#ifndef KANFORGE_B200_H
#define KANFORGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KF_ABI_VERSION 2

/* status codes */
#define KF_OK 0
#define KF_ERR_ARG 1         /* bad argument: null pointer, size, alignment */
#define KF_ERR_UNSUPPORTED 2 /* basis / order / dtype without a kernel */
#define KF_ERR_CUDA 3        /* a CUDA runtime call failed */
#define KF_ERR_DEVICE 4      /* a kernel reported a bounded wait that ran out */

/* basis kinds (kanforge/kernels/plan.py:39-72 plan kinds, plus the rational) */
#define KF_BASIS_BSPLINE 1   /* native derivative order, per-input grid */
#define KF_BASIS_CHEB 2      /* Chebyshev features T_j(g(x)), derivatives folded */
#define KF_BASIS_RATIONAL 3  /* KAT P(x) / (1 + |Q(x)|), per-group parameters */
#define KF_BASIS_FOURIER 4   /* cos(w_j x), sin(w_j x), w_j = 2 pi j / period; derivatives folded */
#define KF_BASIS_BUMP 5      /* bumps on a per-input grid of centres (RBF, wavelets, RSWAF), native order */

#define KF_BUMP_GAUSS 0      /* norm P_m(u) exp(-u^2/2) k^m, u = (x - c_j) k, k = u_scale (count-1) / (c_last - c_first) */
#define KF_BUMP_TANH 1       /* P_m(t) / h^m, t = tanh((x - c_j) / h), h = (c_last - c_first) / (count - 1) */
#define KF_BUMP_MAX_ORDER 5  /* derivative orders with a polynomial in the descriptor */

#define KF_MAP_TANH 0
#define KF_MAP_IDENTITY 1

#define KF_DTYPE_F32 0
#define KF_DTYPE_BF16 1

/* primitive ops of the closed family (kanforge/kernels/__init__.py:5-13) */
#define KF_OP_F 0
#define KF_OP_G 1
#define KF_OP_P 2

typedef struct kf_basis_desc {
  int32_t kind;       /* KF_BASIS_* */
  int32_t size;       /* basis functions per edge: G+k, d+1, or 1 */
  int32_t grid_size;  /* B-spline: intervals G */
  int32_t order;      /* B-spline: spline order k */
  int32_t degree;     /* Chebyshev: degree d; rational: numerator degree */
  int32_t den_degree; /* rational: denominator degree */
  int32_t input_map;  /* Chebyshev: KF_MAP_* */
  int32_t groups;     /* rational: parameter groups (inputs per group = I / groups) */
  float period;       /* Fourier: period (size = 2 frequencies) */
  int32_t bump_mode;  /* bumps: KF_BUMP_*; size = count (grid (I, count) of centres) */
  float u_scale;      /* bumps: scale of u (gauss) */
  float norm;         /* bumps: constant factor (gauss) */
  float bump_poly[KF_BUMP_MAX_ORDER + 1][8]; /* bumps: P_m, coefficients lowest first, m = 0..5 */
} kf_basis_desc;

/* Library ABI version (KF_ABI_VERSION). */
int kf_version(void);

/* Message of the last error on this thread ("" if none). */
const char* kf_last_error(void);

/* 1 if a kernel exists for (basis, op, dtype), else 0.  op: KF_OP_* for the
 * primitives, 16 = fused fwd/dgrad/wgrad, 17 = edge_derivative.
 * Replaces available() + plan_for() (kanforge/torch/kernels.py:19-28,
 * kanforge/kernels/plan.py:104-121). */
int kf_query(const kf_basis_desc* basis, int op, int dtype);

/* SMs that the persistent tensor-core kernels leave free (default 0: they
 * take every SM), so that a kernel launched beside them on another stream --
 * the gradient all-reduce of data parallelism overlapping the backward --
 * finds SMs to run on.  Process-wide; 0 <= n < the SM count.  (No counterpart
 * in the reference, which has no distributed code.) */
int kf_set_reserved_sms(int32_t n);

/* Reads and clears the device-side error word of the current device (set by a
 * kernel whose bounded wait ran out).  Synchronises the device.  *flags = 0 when
 * clean. */
int kf_device_status(int32_t* flags);

/* One launch of the closed primitive family, float32, any derivative order m
 * (kanforge/torch/kernels.py:39-55, triton_kernels.py:128-191):
 *   op F: a = w (B,I),  b = c (O,I,nf) -> out (B,O)    = sum_{i,j} w c phi_j^(m)
 *   op G: a = w (B,I),  b = g (B,O)    -> out (O,I,nf) = sum_b w g phi_j^(m)
 *   op P: a = g (B,O),  b = c (O,I,nf) -> out (B,I)    = sum_{o,j} g c phi_j^(m)
 * For KF_BASIS_CHEB the features are T_0..T_{nf-1}(g(x)) and the caller folds
 * the derivative into c (plan.fold); B-splines evaluate order m natively.
 * grid: (I, G+1) per-input grids for B-splines, else ignored. */
int kf_prim(int op, int m, const float* x, const float* a, const float* b, const float* grid, float* out,
            int64_t B, int32_t I, int32_t O, int32_t nf, const kf_basis_desc* basis, void* stream);

/* Builds the bf16 tensor-core operand of the fused layer kernels:
 *   coef_eff = coef * edge_scale * edge_mask, base_eff = base * edge_mask
 *   (kanforge/torch/layers.py:162-167; a null scale / mask is 1)
 *   packed[o, i, j] = sum_k coef_eff[o,i,k] fold[k,j]   (j < nt; fold = null: j = k)
 *   packed[o, i, f_pad-1] = base_eff[o, i]              (if base != null)
 *   zero elsewhere; f_pad >= nt + 1.
 * coef (O,I,K), base, edge_scale, edge_mask (O,I) in `dtype`; fold (K, nt)
 * float32 row-major.  packed is (O, I*f_pad) bf16, 16-byte aligned. */
int kf_pack_coef(const void* coef, const void* base, const void* edge_scale, const void* edge_mask,
                 const float* fold, void* packed, int32_t O, int32_t I, int32_t K, int32_t nt, int32_t f_pad,
                 int dtype, void* stream);

/* Knot tables of per-input B-spline grids, read by the fused kernels: for each
 * input i, tab[i, 0, r] = extended knot t_r (r < G + 2 order + 1, order mean
 * steps per side, kanforge/bases/spline.py:22-30) and tab[i, q, r] =
 * 1 / (t_{r+q} - t_r) (q = 1..order); rows of 64 floats, zero-padded.
 * grid (I, G+1) float32, tab (I, order+1, 64) float32, 16-byte aligned. */
int kf_knot_tables(const float* grid, float* tab, int32_t I, int32_t grid_size, int32_t order, void* stream);

/* Fused KANLinear forward on tcgen05 (bf16 operands, f32 accumulation):
 *   y[b,o] = sum_{i,j} feat_j(x[b,i]) packed[o,i,j] + bias[o]
 * feat = basis features (B-spline values or T_j(g(x))) and, in the last
 * column f_pad-1, silu(x) when has_base.  x (B,I) bf16, y (B,O) bf16, bias (O) bf16 or null
 * (y and bias 16-byte aligned),
 * knot_tab: kf_knot_tables output for B-splines, else null.  Requires O % 8 == 0.
 * feat: the kf_features matrix of x (the kernel then reads the features by
 * TMA), or null (it evaluates them itself).
 * (kanforge/torch/layers.py:171-192 with kernels.py:143-150.) */
int kf_fwd(const void* x, const void* feat, const void* packed, const void* bias, const float* knot_tab, void* y, int64_t B,
           int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
           void* stream);

/* kf_fwd (feat null) that also writes the basis feature matrix of x, (B, I * f_pad)
 * bf16 as kf_features lays it out, for the coefficient gradient: the forward's
 * producer warps evaluate every feature row anyway, so the backward need not
 * evaluate them again.  KF_BASIS_CHEB and KF_BASIS_FOURIER only.  Same reference
 * interface as kf_fwd (kanforge/torch/layers.py:177-191); the kept matrix is
 * this library's (the reference evaluates the basis in each Triton launch,
 * kanforge/kernels/triton_kernels.py:122-124). */
int kf_fwd_emit_features(const void* x, const void* packed, const void* bias, const float* knot_tab, void* y,
                         void* feat_out, int64_t B, int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base,
                         const kf_basis_desc* basis, void* stream);

/* Fused input gradient on tcgen05:
 *   dx[b,i] = sum_j (sum_o dy[b,o] packed[o,i,j]) dfeat_j(x[b,i])
 * dfeat = d/dx of the forward features (the SiLU column included).
 * dy (B,O) bf16, dx (B,I) bf16.  (kanforge/torch/kernels.py:84 gx = w * P_{m+1}.) */
int kf_dgrad(const void* x, const void* dy, const void* packed, const float* knot_tab, void* dx, int64_t B,
             int32_t I, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
             void* stream);

/* Basis feature matrix of the fused layer, bf16:
 *   feat[b, i*f_pad + j] = feat_j(x[b,i])   (the forward's features: basis
 *   columns 0..nt-1, zero up to f_pad-2, silu(x) in column f_pad-1 when has_base)
 * x (B,I) bf16, feat (B, I*f_pad) bf16, 16-byte aligned.  Input of the fast
 * path of kf_wgrad, which then reads the features by TMA instead of
 * evaluating them once per output tile, and of kf_fwd.  (No reference counterpart: the
 * reference evaluates the basis inside each Triton launch,
 * kanforge/kernels/triton_kernels.py:122-124, 144, 166.) */
int kf_features(const void* x, const float* knot_tab, void* feat, int64_t B, int32_t I, int32_t nt, int32_t f_pad,
                int32_t has_base, const kf_basis_desc* basis, void* stream);

/* Float32 GEMM on tcgen05 with three TF32 products (hi*hi + hi*lo + lo*hi,
 * hi = v truncated to TF32 as the tensor core reads it, lo = v - hi, formed in
 * shared memory), float32 accumulation:
 *   C[m,n] = sum_k A[m,k] B[n,k] (+ bias[n])
 * A is K-major (a_mn_major = 0: element (m,k) at a[m*lda + k]) or MN-major
 * (element (m,k) at a[k*lda + m]); B likewise with n.  lda, ldb multiples of
 * 4 floats, operands 16-byte aligned, K >= 1.  The float32 layer's three
 * contractions: forward y = feat packed^T + b (the reference's F_0,
 * kanforge/torch/kernels.py:143-150), feature gradient dfeat = dy packed
 * (its P_1 before the derivative features, kernels.py:84) and coefficient
 * gradient dpacked = dy^T feat (its G_0, kernels.py:85). */
int kf_gemm_tf32x3(const float* a, int32_t a_mn_major, int64_t lda, const float* b, int32_t b_mn_major, int64_t ldb,
                   const float* bias, float* c, int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream);

/* Float32 feature matrix of the float32 tensor-core path:
 *   feat[b, i*F + j] = phi_j(x[b,i]) (j < nf), 0 up to F-2, silu(x[b,i]) at F-1
 *   when has_base (the column layout of kf_pack_coef; F = 16 or 32).
 * grid (I, G+1) float32 for B-splines, else ignored.  x (B,I) float32; feat
 * 16-byte aligned.
 * (The reference evaluates these inside its Triton launches,
 * kanforge/kernels/triton_kernels.py:32-108.) */
int kf_features_f32(const float* x, const float* grid, float* feat, int64_t B, int32_t I, int32_t nf, int32_t F,
                    int32_t has_base, const kf_basis_desc* basis, void* stream);

/* The same float32 feature matrix for B-spline bases from the knot tables of
 * kf_knot_tables (knot_tab, 16-byte aligned) instead of the raw grid: the
 * knot search and Cox-de Boor steps of kf_features, float32 output, silu(x)
 * at F-1 when has_base.  nt = the basis size; F = 16 or 32. */
int kf_features_spline_f32(const float* x, const float* knot_tab, float* feat, int64_t B, int32_t I, int32_t nt, int32_t F,
                           int32_t has_base, const kf_basis_desc* basis, void* stream);

/* Input gradient from the feature gradient of kf_gemm_tf32x3:
 *   dx[b,i] = sum_{j<nf} dfeat[b, i*F + j] d phi_j / dx (x[b,i])
 *           + dfeat[b, i*F + F-1] silu'(x[b,i])        (when has_base)
 * dfeat 16-byte aligned.  (The reference's gx = w * P_1,
 * kanforge/torch/kernels.py:84, with the base branch of layers.py:185-186.) */
int kf_features_dot_f32(const float* x, const float* grid, const float* dfeat, float* dx, int64_t B, int32_t I,
                        int32_t nf, int32_t F, int32_t has_base, const kf_basis_desc* basis, void* stream);

/* Fused coefficient gradient on tcgen05, with the effective-coefficient chain rule:
 *   dpacked[o,i,j] = sum_b dy[b,o] feat_j(x[b,i])
 *   dC[o,i,k]      = sum_{j<nt} dpacked[o,i,j] fold[k,j]      (fold null: k = j)
 *   dcoef[o,i,k]   = dC[o,i,k] * edge_scale[o,i] * edge_mask[o,i]
 *   dscale[o,i]    = sum_k dC[o,i,k] coef[o,i,k] edge_mask[o,i] (if dscale != null)
 *   dbase[o,i]     = dpacked[o,i,f_pad-1] * edge_mask[o,i]       (if dbase != null)
 * coef, edge_scale, edge_mask (null = 1) and the outputs are bf16.
 * feat: the kf_features matrix of x (fast path), or null (the kernel evaluates
 * the features from x itself).
 * (kanforge/torch/kernels.py:85, 97-98; layers.py:162-167.) */
int kf_wgrad(const void* x, const void* feat, const void* dy, const float* knot_tab, const float* fold, const void* coef,
             const void* edge_scale, const void* edge_mask, void* dcoef, void* dbase, void* dscale, int64_t B,
             int32_t I, int32_t O, int32_t K, int32_t nt, int32_t f_pad, const kf_basis_desc* basis, void* stream);

/* edge_derivative (kanforge/torch/layers.py:206-226), float32:
 *   out[b,o,i] = sum_j phi_j^(order)(x[b,i]) coefT[o,j,i] + s(x[b,i]) base_eff[o,i]
 * coefT (O,nf,I) -- the effective coefficients with the feature axis moved
 * before the input axis: for KF_BASIS_CHEB the caller passes
 * (coef_eff @ fold(order)) transposed and phi_j = T_j(g(x)); otherwise
 * coef_eff transposed and the native derivative.
 * s = silu^(order) given by the polynomials h_order(sigma), h_{order-1}(sigma):
 * silu^(m)(x) = x h_m(s) + m h_{m-1}(s) (kanforge/_calculus.py:90-96), passed as
 * silu_poly = [h_m coefficients (n_poly) , h_{m-1} coefficients (n_poly)];
 * base_eff null: no base term.  out (B,O,I). */
int kf_edge_derivative(const float* x, const float* coefT, const float* base_eff, const float* grid,
                       const float* basis_num, const float* basis_den, float* out, int64_t B, int32_t I,
                       int32_t O, int32_t nf, int32_t order, const kf_basis_desc* basis,
                       const float* silu_poly, int32_t n_poly, void* stream);

/* Backward of kf_edge_derivative: the reference's edge_derivative is an
 * autograd graph (kanforge/torch/layers.py:206-226), so a loss on the edge
 * derivatives trains the layer.  With g = dL/dout (B, O, I) float32:
 *   kf_edge_derivative_dx:    dx[b,i] = sum_o g[b,o,i] (sum_j phi_j^(order)(x) coefT[o,j,i] + s(x) base_eff[o,i])
 *                             -- called with the order, coefficients (coefT of that order, nf features) and
 *                             SiLU polynomials of the forward's order + 1;
 *   kf_edge_derivative_dcoef: dcoefT[o,j,i] = sum_b g[b,o,i] phi_j^(order)(x[b,i]) (O, nf, I) and, when dbase
 *                             is given, dbase[o,i] = sum_b g[b,o,i] s(x[b,i]), s = silu^(order) from silu_poly;
 *                             summed over row splits in a fixed order through `workspace`
 *                             (kf_edge_derivative_workspace floats).
 * The caller applies the fold (Chebyshev, Fourier) and edge_scale / edge_mask chain rule. */
int kf_edge_derivative_dx(const float* x, const float* g, const float* coefT, const float* base_eff, const float* grid,
                          const float* basis_num, const float* basis_den, float* dx, int64_t B, int32_t I, int32_t O,
                          int32_t nf, int32_t order, const kf_basis_desc* basis, const float* silu_poly, int32_t n_poly,
                          void* stream);
int kf_edge_derivative_dcoef(const float* x, const float* g, const float* grid, const float* basis_num,
                             const float* basis_den, float* dcoefT, float* dbase, float* workspace, int64_t B, int32_t I,
                             int32_t O, int32_t nf, int32_t order, const kf_basis_desc* basis, const float* silu_poly,
                             int32_t n_poly, void* stream);
int64_t kf_edge_derivative_workspace(int64_t B, int32_t I, int32_t O, int32_t nf);

/* KAT group rational activation and its order-m derivative, elementwise
 * (kanforge/bases/rational.py:84-101):  out[b,i] = R_g(i)^(m)(x[b,i]).
 * num (groups, p+1), den (groups, q) float32; x, out in `dtype`. */
int kf_rational_act(const void* x, const float* num, const float* den, void* out, int64_t B, int32_t I,
                    int32_t m, const kf_basis_desc* basis, int dtype, void* stream);

/* Backward of the rational activation: dx[b,i] = dr[b,i] R'(x[b,i]) and the
 * per-group parameter gradients dnum (groups, p+1), dden (groups, q), float32,
 * reduced deterministically through `workspace` (float32, at least
 * kf_rational_workspace(B, I, basis) elements). */
int kf_rational_bwd(const void* x, const void* dr, const float* num, const float* den, void* dx, float* dnum,
                    float* dden, float* workspace, int64_t B, int32_t I, const kf_basis_desc* basis,
                    int dtype, void* stream);

/* Workspace (float32 elements) that kf_rational_bwd needs. */
int64_t kf_rational_workspace(int64_t B, int32_t I, const kf_basis_desc* basis);

/* GR-KAN layer contractions on tcgen05 (bf16 operands, f32 accumulation):
 * the linear map of a GRKAN layer, kanforge/torch/layers.py:335-363 (R = the
 * group rational of kf_rational_act, W = coef[..., 0] of shape (O, I)).
 *   kf_grkan_fwd:   y[b,o] = sum_i r[b,i] w[o,i] + bias[o]
 *                   r = R(x) (B,I), w (O,I), bias (O) or null, y (B,O), all bf16;
 *                   I % 16 == 0, O % 8 == 0, r, w, y and bias 16-byte aligned.
 *   kf_grkan_dgrad: dR[b,i] = sum_o dy[b,o] w[o,i] on the tensor cores, then in
 *                   the same kernel dx[b,i] = dR[b,i] R'(x[b,i]) and the partial
 *                   sums of the per-group parameter gradients
 *                   dnum[g,j] = sum dR dR/da_j, dden[g,j] = sum dR dR/db_j
 *                   (float32, reduced in a fixed order through `workspace`,
 *                   kf_grkan_workspace floats).  Rational degrees (5, 4), the
 *                   inputs per group a multiple of 32, O % 8 == 0; x, dy, w, dx
 *                   bf16 and 16-byte aligned; num (groups, 6), den (groups, 4).
 *   kf_grkan_wgrad: dw[o,i] = sum_b dy[b,o] r[b,i], bf16; I % 16 == 0, O % 8 == 0.
 *                   When the (I / 256) x (O / 256) output tiles are too few to
 *                   fill the GPU, the batch is split and the float32 partial
 *                   sums go through `workspace` (kf_grkan_wgrad_workspace
 *                   floats, 16-byte aligned; 0 = none needed), summed in a
 *                   fixed order.
 * Replace Rational._eval + the torch linear map and its autograd
 * (kanforge/bases/rational.py:84-101, kanforge/torch/layers.py:184-191). */
int kf_grkan_fwd(const void* r, const void* w, const void* bias, void* y, int64_t B, int32_t I, int32_t O, void* stream);
int kf_grkan_dgrad(const void* x, const void* dy, const void* w, const float* num, const float* den, void* dx, float* dnum,
                   float* dden, float* workspace, int64_t B, int32_t I, int32_t O, const kf_basis_desc* basis,
                   void* stream);
int64_t kf_grkan_workspace(int64_t B, int32_t I, const kf_basis_desc* basis);
int64_t kf_grkan_wgrad_workspace(int64_t B, int32_t I, int32_t O);
int kf_grkan_wgrad(const void* r, const void* dy, void* dw, float* workspace, int64_t B, int32_t I, int32_t O,
                   void* stream);

/* ---- KAN convolutions (kanforge/torch/conv.py:57-85) ----
 * A KANConvNd applies one KANLinear per channel group to every receptive
 * field.  Its input is an implicit patch matrix of the image img (N, channels,
 * size_0, size_1, size_2), channels-first, unused spatial dimensions of size
 * 1: row (n, o_0, o_1, o_2) over the output positions, column (c, k_0, k_1,
 * k_2) over the group's channels and the kernel offsets (the weight order of
 * torch.nn.ConvNd), value img[n, channel0 + c, o_d stride_d - padding_d +
 * k_d dilation_d] or 0 in the zero padding; out_d = (size_d + 2 padding_d -
 * dilation_d (kernel_d - 1) - 1) / stride_d + 1.  rows = batch prod(out),
 * cols = group_channels prod(kernel).  (Other padding modes: pad the image
 * first and pass padding 0.) */
typedef struct kf_conv_geom {
  int32_t batch;          /* images N */
  int32_t channels;       /* channels of img (all groups) */
  int32_t group_channels; /* channels of this group */
  int32_t channel0;       /* first channel of this group */
  int32_t size[3];
  int32_t kernel[3];
  int32_t stride[3];
  int32_t padding[3];
  int32_t dilation[3];
} kf_conv_geom;

/* The patch matrix itself, (rows, cols) in `dtype` (for the float32 path and
 * the primitives, which take a plain matrix). */
int kf_conv_patches(const void* img, const kf_conv_geom* geom, void* patches, int dtype, void* stream);
/* Its transpose: dimg[n, channel0 + c, p] = sum of dpatches over the
 * (row, column) pairs that read img[n, channel0 + c, p], in a fixed order.
 * Writes this group's channels of dimg only. */
int kf_conv_fold(const void* dpatches, const kf_conv_geom* geom, void* dimg, int dtype, void* stream);
/* kf_fwd / kf_features / kf_dgrad / kf_wgrad with x the implicit patch matrix
 * of img (bf16): the kernels gather each receptive field from the image; no
 * patch matrix is made.  kf_conv_dgrad writes the patch-matrix gradient
 * dpatches (rows, cols), which kf_conv_fold turns into the image gradient. */
int kf_conv_fwd(const void* img, const kf_conv_geom* geom, const void* feat, const void* packed, const void* bias,
                const float* knot_tab, void* y, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base,
                const kf_basis_desc* basis, void* stream);
int kf_conv_features(const void* img, const kf_conv_geom* geom, const float* knot_tab, void* feat, int32_t nt, int32_t f_pad,
                     int32_t has_base, const kf_basis_desc* basis, void* stream);
int kf_conv_dgrad(const void* img, const kf_conv_geom* geom, const void* dy, const void* packed, const float* knot_tab,
                  void* dpatches, int32_t O, int32_t nt, int32_t f_pad, int32_t has_base, const kf_basis_desc* basis,
                  void* stream);
int kf_conv_wgrad(const void* img, const kf_conv_geom* geom, const void* feat, const void* dy, const float* knot_tab,
                  const float* fold, const void* coef, const void* edge_scale, const void* edge_mask, void* dcoef, void* dbase,
                  void* dscale, int32_t O, int32_t K, int32_t nt, int32_t f_pad, const kf_basis_desc* basis, void* stream);

/* kf_rational_bwd for callers that cannot allocate device memory.  Some hosts
 * of this library may not call cudaMalloc: code that runs inside a device
 * memory allocator or pool callback (allocating there would re-enter the
 * allocator), frameworks that own every byte of device memory and hand kernels
 * only the buffers they planned, and runtimes that forbid allocation after
 * start-up to keep latency and memory use fixed.  This entry point takes no
 * workspace: the per-CTA partial sums live in a fixed array of
 * KF_RATIONAL_NOALLOC_MAX_FLOATS floats (4 MiB) that is part of the library's
 * device code, so every GPU that loads the library holds it until the process
 * exits.  Requires I * (p + 1 + q) <= KF_RATIONAL_NOALLOC_MAX_FLOATS (else
 * KF_ERR_ARG with a message) and allocates and frees nothing itself.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * and must come before any stream capture.  With CUDA's lazy module loading
 * (the default) that first call may also be what loads the library's device
 * code onto the device, which places the array in device memory then; a host
 * that must see no device allocation after start-up should make one call per
 * device at start-up.  All calls share the array: calls whose
 * kernels overlap on the GPU race.  The caller still passes inputs and outputs.
 * Has no counterpart in the reference. */
#define KF_RATIONAL_NOALLOC_MAX_FLOATS (1 << 20)
int kf_rational_bwd_noalloc(const void* x, const void* dr, const float* num, const float* den, void* dx, float* dnum,
                            float* dden, int64_t B, int32_t I, const kf_basis_desc* basis, int dtype, void* stream);

/* ---- grid tools (kanforge/grid.py:19-85; kanforge/_layer.py:107-183) -------
 * GridToolsMixin.update_grid / refine_grid / change_basis run on the device:
 * the samples never leave it and the (samples x inputs x outputs) refit
 * targets are never formed. */

#define KF_GRID_MAX_POINTS 192 /* grid points per input of kf_adaptive_grid */
#define KF_FIT_MAX_SIZE 256    /* basis functions per edge of kf_refit (old and new) */

/* Samples x (n, I) row-major in `dtype` -> xt (I, n) float32, one column per
 * input: the sample layout of kf_adaptive_grid and kf_refit. */
int kf_samples_transpose(const void* x, int dtype, int64_t n, int32_t I, float* xt, void* stream);

/* Bytes of workspace kf_adaptive_grid needs. */
int64_t kf_grid_workspace(int64_t n, int32_t I, int32_t n_points);

/* Per-input adaptive grids (I, n_points) float64 from the samples xt (I, n)
 * (kanforge/grid.py:19-31, pykan's update_grid_from_samples):
 *   q_t   = the sample of rank round(linspace(0, n-1, n_points)[t]) (halves to even)
 *   u_t   = lo + (hi - lo) t / (n_points - 1),  lo = min - margin, hi = max + margin
 *           (hi - lo < 1e-8: lo -= 0.5, hi += 0.5 and q = u)
 *   grid  = grid_eps u + (1 - grid_eps) q
 * Equal to the reference's float64 result on the same float32 samples.  NaN
 * samples sort last.  2 <= n_points <= KF_GRID_MAX_POINTS, n >= 1,
 * 0 < grid_eps <= 1. */
int kf_adaptive_grid(const float* xt, int64_t n, int32_t I, int32_t n_points, double margin, double grid_eps,
                     double* grid, void* workspace, void* stream);

/* out (I, n_new) = np.interp(linspace(0, 1, n_new), linspace(0, 1, n_old), grid[i])
 * for every row of grid (I, n_old), float64 (kanforge/grid.py:34-38). */
int kf_resample_grid(const double* grid, int32_t I, int32_t n_old, int32_t n_new, double* out, void* stream);

/* A basis as kf_refit evaluates it (order 0, float64).  Constants are the
 * reference's float64 values (kf_basis_desc holds float32 copies). */
typedef struct kf_fit_basis {
  int32_t kind;        /* KF_BASIS_BSPLINE, KF_BASIS_CHEB, KF_BASIS_FOURIER, KF_BASIS_BUMP */
  int32_t size;        /* basis functions per edge, <= KF_FIT_MAX_SIZE */
  int32_t order;       /* B-spline order k */
  int32_t degree;      /* Chebyshev: features T_0..T_degree; Fourier: frequencies */
  int32_t input_map;   /* Chebyshev: KF_MAP_* */
  int32_t bump_mode;   /* bumps: KF_BUMP_* */
  int32_t n_grid;      /* B-spline: G + 1 grid points; bumps: count; else 0 */
  int32_t n_poly;      /* bumps: coefficients in poly */
  const double* grid;  /* (I, n_grid) per-input grid / centres (device), or null */
  const double* fold;  /* Chebyshev: (size, degree + 1), phi_k = sum_j fold[k, j] T_j (device) */
  double freq;         /* Fourier: 2 pi / period */
  double u_scale;      /* gauss bumps */
  double norm;         /* gauss bumps */
  double poly[8];      /* bumps: order-0 polynomial, lowest coefficient first */
} kf_fit_basis;

/* Bytes of workspace kf_refit needs. */
int64_t kf_refit_workspace(int64_t n, int32_t I, int32_t k_old, int32_t k_new);

/* Refit of a layer onto `new_basis` (kanforge/grid.py:55-85 refit and
 * kanforge/_layer.py:120-137 _refit_to):
 *   samples  xt (I, n) float32 (kf_samples_transpose), or, with xt null,
 *            n evenly spaced points per input over ranges (I, 2) float64
 *            (grid.py:49-52 sample_inputs);
 *   targets  the old edge functions sum_k c_eff[o,i,k] phi_k(x), c_eff = coef * edge_scale;
 *   solution per input the least-squares coefficients in the new basis:
 *            with both sizes <= 64 the minimum-norm solution where the samples
 *            leave them undetermined (eigenvalues of the Gram matrix below 1e-13
 *            of the largest are dropped); above, a Cholesky factorisation whose
 *            pivots below 1e-13 of the largest diagonal entry drop that basis
 *            function (coefficient 0: the minimum-norm choice for functions no
 *            sample reaches); ridge > 0 adds ridge * mean(phi_new^2) * n to the
 *            Gram diagonal (the reference's appended damping rows);
 *   outputs  coef_out (O, I, new size) = solution / s and scale_out (O, I) = s,
 *            s = edge_scale where |edge_scale| > 1e-12 else 1, float64.
 * coef (O, I, old size) and edge_scale (O, I, or null) in `dtype`; scale_out
 * is written when edge_scale is given.  Deterministic. */
int kf_refit(const float* xt, const double* ranges, int64_t n, int32_t I, int32_t O, const kf_fit_basis* old_basis,
             const kf_fit_basis* new_basis, const void* coef, const void* edge_scale, int dtype, double ridge,
             double* coef_out, double* scale_out, void* workspace, void* stream);

/* ---- sparse B-spline layers (kanforge/bases/base.py:15-16 local / support) --
 * A B-spline of order k has at most k+1 non-zero functions at any input, so
 * a float32 B-spline KANLinear needs k+1 coefficients per (token, input):
 * these kernels gather them on the CUDA cores instead of running the dense
 * (G+k+1)-wide contraction, for narrow layers whose few outputs would leave a
 * tensor-core tile idle.  Same inputs and results as the dense layer
 * (kanforge/torch/layers.py:171-192 and its autograd):
 *   kf_sparse_fwd   y = sum_i phi_oi(x_i) + sum_i base[o,i] m silu(x_i) + bias
 *   kf_sparse_dgrad dx[b,i] = sum_o dy[b,o] dphi_oi/dx (x_bi)   (base branch included)
 *   kf_sparse_wgrad dcoef = sum_b dy B_j s m, dbase = sum_b dy silu m,
 *                   dscale = sum_j coef sum_b dy B_j m, dbias = sum_b dy
 *                   (fixed-order sums through `workspace`, kf_sparse_wgrad_workspace floats)
 * phi_oi(x) = sum_j coef[o,i,j] s m B_j(x), s = edge_scale, m = edge_mask (null: 1).
 * x (B, I), coef (O, I, G+k), edge_scale / edge_mask / base (O, I), bias (O),
 * grid (I, G+1), y / dy (B, O), dx (B, I): float32.  Outputs of wgrad may be
 * null when not wanted.  basis: KF_BASIS_BSPLINE, order 1..5. */
int kf_sparse_fwd(const float* x, const float* coef, const float* edge_scale, const float* edge_mask, const float* base,
                  const float* bias, const float* grid, float* y, int64_t B, int32_t I, int32_t O,
                  const kf_basis_desc* basis, void* stream);
int kf_sparse_dgrad(const float* x, const float* dy, const float* coef, const float* edge_scale, const float* edge_mask,
                    const float* base, const float* grid, float* dx, int64_t B, int32_t I, int32_t O,
                    const kf_basis_desc* basis, void* stream);
int64_t kf_sparse_wgrad_workspace(int64_t B, int32_t I, int32_t O, const kf_basis_desc* basis);
int kf_sparse_wgrad(const float* x, const float* dy, const float* coef, const float* edge_scale, const float* edge_mask,
                    const float* grid, float* dcoef, float* dbase, float* dscale, float* dbias, float* workspace,
                    int64_t B, int32_t I, int32_t O, const kf_basis_desc* basis, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KANFORGE_B200_H */
