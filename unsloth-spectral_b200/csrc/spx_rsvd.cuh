// Parameters of the rSVD lift / quantisation epilogue.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace spx {

struct LiftParams {
  int m, n, r, k, rank_pad;
  const float* Q;    // [Nb][m][r] orthonormal basis of the sketch
  const float* Wk;   // [Nb][r][k] top-k eigenvectors of Bp Bp^T
  const float* Sw;   // [Nb][k] singular values
  const float* Vhw;  // [Nb][k][n] right singular vectors
  float* U;          // optional outputs
  float* S;
  float* Vh;
  int8_t* codes;
  int64_t codes_mat_stride, codes_t_stride, codes_j_stride;
  int codes_tiled;
  float* qscale;
  int64_t scale_mat_stride;
  float* qminmax;
  int64_t minmax_mat_stride;
  void* basis;
  int basis_dtype;
  int64_t basis_mat_stride;
};

// Tensor-core products of the subspace iteration (spx_rsvd_tc.cu): mode 0 Y = M X,
// mode 1 Z = M^T Y, for 16-bit M of 128 columns and m % 128 == 0.
bool rsvd_tc_supported(int dtype, const void* M, int64_t ms, int m, int n, int r);
int rsvd_tc_gemm(int mode, int dtype, const void* M, int64_t ms, const float* X, float* Y, int Nb, int m, int r,
                 cudaStream_t st);

// Fused subspace iteration (spx_rsvd_fused.cu): one CTA per matrix keeps M in shared
// memory for every product and orthonormalisation; writes Q [Nb][m][r] and
// Bp^T = M^T Q [Nb][128][r].  16-bit M of 128 columns, 128 <= m <= 512, m % 128 == 0,
// r % 4 == 0, r <= 40.
bool rsvd_fused_supported(int dtype, const void* M, int64_t ms, const void* omega, int m, int n, int r);
size_t rsvd_fused_smem(int m, int r);
int rsvd_fused(int dtype, const void* M, int64_t ms, const float* omega, float* Q, float* Bt, int Nb, int m, int r,
               int n_iter, cudaStream_t st);

// ------------------------------------------------ device helpers of the rSVD kernels
// 1 / sqrt(x) for a positive finite float64 x, to float32 accuracy (it only scales the
// float32 copy of L): x is scaled by an even power of two into [1, 4), the rsqrtf value
// of that is refined by one Newton-Raphson step y <- y (3 - m y^2) / 2 and the power of
// two put back.  Subnormal x takes the library path.
__device__ __forceinline__ float rsqrt_pos_f(double x) {
  if (x < 2.2250738585072014e-308) return (float)(1.0 / sqrt(x));
  const int e = ((__double2hiint(x) >> 20) & 0x7ff) - 1023;
  const int k = e >> 1;   // floor(e / 2)
  const float m = (float)(x * __hiloint2double((1023 - 2 * k) << 20, 0));
  float y = rsqrtf(m);
  y = y * fmaf(-0.5f * m * y, y, 1.5f);
  return (float)((double)y * __hiloint2double((1023 - k) << 20, 0));
}

// 1 / x for a positive finite float64 x: x = m 2^e with m in [1, 2), the float32
// reciprocal of m refined by one Newton-Raphson step y <- y + y (1 - m y) (relative
// error ~6e-8 -> ~4e-15, far below the float32 result the factor feeds), times 2^-e.
// Subnormal or huge x takes the library path.
__device__ __forceinline__ double recip_pos(double x) {
  const int e = ((__double2hiint(x) >> 20) & 0x7ff) - 1023;
  if (e <= -1023 || e >= 1023) return 1.0 / x;
  const double s = __hiloint2double((1023 - e) << 20, 0);   // 2^-e
  const double m = x * s;
  double y = (double)__frcp_rn((float)m);
  y = fma(y, fma(-m, y, 1.0), y);
  return y * s;
}

// 1 / x for a float64 x >= 2^-1022 (normal) and below 2^1022, without branches: the
// hardware approximation rcp.approx.ftz.f64 refined by one cubically convergent
// Newton-Raphson step y (1 + e + e^2), e = 1 - x y (relative error of the seed ~2^-22 ->
// below float64 rounding).  Used on the critical path of the Cholesky factor, where the
// branch of recip_pos would split the step and add ~150 cycles per column.
__device__ __forceinline__ double recip_fast(double x) {
  double y;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(x));
  const double e = fma(-x, y, 1.0);
  return fma(y, fma(e, e, e), y);
}

// Cholesky factor of one r x r float64 matrix (r <= RMAX <= 40) by ONE warp, right-
// looking, rows in registers.  Lane l holds row l (l < H) and, for RMAX > 32, also row
// RMAX - 1 - l (folded, so both register arrays stay short: H = RMAX / 2).  Step j:
// every lane publishes its rows' (still unscaled) column-j entries to colbuf, then
// updates its entries c > j by G[a][c] -= G[a][j] G[c][j] / G[j][j]; the next pivot's
// row is updated first, so that its reciprocal (recip_fast, broadcast by a shuffle) is
// formed while the rest of the update issues.  Steps past r run on zero rows and change
// nothing.  A pivot counts as zero (its column is zeroed) unless it exceeds 1e-30 times
// the largest diagonal entry and is a normal float64.
//   G        lower triangle, row-major with pitch gp (entries c <= a are read)
//   L        strict lower part of L (each entry times 1/sqrt of its column's pivot, float
//            accuracy) and 1 / L[j][j] on the diagonal, pitch lp
//   colbuf   2 * RMAX doubles, scale_s RMAX doubles: shared scratch of this warp
// Returns, in every lane, npass0 raised by the pivot spread (> 1e6: 2, > 1e12: 3).
template <int RMAX>
__device__ __noinline__ int chol_warp(const double* G, int gp, int r, float* L, int lp, double* colbuf,
                                      double* scale_s, int npass0) {
  static_assert(RMAX <= 40, "two rows per lane at most");
  constexpr bool FOLD = RMAX > 32;
  constexpr int H = FOLD ? RMAX / 2 : RMAX, NB = FOLD ? RMAX : 1;
  const int lane = threadIdx.x & 31;
  const int arow = lane, brow = RMAX - 1 - lane;
  const bool hasa = arow < H && arow < r, hasb = FOLD && lane < H && brow < r;
  auto owner = [](int c) { return (FOLD && c >= H) ? RMAX - 1 - c : c; };
  double ra[H], rb[NB];
#pragma unroll
  for (int c = 0; c < H; ++c) ra[c] = (hasa && c <= arow) ? G[arow * gp + c] : 0.0;
#pragma unroll
  for (int c = 0; c < NB; ++c) rb[c] = (hasb && c <= brow) ? G[brow * gp + c] : 0.0;
  double dm = 0.0;
#pragma unroll
  for (int c = 0; c < H; ++c)
    if (c == arow) dm = fmax(dm, ra[c]);
  if (FOLD) {
#pragma unroll
    for (int c = H; c < NB; ++c)
      if (c == brow) dm = fmax(dm, rb[c]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) dm = fmax(dm, __shfl_xor_sync(0xffffffffu, dm, o));
  const double thr = fmax(1e-30 * dm, 2.2250738585072014e-308);
  const bool dpos = dm > 0.0;
  double coef = __shfl_sync(0xffffffffu, ra[0], 0);
  coef = (coef > thr && dpos) ? recip_fast(coef) : 0.0;
#pragma unroll
  for (int j = 0; j < RMAX; ++j) {
    const double vA = j < H ? ra[j] : 0.0;
    const double vB = FOLD ? rb[j] : 0.0;
    double* cb = colbuf + (j & 1) * RMAX;
    if (lane < H) cb[arow] = vA;
    if (FOLD && lane < H) cb[brow] = vB;
    __syncwarp();
    const double tA = -vA * coef, tB = -vB * coef;
    double ncoef = 0.0;
    if (j + 1 < RMAX) {
      const int c = j + 1;
      const double x = cb[c];
      if (c < H) ra[c < H ? c : 0] = fma(tA, x, ra[c < H ? c : 0]);
      if (FOLD) rb[c < NB ? c : 0] = fma(tB, x, rb[c < NB ? c : 0]);
      const double pr = __shfl_sync(0xffffffffu, (!FOLD || c < H) ? ra[c < H ? c : 0] : rb[c < NB ? c : 0], owner(c));
      ncoef = (pr > thr && dpos) ? recip_fast(pr) : 0.0;
    }
#pragma unroll
    for (int c = j + 2; c < RMAX; ++c) {
      const double x = cb[c];
      if (c < H) ra[c < H ? c : 0] = fma(tA, x, ra[c < H ? c : 0]);
      if (FOLD) rb[c < NB ? c : 0] = fma(tB, x, rb[c < NB ? c : 0]);
    }
    coef = ncoef;
  }
  // pivots are the final diagonal entries; their scales and spread
  double pa = 0.0, pb = 0.0;
#pragma unroll
  for (int c = 0; c < H; ++c)
    if (c == arow) pa = ra[c];
  if (FOLD) {
#pragma unroll
    for (int c = H; c < NB; ++c)
      if (c == brow) pb = rb[c];
  }
  pa = (hasa && pa > thr && dpos) ? pa : 0.0;
  pb = (hasb && pb > thr && dpos) ? pb : 0.0;
  if (hasa) scale_s[arow] = pa > 0.0 ? (double)rsqrt_pos_f(pa) : 0.0;
  if (hasb) scale_s[brow] = pb > 0.0 ? (double)rsqrt_pos_f(pb) : 0.0;
  double pmin = 1e300, pmax = 0.0;
  if (pa > 0.0) {
    pmin = pa;
    pmax = pa;
  }
  if (pb > 0.0) {
    pmin = fmin(pmin, pb);
    pmax = fmax(pmax, pb);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    pmin = fmin(pmin, __shfl_xor_sync(0xffffffffu, pmin, o));
    pmax = fmax(pmax, __shfl_xor_sync(0xffffffffu, pmax, o));
  }
  __syncwarp();
  if (hasa) {
#pragma unroll
    for (int c = 0; c < H; ++c)
      if (c < arow) L[arow * lp + c] = (float)(ra[c] * scale_s[c]);
    L[arow * lp + arow] = (float)scale_s[arow];
  }
  if (hasb) {
#pragma unroll
    for (int c = 0; c < NB; ++c)
      if (c < brow) L[brow * lp + c] = (float)(rb[c] * scale_s[c]);
    L[brow * lp + brow] = (float)scale_s[brow];
  }
  __syncwarp();
  int n = npass0;
  if (pmax > 1e6 * pmin && n < 2) n = 2;
  if (pmax > 1e12 * pmin) n = 3;
  return n;
}

// Number of 4 x 4 tile pairs (ta, tb), (ta, tb + 1) covering the upper triangle of an
// nb4 x nb4 grid of 4 x 4 tiles (the Gram tiling of the Cholesky-QR passes).
__host__ __device__ constexpr int gram_npair(int nb4) {
  int n = 0;
  for (int ta = 0; ta < nb4; ++ta) n += (nb4 - ta + 1) / 2;
  return n;
}

}  // namespace spx
