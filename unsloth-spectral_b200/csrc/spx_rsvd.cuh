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

// Number of 4 x 4 tile pairs (ta, tb), (ta, tb + 1) covering the upper triangle of an
// nb4 x nb4 grid of 4 x 4 tiles (the Gram tiling of the Cholesky-QR passes).
__host__ __device__ constexpr int gram_npair(int nb4) {
  int n = 0;
  for (int ta = 0; ta < nb4; ++ta) n += (nb4 - ta + 1) / 2;
  return n;
}

}  // namespace spx
