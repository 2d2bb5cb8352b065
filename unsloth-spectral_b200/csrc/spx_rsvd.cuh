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

}  // namespace spx
