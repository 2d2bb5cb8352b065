// Parameters of the rSVD lift / quantisation epilogue.
#pragma once
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

}  // namespace spx
