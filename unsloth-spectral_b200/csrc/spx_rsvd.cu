// Batched randomized SVD + INT8 block compression (spx_rsvd_compress).
//
// Algorithm (unsloth_spectral/rsvd.py:74-157, spectral_cache.py:345-407):
//   Y = M Omega; Q = orth(Y)
//   repeat n_iter: Z = orth(M^T Q); Q = orth(M Z)      (subspace iteration)
//   Bp^T = M^T Q                                        ([n, r])
//   Bp = W S Vh by one-sided Jacobi on the columns of Bp^T (float32, round-robin)
//   U = Q W (truncated to k)
//   C = U * S -> per-matrix INT8 codes, scale, (min, max); basis = Vh in basis dtype.
// The reference runs the power iterations un-normalised; re-orthonormalising every
// step spans the same subspace in exact arithmetic and avoids the float32 loss of the
// un-normalised form.  orth() is Cholesky-QR with a float64 Gram matrix: two passes for
// the final basis (as stable as Householder QR for these panels), one for intermediate
// bases unless their conditioning asks for more.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "spx_common.cuh"
#include "spx_rsvd.cuh"

namespace spx {

// ------------------------------------------------------------ Y = M X  (CUDA cores)
// X: f32 [n][r] per matrix.  Y: f32 [m][r].  grid (ceil(m/64), Nb), 256 threads.
// Register tiles: thread (row pair rp = tid / 8, column group cg = tid % 8) owns rows
// 2rp, 2rp+1 and columns cg, cg + 8, ... (< r <= 64), so each shared-memory load feeds
// several FMAs.
template <typename T>
__global__ void __launch_bounds__(256) gemm_mx_kernel(const T* __restrict__ M, int64_t ms,
                                                      const float* __restrict__ X, float* __restrict__ Y, int m,
                                                      int n, int r) {
  extern __shared__ float sm[];
  float* sx = sm;            // [n][r]
  float* smt = sx + n * r;   // [64][n + 1]
  const int i = blockIdx.y, row0 = blockIdx.x * 64;
  const T* Mi = M + (int64_t)i * ms;
  const float* Xi = X + (int64_t)i * n * r;
  for (int e = threadIdx.x; e < n * r; e += blockDim.x) sx[e] = Xi[e];
  const int rows = min(64, m - row0);
  for (int e = threadIdx.x; e < 64 * n; e += blockDim.x) {
    const int t = e / n, d = e - t * n;
    smt[t * (n + 1) + d] = t < rows ? to_f(Mi[(int64_t)(row0 + t) * n + d]) : 0.f;
  }
  __syncthreads();
  const int rpi = threadIdx.x >> 3, cg = threadIdx.x & 7;
  float acc0[8], acc1[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) acc0[u] = acc1[u] = 0.f;
  const float* m0 = smt + (2 * rpi) * (n + 1);
  const float* m1 = m0 + (n + 1);
  for (int d = 0; d < n; ++d) {
    const float a0 = m0[d], a1 = m1[d];
    const float* xr = sx + d * r;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = cg + 8 * u;
      if (c < r) {
        const float xv = xr[c];
        acc0[u] = fmaf(a0, xv, acc0[u]);
        acc1[u] = fmaf(a1, xv, acc1[u]);
      }
    }
  }
  float* Yi = Y + (int64_t)i * m * r;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int c = cg + 8 * u;
    if (c < r) {
      if (2 * rpi < rows) Yi[(int64_t)(row0 + 2 * rpi) * r + c] = acc0[u];
      if (2 * rpi + 1 < rows) Yi[(int64_t)(row0 + 2 * rpi + 1) * r + c] = acc1[u];
    }
  }
}

// ---------------------------------------------------------- Z = M^T Y (CUDA cores)
// Y: f32 [m][r]; Z: f32 [n][r].  grid (ceil(n/64), Nb), 256 threads.  Thread (column
// pair dp = tid / 8, group cg = tid % 8) owns columns 2dp, 2dp+1 of M and outputs
// cg, cg + 8, ... of r, accumulated over 64-row tiles of M and Y staged in shared memory.
template <typename T>
__global__ void __launch_bounds__(256) gemm_mty_kernel(const T* __restrict__ M, int64_t ms,
                                                       const float* __restrict__ Y, float* __restrict__ Z, int m,
                                                       int n, int r) {
  __shared__ float smt[64][65];
  __shared__ float sy[64][65];
  const int i = blockIdx.y, col0 = blockIdx.x * 64;
  const int cols = min(64, n - col0);
  const T* Mi = M + (int64_t)i * ms;
  const float* Yi = Y + (int64_t)i * m * r;
  const int dpi = threadIdx.x >> 3, cg = threadIdx.x & 7;
  float acc0[8], acc1[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) acc0[u] = acc1[u] = 0.f;
  for (int t0 = 0; t0 < m; t0 += 64) {
    const int rows = min(64, m - t0);
    __syncthreads();
    for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
      const int t = e >> 6, d = e & 63;
      smt[t][d] = (t < rows && d < cols) ? to_f(Mi[(int64_t)(t0 + t) * n + col0 + d]) : 0.f;
    }
    for (int e = threadIdx.x; e < 64 * r; e += blockDim.x) {
      const int t = e / r, c = e - t * r;
      sy[t][c] = t < rows ? Yi[(int64_t)(t0 + t) * r + c] : 0.f;
    }
    __syncthreads();
    for (int t = 0; t < 64; ++t) {
      const float a0 = smt[t][2 * dpi], a1 = smt[t][2 * dpi + 1];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = cg + 8 * u;
        if (c < r) {
          const float yv = sy[t][c];
          acc0[u] = fmaf(a0, yv, acc0[u]);
          acc1[u] = fmaf(a1, yv, acc1[u]);
        }
      }
    }
  }
  float* Zi = Z + (int64_t)i * n * r;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int c = cg + 8 * u;
    if (c < r) {
      if (2 * dpi < cols) Zi[(int64_t)(col0 + 2 * dpi) * r + c] = acc0[u];
      if (2 * dpi + 1 < cols) Zi[(int64_t)(col0 + 2 * dpi + 1) * r + c] = acc1[u];
    }
  }
}


// ------------------------------------- Cholesky-QR orthonormalisation, three kernels
// X: f32 [rows][r] per matrix, orthonormalised in place.  Each pass forms the Gram
// matrix G = X^T X in float64 (products of two float32 values are exact in float64),
// factors G = L L^T in float64 and solves X := X L^{-T}.  Two passes give an orthonormal
// basis to float32 accuracy while cond(X) <= ~1e6; a third runs when the first pass's
// pivots spread by more than 1e12.  The intermediate bases of the subspace iteration
// (which only need a well-conditioned basis of the right span) ask for one pass; a
// second then runs only when the pivots spread by more than 1e6 (cond(X) > 1e3).  A
// pivot at rounding level of a zero column (relative 1e-30) leaves that column zero.
// A pass is three kernels, so that each step gets the parallelism it needs: a float64
// Gram kernel (the panel streams through shared memory in 128-row chunks), a
// Cholesky-only kernel (one small CTA per matrix, many per SM: the 40-odd dependent
// column steps of many matrices overlap) and a row-parallel triangular solve.  np[i]
// holds the number of passes matrix i needs: the Gram kernel of pass 0 sets it to the
// requested count npass0 and zeroes the list count, and the Cholesky of pass 0 raises it
// from the pivot spread and appends i to a list when it does.  Passes below npass0 run
// one CTA per matrix; a later pass (usually needed by no matrix) runs small grids that
// stride over the listed matrices and skip those that need no more.
constexpr int kGramChunk = 128;
// Gram tiling: 4 x 4 tiles of the upper triangle, taken in pairs (ta, tb), (ta, tb + 1)
// that share the a-block, so a row converts 12 float32 values to float64 per 32 FMAs (16
// for two separate tiles; the float32 -> float64 conversion issues at a quarter of the
// float64 FMA rate).  A pair is split over S interleaved row subsets (rows t = s mod S of
// every chunk) so that most threads are busy; the S partial sums of an entry are added in
// a fixed order, so the result is deterministic.  The chunk's row pitch P covers every
// column a tile reads (columns r .. 4 NB4 - 1 are zero), so the inner loop has no bounds
// tests.  The last pair of an odd row of tiles computes a dummy second tile, not stored.
template <int RMAX>
struct GramTiling {
  static constexpr int NB4 = (RMAX + 3) / 4;
  static constexpr int NTILE = NB4 * (NB4 + 1) / 2;
  static constexpr int NPAIR = gram_npair(NB4);
  static constexpr int NT = RMAX > 40 ? 256 : 128;   // threads
  static constexpr int S = NT / NPAIR >= 8 ? 8 : NT / NPAIR >= 1 ? NT / NPAIR : 1;
  static constexpr int TPT = (NPAIR * S + NT - 1) / NT;   // items per thread
  static constexpr int P = (4 * NB4) | 1;                 // chunk row pitch (floats)
  static constexpr int CHUNK_FLOATS = (kGramChunk * P + 3) & ~3;
  static constexpr size_t SMEM = (size_t)CHUNK_FLOATS * sizeof(float) + (size_t)S * NTILE * 16 * sizeof(double);
};
size_t gram_smem(int r) {
  return r <= 24 ? GramTiling<24>::SMEM : r <= 40 ? GramTiling<40>::SMEM : GramTiling<64>::SMEM;
}
int gram_threads(int r) { return r <= 24 ? GramTiling<24>::NT : r <= 40 ? GramTiling<40>::NT : GramTiling<64>::NT; }

template <int RMAX>
__global__ void __launch_bounds__(GramTiling<RMAX>::NT, RMAX > 40 ? 1 : 4) gram_kernel(const float* __restrict__ X, double* __restrict__ Gw,
                                                   int* __restrict__ np, const int* __restrict__ list,
                                                   int* __restrict__ cnt, int pass, int npass0, int rows, int r) {
  using GT = GramTiling<RMAX>;
  constexpr int NT = GT::NT, P = GT::P;
  const int tid = threadIdx.x;
  const bool listed = pass >= npass0;
  if (pass == 0 && blockIdx.x == 0 && tid == 0) *cnt = 0;
  if (listed && (int)blockIdx.x >= *cnt) return;   // nothing listed for this CTA
  extern __shared__ __align__(16) float gsm[];
  float* sxc = gsm;                                                   // [kGramChunk][P]
  double* red = reinterpret_cast<double*>(gsm + GT::CHUNK_FLOATS);    // [S][NTILE][16]
  // items: (pair, row subset); pair (ta, tb), (ta, tb + 1) of 4 x 4 blocks, ta <= tb
  int it_a[GT::TPT], it_b[GT::TPT], it_c[GT::TPT], it_s[GT::TPT], it_t0[GT::TPT];
  bool it_two[GT::TPT];
#pragma unroll
  for (int q = 0; q < GT::TPT; ++q) {
    const int item = tid + NT * q;
    it_a[q] = -1;
    it_b[q] = it_c[q] = it_s[q] = it_t0[q] = 0;
    it_two[q] = false;
    if (item < GT::NPAIR * GT::S) {
      int p = item / GT::S, ta = 0;
      it_s[q] = item - p * GT::S;
      while (p >= (GT::NB4 - ta + 1) / 2) {
        p -= (GT::NB4 - ta + 1) / 2;
        ++ta;
      }
      const int tb = ta + 2 * p;
      it_two[q] = tb + 1 < GT::NB4;
      it_a[q] = 4 * ta;
      it_b[q] = 4 * tb;
      it_c[q] = it_two[q] ? 4 * (tb + 1) : 4 * ta;   // dummy second tile: any valid columns
      it_t0[q] = ta * GT::NB4 - ta * (ta - 1) / 2 + (tb - ta);   // tile index of (ta, tb)
    }
  }
  const int nk = listed ? *cnt : gridDim.x;
  for (int kk = blockIdx.x; kk < nk; kk += gridDim.x) {
    const int i = listed ? list[kk] : kk;
    if (pass == 0) {
      if (tid == 0) np[i] = npass0;
    } else if (listed && pass >= np[i]) {
      continue;
    }
    double g[GT::TPT][2][16];
#pragma unroll
    for (int q = 0; q < GT::TPT; ++q)
#pragma unroll
      for (int e = 0; e < 16; ++e) g[q][0][e] = g[q][1][e] = 0.0;
    const float* Xi = X + (int64_t)i * rows * r;
    for (int c0 = 0; c0 < rows; c0 += kGramChunk) {
      const int nrow = min(kGramChunk, rows - c0);
      __syncthreads();
      if ((r & 3) == 0) {   // float4 loads, all of a thread's in flight at once
        const int n4 = nrow * r / 4;
        const float4* X4 = reinterpret_cast<const float4*>(Xi + (int64_t)c0 * r);
        constexpr int U = (kGramChunk * RMAX / 4 + NT - 1) / NT;
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int e = tid + NT * u;
          v[u] = e < n4 ? __ldg(X4 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int e = 4 * (tid + NT * u);
          if (e < nrow * r) {
            const int t = e / r, c = e - t * r;   // r % 4 == 0: the four stay in row t
            float* d = sxc + t * P + c;
            d[0] = v[u].x;
            d[1] = v[u].y;
            d[2] = v[u].z;
            d[3] = v[u].w;
          }
        }
      } else {
        for (int e = tid; e < nrow * r; e += NT) {
          const int t = e / r, c = e - t * r;
          sxc[t * P + c] = Xi[(int64_t)c0 * r + e];
        }
      }
      // zero the columns r .. 4 NB4 - 1 (read by edge tiles, never stored)
      for (int e = tid; e < nrow * (4 * GT::NB4 - r); e += NT) {
        const int w4 = 4 * GT::NB4 - r, t = e / w4;
        sxc[t * P + r + (e - t * w4)] = 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < GT::TPT; ++q) {
        if (it_a[q] < 0) continue;
        const float* xa_p = sxc + it_a[q];
        const float* xb_p = sxc + it_b[q];
        const float* xc_p = sxc + it_c[q];
#pragma unroll 2
        for (int t = it_s[q]; t < nrow; t += GT::S) {
          double xa[4], xb[4], xc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            xa[u] = xa_p[t * P + u];
            xb[u] = xb_p[t * P + u];
            xc[u] = xc_p[t * P + u];
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              g[q][0][4 * u + v] = fma(xa[u], xb[v], g[q][0][4 * u + v]);
              g[q][1][4 * u + v] = fma(xa[u], xc[v], g[q][1][4 * u + v]);
            }
        }
      }
    }
    // partial sums -> shared memory; fixed-order sum over the S row subsets
#pragma unroll
    for (int q = 0; q < GT::TPT; ++q) {
      if (it_a[q] < 0) continue;
      // element-major, red[(entry * S + subset) * NTILE + tile]: conflict-free stores
      // from the threads of a warp and consecutive reads for the summing threads
      double* dst = red + (int64_t)it_s[q] * GT::NTILE + it_t0[q];
#pragma unroll
      for (int e = 0; e < 16; ++e) dst[(int64_t)e * GT::S * GT::NTILE] = g[q][0][e];
      if (it_two[q]) {
#pragma unroll
        for (int e = 0; e < 16; ++e) dst[(int64_t)e * GT::S * GT::NTILE + 1] = g[q][1][e];   // tile (ta, tb + 1) is the next index
      }
    }
    __syncthreads();
    double* Gi = Gw + (int64_t)i * r * r;
    for (int e2 = tid; e2 < GT::NTILE * 16; e2 += NT) {
      const int idx = e2 / GT::NTILE, tile = e2 - idx * GT::NTILE, u = idx >> 2, v = idx & 3;
      double sum = 0.0;
      for (int s2 = 0; s2 < GT::S; ++s2) sum += red[((int64_t)idx * GT::S + s2) * GT::NTILE + tile];
      // tile index -> (ta, tb)
      int tb = tile, ta = 0;
      while (tb >= GT::NB4 - ta) {
        tb -= GT::NB4 - ta;
        ++ta;
      }
      tb += ta;
      const int col = 4 * ta + u, row = 4 * tb + v;   // entry (a, b) = (col, row), a <= b for lower storage
      if (row < r && col < r && col <= row) Gi[row * r + col] = sum;
    }
    __syncthreads();   // red is rewritten for the next matrix of a listed pass
  }
}

// Factor G = L L^T of one matrix per CTA, right-looking with one block barrier per
// column.  Each thread owns fixed lower-triangle entries (a, c) and keeps them in
// registers; in step j it updates those with c > j from the still unscaled column j,
// G[a][c] -= G[a][j] G[c][j] / G[j][j], reading column j from a shared copy that the
// owners of its entries published in step j - 1 (two alternating buffers, so one
// barrier per step suffices).  The owner of diagonal entry j + 1 publishes 1 / pivot
// (float64, a Newton-refined reciprocal) for the next step; thread NT - 1 computes
// 1 / sqrt(pivot) at float accuracy (it only scales the float32 copy of L).  Writes
// Lw [r][r] f32: strict lower part L (each entry times the 1 / sqrt(pivot) of its
// column), 1 / L[j][j] on the diagonal.  In pass 0 the pivot spread raises np[i] and
// appends i to the list of matrices that need more passes than requested.
constexpr int kCholThreads = 128;
template <int RMAX>
__global__ void __launch_bounds__(kCholThreads, RMAX <= 24 ? 10 : RMAX <= 40 ? 8 : 6)
    chol_kernel(const double* __restrict__ Gw, float* __restrict__ Lw, int* __restrict__ np,
                int* __restrict__ list, int* __restrict__ cnt, int pass, int npass0, int r) {
  constexpr int NT = kCholThreads;
  constexpr int OWN = (RMAX * (RMAX + 1) / 2 + NT - 1) / NT;
  const int tid = threadIdx.x;
  const bool listed = pass >= npass0;
  if (listed && (int)blockIdx.x >= *cnt) return;   // nothing listed for this CTA
  __shared__ double colj[2][RMAX];   // unscaled column j (rows > j), published in step j - 1
  __shared__ double diag[RMAX];
  __shared__ double dmax_s;
  __shared__ double pivs[RMAX], coef_s[RMAX], scale_s[RMAX];
  int own[OWN];   // a * 256 + c, or -1
  const int ntri = r * (r + 1) / 2;
#pragma unroll
  for (int q = 0; q < OWN; ++q) {
    const int e = tid + NT * q;
    if (e < ntri) {
      int a = (int)((sqrt(8.0 * e + 1.0) - 1.0) * 0.5);
      while (a * (a + 1) / 2 > e) --a;
      while ((a + 1) * (a + 2) / 2 <= e) ++a;
      own[q] = a * 256 + (e - a * (a + 1) / 2);
    } else {
      own[q] = -1;
    }
  }
  const int nk = listed ? *cnt : gridDim.x;
  for (int kk = blockIdx.x; kk < nk; kk += gridDim.x) {
    const int i = listed ? list[kk] : kk;
    if (listed && pass >= np[i]) continue;
    const double* Gi = Gw + (int64_t)i * r * r;
    double g[OWN];
#pragma unroll
    for (int q = 0; q < OWN; ++q) {
      const int a = own[q] >> 8, c = own[q] & 255;
      g[q] = 0.0;
      if (own[q] >= 0) {
        g[q] = Gi[a * r + c];
        if (c == 0) colj[0][a] = g[q];
        if (c == a) diag[a] = g[q];
      }
    }
    __syncthreads();
    if (tid == 0) {
      double dm = 0.0;
      for (int j = 0; j < r; ++j) dm = fmax(dm, diag[j]);
      dmax_s = dm;
      const double p0 = diag[0];
      const bool ok = p0 > 1e-30 * dm && dm > 0.0;
      pivs[0] = ok ? p0 : 0.0;
      coef_s[0] = ok ? recip_pos(p0) : 0.0;
    }
    __syncthreads();
    const double dmax = dmax_s;
    for (int j = 0; j < r; ++j) {
      const double coef = coef_s[j];
      const double* cj = colj[j & 1];
      double* cn = colj[(j + 1) & 1];
#pragma unroll
      for (int q = 0; q < OWN; ++q) {
        const int a = own[q] >> 8, c = own[q] & 255;
        if (own[q] >= 0 && c > j) {
          const double v = fma(-cj[a] * coef, cj[c], g[q]);
          g[q] = v;
          if (c == j + 1) {
            cn[a] = v;
            if (a == j + 1) {
              const bool ok = v > 1e-30 * dmax && dmax > 0.0;
              pivs[j + 1] = ok ? v : 0.0;
              coef_s[j + 1] = ok ? recip_pos(v) : 0.0;
            }
          }
        }
      }
      if (tid == NT - 1) scale_s[j] = pivs[j] > 0.0 ? (double)rsqrt_pos_f(pivs[j]) : 0.0;
      __syncthreads();
    }
    float* Li = Lw + (int64_t)i * r * r;
#pragma unroll
    for (int q = 0; q < OWN; ++q) {
      const int a = own[q] >> 8, c = own[q] & 255;
      if (own[q] >= 0 && a > c) Li[a * r + c] = (float)(g[q] * scale_s[c]);
    }
    for (int j = tid; j < r; j += NT) Li[j * r + j] = (float)scale_s[j];
    if (tid == 0 && pass == 0) {
      double pmin = 1e300, pmax = 0.0;
      for (int j = 0; j < r; ++j)
        if (pivs[j] > 0.0) {
          pmin = fmin(pmin, pivs[j]);
          pmax = fmax(pmax, pivs[j]);
        }
      const int n0 = np[i];
      int n = n0;
      if (pmax > 1e6 * pmin && n < 2) n = 2;
      if (pmax > 1e12 * pmin) n = 3;
      np[i] = n;
      if (n > n0) list[atomicAdd(cnt, 1)] = i;
    }
    __syncthreads();   // shared state is rewritten for the next matrix of a listed pass
  }
}

// The same factor for r <= 40 with one warp per matrix (chol_warp: rows in registers, no
// block barriers, the next pivot's reciprocal formed while a column's update issues):
// 2.6x the throughput of chol_kernel at 4096 matrices on B200.  Same outputs and pass
// rules; a pivot must also be a normal float64 to count.
constexpr int kCholWarps = 2;
template <int RMAX>
__global__ void __launch_bounds__(kCholWarps * 32)
    chol_warp_kernel(const double* __restrict__ Gw, float* __restrict__ Lw, int* __restrict__ np,
                     int* __restrict__ list, int* __restrict__ cnt, int pass, int npass0, int r, int Nb) {
  __shared__ double colbuf[kCholWarps][2 * RMAX];
  __shared__ double scale_s[kCholWarps][RMAX];
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool listed = pass >= npass0;
  const int nk = listed ? *cnt : Nb;
  for (int kk = blockIdx.x * kCholWarps + wi; kk < nk; kk += gridDim.x * kCholWarps) {
    const int i = listed ? list[kk] : kk;
    if (listed && pass >= np[i]) continue;
    const int n0 = np[i];
    const int n = chol_warp<RMAX>(Gw + (int64_t)i * r * r, r, r, Lw + (int64_t)i * r * r, r, colbuf[wi],
                                  scale_s[wi], n0);
    if (lane == 0 && pass == 0) {
      np[i] = n;
      if (n > n0) list[atomicAdd(cnt, 1)] = i;
    }
    __syncwarp();
  }
}

// X := X L^{-T}, grid (matrices, 128-row chunks), 128 threads.  The chunk is staged in
// shared memory with coalesced float4 copies (odd row pitch: a thread reads its own row
// conflict-free), each thread substitutes its row in registers reading L four entries
// at a time (pitch rounded up to 4), and the chunk is copied back the same way.
size_t trsolve_smem(int r) { return ((size_t)r * ((r + 3) & ~3) + 128 * (size_t)(r | 1)) * sizeof(float); }

template <int RMAX>
__global__ void __launch_bounds__(128) trsolve_kernel(float* __restrict__ X, const float* __restrict__ Lw,
                                                      const int* __restrict__ np, const int* __restrict__ list,
                                                      const int* __restrict__ cnt, int pass, int npass0, int rows,
                                                      int r) {
  const int tid = threadIdx.x;
  constexpr int R4 = (RMAX + 3) & ~3;
  extern __shared__ __align__(16) float tsm[];
  const int r4 = (r + 3) & ~3, rp = r | 1;
  float* Ls = tsm;             // [r][r4]
  float* sx = tsm + r * r4;    // [128][rp]
  const bool listed = pass >= npass0;
  const int nk = listed ? *cnt : gridDim.x;
  for (int kk = blockIdx.x; kk < nk; kk += gridDim.x) {
    const int i = listed ? list[kk] : kk;
    if (listed && pass >= np[i]) continue;
    const float* Li = Lw + (int64_t)i * r * r;
    const int t0 = blockIdx.y * 128, nrow = min(128, rows - t0);
    float* Xc = X + ((int64_t)i * rows + t0) * r;
    const bool vec = (r & 3) == 0;
    if (vec) {   // r4 == r: L and the chunk are contiguous; float4 loads, all in flight at once
      constexpr int UL = (RMAX * RMAX / 4 + 127) / 128, UX = (128 * RMAX / 4 + 127) / 128;
      const float4* L4 = reinterpret_cast<const float4*>(Li);
      const float4* X4 = reinterpret_cast<const float4*>(Xc);
      const int nl4 = r * r / 4, nx4 = nrow * r / 4;
      float4 vl[UL], vx[UX];
#pragma unroll
      for (int u = 0; u < UL; ++u) {
        const int e = tid + 128 * u;
        vl[u] = e < nl4 ? __ldg(L4 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < UX; ++u) {
        const int e = tid + 128 * u;
        vx[u] = e < nx4 ? X4[e] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < UL; ++u) {
        const int e = tid + 128 * u;
        if (e < nl4) reinterpret_cast<float4*>(Ls)[e] = vl[u];
      }
#pragma unroll
      for (int u = 0; u < UX; ++u) {
        const int e = tid + 128 * u;
        if (e < nx4) {
          const int t = (4 * e) / r, c = 4 * e - t * r;
          float* d = sx + t * rp + c;
          d[0] = vx[u].x;
          d[1] = vx[u].y;
          d[2] = vx[u].z;
          d[3] = vx[u].w;
        }
      }
    } else {
      for (int e = tid; e < r * r4; e += 128) {
        const int j = e / r4, c = e - j * r4;
        Ls[e] = c < r ? Li[j * r + c] : 0.f;
      }
      for (int e = tid; e < nrow * r; e += 128) {
        const int t = e / r, c = e - t * r;
        sx[t * rp + c] = Xc[e];
      }
    }
    __syncthreads();
    if (tid < nrow) {
      float* xr = sx + tid * rp;
      float x[R4];
#pragma unroll
      for (int c = 0; c < R4; ++c) x[c] = c < r ? xr[c] : 0.f;
#pragma unroll
      for (int j = 0; j < RMAX; ++j) {
        if (j < r) {
          const float4* lj = reinterpret_cast<const float4*>(Ls + j * r4);
          float a0 = x[j], a1 = 0.f;
#pragma unroll
          for (int c = 0; c < (j & ~3); c += 4) {   // entries c < j in whole quads
            const float4 l = lj[c >> 2];
            a0 = fmaf(-x[c], l.x, a0);
            a1 = fmaf(-x[c + 1], l.y, a1);
            a0 = fmaf(-x[c + 2], l.z, a0);
            a1 = fmaf(-x[c + 3], l.w, a1);
          }
          if (j & 3) {   // the partial quad holding columns (j & ~3) .. j - 1 and the diagonal
            const float4 l = lj[j >> 2];
            const int c = j & ~3;
            a0 = fmaf(-x[c], l.x, a0);
            if ((j & 3) > 1) a1 = fmaf(-x[c + 1], l.y, a1);
            if ((j & 3) > 2) a0 = fmaf(-x[c + 2], l.z, a0);
          }
          x[j] = (a0 + a1) * Ls[j * r4 + j];
        }
      }
#pragma unroll
      for (int c = 0; c < R4; ++c)
        if (c < r) xr[c] = x[c];
    }
    __syncthreads();
    if (vec) {
      float4* X4 = reinterpret_cast<float4*>(Xc);
      for (int e = tid; e < nrow * r / 4; e += 128) {
        const int t = (4 * e) / r, c = 4 * e - t * r;
        const float* d = sx + t * rp + c;
        X4[e] = make_float4(d[0], d[1], d[2], d[3]);
      }
    } else {
      for (int e = tid; e < nrow * r; e += 128) {
        const int t = e / r, c = e - t * r;
        Xc[e] = sx[t * rp + c];
      }
    }
    __syncthreads();   // shared memory is rewritten for the next matrix of a listed pass
  }
}

// ------------------------------------------------ small SVD by one-sided Jacobi
// Z = Bp^T: f32 [n][r] (n <= 128, r <= 64).  One-sided (Hestenes) Jacobi on the columns
// of A = Bp^T: plane rotations A J make the columns orthogonal; then A J = Vh^T S (column
// norms are the singular values) and J holds the left singular vectors of Bp, i.e. the
// eigenvectors of Bp Bp^T.  Bp Bp^T is never formed, so small singular values keep their
// relative accuracy in float32.  A round applies rp/2 disjoint rotations (circle
// ordering: index rp-1 meets `round`, pair u >= 1 couples round +- u modulo rp-1), one
// 8-lane group per rotation (four rotations per warp at once); a pair is rotated while
// |a_p . a_q| > 2e-6 |a_p| |a_q| (a few times the float32 rounding of a 128-term dot
// product), and a sweep without rotations ends the iteration.  The squared column norms
// are recomputed at the start of every sweep and updated in between by the exact
// relations |a_p'|^2 = |a_p|^2 - t a_p.a_q, |a_q'|^2 = |a_q|^2 + t a_p.a_q, so a rotation
// needs one reduction (a_p . a_q) instead of three.
// Outputs Wk f32 [r][k], S f32 [k], Vh f32 [k][n] (descending singular values).
__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
size_t small_svd_smem(int n, int r) {
  const int rp = (r + 1) & ~1;
  return ((size_t)rp * 128 + (size_t)rp * rp + 2 * rp) * sizeof(float) + rp * sizeof(int);
}

__global__ void __launch_bounds__(256) small_svd_kernel(const float* __restrict__ Z, float* __restrict__ Wk,
                                                        float* __restrict__ S, float* __restrict__ Vh, int n, int r,
                                                        int k) {
  extern __shared__ float smf[];
  const int rp = (r + 1) & ~1;        // padded to even for the round-robin ordering
  float* A = smf;                     // [rp][128] columns of Bp^T (zero padded)
  float* J = A + rp * 128;            // [rp][rp] column-major: J[c * rp + a] = J(a, c)
  float* nrm = J + rp * rp;           // [rp] column norms
  float* n2 = nrm + rp;               // [rp] squared column norms during the sweeps
  int* perm = reinterpret_cast<int*>(n2 + rp);   // [rp]
  __shared__ int rotated;
  const int i = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const float* Zi = Z + (int64_t)i * n * r;
  for (int e = tid; e < rp * 128; e += blockDim.x) {
    const int c = e >> 7, d = e & 127;
    A[e] = (c < r && d < n) ? Zi[(int64_t)d * r + c] : 0.f;
  }
  for (int e = tid; e < rp * rp; e += blockDim.x) J[e] = (e / rp == e % rp) ? 1.f : 0.f;
  __syncthreads();
  const int np = rp / 2, nn = rp - 1;
  const int grp = lane >> 3, gl = lane & 7;   // rotation slot of this lane's 8-lane group
  const unsigned gmask = 0xFFu << (8 * grp);
  for (int sweep = 0; sweep < 30; ++sweep) {
    for (int c = warp; c < rp; c += nw) {
      const float4 v = reinterpret_cast<const float4*>(A + c * 128)[lane];
      const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      if (lane == 0) n2[c] = ss;
    }
    if (tid == 0) rotated = 0;
    __syncthreads();
    for (int round = 0; round < nn; ++round) {
      for (int u = 4 * warp + grp; u < np; u += 4 * nw) {
        // pair u of the round: 0 <= round < nn and 1 <= u < np <= nn, so one wrap suffices
        int p = round + u, q = round - u;
        if (p >= nn) p -= nn;
        if (q < 0) q += nn;
        if (u == 0) q = nn;
        if (p > q) { const int tmp = p; p = q; q = tmp; }
        if (q >= r) continue;   // the padding column (uniform across the group)
        float4* cp = reinterpret_cast<float4*>(A + p * 128);
        float4* cq = reinterpret_cast<float4*>(A + q * 128);
        float4 ap[4], aq[4];
        float ga = 0.f;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          ap[v] = cp[gl + 8 * v];
          aq[v] = cq[gl + 8 * v];
          ga += ap[v].x * aq[v].x + ap[v].y * aq[v].y + ap[v].z * aq[v].z + ap[v].w * aq[v].w;
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) ga += __shfl_xor_sync(gmask, ga, o);
        const float al = n2[p], be = n2[q];
        if (!(ga * ga > 4e-12f * (al * be)) || ga == 0.f) continue;   // |ga| > 2e-6 sqrt(al be)
        // the rotation: approximate division and square root are enough, since c and s
        // are formed as rsqrt(1 + t^2) and t c, a rotation whatever the rounding of t
        const float zeta = __fdividef(be - al, 2.f * ga);
        const float t = __fdividef(zeta >= 0.f ? 1.f : -1.f, fabsf(zeta) + sqrt_approx(fmaf(zeta, zeta, 1.f)));
        const float c = rsqrtf(fmaf(t, t, 1.f)), sn = t * c;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float4 np4, nq4;
          np4.x = c * ap[v].x - sn * aq[v].x; nq4.x = sn * ap[v].x + c * aq[v].x;
          np4.y = c * ap[v].y - sn * aq[v].y; nq4.y = sn * ap[v].y + c * aq[v].y;
          np4.z = c * ap[v].z - sn * aq[v].z; nq4.z = sn * ap[v].z + c * aq[v].z;
          np4.w = c * ap[v].w - sn * aq[v].w; nq4.w = sn * ap[v].w + c * aq[v].w;
          cp[gl + 8 * v] = np4;
          cq[gl + 8 * v] = nq4;
        }
        for (int a = gl; a < r; a += 8) {
          const float jp = J[p * rp + a], jq = J[q * rp + a];
          J[p * rp + a] = c * jp - sn * jq;
          J[q * rp + a] = sn * jp + c * jq;
        }
        __syncwarp(gmask);
        if (gl == 0) {
          n2[p] = al - t * ga;
          n2[q] = be + t * ga;
          rotated = 1;
        }
      }
      __syncthreads();
    }
    if (!rotated) break;
    __syncthreads();
  }
  // singular values = column norms; order descending (rank, ties by index)
  for (int c = warp; c < r; c += nw) {
    const float4 v = reinterpret_cast<const float4*>(A + c * 128)[lane];
    const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if (lane == 0) nrm[c] = sqrtf(ss);
  }
  __syncthreads();
  for (int a = tid; a < r; a += blockDim.x) {
    const float na = nrm[a];
    int rank = 0;
    for (int b = 0; b < r; ++b) rank += (nrm[b] > na) || (nrm[b] == na && b < a);
    perm[rank] = a;
  }
  __syncthreads();
  const float s0 = nrm[perm[0]];
  for (int j = tid; j < k; j += blockDim.x) S[(int64_t)i * k + j] = nrm[perm[j]];
  for (int e = tid; e < r * k; e += blockDim.x) {
    const int a = e / k, j = e - a * k;
    Wk[(int64_t)i * r * k + e] = J[perm[j] * rp + a];
  }
  for (int e = tid; e < k * n; e += blockDim.x) {
    const int j = e / n, d = e - j * n;
    const int pj = perm[j];
    const float sj = nrm[pj];
    Vh[(int64_t)i * k * n + e] = (sj > 1e-12f * s0 && sj > 0.f) ? A[pj * 128 + d] / sj : 0.f;
  }
}

// ------------------------------------------------- lift, C = U S, INT8 quantisation
// Shared memory of lift_quant_kernel: W^T [k][r4], C [m][k + 1] (odd pitch: the
// row-per-thread writes are bank-conflict free).
// Shared memory of lift_quant_kernel: W^T [k][r4] f32, a chunk of INT8 codes [256][kp].
size_t lift_smem(int m, int r, int k, int kp) {
  const int r4 = (r + 3) & ~3;
  return (size_t)k * r4 * sizeof(float) + (size_t)256 * kp;
}

// One CTA per matrix, two passes over the rows of U = Q W (a thread holds a row of Q in
// registers and reads W^T from shared memory four entries at a time).  Pass 1 writes U
// (when asked for) and reduces min / max / absmax of C = U S; pass 2 recomputes the rows
// with the same instruction sequence - so C is bit-identical - and quantises them, the
// codes of 256 rows at a time staged in shared memory and written out in the
// destination's element order.  Holding C between the passes instead would take
// m (k + 1) floats of shared memory and cap the kernel at three CTAs per SM.
template <int RMAX>
__global__ void __launch_bounds__(256) lift_quant_kernel(LiftParams p) {
  extern __shared__ float sm[];
  const int m = p.m, r = p.r, k = p.k, n = p.n;
  const int r4 = (r + 3) & ~3;
  float* swt = sm;                                           // [k][r4] W^T, zero padded
  int8_t* scodes = reinterpret_cast<int8_t*>(swt + k * r4);  // [256][kp]
  __shared__ float ss[64];
  __shared__ float red[3][32];
  const int i = blockIdx.x;
  for (int e = threadIdx.x; e < k * r4; e += blockDim.x) {
    const int j = e / r4, a = e - j * r4;
    swt[e] = a < r ? p.Wk[(int64_t)i * r * k + (int64_t)a * k + j] : 0.f;
  }
  if (threadIdx.x < k) ss[threadIdx.x] = p.Sw[(int64_t)i * k + threadIdx.x];
  __syncthreads();
  const float* Qi = p.Q + (int64_t)i * m * r;
  auto load_row = [&](int t, float (&q)[RMAX]) {
    if ((r & 3) == 0) {   // rows of 16-byte multiples: float4 loads
      const float4* q4 = reinterpret_cast<const float4*>(Qi + (int64_t)t * r);
#pragma unroll
      for (int a = 0; a < RMAX; a += 4) {
        const float4 v = a < r ? __ldg(q4 + (a >> 2)) : make_float4(0.f, 0.f, 0.f, 0.f);
        q[a] = v.x;
        q[a + 1] = v.y;
        q[a + 2] = v.z;
        q[a + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int a = 0; a < RMAX; ++a) q[a] = a < r ? __ldg(Qi + (int64_t)t * r + a) : 0.f;
    }
  };
  auto u_of = [&](const float (&q)[RMAX], int j) {
    const float4* w4 = reinterpret_cast<const float4*>(swt + j * r4);
    float u0 = 0.f, u1 = 0.f;
#pragma unroll
    for (int a = 0; a < RMAX; a += 4) {
      if (a < r) {
        const float4 w = w4[a >> 2];
        u0 = fmaf(q[a], w.x, u0);
        u1 = fmaf(q[a + 1], w.y, u1);
        u0 = fmaf(q[a + 2], w.z, u0);
        u1 = fmaf(q[a + 3], w.w, u1);
      }
    }
    return u0 + u1;
  };
  float mn = INFINITY, mx = -INFINITY, am = 0.f;
  for (int t = threadIdx.x; t < m; t += blockDim.x) {
    float q[RMAX];
    load_row(t, q);
    for (int j = 0; j < k; ++j) {
      const float u = u_of(q, j);
      if (p.U) p.U[(int64_t)i * m * k + (int64_t)t * k + j] = u;
      const float c = u * ss[j];
      mn = fminf(mn, c);
      mx = fmaxf(mx, c);
      am = fmaxf(am, fabsf(c));
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    red[0][warp] = mn;
    red[1][warp] = mx;
    red[2][warp] = am;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w) {
      mn = fminf(mn, red[0][w]);
      mx = fmaxf(mx, red[1][w]);
      am = fmaxf(am, red[2][w]);
    }
    red[0][0] = mn;
    red[1][0] = mx;
    red[2][0] = __fdiv_rn(fmaxf(am, 1e-8f), 127.0f);
  }
  __syncthreads();
  const float scale = red[2][0];
  if (threadIdx.x == 0) {
    if (p.codes) p.qscale[(int64_t)i * p.scale_mat_stride] = scale;
    if (p.qminmax) {
      p.qminmax[(int64_t)i * p.minmax_mat_stride] = red[0][0];
      p.qminmax[(int64_t)i * p.minmax_mat_stride + 1] = red[1][0];
    }
  }
  if (p.codes) {
    const int kp = p.rank_pad;
    int8_t* ci = p.codes + (int64_t)i * p.codes_mat_stride;
    for (int t0 = 0; t0 < m; t0 += 256) {
      const int nrow = min(256, m - t0);
      if ((int)threadIdx.x < nrow) {
        const int t = t0 + threadIdx.x;
        float q[RMAX];
        load_row(t, q);
        for (int j = 0; j < kp; ++j)
          scodes[threadIdx.x * kp + j] =
              j < k ? (int8_t)(int)rintf(__fdiv_rn(u_of(q, j) * ss[j], scale)) : (int8_t)0;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < nrow * kp; e += blockDim.x) {
        int tl, j;
        if (p.codes_j_stride == 1 || p.codes_tiled) { tl = e / kp; j = e - tl * kp; }
        else { j = e / nrow; tl = e - j * nrow; }
        const int t = t0 + tl;
        const int8_t v = scodes[tl * kp + j];
        if (p.codes_tiled)
          ci[vtile_offset(j, t, kp)] = v;
        else
          ci[(int64_t)t * p.codes_t_stride + (int64_t)j * p.codes_j_stride] = v;
      }
      __syncthreads();
    }
  }
  if (p.S && threadIdx.x < k) p.S[(int64_t)i * k + threadIdx.x] = ss[threadIdx.x];
  const float* Vhw = p.Vhw + (int64_t)i * k * n;
  if (p.Vh)
    for (int e = threadIdx.x; e < k * n; e += blockDim.x) p.Vh[(int64_t)i * k * n + e] = Vhw[e];
  if (p.basis) {
    const int kp = p.rank_pad;
    for (int e = threadIdx.x; e < kp * n; e += blockDim.x) {
      const float v = e < k * n ? Vhw[e] : 0.f;
      const int64_t o = (int64_t)i * p.basis_mat_stride + e;
      if (p.basis_dtype == SPX_F32) reinterpret_cast<float*>(p.basis)[o] = v;
      else if (p.basis_dtype == SPX_F16) reinterpret_cast<__half*>(p.basis)[o] = __float2half_rn(v);
      else reinterpret_cast<__nv_bfloat16*>(p.basis)[o] = __float2bfloat16_rn(v);
    }
  }
}

// ------------------------------------------------------------------- host side ---
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct RsvdWs {
  float *Y, *Z, *Wk, *S, *Vh;
  double* G;   // [Nb][r][r] Gram matrices of the split Cholesky-QR
  float* L;    // [Nb][r][r] its factors
  int* np;     // [Nb] passes each matrix needs
  int* list;   // [Nb] matrices that need more passes than requested
  int* cnt;    // [1] entries of list
  size_t bytes;
};

static RsvdWs carve(const spx_rsvd_args* a, char* base) {
  RsvdWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align256(bytes);
    return reinterpret_cast<float*>(p);
  };
  const size_t Nb = a->num_mats;
  w.Y = take(Nb * a->m * a->r * sizeof(float));
  w.Z = take(Nb * a->n * a->r * sizeof(float));
  w.Wk = take(Nb * a->r * a->k * sizeof(float));
  w.S = take(Nb * a->k * sizeof(float));
  w.Vh = take(Nb * a->k * a->n * sizeof(float));
  w.G = reinterpret_cast<double*>(take(Nb * a->r * a->r * sizeof(double)));
  w.L = take(Nb * a->r * a->r * sizeof(float));
  w.np = reinterpret_cast<int*>(take(Nb * sizeof(int)));
  w.list = reinterpret_cast<int*>(take(Nb * sizeof(int)));
  w.cnt = reinterpret_cast<int*>(take(sizeof(int)));
  w.bytes = off;
  return w;
}

static int validate(const spx_rsvd_args* a) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->num_mats >= 0, SPX_ERR_SHAPE, "num_mats < 0");
  SPX_REQUIRE(a->m >= 16 && a->m <= 1024 && a->n >= 16 && a->n <= 128, SPX_ERR_SHAPE,
              "matrix %dx%d outside [16,1024]x[16,128]", a->m, a->n);
  SPX_REQUIRE(a->k >= 1 && a->k <= 64 && a->r > a->k && a->r <= 64 && a->r <= (a->m < a->n ? a->m : a->n) - 2,
              SPX_ERR_SHAPE, "need 1 <= k < r <= min(64, min(m,n)-2); got k=%d r=%d", a->k, a->r);
  SPX_REQUIRE(a->n_iter >= 0 && a->n_iter <= 8, SPX_ERR_SHAPE, "n_iter %d outside [0, 8]", a->n_iter);
  SPX_REQUIRE(dtype_ok(a->in_dtype), SPX_ERR_UNSUPPORTED, "bad input dtype");
  SPX_REQUIRE((size_t)a->m * a->r * 4 + 4 * 64 <= 200 * 1024, SPX_ERR_UNSUPPORTED, "m*r too large for one CTA");
  SPX_REQUIRE(lift_smem(a->m, a->r, a->k, a->codes_rank_pad > a->k ? a->codes_rank_pad : a->k) <= 200 * 1024,
              SPX_ERR_UNSUPPORTED, "rank too large for one CTA");
  if (a->num_mats == 0) return SPX_OK;
  SPX_REQUIRE(a->M && a->omega, SPX_ERR_NULL, "M and omega are required");
  SPX_REQUIRE(a->M_mat_stride == 0 || a->M_mat_stride >= (int64_t)a->m * a->n, SPX_ERR_SHAPE,
              "M_mat_stride smaller than m*n");
  if (a->codes) {
    SPX_REQUIRE(a->qscale, SPX_ERR_NULL, "qscale is required with codes");
    SPX_REQUIRE(a->codes_rank_pad >= a->k, SPX_ERR_SHAPE, "codes_rank_pad < k");
    SPX_REQUIRE(a->codes_tiled || a->codes_j_stride == 1 || a->codes_t_stride == 1, SPX_ERR_SHAPE,
                "codes must be token-major, rank-major or tiled");
    if (a->codes_tiled)
      SPX_REQUIRE(a->m % 16 == 0 && a->codes_rank_pad % 8 == 0, SPX_ERR_SHAPE,
                  "tiled codes need m %% 16 == 0 and codes_rank_pad %% 8 == 0");
  }
  if (a->basis) {
    SPX_REQUIRE(dtype_ok(a->basis_dtype), SPX_ERR_UNSUPPORTED, "bad basis dtype");
    SPX_REQUIRE(a->codes_rank_pad >= a->k, SPX_ERR_SHAPE, "codes_rank_pad < k");
  }
  return SPX_OK;
}

template <typename T>
static int run_chain(const spx_rsvd_args* a, const RsvdWs& w, cudaStream_t st) {
  const int Nb = a->num_mats, m = a->m, n = a->n, r = a->r, k = a->k;
  const T* M = reinterpret_cast<const T*>(a->M);
  const int64_t ms = a->M_mat_stride > 0 ? a->M_mat_stride : (int64_t)m * n;
  const size_t smx = ((size_t)n * r + 64 * (size_t)(n + 1)) * sizeof(float);
  cudaFuncSetAttribute(gemm_mx_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smx);
  const dim3 gmx((m + 63) / 64, Nb), gmty((n + 63) / 64, Nb);
  cudaFuncSetAttribute(trsolve_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  cudaFuncSetAttribute(gram_kernel<24>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  cudaFuncSetAttribute(gram_kernel<40>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  cudaFuncSetAttribute(gram_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  // Cholesky-QR: npass 2 for the final basis Q (it feeds Bp and the lift), 1 for the
  // intermediate ones; three kernels per pass (Gram, factor, solve).  A pass past the
  // requested count runs grids of about one wave that stride over the listed matrices.
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  auto orth = [&](float* X, int rows, int npass) {
    const int nch = (rows + 127) / 128;
    const size_t sg = gram_smem(r), ts = trsolve_smem(r);
    for (int pass = 0; pass < 3; ++pass) {
      const bool listed = pass >= npass;
      const int gg = listed ? std::min(Nb, 4 * nsm) : Nb;
      const int gc = listed ? std::min(Nb, 8 * nsm) : Nb;
      const int gw = listed ? std::min((Nb + kCholWarps - 1) / kCholWarps, 4 * nsm) : (Nb + kCholWarps - 1) / kCholWarps;
      const dim3 gs(listed ? std::min(Nb, std::max(nsm, 8 * nsm / nch)) : Nb, nch);
      if (r <= 24) {
        gram_kernel<24><<<gg, gram_threads(r), sg, st>>>(X, w.G, w.np, w.list, w.cnt, pass, npass, rows, r);
        chol_warp_kernel<24><<<gw, kCholWarps * 32, 0, st>>>(w.G, w.L, w.np, w.list, w.cnt, pass, npass, r, Nb);
        trsolve_kernel<24><<<gs, 128, ts, st>>>(X, w.L, w.np, w.list, w.cnt, pass, npass, rows, r);
      } else if (r <= 40) {
        gram_kernel<40><<<gg, gram_threads(r), sg, st>>>(X, w.G, w.np, w.list, w.cnt, pass, npass, rows, r);
        chol_warp_kernel<40><<<gw, kCholWarps * 32, 0, st>>>(w.G, w.L, w.np, w.list, w.cnt, pass, npass, r, Nb);
        trsolve_kernel<40><<<gs, 128, ts, st>>>(X, w.L, w.np, w.list, w.cnt, pass, npass, rows, r);
      } else {
        gram_kernel<64><<<gg, gram_threads(r), sg, st>>>(X, w.G, w.np, w.list, w.cnt, pass, npass, rows, r);
        chol_kernel<64><<<gc, kCholThreads, 0, st>>>(w.G, w.L, w.np, w.list, w.cnt, pass, npass, r);
        trsolve_kernel<64><<<gs, 128, ts, st>>>(X, w.L, w.np, w.list, w.cnt, pass, npass, rows, r);
      }
    }
  };
  // 16-bit inputs of 128 columns run the products on the tensor cores (spx_rsvd_tc.cu)
  const bool tc = rsvd_tc_supported(a->in_dtype, a->M, ms, m, n, r);
  auto mx = [&](const float* X, float* Y) {
    if (tc) rsvd_tc_gemm(0, a->in_dtype, M, ms, X, Y, Nb, m, r, st);
    else gemm_mx_kernel<T><<<gmx, 256, smx, st>>>(M, ms, X, Y, m, n, r);
  };
  auto mty = [&](const float* Y, float* Z) {
    if (tc) rsvd_tc_gemm(1, a->in_dtype, M, ms, Y, Z, Nb, m, r, st);
    else gemm_mty_kernel<T><<<gmty, 256, 0, st>>>(M, ms, Y, Z, m, n, r);
  };
  // Two implementations of the same sequence and pass rules: the fused kernel
  // (spx_rsvd_fused.cu: one CTA per matrix, everything on chip, one CTA per SM) and the
  // multi-kernel chain below (each step a grid of its own, several CTAs per SM hiding the
  // latency of the small dense steps).  Measured on B200 at k = 32, q = 2 with the
  // one-warp Cholesky factor in both: fused 488k / 541k / 578k blocks/s at 296 / 1024 /
  // 4096 matrices, chain 363k / 471k / 565k, so the fused kernel runs wherever its shape
  // is supported; SPX_RSVD_PATH=fused|chain forces one.
  const char* path = getenv("SPX_RSVD_PATH");
  const bool can_fuse = rsvd_fused_supported(a->in_dtype, a->M, ms, a->omega, m, n, r);
  bool fused = can_fuse;
  if (path && strcmp(path, "fused") == 0) fused = can_fuse;
  if (path && strcmp(path, "chain") == 0) fused = false;
  int rc = SPX_OK;
  if (fused) {
    rc = rsvd_fused(a->in_dtype, a->M, ms, a->omega, w.Y, w.Z, Nb, m, r, a->n_iter, st);
  } else {
    mx(a->omega, w.Y);
    orth(w.Y, m, a->n_iter == 0 ? 2 : 1);
    for (int it = 0; it < a->n_iter; ++it) {
      mty(w.Y, w.Z);
      orth(w.Z, n, 1);
      mx(w.Z, w.Y);
      orth(w.Y, m, it == a->n_iter - 1 ? 2 : 1);
    }
    mty(w.Y, w.Z);
    rc = launch_status("rsvd gemm/orth chain");
  }
  if (rc != SPX_OK) return rc;
  const size_t ssvd = small_svd_smem(n, r);
  cudaFuncSetAttribute(small_svd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssvd);
  small_svd_kernel<<<Nb, 256, ssvd, st>>>(w.Z, w.Wk, w.S, w.Vh, n, r, k);
  rc = launch_status("small_svd_kernel");
  if (rc != SPX_OK) return rc;
  LiftParams lp;
  lp.m = m; lp.n = n; lp.r = r; lp.k = k;
  lp.Q = w.Y; lp.Wk = w.Wk; lp.Sw = w.S; lp.Vhw = w.Vh;
  lp.U = a->U; lp.S = a->S; lp.Vh = a->Vh;
  lp.codes = a->codes;
  lp.codes_mat_stride = a->codes_mat_stride;
  lp.codes_t_stride = a->codes_t_stride;
  lp.codes_j_stride = a->codes_j_stride;
  lp.codes_tiled = a->codes_tiled;
  lp.rank_pad = a->codes_rank_pad > k ? a->codes_rank_pad : k;
  lp.qscale = a->qscale; lp.scale_mat_stride = a->scale_mat_stride;
  lp.qminmax = a->qminmax; lp.minmax_mat_stride = a->minmax_mat_stride;
  lp.basis = a->basis; lp.basis_dtype = a->basis_dtype; lp.basis_mat_stride = a->basis_mat_stride;
  const size_t slq = lift_smem(m, r, k, lp.rank_pad);
  cudaFuncSetAttribute(lift_quant_kernel<24>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)slq);
  cudaFuncSetAttribute(lift_quant_kernel<40>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)slq);
  cudaFuncSetAttribute(lift_quant_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)slq);
  if (r <= 24) lift_quant_kernel<24><<<Nb, 256, slq, st>>>(lp);
  else if (r <= 40) lift_quant_kernel<40><<<Nb, 256, slq, st>>>(lp);
  else lift_quant_kernel<64><<<Nb, 256, slq, st>>>(lp);
  return launch_status("lift_quant_kernel");
}

}  // namespace spx

using namespace spx;

extern "C" {

size_t spx_rsvd_workspace_size(const spx_rsvd_args* a) {
  if (validate(a) != SPX_OK) return 0;
  return carve(a, nullptr).bytes;
}

int spx_rsvd_compress(const spx_rsvd_args* a, void* stream) {
  int rc = validate(a);
  if (rc != SPX_OK) return rc;
  if (a->num_mats == 0) return SPX_OK;
  const RsvdWs need = carve(a, nullptr);
  SPX_REQUIRE(a->workspace && a->workspace_bytes >= need.bytes, SPX_ERR_WORKSPACE,
              "workspace of %zu bytes required, %zu given", need.bytes, a->workspace_bytes);
  SPX_REQUIRE((reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0, SPX_ERR_ALIGN,
              "workspace must be 256-byte aligned");
  const RsvdWs w = carve(a, reinterpret_cast<char*>(a->workspace));
  return SPX_DISPATCH_DTYPE(a->in_dtype, T, [&] { return run_chain<T>(a, w, (cudaStream_t)stream); });
}

}  // extern "C"
