// Fused subspace iteration of the batched rSVD (sm_100a): every product and every
// orthonormalisation of unsloth_spectral/rsvd.py:95-140 for one matrix in one CTA.
//
//   Y = M Omega; Q = orth(Y)
//   repeat n_iter: Z = orth(M^T Q); Q = orth(M Z)
//   Bp^T = M^T Q                          -> written out with Q for the small SVD / lift
//
// (the same sequence, pass counts and pivot rules as the multi-kernel chain of
// spx_rsvd.cu, so both give the same values up to summation order).
//
// Residency.  The 16-bit matrix M [m][128] (m <= 512: 128 KB) is read from global memory
// once, with cp.async, into shared memory in 16-byte chunks at
//     chunk (row t, column chunk c) -> (t / 128) * 32768 + c * 2048 + ((t % 128) / 8) * 128 + (t % 8) * 16,
// which is both the K-major no-swizzle UMMA layout of M (products M X: LBO 2048, SBO 128)
// and the MN-major layout of M^T (products M^T Y: LBO 128, SBO 2048).  It stays there for
// all 2 + 2 n_iter products.  The panels never leave the chip: Y [m][r] is a float32
// TMEM accumulator (128-row tile tt at columns tt * RP), Z [128][r] another (columns
// 4 RP), and the orthonormalisations read and rewrite them in place.
//
// Products.  tcgen05.mma.kind::f16 (M = 128, N = RP = r rounded up to 16, K = 16), issued
// by one thread, f32 accumulate.  The float32 right-hand side (Omega, Z or a 128-row
// chunk of Y) is split into 16-bit hi + lo halves of the input's type and written as an
// MN-major B operand: element (k, j) at (j / 8) * 2048 + k * 16 + (j % 8) * 2 (LBO 128,
// SBO 2048), so the thread that owns row k writes 16-byte runs, bank-conflict free.
// Omega is scaled by a power of two so that its largest magnitude is below 1; Q and Z
// are orthonormal.  Orthonormalisation is scale-invariant, so the scale is never undone.
//
// Orthonormalisation (Cholesky-QR).  Per pass: the float64 Gram matrix G = X^T X (each
// 128-row tile converted once to float64 while it is staged from TMEM into shared memory
// over the idle B buffers, 4 x 4 register tiles of the upper
// triangle, partial sums over 8 row subsets added in a fixed order), G = L L^T in float64
// by one warp (chol_warp: rows in registers, no block barriers; pivots at rounding level of
// a zero column give zero columns), X := X L^{-T} row by row in registers (thread = TMEM lane = row), written
// back into TMEM.  Passes: 2 for the final basis, 1 for intermediate ones, raised from
// the first pass's pivot spread (> 1e6: 2, > 1e12: 3).
//
// One CTA of 8 warps per matrix (about 220 KB of shared memory: one CTA per SM).  Every
// wait on an mbarrier is bounded in time; an expired wait stops the issue of further
// products and makes the CTA write NaN outputs.
#include <math.h>

#include "spx_common.cuh"
#include "spx_rsvd.cuh"
#include "spx_sm100.cuh"

namespace spx {
namespace rfu {

using namespace sm100;

constexpr int NT = 256;                 // threads
constexpr int TILE = 128 * 128 * 2;     // one 128-row tile of M in bytes
constexpr int TMEM_COLS = 256;

__host__ __device__ constexpr int rp_of(int rmax) { return (rmax + 15) / 16 * 16; }

// Compile-time geometry of one instantiation (RMAX = 24 or 40).
template <int RMAX>
struct Geo {
  static constexpr int RP = rp_of(RMAX);          // MMA N
  static constexpr int R4 = (RMAX + 3) & ~3;
  static constexpr int NB4 = (RMAX + 3) / 4;      // 4-column blocks of the Gram tiling
  static constexpr int NTILE = NB4 * (NB4 + 1) / 2;
  static constexpr int NPAIR = gram_npair(NB4);
  static constexpr int S = NT / NPAIR >= 8 ? 8 : NT / NPAIR;   // row subsets per tile pair
  static constexpr int P = (4 * NB4) | 1;         // Gram staging pitch (elements, odd)
  static constexpr int SP = RMAX + 4;             // output staging pitch (floats)
  static constexpr int BSZ = 128 * RP * 2;        // one 16-bit half of a B operand
  static constexpr int ZC = 4 * RP;               // TMEM column of the Z accumulator
  static_assert(ZC + RP <= TMEM_COLS, "TMEM columns");
  static_assert(NPAIR * S <= NT, "one Gram item per thread");
  static_assert(P <= SP, "staging pitch");
  // shared memory after the M tiles (bytes)
  static constexpr int OFF_B = 0;                          // 2 buffers x (hi, lo)
  static constexpr int OFF_T = OFF_B + 4 * BSZ;            // staging tile [128][SP] f32
  static constexpr int OFF_G = OFF_T + 128 * SP * 4;       // Gram [RMAX][RMAX] f64 (lower)
  static constexpr int OFF_L = OFF_G + RMAX * RMAX * 8;    // L [RMAX][R4] f32
  static constexpr int BYTES = OFF_L + RMAX * R4 * 4;
  static constexpr int RED = S * NTILE * 16 * 8;           // Gram partials, over B + staging
  static_assert(RED <= OFF_G, "Gram partials fit over the B buffers and the staging tile");
  static_assert(128 * P * 8 <= 4 * BSZ, "float64 Gram staging tile fits over the B buffers");
};

__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int a_mn, int b_mn, int n) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 f32 columns of this warp's 32 TMEM lanes (no wait).
__device__ __forceinline__ void tld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int u = 0; u < 16; ++u) v[u] = __uint_as_float(r[u]);
}
__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tst16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded wait on an mbarrier phase by every thread: false once kWaitNs passed.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity))
    if (gtimer() - t0 > kWaitNs) return false;
  return true;
}

template <typename T>
struct H16;
template <>
struct H16<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ static uint32_t pack(float a, float b) {
    return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
  }
  __device__ static float lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))); }
  __device__ static float hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
};
template <>
struct H16<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ static uint32_t pack(float a, float b) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
  }
  __device__ static float lo(uint32_t w) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)(w & 0xffffu))); }
  __device__ static float hi(uint32_t w) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)(w >> 16))); }
};

// Eight consecutive float32 values of row k -> the hi and lo 16-byte runs of j-octet o in
// the MN-major B operand at b (hi half) and b + BSZ (lo half).
template <typename T, int BSZ>
__device__ __forceinline__ void put_b8(uint8_t* b, int k, int o, const float* x) {
  using H = H16<T>;
  uint32_t hw[4], lw[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    hw[u] = H::pack(x[2 * u], x[2 * u + 1]);
    lw[u] = H::pack(x[2 * u] - H::lo(hw[u]), x[2 * u + 1] - H::hi(hw[u]));
  }
  const int off = o * 2048 + k * 16;
  *reinterpret_cast<uint4*>(b + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(b + BSZ + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

struct FusedParams {
  const void* M;
  int64_t ms;            // matrix stride of M (elements)
  const float* omega;    // [Nb][128][r]
  float* Q;              // [Nb][m][r] out: orthonormal basis of the sketch
  float* Bt;             // [Nb][128][r] out: Bp^T = M^T Q
  int m, r, n_iter;
};

template <typename T, int RMAX>
__global__ void __launch_bounds__(NT, 1) rsvd_fused_kernel(FusedParams p) {
  using G = Geo<RMAX>;
  constexpr int RP = G::RP, R4 = G::R4, BSZ = G::BSZ, P = G::P, SP = G::SP, S = G::S, NB4 = G::NB4,
                NTILE = G::NTILE, ZC = G::ZC;
  constexpr uint32_t ID_MX = idesc(H16<T>::kFmt, 0, 1, RP);   // A = M (K-major), B MN-major
  constexpr uint32_t ID_MTY = idesc(H16<T>::kFmt, 1, 1, RP);  // A = M^T (MN-major)
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tslot;
  __shared__ int sflag[2];   // [0]: a wait expired; [1]: passes asked for by the pivots
  __shared__ float sred[8];
  __shared__ double colj[2][RMAX], scale_s[RMAX];   // scratch of the Cholesky warp

  const int m = p.m, r = p.r, nt = m / 128;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, quad = w & 3, half = w >> 2;
  const int64_t i = blockIdx.x;
  uint8_t* sX = smem + (size_t)nt * TILE;
  uint8_t* sB = sX + G::OFF_B;
  float* sT = reinterpret_cast<float*>(sX + G::OFF_T);
  double* sG = reinterpret_cast<double*>(sX + G::OFF_G);
  float* sL = reinterpret_cast<float*>(sX + G::OFF_L);
  double* red = reinterpret_cast<double*>(sX + G::OFF_B);
  double* sTd = reinterpret_cast<double*>(sX + G::OFF_B);   // Gram staging tile [128][P] f64
  const uint32_t sM0 = smem_u32(smem), bar0 = smem_u32(&bars[0]);

  if (w == 0) {
    tmem_alloc(smem_u32(&tslot), TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    sflag[0] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // M -> shared memory (chunk layout above); a warp covers 8 rows x 4 chunks per copy
  const T* Mi = reinterpret_cast<const T*>(p.M) + i * p.ms;
  for (int tt = 0; tt < nt; ++tt) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int e = tid + NT * it, q = e >> 5, l = e & 31;
      const int t = (q & 15) * 8 + (l & 7), c = (q >> 4) * 4 + (l >> 3);
      cp_async16(sM0 + tt * TILE + c * 2048 + (t >> 3) * 128 + (t & 7) * 16, Mi + (int64_t)(tt * 128 + t) * 128 + c * 8);
    }
  }
  cp_async_commit();
  // Omega (rows 0..127, one per thread of the first four warps), scaled by a power of two
  float om[RP];
  float mx = 0.f;
  if (tid < 128) {
    const float4* o4 = reinterpret_cast<const float4*>(p.omega + (i * 128 + tid) * r);
#pragma unroll
    for (int c4 = 0; c4 < RP / 4; ++c4) {
      const float4 v = 4 * c4 < r ? __ldg(o4 + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      om[4 * c4] = v.x;
      om[4 * c4 + 1] = v.y;
      om[4 * c4 + 2] = v.z;
      om[4 * c4 + 3] = v.w;
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
  mx = warp_max(mx);
  if (lane == 0) sred[w] = mx;
  __syncthreads();
  {
    const float ma = fmaxf(fmaxf(sred[0], sred[1]), fmaxf(sred[2], sred[3]));
    int e2 = 0;
    if (ma > 0.f && isfinite(ma)) frexpf(ma, &e2);   // ma = f 2^e2, 0.5 <= f < 1
    const float sc = ldexpf(1.f, -e2);
    if (tid < 128) {
#pragma unroll
      for (int c = 0; c < RP; ++c) om[c] *= sc;
#pragma unroll
      for (int o = 0; o < RP / 8; ++o) put_b8<T, BSZ>(sB, tid, o, om + 8 * o);
    }
  }
  cp_async_wait_all();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tslot;
  const uint32_t tq = tbase + ((uint32_t)(32 * quad) << 16);   // this warp's TMEM lanes
  bool bad = false;
  uint32_t ph[2] = {0u, 0u};

  // ---- products (one thread issues; completion on bars[buf]) ------------------------
  auto mma_mx = [&](int buf) {   // Y tiles = M B
    if (tid == 0 && !bad) {
      tc_fence_after();
      const uint32_t b0 = smem_u32(sB + buf * 2 * BSZ);
      for (int tt = 0; tt < nt; ++tt)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t a = umma_desc(sM0 + tt * TILE + ks * 4096, 2048, 128);
#pragma unroll
          for (int part = 0; part < 2; ++part)
            umma(tbase + tt * RP, a, umma_desc(b0 + part * BSZ + ks * 256, 128, 2048), ID_MX, (ks | part) != 0);
        }
      umma_commit(bar0 + 8 * buf);
    }
  };
  auto mma_mty = [&](int tt, int buf) {   // Z += M_tt^T B (chunk tt of Y in buffer buf)
    if (tid == 0 && !bad) {
      tc_fence_after();
      const uint32_t b0 = smem_u32(sB + buf * 2 * BSZ);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a = umma_desc(sM0 + tt * TILE + ks * 256, 128, 2048);
#pragma unroll
        for (int part = 0; part < 2; ++part)
          umma(tbase + ZC, a, umma_desc(b0 + part * BSZ + ks * 256, 128, 2048), ID_MTY, (tt | ks | part) != 0);
      }
      umma_commit(bar0 + 8 * buf);
    }
  };
  auto wait_buf = [&](int buf) {   // every thread; then the flag is made uniform
    if (!bad) {
      if (!bar_wait(bar0 + 8 * buf, ph[buf])) sflag[0] = 1;
      ph[buf] ^= 1u;
    }
    __syncthreads();
    bad = sflag[0] != 0;
    tc_fence_after();
  };
  // rows of a 128-row TMEM panel (column col) -> MN-major B operand in buffer buf
  auto tmem_to_b = [&](uint32_t col, int buf) {
    uint8_t* b = sB + buf * 2 * BSZ;
    for (int c16 = half; c16 < RP / 16; c16 += 2) {
      float v[16];
      tld16(tq + col + 16 * c16, v);
      tld_wait();
      put_b8<T, BSZ>(b, 32 * quad + lane, 2 * c16, v);
      put_b8<T, BSZ>(b, 32 * quad + lane, 2 * c16 + 1, v + 8);
    }
    fence_async_smem();
  };
  // Z = M^T Y over the nt chunks of Y, two B buffers in turn
  auto mty_all = [&]() {
    for (int tt = 0; tt < nt; ++tt) {
      const int buf = tt & 1;
      if (tt >= 2) wait_buf(buf);
      tmem_to_b((uint32_t)(tt * RP), buf);
      tc_fence_before();
      __syncthreads();
      mma_mty(tt, buf);
    }
    if (nt >= 2) wait_buf(nt & 1);   // chunk nt - 2
    wait_buf((nt - 1) & 1);
  };

  // ---- Cholesky-QR of a TMEM panel: ntl tiles at columns col0 + tt * cstep ----------
  // Gram item of this thread: tile pair (ta, tb), (ta, tb + 1) of 4 x 4 blocks, row subset s
  int it_a = -1, it_b = 0, it_c = 0, it_s = 0, it_t0 = 0;
  bool it_two = false;
  if (tid < G::NPAIR * S) {
    int pp = tid / S, ta = 0;
    it_s = tid - pp * S;
    while (pp >= (NB4 - ta + 1) / 2) {
      pp -= (NB4 - ta + 1) / 2;
      ++ta;
    }
    const int tb = ta + 2 * pp;
    it_two = tb + 1 < NB4;
    it_a = 4 * ta;
    it_b = 4 * tb;
    it_c = it_two ? 4 * (tb + 1) : 4 * ta;
    it_t0 = ta * NB4 - ta * (ta - 1) / 2 + (tb - ta);
  }
  auto orth = [&](int ntl, uint32_t col0, uint32_t cstep, int npass0) {
    int npass = npass0;
    for (int pass = 0; pass < npass; ++pass) {
      // Gram G = X^T X in float64 over the tiles
      double g0[16], g1[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) g0[e] = g1[e] = 0.0;
      for (int tt = 0; tt < ntl; ++tt) {
        __syncthreads();   // the staging tile (and the partials over it) are free
        for (int c16 = half; c16 < RP / 16; c16 += 2) {
          float v[16];
          tld16(tq + col0 + tt * cstep + 16 * c16, v);
          tld_wait();
          double* dst = sTd + (32 * quad + lane) * P + 16 * c16;
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (16 * c16 + u < 4 * NB4) dst[u] = (double)v[u];
        }
        __syncthreads();
        if (it_a >= 0) {
          const double* xa_p = sTd + it_a;
          const double* xb_p = sTd + it_b;
          const double* xc_p = sTd + it_c;
#pragma unroll 2
          for (int t = it_s; t < 128; t += S) {
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
                g0[4 * u + v] = fma(xa[u], xb[v], g0[4 * u + v]);
                g1[4 * u + v] = fma(xa[u], xc[v], g1[4 * u + v]);
              }
          }
        }
      }
      __syncthreads();   // partials overwrite the B buffers and the staging tile
      // partials element-major, red[(entry * S + subset) * NTILE + tile]: the threads of a
      // warp (consecutive subsets and tiles) store to distinct banks, and the summing
      // threads (consecutive tiles) read consecutive words
      if (it_a >= 0) {
        double* dst = red + (size_t)it_s * NTILE + it_t0;
#pragma unroll
        for (int e = 0; e < 16; ++e) dst[(size_t)e * S * NTILE] = g0[e];
        if (it_two) {
#pragma unroll
          for (int e = 0; e < 16; ++e) dst[(size_t)e * S * NTILE + 1] = g1[e];   // tile (ta, tb + 1) is the next index
        }
      }
      __syncthreads();
      for (int e2 = tid; e2 < NTILE * 16; e2 += NT) {
        const int idx = e2 / NTILE, tile = e2 - idx * NTILE, u = idx >> 2, v = idx & 3;
        double sum = 0.0;
        for (int s2 = 0; s2 < S; ++s2) sum += red[((size_t)idx * S + s2) * NTILE + tile];
        int tb = tile, ta = 0;
        while (tb >= NB4 - ta) {
          tb -= NB4 - ta;
          ++ta;
        }
        tb += ta;
        const int col = 4 * ta + u, row = 4 * tb + v;   // entry (col, row), col <= row: lower storage
        if (row < r && col < r && col <= row) sG[row * RMAX + col] = sum;
      }
      __syncthreads();
      // G = L L^T (float64, one warp: chol_warp); L (float32, inverse diagonal) -> sL
      if (w == 0) {
        const int n = chol_warp<RMAX>(sG, RMAX, r, sL, R4, &colj[0][0], scale_s, npass);
        if (lane == 0) sflag[1] = pass == 0 ? n : npass;
      }
      __syncthreads();
      npass = sflag[1];
      // X := X L^{-T}: thread = row; warps of half h take tiles h, h + 2, ...
      for (int tt = half; tt < ntl; tt += 2) {
        const uint32_t ta = tq + col0 + tt * cstep;
        float x[RP];
#pragma unroll
        for (int c16 = 0; c16 < RP / 16; ++c16) tld16(ta + 16 * c16, x + 16 * c16);
        tld_wait();
#pragma unroll
        for (int j = 0; j < RMAX; ++j) {
          if (j < r) {
            const float4* lj = reinterpret_cast<const float4*>(sL + j * R4);
            float a0 = x[j], a1 = 0.f;
#pragma unroll
            for (int c = 0; c < (j & ~3); c += 4) {   // entries c < j in whole quads
              const float4 l = lj[c >> 2];
              a0 = fmaf(-x[c], l.x, a0);
              a1 = fmaf(-x[c + 1], l.y, a1);
              a0 = fmaf(-x[c + 2], l.z, a0);
              a1 = fmaf(-x[c + 3], l.w, a1);
            }
            if (j & 3) {   // the partial quad holding columns (j & ~3) .. j - 1
              const float4 l = lj[j >> 2];
              const int c = j & ~3;
              a0 = fmaf(-x[c], l.x, a0);
              if ((j & 3) > 1) a1 = fmaf(-x[c + 1], l.y, a1);
              if ((j & 3) > 2) a0 = fmaf(-x[c + 2], l.z, a0);
            }
            x[j] = (a0 + a1) * sL[j * R4 + j];
          }
        }
#pragma unroll
        for (int c16 = 0; c16 < RP / 16; ++c16) tst16(ta + 16 * c16, x + 16 * c16);
        tst_wait();
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
  };

  // rows of a 128-row TMEM panel -> dst [128][r] (global), through the staging tile
  auto write_out = [&](uint32_t col, float* dst) {
    __syncthreads();   // staging tile free
    for (int c16 = half; c16 < RP / 16; c16 += 2) {
      float v[16];
      tld16(tq + col + 16 * c16, v);
      tld_wait();
      float* srow = sT + (32 * quad + lane) * SP + 16 * c16;
#pragma unroll
      for (int u = 0; u < 16; u += 4)
        if (16 * c16 + u < r) {
          float4 o = make_float4(v[u], v[u + 1], v[u + 2], v[u + 3]);
          if (bad) o = make_float4(__int_as_float(0x7fc00000), 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(srow + u) = o;
        }
    }
    __syncthreads();
    const int nq4 = r / 4;
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int g = tid; g < 128 * nq4; g += NT) {
      const int rr = g / nq4, c4 = g - rr * nq4;
      d4[g] = *reinterpret_cast<const float4*>(sT + rr * SP + 4 * c4);
    }
  };

  // ---- the subspace iteration ---------------------------------------------------------
  mma_mx(0);   // Y = M Omega
  wait_buf(0);
  orth(nt, 0u, (uint32_t)RP, p.n_iter == 0 ? 2 : 1);
  for (int it = 0; it < p.n_iter; ++it) {
    mty_all();   // Z = M^T Q
    orth(1, (uint32_t)ZC, 0u, 1);
    tmem_to_b((uint32_t)ZC, 0);
    tc_fence_before();
    __syncthreads();
    mma_mx(0);   // Y = M Z
    wait_buf(0);
    orth(nt, 0u, (uint32_t)RP, it == p.n_iter - 1 ? 2 : 1);
  }
  float* Qi = p.Q + i * (int64_t)m * r;
  for (int tt = 0; tt < nt; ++tt) write_out((uint32_t)(tt * RP), Qi + (int64_t)tt * 128 * r);
  mty_all();   // Bp^T = M^T Q
  write_out((uint32_t)ZC, p.Bt + i * 128 * (int64_t)r);
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, TMEM_COLS);
}

}  // namespace rfu

size_t rsvd_fused_smem(int m, int r) {
  const int g = r <= 24 ? rfu::Geo<24>::BYTES : rfu::Geo<40>::BYTES;
  return (size_t)(m / 128) * rfu::TILE + (size_t)g;
}

bool rsvd_fused_supported(int dtype, const void* M, int64_t ms, const void* omega, int m, int n, int r) {
  if (dtype != SPX_F16 && dtype != SPX_BF16) return false;
  if (n != 128 || m % 128 != 0 || m < 128 || m > 512 || r % 4 != 0 || r > 40) return false;
  if ((reinterpret_cast<uintptr_t>(M) & 15u) != 0 || (ms * 2) % 16 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(omega) & 15u) != 0) return false;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  // static shared memory of the kernel: barriers, flags and the Cholesky vectors
  return rsvd_fused_smem(m, r) + 4096 <= (size_t)optin;
}

template <typename T, int RMAX>
static int launch_fused(const rfu::FusedParams& fp, int Nb, cudaStream_t st) {
  const size_t smem = rsvd_fused_smem(fp.m, fp.r);
  auto kern = rfu::rsvd_fused_kernel<T, RMAX>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<Nb, rfu::NT, smem, st>>>(fp);
  return launch_status("rsvd_fused_kernel");
}

int rsvd_fused(int dtype, const void* M, int64_t ms, const float* omega, float* Q, float* Bt, int Nb, int m, int r,
               int n_iter, cudaStream_t st) {
  rfu::FusedParams fp;
  fp.M = M;
  fp.ms = ms;
  fp.omega = omega;
  fp.Q = Q;
  fp.Bt = Bt;
  fp.m = m;
  fp.r = r;
  fp.n_iter = n_iter;
  if (dtype == SPX_F16)
    return r <= 24 ? launch_fused<__half, 24>(fp, Nb, st) : launch_fused<__half, 40>(fp, Nb, st);
  return r <= 24 ? launch_fused<__nv_bfloat16, 24>(fp, Nb, st) : launch_fused<__nv_bfloat16, 40>(fp, Nb, st);
}

}  // namespace spx
