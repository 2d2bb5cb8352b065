// Projection cold-tier decode kernel for sm_100a (FP16 cache, D = 128, linear-phase RoPE).
//
// The reference scores a cold token by rotating the query to the key's position and
// projecting it on the block's key basis (kernels/spectral_attention.py:375-453):
//   score_t = scale_k * sum_k C[t,k] * (B_k . R(-p_t) q).
// With the basis rows and the query as 64 complex pairs (z_i = x_i + j x_{i+64}) and the
// rotation e^{j theta_i p_t}, the bracket is
//   S[t,(h,k)] = Re sum_i gamma[h,k,i] e^{j theta_i tau_t},   tau_t = t - c,
//   gamma[h,k,i] = conj(q_{h,i}) e^{j theta_i (P_j + c)} beta_{k,i},
// where P_j is the block's start position and c = (T - 1) / 2 its centre.  So S is a
// product of a token-feature table that is the same for every block and unit,
//   A[t, f] = [cos(theta_i tau_t), sin(theta_i tau_t)]  (i < n_hi)   and
//             T_n(tau_t / c)                             (Chebyshev terms, n < np),
// and a per-(unit, block) matrix G[f, (h,k)] built from the query, the block's rotation
// factor and the key basis.  The low frequencies (theta_i c small) are folded into the
// Chebyshev terms with the Jacobi-Anger expansion e^{j phi u} = sum_n eps_n j^n J_n(phi)
// T_n(u) (truncation error <= 1e-7 relative, chosen on the host), so A has KF = 64
// columns for RoPE base 1e6 instead of 128.  DISTANCE mode (spectral_attention.py:198)
// indexes by qpos - p_t: the same with gamma conjugated; tokens past the query (clamped
// distance 0) use the unrotated projection B_k . q.
//
// Per unit-block (one (layer, sequence, KV head) x one block of 512 tokens):
//   S = A . G  on tcgen05 (kind::f16, A from tensor memory, G from shared memory,
//              FP32 accumulator in tensor memory, M = 128 tokens per tile, N = n_rep*RK),
//   score[t,h] = scale_k sum_k C[t,k] S[t,(h,k)]  (FP32 packed FMA on the CUDA cores),
//   online softmax, v_lat += codes_V^T P (mma.sync), expansion through B_V once per
//   unit-block, merge across the blocks of a range (as the reconstruct kernel does).
//
// Warp roles (512 threads, one persistent CTA per SM):
//   warps 0-7   consumers: two per tensor-memory lane quadrant, even / odd M-tiles; the
//               last warp done with a code-ring stage refills it;
//   warps 8-10  builders: G for the unit-blocks ahead of the consumers (the exact pairs as
//               block-diagonal 16 x 16 tiles and the Chebyshev rows on mma.sync); thread
//               256 streams the key-basis ring (a 2-D tensor map with the 128-byte swizzle,
//               so the basis is read without bank conflicts) and the query rows;
//   warp 11     lane 0 issues the tcgen05 MMAs;
//   warps 12-15 epilogue: combines the consumers, expands through B_V, merges, and
//               streams the value-basis ring.
// Every wait is bounded in time (an expired wait raises the CTA abort flag and the
// workspace error word; the merge kernel then writes NaN).
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include <cuda.h>

#include "spx_common.cuh"
#include "spx_decode.cuh"
#include "spx_sm100.cuh"

namespace spx {
namespace projk {

using namespace sm100;

constexpr int FD = 128;
constexpr int NPAIR = 64;
constexpr int NCW = 8;             // consumer warps
constexpr int BW0 = 8, NBW = 3;    // builder warps
constexpr int MMA_W = 11;
constexpr int EW0 = 12, NEW = 4;
constexpr int NT = 512;
constexpr int BT0 = BW0 * 32, NBT = NBW * 32, ET0 = EW0 * 32, NEP = NEW * 32;
constexpr int SK = 3, SV = 2, NG = 2, NS0 = 4;
constexpr int BAR_EPI = 3, BAR_BLD = 4;
constexpr int VP = 2 * FD + 16;    // row pitch of the staged Chebyshev operand (<= 128 dims)
constexpr int QP = FD * 2 + 16;    // padded value-basis row pitch (ldmatrix.trans)
constexpr int NPMAX = 16;          // Chebyshev terms at most
constexpr int VROWS = 48;          // n_rep x Chebyshev terms at most
constexpr float kChebErr = 1e-7f;  // truncation error bound of the expansion

// Launch-wide constants of the feature split (kernel parameter).
struct Geom {
  int n_hi;      // pairs i < n_hi use exact cos/sin features (multiple of 8)
  int np;        // Chebyshev terms for the pairs i >= n_hi
  float sg;      // +1: ABSOLUTE RoPE; -1: DISTANCE RoPE (conjugated phase)
};

template <int RK, int RV, int MT, int NREP, int KF>
struct PCfg {
  static constexpr int TB = MT * 128;
  static constexpr int N = NREP * RK;                     // UMMA N: (head, rank) columns
  static constexpr int ACOLS = MT * KF / 2;               // tensor-memory columns of the feature table
  static constexpr int NSR = (512 - ACOLS) / N;
  static constexpr int NS = NSR < 4 ? NSR : 4;            // S accumulator slots
  static constexpr int SC = KF <= 64 ? 3 : 2;             // code-ring stages
  static constexpr int RVP = RV + 4;
  // key ring stage: the basis as two 128-byte-swizzled boxes (dims 0-63, 64-127; RK rows
  // of 128 bytes each), then the query rows
  static constexpr int K_B0 = 0, K_B1 = RK * 128, K_Q = 2 * RK * 128;
  static constexpr int STAGE_K = (K_Q + NREP * FD * 2 + 1023) / 1024 * 1024;
  static constexpr int C_CK = 0, C_CV = TB * RK, STAGE_C = TB * (RK + RV);
  static constexpr int STAGE_V = RV * FD * 2;
  static constexpr int GB = KF * N * 2;                   // one G buffer (f16, K-major core matrices)
  static constexpr int OFF_RK = 0;                        // 1024-aligned (swizzle atoms)
  static constexpr int OFF_RC = OFF_RK + SK * STAGE_K;
  static constexpr int OFF_RV = OFF_RC + SC * STAGE_C;
  static constexpr int OFF_G = OFF_RV + SV * STAGE_V;
  static constexpr int OFF_W = OFF_G + NG * GB;           // [NREP][64] float4 (wa.x, wa.y, wb.x, wb.y)
  static constexpr int OFF_CF = OFF_W + NREP * NPAIR * 16;      // [NPMAX][64] f32 Chebyshev coefficients
  static constexpr int OFF_S0 = OFF_CF + NPMAX * NPAIR * 4;     // [NS0][NREP][RK] f32 unrotated projections
  static constexpr int OFF_V = OFF_S0 + NS0 * NREP * RK * 4;    // [VROWS][VP] f16 Chebyshev operand
  static constexpr int OFF_P = OFF_V + VROWS * VP;              // [NCW][32 tokens][8 heads] f16
  static constexpr int PART = NCW * NREP * 4 * 2 + NCW * NREP * RVP * 4;
  static constexpr int OFF_PT = OFF_P + NCW * 32 * 16;
  static constexpr int OFF_BVP = OFF_PT + 2 * PART;
  static constexpr int OFF_VL = OFF_BVP + RV * QP;
  static constexpr int OFF_ML = OFF_VL + NREP * RV * 4;
  static constexpr int OFF_ST = OFF_ML + NREP * 4 * 4;
  static constexpr int OFF_RW = OFF_ST + GMAX * NREP * 2 * 4;  // [VROWS] (h << 8 | n) of the Chebyshev rows
  static constexpr int OFF_CC = OFF_RW + VROWS * 4;            // [SC] code-stage release counters
  static constexpr int OFF_BAR = (OFF_CC + 4 * 4 + 7) / 8 * 8;
  enum {
    B_KFULL = 0,
    B_CFULL = B_KFULL + SK,
    B_VFULL = B_CFULL + SC,
    B_GFULL = B_VFULL + SV,
    B_GFREE = B_GFULL + NG,
    B_SFULL = B_GFREE + NG,
    B_SFREE = B_SFULL + 4,
    B_PREADY = B_SFREE + 4,
    B_PFREE = B_PREADY + 2,
    B_S0FREE = B_PFREE + 2,
    NBAR = B_S0FREE + NS0
  };
  static constexpr int OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_TM + 16 + 1024;        // + slack to align the base to 1024
  // configurations the kernel is built for (the host checks the same predicate)
  static constexpr bool OK = BYTES <= 227 * 1024 && NSR >= 2 && N % 16 == 0 && N >= 16 && N <= 128 &&
                             KF % 16 == 0 && KF <= 128 && NREP <= 8;
  static_assert(!(RK == 32 && RV == 32 && MT == 4 && NREP == 4 && KF == 64) || OK, "the timed configuration fits");
  static_assert(OFF_RC % 128 == 0 && OFF_RV % 128 == 0 && OFF_G % 128 == 0 && STAGE_C % 128 == 0, "alignment");
};

// ------------------------------------------------------------------ device helpers --
// UMMA with A in tensor memory: D[tmem] (+)= A[tmem] . B[smem], kind::f16.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

#define SPX_R8(r, o) "=r"(r[o + 0]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), "=r"(r[o + 4]), "=r"(r[o + 5]), \
                     "=r"(r[o + 6]), "=r"(r[o + 7])
#define SPX_I8(r, o) "r"(r[o + 0]), "r"(r[o + 1]), "r"(r[o + 2]), "r"(r[o + 3]), "r"(r[o + 4]), "r"(r[o + 5]), \
                     "r"(r[o + 6]), "r"(r[o + 7])
#define SPX_T8(r, o) "+r"(r[o + 0]), "+r"(r[o + 1]), "+r"(r[o + 2]), "+r"(r[o + 3]), "+r"(r[o + 4]), "+r"(r[o + 5]), \
                     "+r"(r[o + 6]), "+r"(r[o + 7])

// 16 / 32 columns of this warp's 32 lanes (one row per thread), without the wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15}, [%16];"
               : SPX_R8(r, 0), SPX_R8(r, 8)
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
               "[%32];"
               : SPX_R8(r, 0), SPX_R8(r, 8), SPX_R8(r, 16), SPX_R8(r, 24)
               : "r"(taddr)
               : "memory");
}
template <int NR>
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[NR]);
template <>
__device__ __forceinline__ void tmem_wait_ld<16>(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : SPX_T8(r, 0), SPX_T8(r, 8) : : "memory");
}
template <>
__device__ __forceinline__ void tmem_wait_ld<32>(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : SPX_T8(r, 0), SPX_T8(r, 8), SPX_T8(r, 16), SPX_T8(r, 24) : : "memory");
}
template <int NR>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[NR]) {
  if constexpr (NR == 16) tmem_ld16(taddr, r);
  else tmem_ld32(taddr, r);
}
// 16 / 32 columns from registers into this warp's lanes.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15, %16};" ::"r"(taddr),
               SPX_I8(r, 0), SPX_I8(r, 8)
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
               "%32};" ::"r"(taddr),
               SPX_I8(r, 0), SPX_I8(r, 8), SPX_I8(r, 16), SPX_I8(r, 24)
               : "memory");
}
#undef SPX_R8
#undef SPX_I8
#undef SPX_T8

// Four INT8 codes -> two float pairs, exact: byte b becomes the float 2^23 + (b ^ 0x80),
// and 2^23 + 128 is subtracted with one packed add.
__device__ __forceinline__ void i8x4_to_f2x2(uint32_t w, float2& lo, float2& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const float2 bias = make_float2(-8388736.f, -8388736.f);
  // result bytes: (byte k of x, 0, 0, 0x4B) -> selector nibbles (k, 4, 5, 7)
  const float2 a = make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540)),
                               __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541)));
  const float2 b = make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7542)),
                               __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7543)));
  lo = __fadd2_rn(a, bias);
  hi = __fadd2_rn(b, bias);
}

// Byte offset of G element (column n, feature f) in the K-major, no-swizzle UMMA layout:
// 8 x 16-byte core matrices, N-adjacent ones 128 bytes apart, K-adjacent ones 16*N apart.
template <int N>
__device__ __forceinline__ int g_off(int n, int f) {
  return ((f >> 3) * (N / 8) + (n >> 3)) * 128 + (n & 7) * 16 + (f & 7) * 2;
}

// -------------------------------------------------------------------- the kernel ---
// The walk position k steps after s (k small): ring refills look ahead without keeping a
// second walk state in registers.
__device__ __forceinline__ Seq ahead(Seq s, int k, const Items& I) {
  for (int q = 0; q < k && s.valid(I); ++q) s.next(I);
  return s;
}

// Event timeline for diagnostics: compiled in only with -DSPX_PROJ_TRACE=1; records the
// clock64 of event `ev` of iteration `it` in CTA 0.
#ifdef SPX_PROJ_TRACE
#define SPX_TRACE(cond, it, ev)                                                         \
  do {                                                                                  \
    if ((cond) && blockIdx.x == 0 && (it) < 64) sc.trace[(it) * 64 + (ev)] = clock64(); \
  } while (0)
#else
#define SPX_TRACE(cond, it, ev) \
  do {                          \
  } while (0)
#endif

// One bulk-copy stage of a ring: `bytes` from `src` into shared memory at `dst`,
// completing on barrier `bar` (single thread).
__device__ __forceinline__ void ring_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  mbar_expect_tx(bar, bytes);
  bulk_g2s_hint(dst, src, bytes, bar, pol);
}
// 2-D tensor-map load of box (x, y) into shared memory at dst (128-byte swizzle; dst
// 1024-aligned), completing on barrier `bar`.
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Byte offset of basis element (row k, dim d) in a key-ring stage: two boxes of RK rows x
// 128 bytes (dims 0-63, 64-127), 16-byte chunks XOR-swizzled by the row (k & 7).
template <int RK>
__device__ __forceinline__ int kb_off(int k, int d) {
  const int box = d >> 6, b = (d & 63) * 2;
  return box * (RK * 128) + k * 128 + ((((b >> 4) ^ (k & 7))) << 4) + (b & 15);
}

// Slot index and phase of a ring of S slots, advanced by a fixed step per use.
struct Ring {
  int slot, phase;
  __device__ __forceinline__ void advance(int step, int n) {
    slot += step;
    while (slot >= n) {
      slot -= n;
      phase ^= 1;
    }
  }
};

template <int RK, int RV, int MT, int NREP, int KF>
__global__ void __launch_bounds__(NT, 1)
    proj_kernel(DecodeParams p, Items I, Geom gm, const __grid_constant__ CUtensorMap tmB) {
  using C = PCfg<RK, RV, MT, NREP, KF>;
  constexpr int N = C::N, TB = C::TB, NS = C::NS, SC = C::SC;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const uint32_t bar0 = smem_u32(sm + C::OFF_BAR);
  auto BAR = [bar0](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tm_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_TM);
  Abort ab{reinterpret_cast<volatile int*>(sm + C::OFF_TM + 4), reinterpret_cast<int*>(p.ws) - 64};
  const ProjScratch sc = proj_scratch(p, KF);

  if (w == 0) {
    tmem_alloc(smem_u32(tm_slot), 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < SK; ++s) mbar_init(BAR(C::B_KFULL + s), 1);
    for (int s = 0; s < SC; ++s) {
      mbar_init(BAR(C::B_CFULL + s), 1);
      reinterpret_cast<int*>(sm + C::OFF_CC)[s] = 0;
    }
    for (int s = 0; s < SV; ++s) mbar_init(BAR(C::B_VFULL + s), 1);
    for (int s = 0; s < NG; ++s) {
      mbar_init(BAR(C::B_GFULL + s), NBW);
      mbar_init(BAR(C::B_GFREE + s), 1);
    }
    for (int s = 0; s < 4; ++s) {
      mbar_init(BAR(C::B_SFULL + s), 1);
      mbar_init(BAR(C::B_SFREE + s), 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(C::B_PREADY + s), NCW);
      mbar_init(BAR(C::B_PFREE + s), 1);
    }
    for (int s = 0; s < NS0; ++s) mbar_init(BAR(C::B_S0FREE + s), NCW);
    *ab.flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  {
    float* cf = reinterpret_cast<float*>(sm + C::OFF_CF);
    for (int e = tid; e < NPMAX * NPAIR; e += NT) cf[e] = e < gm.np * NPAIR ? sc.coef[e] : 0.f;
    int* rw = reinterpret_cast<int*>(sm + C::OFF_RW);
    for (int r = tid; r < VROWS; r += NT) rw[r] = gm.np > 0 ? (((r / gm.np) << 8) | (r % gm.np)) : 0;
    // feature rows past 2 n_hi + np are zero in every G, and so are the Chebyshev
    // operand's padding rows: clear both once
    uint4* gz = reinterpret_cast<uint4*>(sm + C::OFF_G);
    for (int e = tid; e < NG * C::GB / 16; e += NT) gz[e] = make_uint4(0u, 0u, 0u, 0u);
    uint4* vz = reinterpret_cast<uint4*>(sm + C::OFF_V);
    for (int e = tid; e < VROWS * VP / 16; e += NT) vz[e] = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tm_slot;

  // ---- feature table -> tensor memory columns [0, ACOLS): M-tile mt at mt*KF/2, one
  //      token row per lane, two f16 features per 32-bit column
  if (w < NCW) {
    const int qd = w & 3, par = w >> 2;
    for (int mt = par; mt < MT; mt += 2) {
      const int row = mt * 128 + qd * 32 + lane;
      const uint4* src = reinterpret_cast<const uint4*>(sc.atab + (size_t)row * KF);
      uint32_t r[KF / 2];
#pragma unroll
      for (int q = 0; q < KF / 8; ++q) {
        const uint4 v = src[q];
        r[4 * q] = v.x;
        r[4 * q + 1] = v.y;
        r[4 * q + 2] = v.z;
        r[4 * q + 3] = v.w;
      }
      const uint32_t ta = tbase + ((uint32_t)(qd * 32) << 16) + (uint32_t)(mt * (KF / 2));
#pragma unroll
      for (int q = 0; q < KF / 64; ++q) tmem_st32(ta + 32u * q, r + 32 * q);
      if constexpr ((KF / 2) % 32 != 0) tmem_st16(ta + 32u * (KF / 64), r + 32 * (KF / 64));
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  Seq sq;
  sq.x = blockIdx.x;
  if (sq.valid(I)) sq.load_item(I);
  const uint64_t pol = l2_evict_first_policy();

  if (w >= EW0) {
    // ============================================================== epilogue warps ===
    setmaxnreg_dec<80>();
    const int et = tid - ET0, ew = et >> 5;
    int issuedV = 0;
#define SPX_ISSUE_V(at, s)                                                                                        \
  ring_copy(smem_u32(sm + C::OFF_RV + (s) * C::STAGE_V),                                                        \
            reinterpret_cast<const uint8_t*>(p.bv) + ((int64_t)(at).unit() * p.NBc + (at).j()) * C::STAGE_V,   \
            C::STAGE_V, BAR(C::B_VFULL + (s)), pol)
    if (et == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      Seq a = sq;
      for (int k = 0; k < SV && a.valid(I); ++k, a.next(I), ++issuedV) SPX_ISSUE_V(a, k);
    }
    __syncwarp();
    float* sVL = reinterpret_cast<float*>(sm + C::OFF_VL);
    float* sML = reinterpret_cast<float*>(sm + C::OFF_ML);
    float* sST = reinterpret_cast<float*>(sm + C::OFF_ST);
    const uint32_t bvp_u = smem_u32(sm + C::OFF_BVP);
    const bool hl = g < NREP;
    int sv = 0, phv = 0;
    for (int it = 0; sq.valid(I); sq.next(I), ++it) {
      const int b2 = it & 1;
      const uint8_t* st = sm + C::OFF_RV + sv * C::STAGE_V;
      const int64_t unit = sq.unit();
      const bool first_j = sq.jj == 0, last_j = sq.jj == sq.jn - 1;
      const float vscale = __ldg(p.sv + unit * p.NBc + sq.j());
      float* rec = p.ws + (unit * p.nparts + (sq.j0 / I.JR)) * (int64_t)NREP * (FD + 4);
      float2 oold[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        oold[q] = make_float2(0.f, 0.f);
        if (!first_j && hl)
          oold[q] = *reinterpret_cast<const float2*>(rec + g * (FD + 4) + 4 + 8 * (4 * ew + q) + 2 * t4);
      }
      SPX_TRACE(et == 0, it, 40);
      waitw(BAR(C::B_VFULL + sv), (uint32_t)phv, ab);
      SPX_TRACE(et == 0, it, 41);
      waitw(BAR(C::B_PREADY + b2), (uint32_t)((it >> 1) & 1), ab);
      SPX_TRACE(et == 0, it, 42);
      const float* sM = reinterpret_cast<const float*>(sm + C::OFF_PT + b2 * C::PART);
      const float* sL = sM + NCW * NREP;
      const float* sV = sL + NCW * NREP;
      // ---- combine the consumer warps: v_lat[h][r] and the block's (m, l) per head ----
      for (int e = et; e < NREP * RV; e += NEP) {
        const int h = e / RV, r = e - h * RV;
        float M = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < NCW; ++ww) M = fmaxf(M, sM[ww * NREP + h]);
        float v = 0.f, l = 0.f;
#pragma unroll
        for (int ww = 0; ww < NCW; ++ww) {
          const float wt = exp2f(sM[ww * NREP + h] - M);
          v = fmaf(sV[(ww * NREP + h) * C::RVP + r], wt, v);
          l = fmaf(sL[ww * NREP + h], wt, l);
        }
        sVL[h * RV + r] = v;
        if (r == 0) {
          float* stt = sST + (sq.uu * NREP + h) * 2;
          const float mo = first_j ? -INFINITY : stt[0], lo = first_j ? 0.f : stt[1];
          const float Mn = fmaxf(mo, M);
          const float ao = exp2f(mo - Mn), an = exp2f(M - Mn);
          sML[4 * h + 0] = l;
          sML[4 * h + 1] = ao;
          sML[4 * h + 2] = an;
          stt[0] = Mn;
          stt[1] = fmaf(lo, ao, l * an);
        }
      }
      // ---- value basis -> rows padded to QP bytes (conflict-free ldmatrix.trans) -----
      {
        const uint4* src = reinterpret_cast<const uint4*>(st);
        for (int e = et; e < RV * 16; e += NEP)
          *reinterpret_cast<uint4*>(sm + C::OFF_BVP + (e >> 4) * QP + (e & 15) * 16) = src[e];
      }
      named_sync(BAR_EPI, NEP);
      SPX_TRACE(et == 0, it, 43);
      if (et == 0) {
        mbar_arrive(BAR(C::B_PFREE + b2));
        const Seq a = ahead(sq, SV, I);
        if (a.valid(I) && !*ab.flag) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          SPX_ISSUE_V(a, sv);
          ++issuedV;
        }
      }
      __syncwarp();
      if (++sv == SV) {
        sv = 0;
        phv ^= 1;
      }
      // ---- expand once through B_V (mma.sync), merge with the running o --------------
      {
        const float lj = hl ? sML[4 * g] : 1.f;
        const float inv_l = hl ? 1.f / lj : 0.f;
        uint32_t va[RV / 16][2];
#pragma unroll
        for (int ks = 0; ks < RV / 16; ++ks) {
          float2 x0 = make_float2(0.f, 0.f), x1 = x0;
          if (hl) {
            x0 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t4);
            x1 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t4 + 8);
          }
          va[ks][0] = pack_f2(x0.x * inv_l, x0.y * inv_l);
          va[ks][1] = pack_f2(x1.x * inv_l, x1.y * inv_l);
        }
        const float an = hl ? sML[4 * g + 2] * lj * vscale : 0.f;
        const float ao = hl ? sML[4 * g + 1] : 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int n = 4 * ew + q;
          float o[4] = {0.f, 0.f, 0.f, 0.f};
          const int mi = lane >> 3, rr = lane & 7;
          if constexpr (RV == 32) {
            const int R = 16 * (mi >> 1) + 8 * (mi & 1) + rr;
            uint32_t b00, b01, b10, b11;
            ldsm_x4_t(bvp_u + R * QP + n * 16, b00, b01, b10, b11);
            mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
            mma16816(o, va[1][0], 0u, va[1][1], 0u, b10, b11);
          } else {
            const int R = 8 * (mi & 1) + rr;
            uint32_t b00, b01;
            ldsm_x2_t(bvp_u + R * QP + n * 16, b00, b01);
            mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
          }
          if (hl)
            *reinterpret_cast<float2*>(rec + g * (FD + 4) + 4 + 8 * n + 2 * t4) =
                make_float2(fmaf(oold[q].x, ao, o[0] * an), fmaf(oold[q].y, ao, o[1] * an));
        }
        if (last_j && et < NREP) {
          const float* stt = sST + (sq.uu * NREP + et) * 2;
          rec[et * (FD + 4) + 0] = stt[0] * LN2;
          rec[et * (FD + 4) + 1] = stt[1];
        }
      }
      named_sync(BAR_EPI, NEP);
      SPX_TRACE(et == 0, it, 44);
    }
    if (et == 0 && *ab.flag) drain<SV>(BAR(C::B_VFULL), issuedV);
    __syncwarp();
  } else if (w == MMA_W) {
    // ============================================================== MMA issuer ========
    setmaxnreg_dec<80>();
    if (lane == 0) {
      // D f32, A/B f16, both K-major, N columns, M = 128
      const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((128u >> 4) << 24);
      const uint64_t bd0 = umma_desc(smem_u32(sm + C::OFF_G), 16 * N, 128);
      Ring rs{0, 0};
      int pg = 0, last_slot = -1, last_phase = 0;
      int n = 0;
      for (int it = 0; sq.valid(I); sq.next(I), ++it) {
        const int gs = it & 1;
        SPX_TRACE(true, it, 8);
        bool ok = wait1(BAR(C::B_GFULL + gs), (uint32_t)pg, ab);
        SPX_TRACE(true, it, 9);
        if (gs == 1) pg ^= 1;
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt, ++n) {
          if (n >= NS) ok = wait1(BAR(C::B_SFREE + rs.slot), (uint32_t)(rs.phase ^ 1), ab) && ok;
          SPX_TRACE(true, it, 10 + mt);
          if (ok && !*ab.flag) {
            tc_fence_after();
            const uint32_t d = tbase + (uint32_t)(C::ACOLS + rs.slot * N);
            const uint32_t a = tbase + (uint32_t)(mt * (KF / 2));
#pragma unroll
            for (int ks = 0; ks < KF / 16; ++ks)
              umma_ts(d, a + 8u * ks, bd0 + (uint64_t)((gs * C::GB + ks * 32 * N) >> 4), idesc, ks > 0 ? 1u : 0u);
            umma_commit(BAR(C::B_SFULL + rs.slot));
            last_slot = rs.slot;
            last_phase = rs.phase;
          }
          rs.advance(1, NS);
        }
        if (ok && !*ab.flag) umma_commit(BAR(C::B_GFREE + gs));
      }
      if (*ab.flag && last_slot >= 0) {
        const uint64_t t0 = gtimer();
        while (!mbar_try_wait_sleep(BAR(C::B_SFULL + last_slot), (uint32_t)last_phase) && gtimer() - t0 < kWaitNs) {
        }
      }
    }
    __syncwarp();
  } else if (w >= BW0) {
    // ============================================================== builders ==========
    setmaxnreg_dec<80>();
    const int bt = tid - BT0, bw = w - BW0;
    float4* sW = reinterpret_cast<float4*>(sm + C::OFF_W);
    const float* sCF = reinterpret_cast<const float*>(sm + C::OFF_CF);
    const int* sRW = reinterpret_cast<const int*>(sm + C::OFF_RW);
    uint8_t* sV = sm + C::OFF_V;
    int issuedK = 0;
#define SPX_ISSUE_K(at, s)                                                                                        \
  do {                                                                                                            \
    const int64_t unit_ = (at).unit();                                                                            \
    const int row_ = (int)((unit_ * p.NBc + (at).j()) * RK);                                                      \
    uint8_t* st_ = sm + C::OFF_RK + (s) * C::STAGE_K;                                                             \
    const uint32_t bar_ = BAR(C::B_KFULL + (s));                                                                  \
    mbar_expect_tx(bar_, 2 * RK * 128 + NREP * FD * 2);                                                           \
    tma2d(smem_u32(st_ + C::K_B0), &tmB, 0, row_, bar_);                                                          \
    tma2d(smem_u32(st_ + C::K_B1), &tmB, 64, row_, bar_);                                                         \
    bulk_g2s(smem_u32(st_ + C::K_Q),                                                                              \
             reinterpret_cast<const uint8_t*>(p.q) + (((unit_ / p.H) * p.Hq) + (unit_ % p.H) * NREP) * FD * 2,    \
             NREP * FD * 2, bar_);                                                                                \
  } while (0)
    if (bt == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      Seq a = sq;
      for (int k = 0; k < SK && a.valid(I); ++k, a.next(I), ++issuedK) SPX_ISSUE_K(a, k);
    }
    __syncwarp();
    const int nhc = gm.n_hi / 8;               // row tiles of exact pairs (8 pairs each)
    const int nlo = NPAIR - gm.n_hi;           // low pairs
    const int nrows = NREP * gm.np;            // Chebyshev rows
    const int mlt = (nrows + 15) / 16;         // their m-tiles
    const int kls = (2 * nlo) / 16;            // their k-steps (2 nlo dims, a multiple of 16)
    const uint32_t sV_u = smem_u32(sV);
    int sk = 0, phk = 0, pgf = 0, s0i = 0, phs0 = 0;
    // block factor of the first unit-block (pair bt), then prefetched one unit-block ahead
    float2 rot_n = make_float2(0.f, 0.f);
    if (bt < NPAIR && sq.valid(I)) rot_n = sc.rot[(int64_t)sq.j() * NPAIR + bt];
    for (int it = 0; sq.valid(I); sq.next(I), ++it) {
      const int gs = it & 1;
      const uint8_t* st = sm + C::OFF_RK + sk * C::STAGE_K;
      const int clampj = sc.clamp[sq.j()];
      const float2 rot = rot_n;
      {
        const Seq nx = ahead(sq, 1, I);
        if (bt < NPAIR && nx.valid(I)) rot_n = sc.rot[(int64_t)nx.j() * NPAIR + bt];
      }
      SPX_TRACE(bt == 0, it, 0);
      bool ok = waitw(BAR(C::B_KFULL + sk), (uint32_t)phk, ab);
      if (it >= NG) ok = waitw(BAR(C::B_GFREE + gs), (uint32_t)(pgf ^ 1), ab) && ok;
      if (gs == 1) pgf ^= 1;
      const bool need_s0 = clampj < TB;
      if (need_s0 && it >= NS0) ok = waitw(BAR(C::B_S0FREE + s0i), (uint32_t)(phs0 ^ 1), ab) && ok;
      SPX_TRACE(bt == 0, it, 1);
      // ---- query pairs rotated by the block factor: W = conj(q) * rot -----------------
      if (bt < NPAIR) {
        const __half* qh = reinterpret_cast<const __half*>(st + C::K_Q);
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const float q1 = __half2float(qh[h * FD + bt]), q2 = __half2float(qh[h * FD + bt + NPAIR]);
          const float wr = fmaf(q1, rot.x, q2 * rot.y), wi = fmaf(q1, rot.y, -q2 * rot.x);
          sW[h * NPAIR + bt] = make_float4(wr, -gm.sg * wi, -wi, -gm.sg * wr);
        }
      }
      named_sync(BAR_BLD, NBT);
      SPX_TRACE(bt == 0, it, 2);
      uint8_t* G = sm + C::OFF_G + gs * C::GB;
      // ---- Chebyshev operand V[(h, n), d] -> shared memory (f16):
      //      d < nlo: pair i = n_hi + d against B[k][i]; d >= nlo: pair n_hi + d - nlo against
      //      B[k][i + 64]; value c'[n][i] * (n even ? wa.x | wb.x : wa.y | wb.y)
      for (int row = bw; row < nrows; row += NBW) {
        const int hn = sRW[row];
        const int h = hn >> 8, n = hn & 255;
        const bool odd = n & 1;
        __half* vr = reinterpret_cast<__half*>(sV + row * VP);
#pragma unroll 2
        for (int il = lane; il < nlo; il += 32) {
          const int i = gm.n_hi + il;
          const float4 W = sW[h * NPAIR + i];
          const float c = sCF[n * NPAIR + i];
          vr[il] = __float2half_rn(c * (odd ? W.y : W.x));
          vr[nlo + il] = __float2half_rn(c * (odd ? W.w : W.z));
        }
      }
      SPX_TRACE(bt == 0, it, 3);
      // ---- exact pairs on mma.sync: row tile r holds features 16r..16r+15 (pairs 8r..8r+7,
      //      Re and -sg Im) as a block-diagonal 16 x 16 A, per head, against the basis dims
      //      (8r.., 64 + 8r..) as the 16-long K dimension; the basis fragments serve every head
      for (int r = bw; r < nhc; r += NBW) {
        uint32_t a[NREP][4];
        {
          const int pl = 8 * r + (g >> 1);       // pair of row g (row g + 8: pl + 4)
          const bool c1 = g & 1;                 // 0: Re gamma row, 1: -sg Im gamma row
          const bool lo_col = t4 == (g >> 2), hi_col = t4 == (g >> 2) + 2;
          const int e = (g >> 1) & 1;            // which of the thread's two columns
#pragma unroll
          for (int h = 0; h < NREP; ++h) {
            const float4 W1 = sW[h * NPAIR + pl], W2 = sW[h * NPAIR + pl + 4];
            const float f1 = c1 ? W1.y : W1.x, s1 = c1 ? W1.w : W1.z;
            const float f2 = c1 ? W2.y : W2.x, s2 = c1 ? W2.w : W2.z;
            const float v0 = lo_col ? f1 : 0.f, v1 = hi_col ? f2 : 0.f, v2 = lo_col ? s1 : 0.f, v3 = hi_col ? s2 : 0.f;
            a[h][0] = pack_f2(e ? 0.f : v0, e ? v0 : 0.f);
            a[h][1] = pack_f2(e ? 0.f : v1, e ? v1 : 0.f);
            a[h][2] = pack_f2(e ? 0.f : v2, e ? v2 : 0.f);
            a[h][3] = pack_f2(e ? 0.f : v3, e ? v3 : 0.f);
          }
        }
        // basis row k = 8 nt + g, dims 8r + 2t4 (box 0) and 64 + 8r + 2t4 (box 1), swizzled
        const int boff = g * 128 + ((r ^ g) << 4) + 4 * t4;
#pragma unroll
        for (int nt = 0; nt < RK / 8; ++nt) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(st + C::K_B0 + nt * 1024 + boff);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(st + C::K_B1 + nt * 1024 + boff);
#pragma unroll
          for (int h = 0; h < NREP; ++h) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(d, a[h][0], a[h][1], a[h][2], a[h][3], b0, b1);
            // d: (feature 16r + g | + 8, column 8 nt + 2t4 | + 1); transposing the 8 x 8
            // halves gives each thread two consecutive features of column 8 nt + g
            const uint32_t x = movm_t(pack_f2(d[0], d[1])), y = movm_t(pack_f2(d[2], d[3]));
            const int col = h * RK + nt * 8 + g;
            *reinterpret_cast<uint32_t*>(G + ((2 * r) * (N / 8) + (col >> 3)) * 128 + (col & 7) * 16 + 4 * t4) = x;
            *reinterpret_cast<uint32_t*>(G + ((2 * r + 1) * (N / 8) + (col >> 3)) * 128 + (col & 7) * 16 + 4 * t4) = y;
          }
        }
      }
      named_sync(BAR_BLD, NBT);   // the Chebyshev operand is complete
      SPX_TRACE(bt == 0, it, 4);
      // ---- Chebyshev rows: G[2 n_hi + n, (h, k)] = sum_d V[(h, n), d] B[k][dim(d)] --------
      for (int mtl = bw; mtl < mlt; mtl += NBW) {
        float acc[RK / 8][4];
#pragma unroll
        for (int nt = 0; nt < RK / 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        const uint32_t vbase = sV_u + (uint32_t)((mtl * 16 + (lane & 15)) * VP + (lane >> 4) * 16);
        for (int ks = 0; ks < kls; ++ks) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(vbase + ks * 32, a0, a1, a2, a3);
          int off[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int cc = 16 * ks + 2 * t4 + 8 * hh;
            const int dim = cc >= nlo ? FD / 2 + gm.n_hi + cc - nlo : gm.n_hi + cc;
            const int bb = (dim & 63) * 2;
            off[hh] = (dim >> 6) * (RK * 128) + g * 128 + (((bb >> 4) ^ g) << 4) + (bb & 15);
          }
#pragma unroll
          for (int nt = 0; nt < RK / 8; ++nt) {
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(st + off[0] + nt * 1024);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(st + off[1] + nt * 1024);
            mma16816(acc[nt], a0, a1, a2, a3, b0, b1);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int row = mtl * 16 + g + 8 * (q >> 1);
          if (row < nrows) {
            const int hn = sRW[row];
            const int f = 2 * gm.n_hi + (hn & 255);
#pragma unroll
            for (int nt = 0; nt < RK / 8; ++nt) {
              const int col = (hn >> 8) * RK + nt * 8 + 2 * t4 + (q & 1);
              *reinterpret_cast<__half*>(G + g_off<N>(col, f)) = __float2half_rn(acc[nt][q]);
            }
          }
        }
      }
      SPX_TRACE(bt == 0, it, 5);
      // ---- unrotated projections B_k . q for tokens past the query (DISTANCE mode) -------
      if (need_s0) {
        float* s0 = reinterpret_cast<float*>(sm + C::OFF_S0) + s0i * NREP * RK;
        const __half* qh = reinterpret_cast<const __half*>(st + C::K_Q);
        for (int col = bt; col < N; col += NBT) {
          const int h = col / RK, k = col - h * RK;
          float acc = 0.f;
          for (int d = 0; d < FD; ++d)
            acc = fmaf(__half2float(*reinterpret_cast<const __half*>(st + kb_off<RK>(k, d))), __half2float(qh[h * FD + d]),
                       acc);
          s0[h * RK + k] = acc;
        }
      }
      if (++s0i == NS0) {
        s0i = 0;
        phs0 ^= 1;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(BAR(C::B_GFULL + gs));
      named_sync(BAR_BLD, NBT);
      SPX_TRACE(bt == 0, it, 6);
      // every builder warp is done with stage sk of the key ring: refill it
      if (bt == 0 && !*ab.flag) {
        const Seq a = ahead(sq, SK, I);
        if (a.valid(I)) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          SPX_ISSUE_K(a, sk);
          ++issuedK;
        }
      }
      __syncwarp();
      if (++sk == SK) {
        sk = 0;
        phk ^= 1;
      }
    }
    if (bt == 0 && *ab.flag) drain<SK>(BAR(C::B_KFULL), issuedK);
    __syncwarp();
  } else {
    // ============================================================== consumer warps ===
    setmaxnreg_inc<176>();
    const int qd = w & 3, par = w >> 2;
    const uint32_t lrow = (uint32_t)(qd * 32) << 16;
    uint8_t* sP = sm + C::OFF_P + w * 512;
    const uint32_t sP_u = smem_u32(sP);
    const int* sRW = reinterpret_cast<const int*>(sm + C::OFF_RW);
    const float* sCF = reinterpret_cast<const float*>(sm + C::OFF_CF);
    // code ring: stage it % SC holds iteration it; the last consumer warp done with a
    // stage refills it with iteration it + SC
    int* ccnt = reinterpret_cast<int*>(sm + C::OFF_CC);
#define SPX_ISSUE_C(at, stage)                                                                                    \
  do {                                                                                                            \
    const int64_t slot_ = (int64_t)(at).unit() * p.NBc + (at).j();                                                \
    uint8_t* dst_ = sm + C::OFF_RC + (stage) * C::STAGE_C;                                                        \
    const uint32_t bar_ = BAR(C::B_CFULL + (stage));                                                              \
    mbar_expect_tx(bar_, C::STAGE_C);                                                                             \
    bulk_g2s_hint(smem_u32(dst_ + C::C_CK), p.ck + slot_ * (TB * RK), TB * RK, bar_, pol);                        \
    bulk_g2s_hint(smem_u32(dst_ + C::C_CV), p.cv + slot_ * (RV * TB), RV * TB, bar_, pol);                        \
  } while (0)
    if (tid == 0) {
      Seq a = sq;
      for (int k = 0; k < SC && a.valid(I); ++k, a.next(I)) SPX_ISSUE_C(a, k);
    }
    constexpr int NTL = MT / 2;   // M-tiles per consumer warp per unit-block
    Ring rs{par % NS, par / NS};  // S slot of this warp's next M-tile (tile index n = par, par + 2, ...)
    int scs = 0, phc = 0, s0i = 0;
    for (int it = 0; sq.valid(I); sq.next(I), ++it) {
      const int b2 = it & 1;
      const int tb = 16 + 12 * par;
      const bool tw = qd == 0 && lane == 0;
      SPX_TRACE(tw, it, tb);
      const uint8_t* st = sm + C::OFF_RC + scs * C::STAGE_C;
      const int j = sq.j();
      // the scale is first needed after the scores: its load latency hides behind them
      const float kscale = __ldg(p.sk + (int64_t)sq.unit() * p.NBc + j) * p.scale * LOG2E;
      const int clampj = sc.clamp[j];
      waitw(BAR(C::B_CFULL + scs), (uint32_t)phc, ab);
      SPX_TRACE(tw, it, tb + 1);
      float lg[NTL][NREP];
#pragma unroll
      for (int ti = 0; ti < NTL; ++ti) {
        const int mt = par + 2 * ti;
        const int t = mt * 128 + qd * 32 + lane;
        // codes of token t: RK bytes (two 16-byte halves read in a lane-dependent order,
        // so that the lanes of a quarter-warp hit distinct banks)
        float2 cf[RK / 2];
        {
          const uint8_t* crow = st + C::C_CK + t * RK;
          if constexpr (RK == 32) {
            const int sw = (lane >> 2) & 1;
            const uint4 u0 = *reinterpret_cast<const uint4*>(crow + 16 * sw);
            const uint4 u1 = *reinterpret_cast<const uint4*>(crow + 16 * (sw ^ 1));
            const uint4 lo = sw ? u1 : u0, hi = sw ? u0 : u1;
            i8x4_to_f2x2(lo.x, cf[0], cf[1]);
            i8x4_to_f2x2(lo.y, cf[2], cf[3]);
            i8x4_to_f2x2(lo.z, cf[4], cf[5]);
            i8x4_to_f2x2(lo.w, cf[6], cf[7]);
            i8x4_to_f2x2(hi.x, cf[8], cf[9]);
            i8x4_to_f2x2(hi.y, cf[10], cf[11]);
            i8x4_to_f2x2(hi.z, cf[12], cf[13]);
            i8x4_to_f2x2(hi.w, cf[14], cf[15]);
          } else {
            const uint4 u0 = *reinterpret_cast<const uint4*>(crow);
            i8x4_to_f2x2(u0.x, cf[0], cf[1]);
            i8x4_to_f2x2(u0.y, cf[2], cf[3]);
            i8x4_to_f2x2(u0.z, cf[4], cf[5]);
            i8x4_to_f2x2(u0.w, cf[6], cf[7]);
          }
        }
        waitw(BAR(C::B_SFULL + rs.slot), (uint32_t)rs.phase, ab);
        SPX_TRACE(tw, it, tb + 2 + 2 * ti);
        tc_fence_after();
        const uint32_t ts = tbase + lrow + (uint32_t)(C::ACOLS + rs.slot * N);
        uint32_t r[2][RK];
        tmem_ld<RK>(ts, r[0]);
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          tmem_wait_ld<RK>(r[h & 1]);
          if (h + 1 < NREP) tmem_ld<RK>(ts + (uint32_t)((h + 1) * RK), r[(h + 1) & 1]);
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int k2 = 0; k2 < RK / 2; ++k2)
            acc = __ffma2_rn(cf[k2], make_float2(__uint_as_float(r[h & 1][2 * k2]), __uint_as_float(r[h & 1][2 * k2 + 1])),
                             acc);
          lg[ti][h] = (acc.x + acc.y) * kscale;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(C::B_SFREE + rs.slot));
        SPX_TRACE(tw, it, tb + 3 + 2 * ti);
        rs.advance(2, NS);
        if (__any_sync(0xffffffffu, t >= clampj)) {
          // DISTANCE mode, tokens past the query: distance clamped to 0, no rotation
          const float* s0 = reinterpret_cast<const float*>(sm + C::OFF_S0) + s0i * NREP * RK;
          if (t >= clampj) {
#pragma unroll
            for (int h = 0; h < NREP; ++h) {
              float a = 0.f;
#pragma unroll
              for (int k2 = 0; k2 < RK / 2; ++k2)
                a = fmaf(cf[k2].x, s0[h * RK + 2 * k2], fmaf(cf[k2].y, s0[h * RK + 2 * k2 + 1], a));
              lg[ti][h] = a * kscale;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(C::B_S0FREE + s0i));
      if (++s0i == NS0) s0i = 0;
      // ---- per-warp softmax over its tokens (log2 domain) ------------------------------
      float mx[NREP], l[NREP];
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        float m = lg[0][h];
#pragma unroll
        for (int ti = 1; ti < NTL; ++ti) m = fmaxf(m, lg[ti][h]);
        asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(mx[h]) : "f"(m));
        l[h] = 0.f;
      }
      SPX_TRACE(tw, it, tb + 6);
      float vacc[RV / 16][4];
#pragma unroll
      for (int rt = 0; rt < RV / 16; ++rt) vacc[rt][0] = vacc[rt][1] = vacc[rt][2] = vacc[rt][3] = 0.f;
      const uint32_t cV_u = smem_u32(st + C::C_CV);
#pragma unroll
      for (int ti = 0; ti < NTL; ++ti) {
        const int mt = par + 2 * ti;
        float pr[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          pr[h] = 0.f;
          if (h < NREP) {
            pr[h] = exp2f(lg[ti][h] - mx[h]);
            l[h] += pr[h];
          }
        }
        *reinterpret_cast<uint4*>(sP + lane * 16) =
            make_uint4(pack_f2(pr[0], pr[1]), pack_f2(pr[2], pr[3]), pack_f2(pr[4], pr[5]), pack_f2(pr[6], pr[7]));
        __syncwarp();
        uint32_t pb[4];
        ldsm_x4_t(sP_u + lane * 16, pb[0], pb[1], pb[2], pb[3]);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int tt = (mt * 128 + qd * 32) / 16 + half;
          const uint32_t b0 = pb[2 * half], b1 = pb[2 * half + 1];
          if constexpr (RV == 32) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4(cV_u + ((tt * RV + (lane ^ (tt & 7))) << 4), v0, v1, v2, v3);
            uint32_t a0, a1, a2, a3;
            i8x4_to_h2(v0, a0, a2);
            i8x4_to_h2(v1, a1, a3);
            mma16816(vacc[0], a0, a1, a2, a3, b0, b1);
            i8x4_to_h2(v2, a0, a2);
            i8x4_to_h2(v3, a1, a3);
            mma16816(vacc[1], a0, a1, a2, a3, b0, b1);
          } else {
            uint32_t v0, v1;
            ldsm_x2(cV_u + ((tt * RV + ((lane & 15) ^ (tt & 7))) << 4), v0, v1);
            uint32_t a0, a1, a2, a3;
            i8x4_to_h2(v0, a0, a2);
            i8x4_to_h2(v1, a1, a3);
            mma16816(vacc[0], a0, a1, a2, a3, b0, b1);
          }
        }
        __syncwarp();
      }
      SPX_TRACE(tw, it, tb + 7);
      // the code stage is consumed; the last warp to finish refills it
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(ccnt + scs, 1) == NCW - 1) {
          atomicExch(ccnt + scs, 0);
          const Seq a = ahead(sq, SC, I);
          if (a.valid(I) && !*ab.flag) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            SPX_ISSUE_C(a, scs);
          }
        }
      }
      if (++scs == SC) {
        scs = 0;
        phc ^= 1;
      }
#pragma unroll
      for (int h = 0; h < NREP; ++h) l[h] = warp_sum(l[h]);
      // ---- hand (m, l, v_lat) of this warp to the epilogue ----------------------------
      SPX_TRACE(tw, it, tb + 8);
      if (it >= 2) waitw(BAR(C::B_PFREE + b2), (uint32_t)(((it >> 1) - 1) & 1), ab);
      SPX_TRACE(tw, it, tb + 9);
      float* sM = reinterpret_cast<float*>(sm + C::OFF_PT + b2 * C::PART);
      float* sL = sM + NCW * NREP;
      float* sV = sL + NCW * NREP;
      if (lane < NREP) {
        float mv = mx[0], lv = l[0];
#pragma unroll
        for (int h = 1; h < NREP; ++h)
          if (lane == h) {
            mv = mx[h];
            lv = l[h];
          }
        sM[w * NREP + lane] = mv;
        sL[w * NREP + lane] = lv;
      }
#pragma unroll
      for (int rt = 0; rt < RV / 16; ++rt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int head = 2 * t4 + (q & 1), rank = rt * 16 + g + 8 * (q >> 1);
          if (head < NREP) sV[(w * NREP + head) * C::RVP + rank] = vacc[rt][q];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(C::B_PREADY + b2));
      SPX_TRACE(tw, it, tb + 10);
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, 512);
}
#undef SPX_ISSUE_V
#undef SPX_ISSUE_C
#undef SPX_ISSUE_K
#undef SPX_TRACE

// -------------------------------------------------------------- per-call set-up ----
// Block factors, clamp points, the feature table and the Chebyshev coefficients.
//   rot[j][i]  = table row (P_j | qpos - P_j) * e^{+-j theta_i c}   (complex, f32)
//   clamp[j]   = first token of block j past the query (DISTANCE mode), else T
//   atab[t][f] = cos / sin(theta_i (t - c)) for f < 2 n_hi, T_n((t - c) / c) after, 0 pad
//   coef[n][i] = eps_n J_n(theta_i c) (+1, +1, -1, -1 for n mod 4), zero for i < n_hi
struct SetupArgs {
  float theta[NPAIR];
  int n_hi, np, kf;
};

__device__ double bessel_j(int n, double x) {
  // series sum_m (-1)^m (x/2)^(2m+n) / (m! (m+n)!); x <= ~16 here
  double term = 1.0;
  const double h = 0.5 * x;
  for (int k = 1; k <= n; ++k) term *= h / k;
  double s = term;
  for (int m = 1; m < 80; ++m) {
    term *= -(h * h) / ((double)m * (double)(m + n));
    s += term;
    if (fabs(term) < 1e-18 * fabs(s) && m > 4) break;
  }
  return s;
}

__global__ void __launch_bounds__(256) proj_setup_kernel(DecodeParams p, SetupArgs a, ProjScratch sc) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const int T = p.Tb;
  const double c = 0.5 * (T - 1);
  if (b < p.nblk) {
    // ---- block factor and clamp point of block j ----
    const int j = b;
    const int64_t P = p.bpos[j];
    if (tid < NPAIR) {
      const int i = tid;
      int64_t row = p.mode == SPX_ROPE_DISTANCE ? p.qpos - P : P;
      row = row < 0 ? 0 : (row >= p.rope_len ? p.rope_len - 1 : row);
      const double tc = p.cosT[row * FD + i], ts = p.sinT[row * FD + i];
      double sn, cs;
      sincos((double)a.theta[i] * c, &sn, &cs);
      if (p.mode == SPX_ROPE_DISTANCE) sn = -sn;
      sc.rot[(int64_t)j * NPAIR + i] = make_float2((float)(tc * cs - ts * sn), (float)(tc * sn + ts * cs));
    }
    if (tid == 0) {
      int cl = T;
      if (p.mode == SPX_ROPE_DISTANCE) {
        const int64_t f = p.qpos - P + 1;   // first t with P + t > qpos
        cl = f < 0 ? 0 : (f > T ? T : (int)f);
      }
      sc.clamp[j] = cl;
    }
    return;
  }
  const int b2 = b - p.nblk;
  const int KF = a.kf;
  const int ntab = T * KF;
  const int e = b2 * 256 + tid;
  if (e < ntab) {
    const int t = e / KF, f = e - t * KF;
    const double tau = t - c;
    double v = 0.0;
    if (f < 2 * a.n_hi) {
      double sn, cs;
      sincos((double)a.theta[f >> 1] * tau, &sn, &cs);
      v = (f & 1) ? sn : cs;
    } else if (f < 2 * a.n_hi + a.np) {
      const int n = f - 2 * a.n_hi;
      double u = tau / c;
      u = u > 1.0 ? 1.0 : (u < -1.0 ? -1.0 : u);
      v = cos(n * acos(u));
    }
    sc.atab[e] = __float2half_rn((float)v);
    return;
  }
  const int e2 = e - ntab;
  if (e2 < a.np * NPAIR) {
    const int n = e2 / NPAIR, i = e2 - n * NPAIR;
    double v = 0.0;
    if (i >= a.n_hi) {
      const double phi = (double)a.theta[i] * c;
      v = (n == 0 ? 1.0 : 2.0) * bessel_j(n, phi) * ((n & 3) < 2 ? 1.0 : -1.0);
    }
    sc.coef[e2] = (float)v;
  }
}

// ----------------------------------------------------------------- host side -------
// Error bound of the truncated expansion: 2 sum_{n >= np} |J_n(phi)| <= 2 (phi/2)^np / np!
// / (1 - (phi/2) / (np + 1)).
static double cheb_bound(double phi, int np) {
  const double h = 0.5 * fabs(phi);
  if (h >= np + 1) return 1e30;
  double t = 1.0;
  for (int k = 1; k <= np; ++k) t *= h / k;
  return 2.0 * t / (1.0 - h / (np + 1));
}

struct Split {
  int kf, n_hi, np;
};
// The smallest feature count KF in {64, 96, 128} (tensor time), then the cheapest
// builder work: n_hi exact pairs (multiple of 8) and np <= 16 Chebyshev terms for the
// rest, with truncation error <= kChebErr.  KF = 128 with every pair exact always fits.
static bool fits(int RK, int RV, int T, int nrep, int kf);
static Split choose_split(const float* theta, int T, int nrep, int RK, int RV) {
  const double c = 0.5 * (T - 1);
  for (int kf : {64, 96, 128}) {
    if (!fits(RK, RV, T, nrep, kf)) continue;
    Split best{0, 0, 0};
    double best_cost = 1e30;
    for (int n_hi = 0; n_hi <= NPAIR && 2 * n_hi <= kf; n_hi += 8) {
      double phi = 0.0;
      for (int i = n_hi; i < NPAIR; ++i) phi = fmax(phi, fabs((double)theta[i]) * c);
      int np = -1;
      if (n_hi == NPAIR) {
        np = 0;
      } else {
        for (int q = 1; q <= NPMAX && 2 * n_hi + q <= kf && nrep * q <= VROWS; ++q)
          if (cheb_bound(phi, q) <= kChebErr) {
            np = q;
            break;
          }
      }
      if (np < 0) continue;
      const int mlt = (nrep * np + 15) / 16, kls = (2 * (NPAIR - n_hi)) / 16;
      const double cost = 6.0 * n_hi + 12.0 * mlt * kls;
      if (cost < best_cost) {
        best_cost = cost;
        best = Split{kf, n_hi, np};
      }
    }
    if (best.kf) return best;
  }
  return Split{0, 0, 0};
}

// cuTensorMapEncodeTiled, looked up through the runtime (the library does not link the
// driver, so that it loads on machines without one).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

template <int RK, int RV, int MT, int NREP, int KF>
static int launch_cfg(const DecodeParams& p, const Split& s, cudaStream_t st) {
  using C = PCfg<RK, RV, MT, NREP, KF>;
  if constexpr (!C::OK) {
    set_error("projection kernel not built for RK=%d RV=%d T=%d n_rep=%d KF=%d", RK, RV, MT * 128, NREP, KF);
    return SPX_ERR_UNSUPPORTED;
  } else {
  const int units = p.L * p.B * p.H;
  const Plan pl = plan(units, p.nblk, num_sms());
  cudaError_t e = cudaFuncSetAttribute(proj_kernel<RK, RV, MT, NREP, KF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::BYTES);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(proj_kernel): %s", cudaGetErrorString(e));
    return SPX_ERR_CUDA;
  }
  const Items items{pl.G, pl.JR, pl.ngroups, pl.nitems, p.nblk, units};
  Geom gm{s.n_hi, s.np, p.mode == SPX_ROPE_DISTANCE ? -1.f : 1.f};
  // the key bases as a 2-D tensor of rows of 128 f16 dims (one row per (slot, rank)),
  // loaded in boxes of 64 dims x RK rows with the 128-byte swizzle
  CUtensorMap tm;
  const cuuint64_t dims[2] = {(cuuint64_t)FD, (cuuint64_t)p.L * p.B * p.H * p.NBc * RK};
  const cuuint64_t strides[1] = {(cuuint64_t)FD * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)RK};
  const cuuint32_t estr[2] = {1, 1};
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return SPX_ERR_CUDA;
  }
  const CUresult cr = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p.bk), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled(key basis): error %d", (int)cr);
    return SPX_ERR_CUDA;
  }
  proj_kernel<RK, RV, MT, NREP, KF><<<pl.grid, NT, C::BYTES, st>>>(p, items, gm, tm);
  return launch_status("proj_kernel");
  }
}

template <int RK, int RV, int MT, int NREP>
static bool fits_kf(int kf) {
  return kf == 64 ? PCfg<RK, RV, MT, NREP, 64>::OK : kf == 96 ? PCfg<RK, RV, MT, NREP, 96>::OK
                                                              : PCfg<RK, RV, MT, NREP, 128>::OK;
}
template <int RK, int RV, int MT>
static bool fits_nrep(int nrep, int kf) {
  switch (nrep) {
    case 1: return fits_kf<RK, RV, MT, 1>(kf);
    case 2: return fits_kf<RK, RV, MT, 2>(kf);
    case 4: return fits_kf<RK, RV, MT, 4>(kf);
    case 8: return fits_kf<RK, RV, MT, 8>(kf);
    default: return false;
  }
}
// True when the kernel is built for this shape and feature count.
static bool fits(int RK, int RV, int T, int nrep, int kf) {
  auto mt = [&](auto rk, auto rv) {
    constexpr int A = decltype(rk)::value, B = decltype(rv)::value;
    return T == 256 ? fits_nrep<A, B, 2>(nrep, kf) : T == 512 ? fits_nrep<A, B, 4>(nrep, kf) : false;
  };
  using I16 = std::integral_constant<int, 16>;
  using I32 = std::integral_constant<int, 32>;
  if (RK == 32) return RV == 32 ? mt(I32(), I32()) : mt(I32(), I16());
  return RV == 32 ? mt(I16(), I32()) : mt(I16(), I16());
}

template <int RK, int RV, int MT, int NREP>
static int launch_kf(const DecodeParams& p, const Split& s, cudaStream_t st) {
  if (s.kf == 64) return launch_cfg<RK, RV, MT, NREP, 64>(p, s, st);
  if (s.kf == 96) return launch_cfg<RK, RV, MT, NREP, 96>(p, s, st);
  return launch_cfg<RK, RV, MT, NREP, 128>(p, s, st);
}

template <int RK, int RV, int MT>
static int launch_nrep(const DecodeParams& p, const Split& s, cudaStream_t st) {
  switch (p.nrep) {
    case 1: return launch_kf<RK, RV, MT, 1>(p, s, st);
    case 2: return launch_kf<RK, RV, MT, 2>(p, s, st);
    case 4: return launch_kf<RK, RV, MT, 4>(p, s, st);
    default: return launch_kf<RK, RV, MT, 8>(p, s, st);
  }
}

template <int RK, int RV>
static int launch_mt(const DecodeParams& p, const Split& s, cudaStream_t st) {
  return p.Tb == 256 ? launch_nrep<RK, RV, 2>(p, s, st) : launch_nrep<RK, RV, 4>(p, s, st);
}

}  // namespace projk

bool decode_proj_supported(const DecodeParams& p) {
  if (p.nblk <= 0 || p.D != 128 || p.dtype != SPX_F16 || p.mask != nullptr || !p.freq) return false;
  if (!(p.tied || p.mode == SPX_ROPE_DISTANCE)) return false;
  if (!(p.RK == 16 || p.RK == 32) || !(p.RV == 16 || p.RV == 32)) return false;
  if (!(p.Tb == 256 || p.Tb == 512)) return false;
  if (!(p.nrep == 1 || p.nrep == 2 || p.nrep == 4 || p.nrep == 8)) return false;
  if (p.nrep * p.RK > 128 || p.nrep * p.RK < 16) return false;
  if (reinterpret_cast<uintptr_t>(p.q) & 15) return false;
  return projk::choose_split(p.freq, p.Tb, p.nrep, p.RK, p.RV).kf != 0;
}

int decode_proj_ncold(const DecodeParams& p) { return sm100::plan(p.L * p.B * p.H, p.nblk, sm100::num_sms()).nranges; }

size_t decode_proj_scratch_bytes(const DecodeParams& p) {
  return proj_scratch_bytes(p.nblk, p.Tb, 128);
}

int decode_proj_cold(const DecodeParams& p, cudaStream_t st) {
  using namespace projk;
  const Split s = choose_split(p.freq, p.Tb, p.nrep, p.RK, p.RV);
  SPX_REQUIRE(s.kf != 0, SPX_ERR_UNSUPPORTED, "projection kernel: no feature split fits");
  const ProjScratch sc = proj_scratch(p, s.kf);
  SetupArgs a;
  for (int i = 0; i < NPAIR; ++i) a.theta[i] = p.freq[i];
  a.n_hi = s.n_hi;
  a.np = s.np;
  a.kf = s.kf;
  const int nb = p.nblk + (p.Tb * s.kf + s.np * NPAIR + 255) / 256;
  proj_setup_kernel<<<nb, 256, 0, st>>>(p, a, sc);
  int rc = launch_status("proj_setup_kernel");
  if (rc != SPX_OK) return rc;
  if (p.RK == 32) return p.RV == 32 ? launch_mt<32, 32>(p, s, st) : launch_mt<32, 16>(p, s, st);
  return p.RV == 32 ? launch_mt<16, 32>(p, s, st) : launch_mt<16, 16>(p, s, st);
}

}  // namespace spx
