// Fast cold-tier decode kernel for sm_100a (FP16 cache, D = 128, tied RoPE tables).
//
// Work item: one CTA per (cold block j, chunk of units), a unit being one (layer,
// sequence, KV head).  Every unit of the chunk shares block j's token positions, so the
// block's RoPE rows are read once per CTA and parked in tensor memory (TMEM, used here as
// an extension of the register file: each warp writes its own tokens' rows with
// tcgen05.st and reads them back per unit with tcgen05.ld of the same shape).
//
// Per unit the CTA streams, through a 3-stage TMA bulk-copy + mbarrier pipeline:
//   INT8 key codes [T][RK] (token-major), INT8 value codes [RV][T] (rank-major),
//   FP16 bases [RK][128] and [RV][128], and the unit's query rows (n_rep x 128 FP16).
// A swizzle pass copies codes and key basis into bank-conflict-free layouts.  Each warp
// owns 64 tokens (four 16-token m-tiles) and computes, with mma.sync m16n8k16:
//   K~ = codes_K @ B_K (FP32 accumulate)   -> RoPE rotation in packed f16x2 registers
//   scores = rot(K~) . Q                   -> online softmax (exp2, per-warp running max)
//   v_lat += P^T-weighted codes_V          -> [RV x heads]
// Warps combine (m, l, v_lat) in shared memory; v_lat is expanded once through B_V and
// written as the unit's partial (m, l, o[128]) for the hot-tier/merge kernel.
//
// Token order inside a 16-token m-tile is the permutation PI below, chosen so that the
// value codes load with one ldmatrix per m-tile; softmax is order-invariant.
#include <math.h>

#include "spx_common.cuh"
#include "spx_decode.cuh"

namespace spx {
namespace fastk {

constexpr int FD = 128;
constexpr int STAGES = 3;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr unsigned kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier / TMA --
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(cnt) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the phase did not complete within the iteration limit.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity) {
  for (unsigned it = 0; it < kWaitLimit; ++it)
    if (mbar_try_wait(a, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// ------------------------------------------------------------------------- TMEM -----
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16x256_x2(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Load + wait in one statement so no use of the registers can be scheduled early.
__device__ __forceinline__ void tmem_ld16x256_x2(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
}

// ------------------------------------------------------------- warp MMA helpers -----
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t pack_f2(float lo, float hi) { return h2u(__floats2half2_rn(lo, hi)); }

// Four INT8 codes -> two f16x2 (bytes 0,1 -> lo; bytes 2,3 -> hi), exact: the biased byte
// becomes the mantissa of 1024 + byte, then 1152 = 1024 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  uint32_t l, h;
  asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(l) : "r"(x), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(h) : "r"(x), "r"(0x64646464u));
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152.0
  lo = h2u(__hsub2(u2h(l), bias));
  hi = h2u(__hsub2(u2h(h), bias));
}

// Slot s of an m-tile holds token PI(s); PI_INV maps a token back to its slot.
__host__ __device__ __forceinline__ int slot_to_token(int s) {
  return s < 8 ? 4 * (s >> 1) + (s & 1) : 4 * ((s - 8) >> 1) + 2 + (s & 1);
}
__host__ __device__ __forceinline__ int token_to_slot(int tau) { return 2 * (tau >> 2) + (tau & 1) + 8 * ((tau & 3) >> 1); }

template <int RK, int RV, int NW>
struct Cfg {
  static constexpr int NT = NW * 32;
  static constexpr int TB = NW * 64;
  static constexpr int G = RK / 4;                      // key-code bytes per thread-row
  static constexpr int CK = TB * RK;
  static constexpr int CV = RV * TB;
  static constexpr int BK = RK * FD * 2;
  static constexpr int BV = RV * FD * 2;
  static constexpr int QB = 8 * FD * 2;
  static constexpr int STAGE = CK + CV + BK + BV + QB;
  static constexpr int OFF_CK = STAGES * STAGE;         // swizzled compute copies
  static constexpr int OFF_CV = OFF_CK + CK;
  static constexpr int OFF_BK = OFF_CV + CV;
  static constexpr int OFF_SM = OFF_BK + BK;            // per-warp m [NW][8]
  static constexpr int OFF_SL = OFF_SM + NW * 8 * 4;    // per-warp l [NW][8]
  static constexpr int OFF_SV = OFF_SL + NW * 8 * 4;    // per-warp v_lat [NW][RV][8]
  static constexpr int OFF_VL = OFF_SV + NW * RV * 8 * 4;   // combined v_lat [8][RV]
  static constexpr int OFF_ML = OFF_VL + 8 * RV * 4;    // combined (m, l) [8][2]
  static constexpr int OFF_BAR = OFF_ML + 16 * 4;
  static constexpr int OFF_TM = OFF_BAR + STAGES * 8;
  static constexpr int BYTES = OFF_TM + 16;
  static_assert(STAGE % 16 == 0 && OFF_BAR % 8 == 0, "alignment");
};

// Bank-conflict-free chunk index for row R of the key basis (see the loader below).
template <int G>
__device__ __forceinline__ int bk_swz(int R) { return (((R / G) & 3) << 1) | (R & 1); }

template <int RK, int RV, int NW>
__global__ void __launch_bounds__(NW * 32, 1) cold_fast_kernel(DecodeParams p, int units_per_cta) {
  using C = Cfg<RK, RV, NW>;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int j = blockIdx.x;
  const int units = p.L * p.B * p.H;
  const int u0 = blockIdx.y * units_per_cta;
  const int nu = min(units_per_cta, units - u0);
  const int nrep = p.nrep;
  const uint32_t bar0 = smem_u32(sm + C::OFF_BAR);
  uint32_t* tm_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_TM);
  int* err = reinterpret_cast<int*>(p.ws) - 64;   // status word in the workspace header

  if (w == 0) {
    tmem_alloc(smem_u32(tm_slot), 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tm_slot;

  auto issue = [&](int u) {  // one thread: TMA bulk loads of unit u into stage u % STAGES
    const int s = u % STAGES;
    const int64_t unit = u0 + u;
    const int64_t slot = unit * p.NBc + j;
    const int64_t lb = unit / p.H, gg = unit % p.H;
    uint8_t* st = sm + s * C::STAGE;
    const uint32_t bar = bar0 + 8 * s;
    const uint32_t qbytes = nrep * FD * 2;
    mbar_expect_tx(bar, C::CK + C::CV + C::BK + C::BV + qbytes);
    bulk_g2s(smem_u32(st), p.ck + slot * C::CK, C::CK, bar);
    bulk_g2s(smem_u32(st + C::CK), p.cv + slot * C::CV, C::CV, bar);
    bulk_g2s(smem_u32(st + C::CK + C::CV), reinterpret_cast<const uint8_t*>(p.bk) + slot * C::BK, C::BK, bar);
    bulk_g2s(smem_u32(st + C::CK + C::CV + C::BK), reinterpret_cast<const uint8_t*>(p.bv) + slot * C::BV, C::BV, bar);
    bulk_g2s(smem_u32(st + C::CK + C::CV + C::BK + C::BV),
             reinterpret_cast<const uint8_t*>(p.q) + ((lb * p.Hq) + gg * nrep) * FD * 2, qbytes, bar);
  };
  if (tid == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int u = 0; u < min(STAGES, nu); ++u) issue(u);
  }

  // ---- RoPE rows of this warp's 64 tokens -> TMEM (f16 pairs), once per CTA ----------
  const int64_t p0 = p.bpos[j];
  const uint32_t lane_q = (uint32_t)(32 * (w & 3));
  auto taddr = [&](int i) {  // TMEM address of m-tile i of this warp
    return tbase + ((lane_q + 16u * (uint32_t)(i & 1)) << 16) + (uint32_t)(((w >> 2) * 2 + (i >> 1)) * 64);
  };
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    int64_t a[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int tok = w * 64 + i * 16 + slot_to_token(g + 8 * hh);
      const int64_t pos = p0 + tok;
      int64_t aa = p.mode == SPX_ROPE_DISTANCE ? (p.qpos - pos > 0 ? p.qpos - pos : 0) : pos;
      a[hh] = aa < 0 ? 0 : (aa >= p.rope_len ? p.rope_len - 1 : aa);
    }
#pragma unroll 1
    for (int s = 0; s < 4; ++s) {
      uint32_t r[8];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int f = 8 * (2 * s + cc) + 2 * t;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float2 cv = *reinterpret_cast<const float2*>(p.cosT + a[hh] * FD + f);
          const float2 sv = *reinterpret_cast<const float2*>(p.sinT + a[hh] * FD + f);
          r[4 * cc + 2 * hh + 0] = pack_f2(cv.x, cv.y);
          r[4 * cc + 2 * hh + 1] = pack_f2(sv.x, sv.y);
        }
      }
      tmem_st16x256_x2(taddr(i) + 16 * s, r);
    }
  }
  tmem_wait_st();

  float* sM = reinterpret_cast<float*>(sm + C::OFF_SM);
  float* sL = reinterpret_cast<float*>(sm + C::OFF_SL);
  float* sV = reinterpret_cast<float*>(sm + C::OFF_SV);
  float* sVL = reinterpret_cast<float*>(sm + C::OFF_VL);
  float* sML = reinterpret_cast<float*>(sm + C::OFF_ML);
  uint8_t* cK = sm + C::OFF_CK;
  uint8_t* cV = sm + C::OFF_CV;
  uint8_t* bK = sm + C::OFF_BK;
  const uint32_t cK_u = smem_u32(cK), cV_u = smem_u32(cV), bK_u = smem_u32(bK);
  int failed_at = -1;

#pragma unroll 1
  for (int u = 0; u < nu; ++u) {
    const int s = u % STAGES;
    uint8_t* st = sm + s * C::STAGE;
    const bool ok = mbar_wait(bar0 + 8 * s, (uint32_t)((u / STAGES) & 1));
    if (__syncthreads_or(!ok)) {   // every thread takes the same decision
      failed_at = u;
      break;
    }
    // ---- swizzle pass: codes and key basis into conflict-free layouts --------------
    {
      const uint4* src = reinterpret_cast<const uint4*>(st);
      for (int e = tid; e < C::CK / 16; e += C::NT) {       // key codes -> slot order
        const int tok = e / (RK / 16), ch = e % (RK / 16);
        const int row = (tok & ~15) + token_to_slot(tok & 15);
        reinterpret_cast<uint4*>(cK + row * RK)[ch] = src[e];
      }
      const uint4* srcv = reinterpret_cast<const uint4*>(st + C::CK);
      for (int e = tid; e < C::CV / 16; e += C::NT) {       // value codes -> [T/16][RV][16]
        const int r = e / (C::TB / 16), tt = e % (C::TB / 16);
        reinterpret_cast<uint4*>(cV)[tt * RV + r] = srcv[e];
      }
      const uint4* srcb = reinterpret_cast<const uint4*>(st + C::CK + C::CV);
      for (int e = tid; e < C::BK / 16; e += C::NT) {       // key basis, XOR-swizzled chunks
        const int R = e >> 4, n = e & 15;
        reinterpret_cast<uint4*>(bK + R * 256)[n ^ bk_swz<C::G>(R)] = srcb[e];
      }
    }
    __syncthreads();
    const int64_t unit = u0 + u;
    const int64_t slotid = unit * p.NBc + j;
    const float kscale = p.sk[slotid] * p.scale * LOG2E;
    const float vscale = p.sv[slotid];

    // ---- query fragments (B operand of the score MMA), padded heads zeroed ---------
    const uint8_t* sq = st + C::CK + C::CV + C::BK + C::BV;
    uint32_t qf[8][2];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      if (g < nrep) {
        qf[ks][0] = *reinterpret_cast<const uint32_t*>(sq + (g * FD + 16 * ks + 2 * t) * 2);
        qf[ks][1] = *reinterpret_cast<const uint32_t*>(sq + (g * FD + 16 * ks + 2 * t + 8) * 2);
      } else {
        qf[ks][0] = qf[ks][1] = 0u;
      }
    }
    // ---- key-code A fragments of the warp's four m-tiles ---------------------------
    uint32_t af[4][RK / 16][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = w * 64 + i * 16 + g;
      if constexpr (RK == 32) {
        const uint2 v0 = *reinterpret_cast<const uint2*>(cK + row * 32 + 8 * t);
        const uint2 v1 = *reinterpret_cast<const uint2*>(cK + (row + 8) * 32 + 8 * t);
        i8x4_to_h2(v0.x, af[i][0][0], af[i][0][2]);
        i8x4_to_h2(v1.x, af[i][0][1], af[i][0][3]);
        i8x4_to_h2(v0.y, af[i][1][0], af[i][1][2]);
        i8x4_to_h2(v1.y, af[i][1][1], af[i][1][3]);
      } else {
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(cK + row * 16 + 4 * t);
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(cK + (row + 8) * 16 + 4 * t);
        i8x4_to_h2(v0, af[i][0][0], af[i][0][2]);
        i8x4_to_h2(v1, af[i][0][1], af[i][0][3]);
      }
    }
    // ---- scores: reconstruct, rotate, dot ------------------------------------------
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
    const int mrow = lane & 7, mid = lane >> 3;
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      uint32_t bf[4][RK / 16][2];   // n-tiles {2s, 2s+1, 2s+8, 2s+9}
      if constexpr (RK == 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int n = 2 * s4 + (q & 1) + 8 * (q >> 1);
          const int ks = mid >> 1, h = mid & 1;
          const int R = C::G * (mrow >> 1) + 4 * ks + 2 * h + (mrow & 1);
          ldsm_x4_t(bK_u + R * 256 + ((n ^ bk_swz<C::G>(R)) << 4), bf[q][0][0], bf[q][0][1], bf[q][1][0],
                    bf[q][1][1]);
        }
      } else {
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int n = 2 * s4 + (mid >> 1) + 8 * q2;
          const int h = mid & 1;
          const int R = C::G * (mrow >> 1) + 2 * h + (mrow & 1);
          ldsm_x4_t(bK_u + R * 256 + ((n ^ bk_swz<C::G>(R)) << 4), bf[2 * q2][0][0], bf[2 * q2][0][1],
                    bf[2 * q2 + 1][0][0], bf[2 * q2 + 1][0][1]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float acc[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < RK / 16; ++ks)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            mma16816(acc[q], af[i][ks][0], af[i][ks][1], af[i][ks][2], af[i][ks][3], bf[q][ks][0], bf[q][ks][1]);
        uint32_t tr[8];
        tmem_ld16x256_x2(taddr(i) + 16 * s4, tr);
        uint32_t k1[4], k2[4];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // hh: row g (0) or g+8 (1)
            const __half2 a1 = u2h(pack_f2(acc[cc][2 * hh], acc[cc][2 * hh + 1]));
            const __half2 a2 = u2h(pack_f2(acc[2 + cc][2 * hh], acc[2 + cc][2 * hh + 1]));
            const __half2 c = u2h(tr[4 * cc + 2 * hh]), sn = u2h(tr[4 * cc + 2 * hh + 1]);
            k1[2 * cc + hh] = h2u(__hfma2(c, a1, __hneg2(__hmul2(sn, a2))));   // c K1 - s K2
            k2[2 * cc + hh] = h2u(__hfma2(c, a2, __hmul2(sn, a1)));            // s K1 + c K2
          }
        }
        mma16816(sc[i], k1[0], k1[1], k1[2], k1[3], qf[s4][0], qf[s4][1]);
        mma16816(sc[i], k2[0], k2[1], k2[2], k2[3], qf[s4 + 4][0], qf[s4 + 4][1]);
      }
    }
    // ---- per-warp softmax over 64 tokens (log2 domain) ----------------------------
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[i][e] *= kscale;
      mx0 = fmaxf(mx0, fmaxf(sc[i][0], sc[i][2]));
      mx1 = fmaxf(mx1, fmaxf(sc[i][1], sc[i][3]));
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const bool live0 = 2 * t < nrep, live1 = 2 * t + 1 < nrep;
    float l0 = 0.f, l1 = 0.f;
    float vacc[RV / 16][4];
#pragma unroll
    for (int rt = 0; rt < RV / 16; ++rt) vacc[rt][0] = vacc[rt][1] = vacc[rt][2] = vacc[rt][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sc[i][0] = live0 ? exp2f(sc[i][0] - mx0) : 0.f;
      sc[i][2] = live0 ? exp2f(sc[i][2] - mx0) : 0.f;
      sc[i][1] = live1 ? exp2f(sc[i][1] - mx1) : 0.f;
      sc[i][3] = live1 ? exp2f(sc[i][3] - mx1) : 0.f;
      l0 += sc[i][0] + sc[i][2];
      l1 += sc[i][1] + sc[i][3];
      // ---- v_lat[rank][head] += codes_V^T . P  (one ldmatrix per m-tile) ------------
      const uint32_t b0 = movm_t(pack_f2(sc[i][0], sc[i][1]));
      const uint32_t b1 = movm_t(pack_f2(sc[i][2], sc[i][3]));
      const int tt = w * 4 + i;
      if constexpr (RV == 32) {
        uint32_t v0, v1, v2, v3;
        ldsm_x4(cV_u + ((tt * RV + lane) << 4), v0, v1, v2, v3);
        uint32_t a0, a1, a2, a3;
        i8x4_to_h2(v0, a0, a2);
        i8x4_to_h2(v1, a1, a3);
        mma16816(vacc[0], a0, a1, a2, a3, b0, b1);
        i8x4_to_h2(v2, a0, a2);
        i8x4_to_h2(v3, a1, a3);
        mma16816(vacc[1], a0, a1, a2, a3, b0, b1);
      } else {
        uint32_t v0, v1;
        ldsm_x2(cV_u + ((tt * RV + (lane & 15)) << 4), v0, v1);
        uint32_t a0, a1, a2, a3;
        i8x4_to_h2(v0, a0, a2);
        i8x4_to_h2(v1, a1, a3);
        mma16816(vacc[0], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (g == 0) {
      sM[w * 8 + 2 * t] = mx0;
      sM[w * 8 + 2 * t + 1] = mx1;
      sL[w * 8 + 2 * t] = l0;
      sL[w * 8 + 2 * t + 1] = l1;
    }
#pragma unroll
    for (int rt = 0; rt < RV / 16; ++rt) {
      float* base = sV + (w * RV + rt * 16) * 8;
      base[g * 8 + 2 * t] = vacc[rt][0];
      base[g * 8 + 2 * t + 1] = vacc[rt][1];
      base[(g + 8) * 8 + 2 * t] = vacc[rt][2];
      base[(g + 8) * 8 + 2 * t + 1] = vacc[rt][3];
    }
    __syncthreads();
    // ---- combine warps: v_lat[h][r], m, l ------------------------------------------
    for (int e = tid; e < nrep * RV; e += C::NT) {
      const int h = e / RV, r = e % RV;
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) M = fmaxf(M, sM[ww * 8 + h]);
      float v = 0.f, l = 0.f;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) {
        const float wt = exp2f(sM[ww * 8 + h] - M);
        v = fmaf(sV[(ww * RV + r) * 8 + h], wt, v);
        l = fmaf(sL[ww * 8 + h], wt, l);
      }
      sVL[h * RV + r] = v;
      if (r == 0) {
        sML[2 * h] = M;
        sML[2 * h + 1] = l;
      }
    }
    __syncthreads();
    // ---- expand once through B_V and write the partial ----------------------------
    {
      const __half* bv = reinterpret_cast<const __half*>(st + C::CK + C::CV + C::BK);
      float* rec = p.ws + (unit * p.nparts + j) * (int64_t)nrep * (FD + 4);
      for (int e = tid; e < nrep * (FD / 2); e += C::NT) {
        const int h = e / (FD / 2), d = 2 * (e % (FD / 2));
        float o0 = 0.f, o1 = 0.f;
#pragma unroll 8
        for (int r = 0; r < RV; ++r) {
          const float2 bb = __half22float2(*reinterpret_cast<const __half2*>(bv + r * FD + d));
          const float vl = sVL[h * RV + r];
          o0 = fmaf(vl, bb.x, o0);
          o1 = fmaf(vl, bb.y, o1);
        }
        *reinterpret_cast<float2*>(rec + h * (FD + 4) + 4 + d) = make_float2(o0 * vscale, o1 * vscale);
      }
      if (tid < nrep) {
        rec[tid * (FD + 4) + 0] = sML[2 * tid] * LN2;
        rec[tid * (FD + 4) + 1] = sML[2 * tid + 1];
      }
    }
    __syncthreads();
    if (tid == 0 && u + STAGES < nu) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(u + STAGES);
    }
  }
  if (failed_at >= 0 && tid == 0) {
    atomicExch(err, 1);
    // drain the copies still in flight (bounded) before the shared memory goes away:
    // units failed_at .. failed_at + STAGES - 1 were issued and not yet consumed
    for (int u = failed_at; u < min(failed_at + STAGES, nu); ++u)
      mbar_wait(bar0 + 8 * (u % STAGES), (uint32_t)((u / STAGES) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, 256);
}

template <int RK, int RV, int NW>
int launch(const DecodeParams& p, cudaStream_t st) {
  using C = Cfg<RK, RV, NW>;
  const int units = p.L * p.B * p.H;
  long want = (long)units * p.nblk / (148L * 4);
  int upc = (int)(want < 1 ? 1 : (want > 64 ? 64 : want));
  const int chunks = (units + upc - 1) / upc;
  SPX_REQUIRE(chunks <= 65535, SPX_ERR_UNSUPPORTED, "too many units for one launch");
  cudaFuncSetAttribute(cold_fast_kernel<RK, RV, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
  dim3 grid(p.nblk, chunks);
  cold_fast_kernel<RK, RV, NW><<<grid, C::NT, C::BYTES, st>>>(p, upc);
  return launch_status("cold_fast_kernel");
}

}  // namespace fastk

bool decode_fast_supported(const DecodeParams& p) {
  if (p.nblk <= 0 || p.D != 128 || p.dtype != SPX_F16 || p.mask != nullptr) return false;
  if (!(p.tied || p.mode == SPX_ROPE_DISTANCE)) return false;
  if (!(p.RK == 16 || p.RK == 32) || !(p.RV == 16 || p.RV == 32)) return false;
  if (!(p.Tb == 128 || p.Tb == 256 || p.Tb == 512)) return false;
  if (!(p.nrep == 1 || p.nrep == 2 || p.nrep == 4 || p.nrep == 8)) return false;
  if (reinterpret_cast<uintptr_t>(p.q) & 15) return false;
  return true;
}

template <int RK, int RV>
static int launch_nw(const DecodeParams& p, cudaStream_t st) {
  switch (p.Tb) {
    case 128: return fastk::launch<RK, RV, 2>(p, st);
    case 256: return fastk::launch<RK, RV, 4>(p, st);
    default: return fastk::launch<RK, RV, 8>(p, st);
  }
}

int decode_fast_cold(const DecodeParams& p, cudaStream_t st) {
  if (p.RK == 32) return p.RV == 32 ? launch_nw<32, 32>(p, st) : launch_nw<32, 16>(p, st);
  return p.RV == 32 ? launch_nw<16, 32>(p, st) : launch_nw<16, 16>(p, st);
}

}  // namespace spx
