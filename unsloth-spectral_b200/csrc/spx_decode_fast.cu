// Fast cold-tier decode kernel for sm_100a (FP16 cache, D = 128, tied RoPE tables).
//
// Work item: one CTA per (cold block j, chunk of units), a unit being one (layer,
// sequence, KV head).  Every unit of the chunk shares block j's token positions, so the
// block's RoPE rows are read once per CTA and parked in tensor memory (TMEM columns
// 0..255, used as an extension of the register file: each warp writes its own tokens'
// rows with tcgen05.st and reads them back per unit with tcgen05.ld of the same shape).
//
// Per unit the CTA streams, through a 3-stage TMA bulk-copy + mbarrier pipeline:
//   INT8 key codes [T][RK] (token-major), INT8 value codes (value-tile layout),
//   FP16 bases [RK][128] and [RV][128], and the unit's query rows (n_rep x 128 FP16).
// A conversion pass turns the key codes into FP16 UMMA operand tiles (K-major, no
// swizzle) and the key basis into the MN-major operand; one thread then issues
//   tcgen05.mma kind::f16  M=128 tokens x N=128 dims x K=16   (K~ = codes_K @ B_K)
// into one of two TMEM accumulators (columns 256..511), per 128-token M-tile.  Warps
// read K~ back with tcgen05.ld.16x256b, which lands in the mma.sync fragment layout:
//   rotate K~ by the token's RoPE row in packed f16x2   -> A fragment
//   scores = rot(K~) . Q          (mma.sync m16n8k16)   -> online softmax (exp2)
//   v_lat += codes_V^T . P        (mma.sync m16n8k16)   -> [RV x heads]
// Warps combine (m, l, v_lat) in shared memory; v_lat is expanded once through B_V and
// written as the unit's partial (m, l, o[128]) for the hot-tier/merge kernel.
//
// Value codes arrive in the value-tile layout (16-token tiles, XOR-swizzled rows, tokens
// ordered 0,1,8,9, 2,3,10,11, ...), so one ldmatrix per 16 tokens yields mma.sync A
// fragments directly.
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

// ------------------------------------------------------------------- tcgen05.mma ----
// Shared-memory matrix descriptor, no swizzle: start address, leading-dimension byte
// offset and stride-dimension byte offset (all >> 4), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor: D f32, A/B f16, A K-major, B MN-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) | ((128u >> 3) << 17) |
                            ((128u >> 4) << 24);
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Three 16x256b.x2 loads (24 registers) issued without waiting.
__device__ __forceinline__ void tmem_ld3(uint32_t ta, uint32_t tb, uint32_t tc, uint32_t (&r)[24]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%24];\n\t"
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%25];\n\t"
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%26];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23])
      : "r"(ta), "r"(tb), "r"(tc)
      : "memory");
}
// Wait for this thread's TMEM loads; the registers are tied to the wait so that no use
// of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld_tied(uint32_t (&r)[24]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]) :: "memory");
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
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
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

template <int RK, int RV, int NW>
struct Cfg {
  static constexpr int NT = NW * 32;
  static constexpr int TB = NW * 64;
  static constexpr int MT = TB / 128;                   // 128-token UMMA M-tiles per unit
  static constexpr int CK = TB * RK;
  static constexpr int CV = RV * TB;
  static constexpr int BK = RK * FD * 2;
  static constexpr int BV = RV * FD * 2;
  static constexpr int QB = 8 * FD * 2;
  static constexpr int STAGE = CK + CV + BK + BV + QB;
  static constexpr int ATILE = 128 * RK * 2;            // one M-tile of FP16 key codes
  static constexpr int OFF_A = STAGES * STAGE;          // UMMA A tiles [MT][RK/8][16][8 rows][16 B]
  static constexpr int OFF_B = OFF_A + MT * ATILE;      // UMMA B tile  [16 n-chunks][RK rows][16 B]
  static constexpr int OFF_CV = OFF_B + BK;             // value codes [T/16][RV][16 B], XOR-swizzled rows
  static constexpr int OFF_Q = OFF_CV + CV;             // query [8][16 chunks], XOR-swizzled chunks
  static constexpr int OFF_BV = OFF_Q + QB;             // value basis [RV][16 chunks], XOR-swizzled
  static constexpr int OFF_SM = OFF_BV + BV;            // per-warp m [NW][8]
  static constexpr int OFF_SL = OFF_SM + NW * 8 * 4;    // per-warp l [NW][8]
  static constexpr int OFF_SV = OFF_SL + NW * 8 * 4;    // per-warp v_lat [NW][RV][8]
  static constexpr int OFF_VL = OFF_SV + NW * RV * 8 * 4;   // combined v_lat [8][RV]
  static constexpr int OFF_ML = OFF_VL + 8 * RV * 4;    // combined (m, l) [8][2]
  static constexpr int OFF_BAR = OFF_ML + 16 * 4;       // STAGES load barriers + 2 MMA barriers
  static constexpr int OFF_TM = OFF_BAR + (STAGES + 2) * 8;
  static constexpr int BYTES = OFF_TM + 16;
  static_assert(STAGE % 16 == 0 && OFF_BAR % 8 == 0 && OFF_A % 128 == 0, "alignment");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

template <int NW>
struct Group {
  int mt, lane_off, tcol;
  __device__ __forceinline__ Group(int w, int i) {
    if constexpr (NW == 8) {
      mt = i;
      lane_off = 32 * (w & 3) + 16 * (w >> 2);
      tcol = 64 * i;
    } else {
      mt = i >> 1;
      lane_off = 32 * w + 16 * (i & 1);
      tcol = 64 * (i >> 1);
    }
  }
  __device__ __forceinline__ int token0() const { return mt * 128 + lane_off; }
};

template <int RK, int RV, int NW>
__global__ void __launch_bounds__(NW * 32, 1) cold_fast_kernel(DecodeParams p, int units_per_cta) {
  using C = Cfg<RK, RV, NW>;
  static_assert(NW == 8 || NW == 4, "one or two warps per TMEM lane quadrant");
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int j = blockIdx.x;
  const int units = p.L * p.B * p.H;
  const int u0 = blockIdx.y * units_per_cta;
  const int nu = min(units_per_cta, units - u0);
  const int nrep = p.nrep;
  const uint32_t bar0 = smem_u32(sm + C::OFF_BAR);      // TMA stage barriers
  const uint32_t mbar0 = bar0 + 8 * STAGES;              // MMA-done barriers, one per accumulator
  uint32_t* tm_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_TM);
  int* err = reinterpret_cast<int*>(p.ws) - 64;   // status word in the workspace header

  if (w == 0) {
    tmem_alloc(smem_u32(tm_slot), 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES + 2; ++s) mbar_init(bar0 + 8 * s, 1);
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
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const Group<NW> G(w, i);
    int64_t a[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int64_t pos = p0 + G.token0() + g + 8 * hh;
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
      tmem_st16x256_x2(tbase + ((uint32_t)G.lane_off << 16) + (uint32_t)(G.tcol + 16 * s), r);
    }
  }
  tmem_wait_st();

  float* sM = reinterpret_cast<float*>(sm + C::OFF_SM);
  float* sL = reinterpret_cast<float*>(sm + C::OFF_SL);
  float* sV = reinterpret_cast<float*>(sm + C::OFF_SV);
  float* sVL = reinterpret_cast<float*>(sm + C::OFF_VL);
  float* sML = reinterpret_cast<float*>(sm + C::OFF_ML);
  uint8_t* sA = sm + C::OFF_A;
  uint8_t* sB = sm + C::OFF_B;
  uint8_t* cV = sm + C::OFF_CV;
  uint8_t* sQ = sm + C::OFF_Q;
  const uint32_t sA_u = smem_u32(sA), sB_u = smem_u32(sB), cV_u = smem_u32(cV);
  int failed_at = -1;
  uint32_t mma_uses[2] = {0u, 0u};   // completed waits per accumulator (phase parity)

  auto issue_mma = [&](int mt) {   // one thread: K~ of M-tile mt into accumulator mt & 1
    tc_fence_after();
    const uint32_t d = tbase + 256u + 128u * (uint32_t)(mt & 1);
#pragma unroll
    for (int ks = 0; ks < RK / 16; ++ks) {
      const uint64_t ad = umma_desc(sA_u + mt * C::ATILE + ks * 2 * 2048, 2048, 128);
      const uint64_t bd = umma_desc(sB_u + ks * 256, 128, RK * 16);
      umma_f16(d, ad, bd, ks > 0 ? 1u : 0u);
    }
    umma_commit(mbar0 + 8 * (mt & 1));
  };

#pragma unroll 1
  for (int u = 0; u < nu; ++u) {
    const int s = u % STAGES;
    uint8_t* st = sm + s * C::STAGE;
    const bool ok = mbar_wait(bar0 + 8 * s, (uint32_t)((u / STAGES) & 1));
    if (__syncthreads_or(!ok)) {   // every thread takes the same decision
      failed_at = u;
      break;
    }
    // ---- conversion pass -----------------------------------------------------------
    {
      // key codes -> FP16 A tiles (row m of M-tile mt = token mt*128 + m), 16-byte
      // K-chunks of 8 codes, K-major, no swizzle; one item = 16 codes of one token
      for (int e = tid; e < C::TB * (RK / 16); e += C::NT) {
        const int tau = e % C::TB, hf = e / C::TB;
        const uint4 v = *reinterpret_cast<const uint4*>(st + tau * RK + hf * 16);
        const int m = tau & 127;
        uint8_t* dst = sA + (tau >> 7) * C::ATILE + 2 * hf * 2048 + (m >> 3) * 128 + (m & 7) * 16;
        uint4 o0, o1;
        i8x4_to_h2(v.x, o0.x, o0.y);
        i8x4_to_h2(v.y, o0.z, o0.w);
        i8x4_to_h2(v.z, o1.x, o1.y);
        i8x4_to_h2(v.w, o1.z, o1.w);
        *reinterpret_cast<uint4*>(dst) = o0;
        *reinterpret_cast<uint4*>(dst + 2048) = o1;
      }
      // key basis [RK][128] -> MN-major B tile [16 n-chunks][RK rows][16 B]
      const uint4* srcb = reinterpret_cast<const uint4*>(st + C::CK + C::CV);
      for (int e = tid; e < RK * 16; e += C::NT) {
        const int k = e % RK, nc = e / RK;
        reinterpret_cast<uint4*>(sB)[nc * RK + k] = srcb[k * 16 + nc];
      }
      // value codes are stored in the value-tile layout the ldmatrix below reads
      const uint4* srcv = reinterpret_cast<const uint4*>(st + C::CK);
      for (int e = tid; e < C::CV / 16; e += C::NT) reinterpret_cast<uint4*>(cV)[e] = srcv[e];
      // value basis [RV][128] -> chunk index XOR (rank & 7) (conflict-free ldmatrix)
      const uint4* srcbv = reinterpret_cast<const uint4*>(st + C::CK + C::CV + C::BK);
      for (int e = tid; e < RV * 16; e += C::NT) {
        const int R = e >> 4, n = e & 15;
        reinterpret_cast<uint4*>(sm + C::OFF_BV)[R * 16 + (n ^ (R & 7))] = srcbv[e];
      }
      // query rows, 16-byte chunk index XOR head
      const uint4* srcq = reinterpret_cast<const uint4*>(st + C::CK + C::CV + C::BK + C::BV);
      for (int e = tid; e < nrep * 16; e += C::NT) {
        const int h = e >> 4, n = e & 15;
        reinterpret_cast<uint4*>(sQ)[h * 16 + (n ^ h)] = srcq[e];
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      issue_mma(0);
      if (C::MT > 1) issue_mma(1);
    }
    const int64_t unit = u0 + u;
    const int64_t slotid = unit * p.NBc + j;
    const float kscale = p.sk[slotid] * p.scale * LOG2E;
    const float vscale = p.sv[slotid];

    // ---- query fragments (B operand of the score MMA), padded heads zeroed ---------
    uint32_t qf[8][2];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      if (g < nrep) {
        qf[ks][0] = *reinterpret_cast<const uint32_t*>(sQ + (g * 16 + ((2 * ks) ^ g)) * 16 + 4 * t);
        qf[ks][1] = *reinterpret_cast<const uint32_t*>(sQ + (g * 16 + ((2 * ks + 1) ^ g)) * 16 + 4 * t);
      } else {
        qf[ks][0] = qf[ks][1] = 0u;
      }
    }
    // ---- scores: K~ from TMEM, rotate, dot ----------------------------------------
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const Group<NW> G(w, i);
      const bool first_of_tile = (NW == 8) || ((i & 1) == 0);
      const int b = G.mt & 1;
      if (first_of_tile) {
        const bool mok = mbar_wait(mbar0 + 8 * b, mma_uses[b] & 1u);
        mma_uses[b]++;
        if (!mok) atomicExch(err, 1);
        tc_fence_after();
      }
      const uint32_t lrow = (uint32_t)G.lane_off << 16;
      const uint32_t dcol = tbase + lrow + 256u + 128u * (uint32_t)b;
      const uint32_t tcol = tbase + lrow + (uint32_t)G.tcol;
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t cur[24];
      tmem_ld3(dcol, dcol + 64, tcol, cur);
      tmem_wait_ld_tied(cur);
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        uint32_t nxt[24];
        if (s4 < 3) tmem_ld3(dcol + 16 * (s4 + 1), dcol + 64 + 16 * (s4 + 1), tcol + 16 * (s4 + 1), nxt);
        uint32_t k1[4], k2[4];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // hh: row g (0) or g+8 (1)
            const int e = 4 * cc + 2 * hh;
            const __half2 a1 = u2h(pack_f2(__uint_as_float(cur[e]), __uint_as_float(cur[e + 1])));
            const __half2 a2 = u2h(pack_f2(__uint_as_float(cur[8 + e]), __uint_as_float(cur[8 + e + 1])));
            const __half2 c = u2h(cur[16 + e]), sn = u2h(cur[16 + e + 1]);
            k1[2 * cc + hh] = h2u(__hfma2(c, a1, __hneg2(__hmul2(sn, a2))));   // c K1 - s K2
            k2[2 * cc + hh] = h2u(__hfma2(c, a2, __hmul2(sn, a1)));            // s K1 + c K2
          }
        }
        mma16816(sa, k1[0], k1[1], k1[2], k1[3], qf[s4][0], qf[s4][1]);
        mma16816(sb, k2[0], k2[1], k2[2], k2[3], qf[s4 + 4][0], qf[s4 + 4][1]);
        if (s4 < 3) {
          tmem_wait_ld_tied(nxt);
#pragma unroll
          for (int q = 0; q < 24; ++q) cur[q] = nxt[q];
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[i][e] = sa[e] + sb[e];
      // accumulator b is free once every warp has read this M-tile: refill it
      const bool last_of_tile = (NW == 8) || ((i & 1) == 1);
      if (last_of_tile && G.mt + 2 < C::MT) {
        tc_fence_before();
        __syncthreads();
        if (tid == 0) issue_mma(G.mt + 2);
      }
    }
    // ---- per-warp softmax over 64 tokens (log2 domain) ----------------------------
    // raw scores times kscale (> 0) are the logits in log2 units; fold the scale into
    // the exp2 argument instead of scaling every score
    // (the max of the scaled logits is max*k for k >= 0 and min*k for k < 0)
    const bool kpos = kscale >= 0.f;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mx0 = fmaxf(mx0, kpos ? fmaxf(sc[i][0], sc[i][2]) : -fminf(sc[i][0], sc[i][2]));
      mx1 = fmaxf(mx1, kpos ? fmaxf(sc[i][1], sc[i][3]) : -fminf(sc[i][1], sc[i][3]));
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    mx0 = kpos ? mx0 * kscale : -mx0 * kscale;
    mx1 = kpos ? mx1 * kscale : -mx1 * kscale;
    const bool live0 = 2 * t < nrep, live1 = 2 * t + 1 < nrep;
    float l0 = 0.f, l1 = 0.f;
    float vacc[RV / 16][4];
#pragma unroll
    for (int rt = 0; rt < RV / 16; ++rt) vacc[rt][0] = vacc[rt][1] = vacc[rt][2] = vacc[rt][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sc[i][0] = live0 ? exp2f(fmaf(sc[i][0], kscale, -mx0)) : 0.f;
      sc[i][2] = live0 ? exp2f(fmaf(sc[i][2], kscale, -mx0)) : 0.f;
      sc[i][1] = live1 ? exp2f(fmaf(sc[i][1], kscale, -mx1)) : 0.f;
      sc[i][3] = live1 ? exp2f(fmaf(sc[i][3], kscale, -mx1)) : 0.f;
      l0 += sc[i][0] + sc[i][2];
      l1 += sc[i][1] + sc[i][3];
      // ---- v_lat[rank][head] += codes_V^T . P  (one ldmatrix per 16 tokens) ---------
      const uint32_t b0 = movm_t(pack_f2(sc[i][0], sc[i][1]));
      const uint32_t b1 = movm_t(pack_f2(sc[i][2], sc[i][3]));
      const int tt = Group<NW>(w, i).token0() >> 4;
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
    // ---- expand once through B_V (mma.sync) and write the partial -----------------
    // o[h][d] = l_h * sum_r (v_lat[h][r] / l_h) B_V[r][d]: the normalised v_lat is a
    // weighted mean of INT8 codes (|.| <= 127), safe as an f16 operand.
    {
      float* rec = p.ws + (unit * p.nparts + j) * (int64_t)nrep * (FD + 4);
      const uint32_t bv_u = smem_u32(sm + C::OFF_BV);
      const bool hl = g < nrep;
      const float inv_l = hl ? 1.f / sML[2 * g + 1] : 0.f;
      uint32_t va[RV / 16][2];
#pragma unroll
      for (int ks = 0; ks < RV / 16; ++ks) {
        const float2 x0 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t);
        const float2 x1 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t + 8);
        va[ks][0] = hl ? pack_f2(x0.x * inv_l, x0.y * inv_l) : 0u;
        va[ks][1] = hl ? pack_f2(x1.x * inv_l, x1.y * inv_l) : 0u;
      }
      const float oscale = hl ? sML[2 * g + 1] * vscale : 0.f;
      constexpr int NTW = 16 / NW;   // n-tiles (8 dims each) per warp
#pragma unroll
      for (int q = 0; q < NTW; ++q) {
        const int n = w * NTW + q;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        const int mi = lane >> 3, rr = lane & 7;
        if constexpr (RV == 32) {
          const int R = 16 * (mi >> 1) + 8 * (mi & 1) + rr;
          uint32_t b00, b01, b10, b11;
          ldsm_x4_t(bv_u + R * 256 + ((n ^ (R & 7)) << 4), b00, b01, b10, b11);
          mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
          mma16816(o, va[1][0], 0u, va[1][1], 0u, b10, b11);
        } else {
          const int R = 8 * (mi & 1) + rr;
          uint32_t b00, b01;
          ldsm_x2_t(bv_u + R * 256 + ((n ^ (R & 7)) << 4), b00, b01);
          mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
        }
        if (hl)
          *reinterpret_cast<float2*>(rec + g * (FD + 4) + 4 + 8 * n + 2 * t) =
              make_float2(o[0] * oscale, o[1] * oscale);
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
  if (w == 0) tmem_dealloc(tbase, 512);
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
  if (!(p.Tb == 256 || p.Tb == 512)) return false;
  if (!(p.nrep == 1 || p.nrep == 2 || p.nrep == 4 || p.nrep == 8)) return false;
  if (reinterpret_cast<uintptr_t>(p.q) & 15) return false;
  return true;
}

template <int RK, int RV>
static int launch_nw(const DecodeParams& p, cudaStream_t st) {
  return p.Tb == 256 ? fastk::launch<RK, RV, 4>(p, st) : fastk::launch<RK, RV, 8>(p, st);
}

int decode_fast_cold(const DecodeParams& p, cudaStream_t st) {
  if (p.RK == 32) return p.RV == 32 ? launch_nw<32, 32>(p, st) : launch_nw<32, 16>(p, st);
  return p.RV == 32 ? launch_nw<16, 32>(p, st) : launch_nw<16, 16>(p, st);
}

}  // namespace spx
