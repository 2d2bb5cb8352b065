// Fast cold-tier decode kernel for sm_100a (FP16 or BF16 cache, D = 128, tied or distance
// RoPE).  A BF16 cache has its bases and queries converted to FP16 where they are staged in
// shared memory (key basis -> B tile, value basis -> padded rows, query fragments); the
// arithmetic below is the same for both.
//
// Work decomposition.  A unit is one (layer, sequence, KV head); a unit-block is one unit
// restricted to one cold block j.  The launch covers items = (group of G units) x (range
// of JR blocks); a persistent CTA per SM walks its items block-major (for j in range:
// for u in group), so block j's RoPE rows are parked in tensor memory once per j and the
// unit's softmax state (m, l, o) is merged across the j of the range inside the CTA: one
// partial record per (unit, range) is written for the hot-tier/merge kernel.
//
// Warp roles (4 warpgroups, 512 threads, one CTA per SM; registers rebalanced with
// setmaxnreg: 176 for the consumers, 80 for the others):
//   warpgroup 2  warps 8-9 convert ring A (INT8 key codes [T][RK], FP16 key basis
//                [RK][128]) -> FP16 UMMA A tiles (K-major, no swizzle) and the MN-major B
//                tile, signalling each tile on an mbarrier; lane 0 of warp 10 (even
//                M-tiles) and of warp 11 (odd M-tiles) issue
//                  tcgen05.mma kind::f16  M=128 tokens x N=128 dims x K=16, D = f16
//                (K~ = codes_K @ B_K) into TMEM accumulator 0 / 1, so the two
//                accumulators cycle independently; lane 0 of warp 11 also bulk-copies
//                ring A 3 stages ahead.
//   warpgroups 0-1  consumers, two warps per TMEM lane quadrant, 16 tokens of each
//                M-tile: K~ via tcgen05.ld 16x256b.pack::16b (already f16 pairs; the next
//                M-tile loads while this one computes), RoPE rows via tcgen05.ld 16x256b,
//                rotate in f16x2, scores = rot(K~) . Q (mma.sync m16n8k16), softmax
//                (exp2), v_lat += codes_V^T P (mma.sync) with the value codes of ring B
//                (value-tile layout); each warp hands (m, l, v_lat) to the epilogue.
//   warpgroup 3  epilogue: combines the 8 warps, expands v_lat once through B_V, merges
//                into the unit's running (m, l, o); thread 384 bulk-copies ring B (value
//                codes, value basis, query rows at a padded pitch) 3 stages ahead.
// Every wait is bounded in time; a wait that expires raises the CTA's abort flag and the
// workspace error word, after which all waits return at once and no new copies or MMAs
// are issued, so every role still reaches each named barrier and the CTA exits.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "spx_common.cuh"
#include "spx_decode.cuh"
#include "spx_sm100.cuh"

namespace spx {
namespace fastk {

constexpr int FD = 128;
constexpr int STAGES = 3;
constexpr int NA = 2;                      // A-tile slots, paired with the two TMEM accumulators
constexpr int NCW = 8;                     // consumer warps (warpgroups 0, 1)
constexpr int NPW = 4;                     // converter warps (warpgroup 2)
constexpr int NEW = 4;                     // epilogue warps (warpgroup 3)
constexpr int NT = (NCW + NPW + NEW) * 32;
constexpr int PT0 = NCW * 32;              // first converter thread
constexpr int ET0 = (NCW + NPW) * 32;      // first epilogue thread
constexpr int NEP = NEW * 32;
constexpr int NCV = NPW - 2;               // converter warps that convert; the other two issue MMAs
constexpr int BAR_EPI = 3;                 // named barrier of the epilogue warps

using namespace sm100;

#define SPX_R8(r, o) "=r"(r[o + 0]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), "=r"(r[o + 4]), "=r"(r[o + 5]), \
                     "=r"(r[o + 6]), "=r"(r[o + 7])
#define SPX_I8(r, o) "r"(r[o + 0]), "r"(r[o + 1]), "r"(r[o + 2]), "r"(r[o + 3]), "r"(r[o + 4]), "r"(r[o + 5]), \
                     "r"(r[o + 6]), "r"(r[o + 7])

// 32 registers of RoPE words (16x256b.x8, 64 columns) -> TMEM, then wait for the store.
__device__ __forceinline__ void tmem_st_rope(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      SPX_I8(r, 0), SPX_I8(r, 8), SPX_I8(r, 16), SPX_I8(r, 24)
      : "memory");
}
// K~ (f16 accumulator, 128 columns, packed pairs) and the RoPE words (64 columns) of one
// 16-lane slab, without the wait: the registers are valid only after tmem_wait_ld_64.
__device__ __forceinline__ void tmem_ld_k_rope_nowait(uint32_t tk, uint32_t tr, uint32_t (&k)[32], uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.pack::16b.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, "
      "%45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];"
      : SPX_R8(k, 0), SPX_R8(k, 8), SPX_R8(k, 16), SPX_R8(k, 24), SPX_R8(r, 0), SPX_R8(r, 8), SPX_R8(r, 16),
        SPX_R8(r, 24)
      : "r"(tk), "r"(tr)
      : "memory");
}
#define SPX_T8(r, o) "+r"(r[o + 0]), "+r"(r[o + 1]), "+r"(r[o + 2]), "+r"(r[o + 3]), "+r"(r[o + 4]), "+r"(r[o + 5]), \
                     "+r"(r[o + 6]), "+r"(r[o + 7])
// Wait for this thread's TMEM loads; the registers are tied to the wait so that no use
// of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld_64(uint32_t (&k)[32], uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : SPX_T8(k, 0), SPX_T8(k, 8), SPX_T8(k, 16), SPX_T8(k, 24), SPX_T8(r, 0), SPX_T8(r, 8), SPX_T8(r, 16),
                 SPX_T8(r, 24)
               :
               : "memory");
}
#undef SPX_T8
#undef SPX_R8
#undef SPX_I8

// Instruction descriptor: D f16, A/B f16, A K-major, B MN-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (0u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) | ((128u >> 3) << 17) |
                            ((128u >> 4) << 24);
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
// ------------------------------------------------------------------ configuration ---
template <int RK, int RV, int MT>
struct Cfg {
  static_assert(MT % 2 == 0, "M-tile n uses accumulator n & 1 == mt & 1 only for an even tile count");
  static constexpr int TB = MT * 128;                  // tokens per block
  static constexpr int CK = TB * RK;                   // INT8 key codes
  static constexpr int CV = RV * TB;                   // INT8 value codes (value-tile layout)
  static constexpr int BK = RK * FD * 2;               // FP16 key basis
  static constexpr int BV = RV * FD * 2;               // FP16 value basis
  static constexpr int QP = FD * 2 + 16;               // padded query row pitch (conflict-free reads)
  static constexpr int QB = 8 * QP;                    // query rows (up to 8 heads)
  // ring A (keys: converters) and ring B (values, queries: consumers and epilogue)
  static constexpr int A_CK = 0, A_BK = CK, STAGE_A = CK + BK;
  static constexpr int B_CV = 0, B_BV = CV, B_Q = CV + BV, STAGE_B = B_Q + QB;
  static constexpr int OFF_RA = 0;
  static constexpr int OFF_RB = OFF_RA + STAGES * STAGE_A;
  // one M-tile of FP16 key codes: per K-step of 16 codes a [2 k-chunks][16 groups][8 rows]
  // [16 B] block; K-step blocks 4096 + 64 bytes apart, so that the converters' two stores
  // of a token's halves fall into different banks
  static constexpr int KSTR = 128 * 16 * 2 + 64;
  static constexpr int ATILE = ((RK / 16) * KSTR + 127) / 128 * 128;
  static constexpr int OFF_A = OFF_RB + STAGES * STAGE_B;   // [NA] x ATILE
  static constexpr int OFF_B = OFF_A + NA * ATILE;     // [2] x [16 n-chunks][RK rows][16 B]
  // consumer -> epilogue partials, double-buffered: m [8][8], l [8][8], v_lat [8 warps][8 heads][RVP]
  static constexpr int RVP = RV + 4;                   // padded rank pitch (conflict-free both ways)
  static constexpr int PART = NCW * 8 * 4 * 2 + NCW * 8 * RVP * 4;
  static constexpr int OFF_P = OFF_B + 2 * BK;
  static constexpr int OFF_BVP = OFF_P + 2 * PART;     // value basis, rows padded to QP bytes
  static constexpr int OFF_VL = OFF_BVP + RV * QP;     // combined v_lat [8][RV]
  static constexpr int OFF_ML = OFF_VL + 8 * RV * 4;   // per head (l_j, a_old, a_new, -) [8][4]
  static constexpr int OFF_ST = OFF_ML + 8 * 4 * 4;    // running (m, l) per unit of the item [GMAX][8][2]
  static constexpr int OFF_BAR = OFF_ST + GMAX * 8 * 2 * 4;
  // barriers: fullA[S], fullB[S], bslot[2], accf[2], acce[2], pready[2], pfree[2], aready[NA]
  static constexpr int NBAR = 2 * STAGES + NA + 10;
  static constexpr int OFF_TM = OFF_BAR + NBAR * 8;    // TMEM base address, abort flag
  static constexpr int BYTES = OFF_TM + 16;
  static_assert(STAGE_A % 128 == 0 && STAGE_B % 128 == 0 && OFF_A % 128 == 0 && OFF_BAR % 8 == 0, "alignment");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

// Eight 16-bit values of the input type -> eight f16 (bf16 input: exact for magnitudes the
// f16 range holds; bases are orthonormal rows, queries are O(1)).
template <bool BF>
__device__ __forceinline__ uint32_t to_h2(uint32_t w) {
  if (!BF) return w;
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
  return pack_f2(lo, hi);
}
template <bool BF>
__device__ __forceinline__ uint4 to_h8(uint4 v) {
  return BF ? make_uint4(to_h2<BF>(v.x), to_h2<BF>(v.y), to_h2<BF>(v.z), to_h2<BF>(v.w)) : v;
}

template <int RK, int RV, int MT, bool BF>
__global__ void __launch_bounds__(NT, 1) cold_fast_kernel(DecodeParams p, Items I) {
  using C = Cfg<RK, RV, MT>;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int nrep = p.nrep;
  const uint32_t bar0 = smem_u32(sm + C::OFF_BAR);
  const uint32_t b_fullA = bar0, b_fullB = bar0 + 8 * STAGES;
  const uint32_t b_bslot = bar0 + 16 * STAGES, b_accf = b_bslot + 16, b_acce = b_accf + 16, b_pready = b_acce + 16,
                 b_pfree = b_pready + 16;
  const uint32_t b_aready = b_pfree + 16;   // A tile (and, for the first, the B tile) converted
  uint32_t* tm_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_TM);
  Abort ab{reinterpret_cast<volatile int*>(sm + C::OFF_TM + 4), reinterpret_cast<int*>(p.ws) - 64};

  if (w == 0) {
    tmem_alloc(smem_u32(tm_slot), 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(b_fullA + 8 * s, 1);
      mbar_init(b_fullB + 8 * s, 1);
    }
    for (int a = 0; a < NA; ++a) mbar_init(b_aready + 8 * a, NCV);
    for (int b = 0; b < 2; ++b) {
      mbar_init(b_bslot + 8 * b, 2);   // one commit per MMA-issue lane
      mbar_init(b_accf + 8 * b, 1);
      mbar_init(b_acce + 8 * b, NCW);
      mbar_init(b_pready + 8 * b, NCW);
      mbar_init(b_pfree + 8 * b, 1);
    }
    *ab.flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tm_slot;

  Seq sq;
  sq.x = blockIdx.x;
  if (sq.valid(I)) sq.load_item(I);
  const uint64_t stream_policy = l2_evict_first_policy();

  if (w >= NCW + NPW) {
    // ============================================================== epilogue warps ===
    // combine the consumer warps' partials, expand v_lat through B_V, merge into the
    // unit's running (m, l, o); thread 384 also streams ring B (values, queries).
    setmaxnreg_dec<80>();
    const int et = tid - ET0, ew = et >> 5;
    Seq sqB = sq;   // ring-B copies run STAGES iterations ahead
    int issuedB = 0;
    auto issueB = [&]() {
      const int s = issuedB % STAGES;
      const int64_t unit = sqB.unit();
      const int64_t slot = unit * p.NBc + sqB.j();
      const int64_t lb = unit / p.H, gg = unit % p.H;
      uint8_t* st = sm + C::OFF_RB + s * C::STAGE_B;
      const uint32_t bar = b_fullB + 8 * s;
      mbar_expect_tx(bar, C::CV + C::BV + nrep * FD * 2);
      bulk_g2s_hint(smem_u32(st + C::B_CV), p.cv + slot * C::CV, C::CV, bar, stream_policy);
      bulk_g2s_hint(smem_u32(st + C::B_BV), reinterpret_cast<const uint8_t*>(p.bv) + slot * C::BV, C::BV, bar,
                    stream_policy);
      const uint8_t* q = reinterpret_cast<const uint8_t*>(p.q) + ((lb * p.Hq) + gg * nrep) * FD * 2;
      for (int h = 0; h < nrep; ++h) bulk_g2s(smem_u32(st + C::B_Q + h * C::QP), q + h * FD * 2, FD * 2, bar);
      ++issuedB;
      sqB.next(I);
    };
    if (et == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int k = 0; k < STAGES && sqB.valid(I); ++k) issueB();
    }
    __syncwarp();
    float* sVL = reinterpret_cast<float*>(sm + C::OFF_VL);
    float* sML = reinterpret_cast<float*>(sm + C::OFF_ML);
    float* sST = reinterpret_cast<float*>(sm + C::OFF_ST);
    const uint32_t bvp_u = smem_u32(sm + C::OFF_BVP);
    const bool hl = g < nrep;
    int it = 0;
    for (; sq.valid(I); sq.next(I), ++it) {
      const int s = it % STAGES, b2 = it & 1;
      const uint8_t* st = sm + C::OFF_RB + s * C::STAGE_B;
      const int64_t unit = sq.unit();
      const bool first_j = sq.jj == 0, last_j = sq.jj == sq.jn - 1;
      const float vscale = __ldg(p.sv + unit * p.NBc + sq.j());
      float* rec = p.ws + (unit * p.nparts + (sq.j0 / I.JR)) * (int64_t)nrep * (FD + 4);
      float2 oold[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        oold[q] = make_float2(0.f, 0.f);
        if (!first_j && hl)
          oold[q] = *reinterpret_cast<const float2*>(rec + g * (FD + 4) + 4 + 8 * (4 * ew + q) + 2 * t);
      }
      waitw(b_fullB + 8 * s, (uint32_t)((it / STAGES) & 1), ab);
      waitw(b_pready + 8 * b2, (uint32_t)((it / 2) & 1), ab);
      const float* sM = reinterpret_cast<const float*>(sm + C::OFF_P + b2 * C::PART);
      const float* sL = sM + NCW * 8;
      const float* sV = sL + NCW * 8;
      // ---- combine the warps: v_lat[h][r], block (m_j, l_j); merge into the state ----
      for (int e = et; e < nrep * RV; e += NEP) {
        const int h = e / RV, r = e - h * RV;
        float M = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < NCW; ++ww) M = fmaxf(M, sM[ww * 8 + h]);
        float v = 0.f, l = 0.f;
#pragma unroll
        for (int ww = 0; ww < NCW; ++ww) {
          const float wt = exp2f(sM[ww * 8 + h] - M);
          v = fmaf(sV[(ww * 8 + h) * C::RVP + r], wt, v);
          l = fmaf(sL[ww * 8 + h], wt, l);
        }
        sVL[h * RV + r] = v;
        if (r == 0) {
          float* stt = sST + (sq.uu * 8 + h) * 2;
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
      __syncwarp();
      // ---- value basis -> rows padded to QP bytes (conflict-free ldmatrix.trans) -----
      {
        const uint4* src = reinterpret_cast<const uint4*>(st + C::B_BV);
        for (int e = et; e < RV * 16; e += NEP)
          *reinterpret_cast<uint4*>(sm + C::OFF_BVP + (e >> 4) * C::QP + (e & 15) * 16) = to_h8<BF>(src[e]);
      }
      named_sync(BAR_EPI, NEP);
      // partials and stage s are consumed: hand them back, refill the stage
      if (et == 0) {
        mbar_arrive(b_pfree + 8 * b2);
        if (sqB.valid(I) && !*ab.flag) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issueB();
        }
      }
      __syncwarp();
      // ---- expand once through B_V (mma.sync), merge with the running o --------------
      // o_j[h][d] = l_j * vscale * sum_r (v_lat[h][r] / l_j) B_V[r][d]: the normalised
      // v_lat is a weighted mean of INT8 codes (|.| <= 127), safe as an f16 operand.
      {
        const float lj = hl ? sML[4 * g] : 1.f;
        const float inv_l = hl ? 1.f / lj : 0.f;
        uint32_t va[RV / 16][2];
#pragma unroll
        for (int ks = 0; ks < RV / 16; ++ks) {
          const float2 x0 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t);
          const float2 x1 = *reinterpret_cast<const float2*>(sVL + g * RV + 16 * ks + 2 * t + 8);
          va[ks][0] = hl ? pack_f2(x0.x * inv_l, x0.y * inv_l) : 0u;
          va[ks][1] = hl ? pack_f2(x1.x * inv_l, x1.y * inv_l) : 0u;
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
            ldsm_x4_t(bvp_u + R * C::QP + n * 16, b00, b01, b10, b11);
            mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
            mma16816(o, va[1][0], 0u, va[1][1], 0u, b10, b11);
          } else {
            const int R = 8 * (mi & 1) + rr;
            uint32_t b00, b01;
            ldsm_x2_t(bvp_u + R * C::QP + n * 16, b00, b01);
            mma16816(o, va[0][0], 0u, va[0][1], 0u, b00, b01);
          }
          if (hl)
            *reinterpret_cast<float2*>(rec + g * (FD + 4) + 4 + 8 * n + 2 * t) =
                make_float2(fmaf(oold[q].x, ao, o[0] * an), fmaf(oold[q].y, ao, o[1] * an));
        }
        if (last_j && et < nrep) {
          const float* stt = sST + (sq.uu * 8 + et) * 2;
          rec[et * (FD + 4) + 0] = stt[0] * LN2;
          rec[et * (FD + 4) + 1] = stt[1];
        }
      }
      __syncwarp();
      named_sync(BAR_EPI, NEP);
    }
    if (et == 0 && *ab.flag) drain<STAGES>(b_fullB, issuedB);
    __syncwarp();
  } else if (w >= NCW) {
    // ============================================================= converter warps ===
    // Warps 8-9 convert: key basis -> B tile, key codes -> FP16 A tiles; each warp
    // arrives on aready[slot] once its share of a tile is written.  Lane 0 of warps 10
    // and 11 issue the MMAs (and warp 11 the ring-A copies), so conversion never waits
    // behind an issue.
    setmaxnreg_dec<80>();
    const int wc = w - NCW;
    if (wc < NCV) {
      const int ct = tid - PT0;   // 0 .. 32 NCV - 1
      int it = 0;
      for (; sq.valid(I); sq.next(I), ++it) {
        const int s = it % STAGES;
        const uint8_t* st = sm + C::OFF_RA + s * C::STAGE_A;
        bool ok = waitw(b_fullA + 8 * s, (uint32_t)((it / STAGES) & 1), ab);
        // key basis [RK][16 chunks] -> B tile [16 n-chunks][RK rows] (conflict-free walk)
        const int bs = it & 1;
        if (it >= 2) ok = waitw(b_bslot + 8 * bs, (uint32_t)((it / 2 - 1) & 1), ab) && ok;
        if (ok) {
          const uint4* srcb = reinterpret_cast<const uint4*>(st + C::A_BK);
          uint4* dstb = reinterpret_cast<uint4*>(sm + C::OFF_B + bs * C::BK);
          for (int idx = ct; idx < RK * 16; idx += NCV * 32) {
            const int l = idx & 31, W = idx >> 5, a = l & 7, b = l >> 3;
            int k, nc;
            if (RK == 32) {
              nc = a + 8 * (W & 1);
              k = 8 * b + ((a + (W >> 1)) & 7);
            } else {
              nc = a + 8 * (b >> 1);
              k = 8 * (b & 1) + ((a + W) & 7);
            }
            dstb[nc * RK + k] = to_h8<BF>(srcb[k * 16 + nc]);
          }
        }
        // key codes -> FP16 A tiles, one M-tile at a time
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt) {
          const int64_t n = (int64_t)it * MT + mt;
          // A slot n & 1 is free once M-tile n - 2, the last one read from it, is done:
          // that is the completion of accumulator n & 1's previous phase
          const int as = (int)(n & 1);
          bool oka = ok;
          if (n >= 2) oka = waitw(b_accf + 8 * as, (uint32_t)(((n - 2) / 2) & 1), ab) && oka;
          if (oka) {
            const uint8_t* src = st + C::A_CK + mt * 128 * RK;
            uint8_t* dst = sm + C::OFF_A + as * C::ATILE;
            for (int e = ct; e < 128 * (RK / 16); e += NCV * 32) {
              const int tau = RK == 32 ? (e >> 1) : e, hf = RK == 32 ? (e & 1) : 0;
              const uint4 v = *reinterpret_cast<const uint4*>(src + tau * RK + hf * 16);
              uint4 o0, o1;
              i8x4_to_h2(v.x, o0.x, o0.y);
              i8x4_to_h2(v.y, o0.z, o0.w);
              i8x4_to_h2(v.z, o1.x, o1.y);
              i8x4_to_h2(v.w, o1.z, o1.w);
              uint8_t* d = dst + hf * C::KSTR + (tau >> 3) * 128 + (tau & 7) * 16;
              *reinterpret_cast<uint4*>(d) = o0;
              *reinterpret_cast<uint4*>(d + 2048) = o1;
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(b_aready + 8 * as);
          __syncwarp();
        }
      }
    } else {
      // ---- MMA issuers: lane 0 of warp 10 (even M-tiles, accumulator 0) and of warp 11
      //      (odd M-tiles, accumulator 1, and the ring-A copies), so that each
      //      accumulator cycles independently of the other -----------------------------
      const int par = wc - NCV;
      if (lane == 0) {
        const uint32_t sA_u = smem_u32(sm + C::OFF_A), sB_u = smem_u32(sm + C::OFF_B);
        Seq sqA = sq;   // ring-A copies run STAGES iterations ahead
        int issuedA = 0;
        auto issueA = [&]() {
          const int s = issuedA % STAGES;
          const int64_t slot = (int64_t)sqA.unit() * p.NBc + sqA.j();
          uint8_t* st = sm + C::OFF_RA + s * C::STAGE_A;
          const uint32_t bar = b_fullA + 8 * s;
          mbar_expect_tx(bar, C::CK + C::BK);
          bulk_g2s_hint(smem_u32(st + C::A_CK), p.ck + slot * C::CK, C::CK, bar, stream_policy);
          bulk_g2s_hint(smem_u32(st + C::A_BK), reinterpret_cast<const uint8_t*>(p.bk) + slot * C::BK, C::BK, bar,
                        stream_policy);
          ++issuedA;
          sqA.next(I);
        };
        if (par == 1) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          for (int k = 0; k < STAGES && sqA.valid(I); ++k) issueA();
        }
        // descriptors of A slot 0 / B slot 0, k-step 0; other slots and k-steps differ
        // only in the start-address field (address >> 4 in the low 14 bits)
        const uint64_t ad0 = umma_desc(sA_u, 2048, 128), bd0 = umma_desc(sB_u, 128, RK * 16);
        int it = 0;
        int64_t n_issued = 0;   // M-tiles handed to the tensor core
        for (; sq.valid(I); sq.next(I), ++it) {
          const int bs = it & 1;
#pragma unroll 1
          for (int mt = par; mt < MT; mt += 2) {
            const int64_t n = (int64_t)it * MT + mt;
            const int as = (int)(n & 1), b = as;
            // test both barriers at once; sleep on whichever is not there yet
            bool ra, re;
            mbar_test2(b_aready + 8 * as, (uint32_t)((n / 2) & 1), b_acce + 8 * b, (uint32_t)((n / 2 + 1) & 1), ra, re);
            re = re || n < 2;   // (n / 2 + 1) & 1 == (n / 2 - 1) & 1: the previous release of buffer b
            bool ok = ra || wait1(b_aready + 8 * as, (uint32_t)((n / 2) & 1), ab);
            if (!re) ok = wait1(b_acce + 8 * b, (uint32_t)((n / 2 - 1) & 1), ab) && ok;
            if (ok && !*ab.flag) {
              tc_fence_after();
              const uint32_t d = tbase + 256u + 128u * (uint32_t)b;
              const uint64_t ad = ad0 + (uint64_t)((as * C::ATILE) >> 4), bd = bd0 + (uint64_t)((bs * C::BK) >> 4);
#pragma unroll
              for (int ks = 0; ks < RK / 16; ++ks)
                umma_f16(d, ad + (uint64_t)((ks * C::KSTR) >> 4), bd + (uint64_t)((ks * 256) >> 4), ks > 0 ? 1u : 0u);
              umma_commit(b_accf + 8 * b);
              if (mt >= MT - 2) umma_commit(b_bslot + 8 * bs);
              n_issued = n + 1;
            }
          }
          // every converter warp has finished with stage it % STAGES of ring A (the last
          // M-tile, converted last, is ready): refill it
          if (par == 1 && sqA.valid(I) && !*ab.flag) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issueA();
          }
        }
        if (*ab.flag) {
          if (par == 1) drain<STAGES>(b_fullA, issuedA);
          if (n_issued > 0) {   // the last MMAs handed to the tensor core
            const int64_t n = n_issued - 1;
            const uint64_t t0 = gtimer();
            while (!mbar_try_wait_sleep(b_accf + 8 * (n & 1), (uint32_t)((n / 2) & 1)) && gtimer() - t0 < kWaitNs) {
            }
          }
        }
      }
      __syncwarp();
    }
  } else {
    // ============================================================== consumer warps ===
    setmaxnreg_inc<176>();
    const int lane_off = 32 * (w & 3) + 16 * (w >> 2);
    const uint4* rope_tab = reinterpret_cast<const uint4*>(p.rope);
    const bool live0 = 2 * t < nrep, live1 = 2 * t + 1 < nrep, hl = g < nrep;
    const uint32_t lrow = (uint32_t)lane_off << 16;
    int prev_j = -1;
    Seq sqn = sq;   // one iteration ahead: scale prefetch
    float ks_next = sq.valid(I) ? __ldg(p.sk + (int64_t)sq.unit() * p.NBc + sq.j()) : 0.f;
    sqn.next(I);
    int it = 0;
    for (; sq.valid(I); sq.next(I), ++it) {
      const int s = it % STAGES, b2 = it & 1;
      const uint8_t* st = sm + C::OFF_RB + s * C::STAGE_B;
      const int j = sq.j();
      // ---- RoPE rows of block j for this warp's 16-lane slabs -> TMEM --------------
      if (j != prev_j) {
        prev_j = j;
        uint32_t r[MT][32];
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const int tile16 = (i * 128 + lane_off) >> 4;
          const uint4* src = rope_tab + (((int64_t)j * (C::TB / 16) + tile16) * 32 + lane) * 8;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 v = __ldg(src + q);
            r[i][4 * q] = v.x;
            r[i][4 * q + 1] = v.y;
            r[i][4 * q + 2] = v.z;
            r[i][4 * q + 3] = v.w;
          }
        }
#pragma unroll
        for (int i = 0; i < MT; ++i) tmem_st_rope(tbase + lrow + (uint32_t)(64 * i), r[i]);
      }
      const float kscale = ks_next * p.scale * LOG2E;
      if (sqn.valid(I)) ks_next = __ldg(p.sk + (int64_t)sqn.unit() * p.NBc + sqn.j());
      sqn.next(I);
      waitw(b_fullB + 8 * s, (uint32_t)((it / STAGES) & 1), ab);
      // ---- query fragments: dims 16k + 4t .. +3 of head g ----------------------------
      uint2 qf[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
      {
        const uint2 v = hl ? *reinterpret_cast<const uint2*>(st + C::B_Q + g * C::QP + 32 * k + 8 * t) : make_uint2(0u, 0u);
        qf[k] = make_uint2(to_h2<BF>(v.x), to_h2<BF>(v.y));
      }
      // ---- scores: K~ from TMEM (next M-tile loading while this one computes) --------
      float sc[MT][4];
      uint32_t kr[2][32], ro[2][32];
      {
        const int64_t n = (int64_t)it * MT;
        waitw(b_accf + 8 * (int)(n & 1), (uint32_t)((n / 2) & 1), ab);
        tc_fence_after();
        tmem_ld_k_rope_nowait(tbase + lrow + 256u + 128u * (uint32_t)(n & 1), tbase + lrow, kr[0], ro[0]);
        tmem_wait_ld_64(kr[0], ro[0]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_acce + 8 * (int)(n & 1));
        __syncwarp();
      }
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int cb = i & 1, nb = cb ^ 1;
        const int64_t n1 = (int64_t)it * MT + i + 1;
        if (i + 1 < MT) {
          waitw(b_accf + 8 * (int)(n1 & 1), (uint32_t)((n1 / 2) & 1), ab);
          tc_fence_after();
          tmem_ld_k_rope_nowait(tbase + lrow + 256u + 128u * (uint32_t)(n1 & 1), tbase + lrow + (uint32_t)(64 * (i + 1)),
                                kr[nb], ro[nb]);
        }
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t k1[4], k2[4];   // [2hh + c]
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int hh = q >> 1, c = q & 1;
            const __half2 x = u2h(kr[cb][4 * k + q]), y = u2h(kr[cb][16 + 4 * k + q]);
            const __half2 cs = u2h(ro[cb][8 * k + 4 * c + 2 * hh]), sn = u2h(ro[cb][8 * k + 4 * c + 2 * hh + 1]);
            k1[q] = h2u(__hfma2(cs, x, __hneg2(__hmul2(sn, y))));   // c K1 - s K2
            k2[q] = h2u(__hfma2(cs, y, __hmul2(sn, x)));            // s K1 + c K2
          }
          mma16816(sa, k1[0], k1[2], k1[1], k1[3], qf[k].x, qf[k].y);
          mma16816(sb, k2[0], k2[2], k2[1], k2[3], qf[k + 4].x, qf[k + 4].y);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[i][e] = sa[e] + sb[e];
        if (i + 1 < MT) {
          tmem_wait_ld_64(kr[nb], ro[nb]);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(b_acce + 8 * (int)(n1 & 1));
          __syncwarp();
        }
      }
      // ---- per-warp softmax over its tokens (log2 domain) ------------------------------
      // raw scores times kscale are the logits in log2 units; the max of the scaled
      // logits is max*k for k >= 0 and min*k for k < 0
      const bool kpos = kscale >= 0.f;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < MT; ++i) {
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
      float l0 = 0.f, l1 = 0.f;
      float vacc[RV / 16][4];
#pragma unroll
      for (int rt = 0; rt < RV / 16; ++rt) vacc[rt][0] = vacc[rt][1] = vacc[rt][2] = vacc[rt][3] = 0.f;
      const uint32_t cV_u = smem_u32(st + C::B_CV);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        sc[i][0] = live0 ? exp2f(fmaf(sc[i][0], kscale, -mx0)) : 0.f;
        sc[i][2] = live0 ? exp2f(fmaf(sc[i][2], kscale, -mx0)) : 0.f;
        sc[i][1] = live1 ? exp2f(fmaf(sc[i][1], kscale, -mx1)) : 0.f;
        sc[i][3] = live1 ? exp2f(fmaf(sc[i][3], kscale, -mx1)) : 0.f;
        l0 += sc[i][0] + sc[i][2];
        l1 += sc[i][1] + sc[i][3];
        // ---- v_lat[rank][head] += codes_V^T . P  (one ldmatrix per 16 tokens) ---------
        const uint32_t b0 = movm_t(pack_f2(sc[i][0], sc[i][1]));
        const uint32_t b1 = movm_t(pack_f2(sc[i][2], sc[i][3]));
        const int tt = (i * 128 + lane_off) >> 4;
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
      // ---- hand (m, l, v_lat) of this warp to the epilogue ----------------------------
      if (it >= 2) waitw(b_pfree + 8 * b2, (uint32_t)((it / 2 - 1) & 1), ab);
      float* sM = reinterpret_cast<float*>(sm + C::OFF_P + b2 * C::PART);
      float* sL = sM + NCW * 8;
      float* sV = sL + NCW * 8;
      if (g == 0) {
        sM[w * 8 + 2 * t] = mx0;
        sM[w * 8 + 2 * t + 1] = mx1;
        sL[w * 8 + 2 * t] = l0;
        sL[w * 8 + 2 * t + 1] = l1;
      }
#pragma unroll
      for (int rt = 0; rt < RV / 16; ++rt) {
        float* base = sV + (w * 8 + 2 * t) * C::RVP + rt * 16 + g;   // [warp][head][rank]
        base[0] = vacc[rt][0];
        base[C::RVP] = vacc[rt][1];
        base[8] = vacc[rt][2];
        base[C::RVP + 8] = vacc[rt][3];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(b_pready + 8 * b2);
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, 512);
}

// RoPE words of every cold block, in the per-lane register order the consumers store to
// TMEM: [block][token/16][lane][32 words]; word 4e + 2hh + cc of lane (g, t) is the f16
// pair (f0, f0 + 1) of cos (cc = 0) or sin (cc = 1) for token 16*tile + g + 8hh, with
// f0 = 16*(e/2) + 4t + 2*(e%2).  First-half table entries (tied or distance RoPE).
__global__ void __launch_bounds__(128) rope_pack_kernel(DecodeParams p) {
  const int j = blockIdx.x, tile = blockIdx.y * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (tile >= p.Tb / 16) return;
  const int g = lane >> 2, t = lane & 3;
  uint32_t r[32];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int64_t pos = p.bpos[j] + tile * 16 + g + 8 * hh;
    int64_t a = p.mode == SPX_ROPE_DISTANCE ? (p.qpos - pos > 0 ? p.qpos - pos : 0) : pos;
    a = a < 0 ? 0 : (a >= p.rope_len ? p.rope_len - 1 : a);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int f0 = 16 * (e >> 1) + 4 * t + 2 * (e & 1);
      const float2 c = *reinterpret_cast<const float2*>(p.cosT + a * FD + f0);
      const float2 s = *reinterpret_cast<const float2*>(p.sinT + a * FD + f0);
      r[4 * e + 2 * hh + 0] = pack_f2(c.x, c.y);
      r[4 * e + 2 * hh + 1] = pack_f2(s.x, s.y);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(p.rope) + (((int64_t)j * (p.Tb / 16) + tile) * 32 + lane) * 8;
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
}

template <int RK, int RV, int MT>
int launch(DecodeParams p, cudaStream_t st) {
  using C = Cfg<RK, RV, MT>;
  const int units = p.L * p.B * p.H;
  const Plan pl = plan(units, p.nblk, num_sms());
  dim3 rg(p.nblk, (p.Tb / 16 + 3) / 4);
  rope_pack_kernel<<<rg, 128, 0, st>>>(p);
  int rc = launch_status("rope_pack_kernel");
  if (rc != SPX_OK) return rc;
  const Items items{pl.G, pl.JR, pl.ngroups, pl.nitems, p.nblk, units};
  if (p.dtype == SPX_BF16) {
    cudaFuncSetAttribute(cold_fast_kernel<RK, RV, MT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
    cold_fast_kernel<RK, RV, MT, true><<<pl.grid, NT, C::BYTES, st>>>(p, items);
  } else {
    cudaFuncSetAttribute(cold_fast_kernel<RK, RV, MT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
    cold_fast_kernel<RK, RV, MT, false><<<pl.grid, NT, C::BYTES, st>>>(p, items);
  }
  return launch_status("cold_fast_kernel");
}

}  // namespace fastk

bool decode_fast_supported(const DecodeParams& p) {
  if (p.nblk <= 0 || p.D != 128 || (p.dtype != SPX_F16 && p.dtype != SPX_BF16) || p.mask != nullptr) return false;
  if (!(p.tied || p.mode == SPX_ROPE_DISTANCE)) return false;
  if (!(p.RK == 16 || p.RK == 32) || !(p.RV == 16 || p.RV == 32)) return false;
  if (!(p.Tb == 256 || p.Tb == 512)) return false;
  if (!(p.nrep == 1 || p.nrep == 2 || p.nrep == 4 || p.nrep == 8)) return false;
  if (reinterpret_cast<uintptr_t>(p.q) & 15) return false;
  return true;
}

int decode_fast_ncold(const DecodeParams& p) {
  return fastk::plan(p.L * p.B * p.H, p.nblk, fastk::num_sms()).nranges;
}

template <int RK, int RV>
static int launch_mt(const DecodeParams& p, cudaStream_t st) {
  return p.Tb == 256 ? fastk::launch<RK, RV, 2>(p, st) : fastk::launch<RK, RV, 4>(p, st);
}

int decode_fast_cold(const DecodeParams& p, cudaStream_t st) {
  if (p.RK == 32) return p.RV == 32 ? launch_mt<32, 32>(p, st) : launch_mt<32, 16>(p, st);
  return p.RV == 32 ? launch_mt<16, 32>(p, st) : launch_mt<16, 16>(p, st);
}

}  // namespace spx
