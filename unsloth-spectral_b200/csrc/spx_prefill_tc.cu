// Multi-query (prefill) attention over the compressed cache on the 5th-generation tensor
// cores: the same computation as spx_prefill.cu's flash-attention loop (integration.py:
// 292-346: keys rotated at their cached positions with the first half of the tables,
// softmax(Q K^T * scale + mask) V), with every product on tcgen05 and the running
// accumulators in tensor memory.
//
// A CTA (8 warps, one per SM: 192 KB of shared memory, all 512 TMEM columns) owns 128
// query rows of one (sequence, KV head) -- 128 / n_rep queries of each of the n_rep query
// heads that read the head -- and walks the keys in cache order in tiles of 128 tokens.
// Per tile:
//   1. cold tiles: the INT8 codes of the tile's keys and values are converted to 16-bit
//      A operands (thread = key) and the block's bases staged as MN-major B operands;
//      tcgen05 rebuilds K~ = codes_K B_K and V~ = codes_V B_V into TMEM (f32, columns
//      0-127 / 128-255); warps w and w + 4 (TMEM lane = key) each take half of the
//      dimensions: scale K~, rotate it in f32 at the keys' positions and store it as the
//      K-major B operand of the scores, and scale V~ into the B operand of the value
//      product.  Hot tiles are copied and rotated instead.
//   2. S = Q K~^T (M = 128 rows, N = 128 keys, K = 128 dims) into TMEM columns 256-383.
//   3. Thread = (query row, half of the tile's keys; warps w and w + 4 share a row, the
//      halves' maxima and sums exchanged through shared memory): scale (log2 units),
//      causal rule (one threshold per row on a cold tile), additive mask, row maximum; the running maximum used for the exponentials moves
//      only when the row's maximum exceeds it by more than 8 (then the row of O in TMEM
//      and the row sum are rescaled), so P = exp2(s - m_used) <= 256 fits the 16-bit
//      operand; P is stored as the K-major A operand of the value product.
//   4. O += P V~ (N = 128 dims, K = 128 keys) into TMEM columns 384-511.
// Finally thread = row reads O, divides by the row sum and writes the output.
//
// All operands use the no-swizzle canonical layouts: 16-byte core rows of 8 elements,
// an operand [rows][K] stored as (k / 8) * 2048 + row * 16 + (k % 8) * 2 (K-major: LBO
// 2048 along K, SBO 128 along rows), the bases [R][128] as (dim / 8) * 16 R + rank * 16 +
// (dim % 8) * 2 (MN-major: LBO 128, SBO 16 R).  One thread issues every MMA; completion
// is an mbarrier every thread waits on, bounded in time (an expired wait stops further
// MMAs and the CTA writes NaN).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "spx_common.cuh"
#include "spx_prefill.cuh"
#include "spx_sm100.cuh"

namespace spx {
namespace ptc {

using namespace sm100;

constexpr int NT = 256;
constexpr int KT = 128;          // keys per tile
constexpr int RMAX = 64;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float RESCALE = 8.f;   // log2 headroom of P before the running maximum moves

// shared memory (bytes)
constexpr int SZ_OP = 128 * 128 * 2;          // a 128 x 128 16-bit operand
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + SZ_OP;          // K~ (B of the scores)
constexpr int OFF_V = OFF_K + SZ_OP;          // V~ (B of the value product)
constexpr int OFF_P = OFF_V + SZ_OP;          // P (A of the value product)
constexpr int OFF_CK = OFF_P + SZ_OP;         // key codes, A [128 keys][RK]
constexpr int OFF_CV = OFF_CK + 128 * RMAX * 2;
constexpr int OFF_BK = OFF_CV + 128 * RMAX * 2;   // key basis, B MN-major
constexpr int OFF_BV = OFF_BK + RMAX * 128 * 2;
constexpr int OFF_RAW = OFF_BV + RMAX * 128 * 2;  // value codes of the tile, as stored
constexpr int OFF_POS = OFF_RAW + 128 * RMAX;     // key positions [128] int64
constexpr int SMEM = OFF_POS + 128 * 8;
static_assert(SMEM <= 227 * 1024, "shared memory");

using Params = PrefillParams;

template <typename T>
struct Ty;
template <>
struct Ty<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static float2 unpack(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  __device__ static float lo(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <>
struct Ty<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static float2 unpack(uint32_t w) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w);
    return __bfloat1622float2(h);
  }
  __device__ static float lo(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
};

__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int a_mn, int b_mn) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(128 >> 3) << 17) | ((128u >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int u = 0; u < 32; ++u) v[u] = __uint_as_float(r[u]);
}
__device__ __forceinline__ void tst32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity))
    if (gtimer() - t0 > kWaitNs) return false;
  return true;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <typename T>
__global__ void __launch_bounds__(NT, 1) prefill_tc_kernel(Params p) {
  using Y = Ty<T>;
  constexpr uint32_t ID_RB = idesc(Ty<T>::kFmt, 0, 1);   // codes (K-major) x basis (MN-major)
  constexpr uint32_t ID_S = idesc(Ty<T>::kFmt, 0, 0);    // Q (K-major) x K~ (K-major)
  constexpr uint32_t ID_PV = idesc(Ty<T>::kFmt, 0, 1);   // P (K-major) x V~ (MN-major)
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ int sbad;
  __shared__ float s_scale[2];
  __shared__ long long s_qmax[8];
  __shared__ float s_pair[2][128];   // per-row partial maxima / sums of the two halves
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, quad = w & 3;
  const int h = blockIdx.y % p.H, b = blockIdx.y / p.H;
  const int64_t u = (int64_t)b * p.H + h;
  const uint32_t s0 = smem_u32(sm);
  const uint32_t sQ = s0 + OFF_Q, sKo = s0 + OFF_K, sVo = s0 + OFF_V, sPo = s0 + OFF_P;
  const uint32_t sCK = s0 + OFF_CK, sCV = s0 + OFF_CV, sBK = s0 + OFF_BK, sBV = s0 + OFF_BV;
  uint8_t* raw = sm + OFF_RAW;
  int64_t* sPos = reinterpret_cast<int64_t*>(sm + OFF_POS);
  const uint32_t barA = smem_u32(&bar);

  if (w == 0) {
    tmem_alloc(smem_u32(&tslot), 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(barA, 1);
    sbad = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // this thread's query row (warps 0-3; TMEM lane = row): head hq, query qi
  // this thread's query row (TMEM lane = row; warps w and w + 4 share the row, each taking
  // half of its keys / dims): head hq, query qi
  const int row = tid & 127, hlf = tid >> 7;
  const int hq = h * p.nrep + row / p.QT;
  const int qi = blockIdx.x * p.QT + row % p.QT;
  const bool rowv = qi < p.qlen;
  const long long qp = rowv ? (long long)p.qpos[qi] : -1;
  {
    long long mq = qp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long x = __shfl_xor_sync(0xffffffffu, mq, o);
      mq = x > mq ? x : mq;
    }
    if (lane == 0) s_qmax[w] = mq;
  }
  // queries -> K-major A operand: row r, 8-dim chunk c at c * 2048 + r * 16
  {
    const T* qg = reinterpret_cast<const T*>(p.q);
    for (int e = tid; e < 2048; e += NT) {
      const int rr = e & 127, c = e >> 7;
      const int qr = blockIdx.x * p.QT + rr % p.QT, hr = h * p.nrep + rr / p.QT;
      const uint32_t dst = sQ + c * 2048 + rr * 16;
      if (qr < p.qlen)
        cp_async16(dst, qg + (((int64_t)b * p.Hq + hr) * p.qlen + qr) * 128 + c * 8);
      else
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tslot;
  const uint32_t tq = tbase + ((uint32_t)(32 * quad) << 16);   // this warp's TMEM lanes
  long long qmax = s_qmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) qmax = s_qmax[i] > qmax ? s_qmax[i] : qmax;

  float m_used = -INFINITY, lsum = 0.f;
  bool o_init = false, bad = false;
  uint32_t ph = 0;
  const float sl2 = p.scale * LOG2E_F;
  const int tpb = p.T / KT;
  const int ncold = p.nblk * tpb, nhot = (p.hot + KT - 1) / KT;
  int cur = -1;
  auto wait_mma = [&]() {
    if (!bad && !bar_wait(barA, ph)) sbad = 1;
    ph ^= 1u;
    __syncthreads();
    bad = sbad != 0;
    tc_fence_after();
  };
  auto sync_ops = [&]() {   // shared-memory operands written by threads -> visible to the MMA
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };

  for (int it = 0; it < ncold + nhot; ++it) {
    const bool cold = it < ncold;
    const int j = cold ? it / tpb : 0;
    const int t0 = cold ? (it - j * tpb) * KT : (it - ncold) * KT;
    const int nk = cold ? KT : min(KT, p.hot - t0);
    if (p.causal && cold && p.bpos[j] + t0 > qmax) continue;   // every key of the tile lies in the future
    const int64_t kbase = cold ? (int64_t)j * p.T + t0 : (int64_t)p.nblk * p.T + t0;
    // ---- stage the tile's operands ------------------------------------------------
    if (cold) {
      const int64_t ub = u * p.nbc + j;
      if (j != cur) {
        // bases -> MN-major B: (rank r, dim d) at (d / 8) * 16 R + r * 16 + (d % 8) * 2
        const T* bk = reinterpret_cast<const T*>(p.bk) + ub * p.RK * 128;
        const T* bv = reinterpret_cast<const T*>(p.bv) + ub * p.RV * 128;
        for (int e = tid; e < p.RK * 16; e += NT) {
          const int rr = e >> 4, o = e & 15;
          *reinterpret_cast<uint4*>(sm + OFF_BK + o * (p.RK * 16) + rr * 16) =
              *reinterpret_cast<const uint4*>(bk + rr * 128 + o * 8);
        }
        for (int e = tid; e < p.RV * 16; e += NT) {
          const int rr = e >> 4, o = e & 15;
          *reinterpret_cast<uint4*>(sm + OFF_BV + o * (p.RV * 16) + rr * 16) =
              *reinterpret_cast<const uint4*>(bv + rr * 128 + o * 8);
        }
        if (tid == 0) {
          s_scale[0] = p.sk[ub];
          s_scale[1] = p.sv[ub];
        }
        cur = j;
      }
      if (tid < KT) {
        // key codes of key tid -> K-major A: (key, rank r) at (r / 8) * 2048 + key * 16 + (r % 8) * 2
        const int8_t* src = p.ck + (ub * p.T + t0 + tid) * p.RK;
        for (int c16 = 0; c16 < p.RK / 16; ++c16) {
          const uint4 v = *reinterpret_cast<const uint4*>(src + 16 * c16);
          const uint32_t wds[4] = {v.x, v.y, v.z, v.w};
          uint32_t hw[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int x0 = (int8_t)(wds[q] & 0xff), x1 = (int8_t)((wds[q] >> 8) & 0xff);
            const int x2 = (int8_t)((wds[q] >> 16) & 0xff), x3 = (int8_t)(wds[q] >> 24);
            hw[2 * q] = Y::pack((float)x0, (float)x1);
            hw[2 * q + 1] = Y::pack((float)x2, (float)x3);
          }
          *reinterpret_cast<uint4*>(sm + OFF_CK + (2 * c16) * 2048 + tid * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(sm + OFF_CK + (2 * c16 + 1) * 2048 + tid * 16) =
              make_uint4(hw[4], hw[5], hw[6], hw[7]);
        }
        sPos[tid] = p.bpos[j] + t0 + tid;
      } else {
        // the tile's value codes as stored: 8 value tiles of 16 tokens, contiguous
        const int8_t* src = p.cv + ub * (int64_t)p.RV * p.T + (int64_t)(t0 >> 4) * p.RV * 16;
        for (int e = tid - 128; e < 8 * p.RV; e += 128)
          *reinterpret_cast<uint4*>(raw + 16 * e) = *reinterpret_cast<const uint4*>(src + 16 * e);
      }
      __syncthreads();
      if (tid >= KT) {
        // value codes of key tid - 128 -> K-major A (gathered from the value-tile layout)
        const int key = tid - KT, tg = t0 + key, vb = (t0 >> 4) * p.RV * 16;
        for (int c = 0; c < p.RV / 8; ++c) {
          uint32_t hw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int r0 = 8 * c + 2 * q;
            hw[q] = Y::pack((float)(int8_t)raw[vtile_offset(r0, tg, p.RV) - vb],
                            (float)(int8_t)raw[vtile_offset(r0 + 1, tg, p.RV) - vb]);
          }
          *reinterpret_cast<uint4*>(sm + OFF_CV + c * 2048 + key * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
      }
    } else {
      // hot tile: keys rotated at their positions (thread = key), values copied
      const int key = tid & 127;
      if (tid < KT) {
        long long kp = key < nk ? (long long)p.hpos[t0 + key] : 0;
        sPos[key] = kp;
        kp = kp < 0 ? 0 : (kp >= p.rope_len ? p.rope_len - 1 : kp);
        const T* rowk = reinterpret_cast<const T*>(p.hk) + (u * p.HC + t0 + key) * 128;
#pragma unroll 2
        for (int i = 0; i < 8; ++i) {
          uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
          if (key < nk) {
            const uint4 x = *reinterpret_cast<const uint4*>(rowk + 8 * i);
            const uint4 y = *reinterpret_cast<const uint4*>(rowk + 64 + 8 * i);
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
            uint32_t lw[4], hw[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int d = 8 * i + 2 * q;
              const float2 c = *reinterpret_cast<const float2*>(p.cosT + kp * 128 + d);
              const float2 sn = *reinterpret_cast<const float2*>(p.sinT + kp * 128 + d);
              const float2 a = Y::unpack(xs[q]), bb = Y::unpack(ys[q]);
              lw[q] = Y::pack(a.x * c.x - bb.x * sn.x, a.y * c.y - bb.y * sn.y);
              hw[q] = Y::pack(bb.x * c.x + a.x * sn.x, bb.y * c.y + a.y * sn.y);
            }
            lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          }
          *reinterpret_cast<uint4*>(sm + OFF_K + i * 2048 + key * 16) = lo;
          *reinterpret_cast<uint4*>(sm + OFF_K + (8 + i) * 2048 + key * 16) = hi;
        }
      } else {
        const T* rowv_ = reinterpret_cast<const T*>(p.hv) + (u * p.HC + t0 + key) * 128;
#pragma unroll 4
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(sm + OFF_V + c * 2048 + key * 16) =
              key < nk ? *reinterpret_cast<const uint4*>(rowv_ + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    sync_ops();
    if (cold) {
      // the key's table rows (half hlf of the first-half dims), loaded while the tensor
      // core rebuilds the tile
      const int key = 32 * quad + lane;   // TMEM lane = key
      float4 c4[8], s4[8];
      {
        long long kp = sPos[key];
        kp = kp < 0 ? 0 : (kp >= p.rope_len ? p.rope_len - 1 : kp);
        const float4* crow = reinterpret_cast<const float4*>(p.cosT + kp * 128 + 32 * hlf);
        const float4* srow = reinterpret_cast<const float4*>(p.sinT + kp * 128 + 32 * hlf);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          c4[i] = __ldg(crow + i);
          s4[i] = __ldg(srow + i);
        }
      }
      // ---- K~ and V~ on the tensor cores (TMEM columns 0 and 128) ---------------------
      if (tid == 0 && !bad) {
        for (int ks = 0; ks < p.RK / 16; ++ks)
          umma(tbase, umma_desc(sCK + ks * 4096, 2048, 128), umma_desc(sBK + ks * 256, 128, p.RK * 16), ID_RB,
               ks > 0 ? 1u : 0u);
        for (int ks = 0; ks < p.RV / 16; ++ks)
          umma(tbase + 128, umma_desc(sCV + ks * 4096, 2048, 128), umma_desc(sBV + ks * 256, 128, p.RV * 16), ID_RB,
               ks > 0 ? 1u : 0u);
        umma_commit(barA);
      }
      wait_mma();
      {
        // K~ half hlf (dims 32 hlf .. and 64 + 32 hlf ..): scale, rotate at the key's
        // position (f32), store as the K-major B operand
        const float sc = s_scale[0];
        const int hf = hlf;
        float x[32], y[32];
        tld32(tq + 32 * hf, x);
        tld32(tq + 64 + 32 * hf, y);
        const float* cf = reinterpret_cast<const float*>(c4);
        const float* sf = reinterpret_cast<const float*>(s4);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t lw[4], hw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 8 * q + 2 * e;
            const float x0 = sc * x[i], x1 = sc * x[i + 1], y0 = sc * y[i], y1 = sc * y[i + 1];
            lw[e] = Y::pack(x0 * cf[i] - y0 * sf[i], x1 * cf[i + 1] - y1 * sf[i + 1]);
            hw[e] = Y::pack(y0 * cf[i] + x0 * sf[i], y1 * cf[i + 1] + x1 * sf[i + 1]);
          }
          const int ch = 4 * hf + q;   // 8-dim chunk of the first half
          *reinterpret_cast<uint4*>(sm + OFF_K + ch * 2048 + key * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          *reinterpret_cast<uint4*>(sm + OFF_K + (8 + ch) * 2048 + key * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
        // V~ dims 64 hlf .. + 63: scale and store as the MN-major B operand (same layout)
        const float sv = s_scale[1];
#pragma unroll 1
        for (int c32 = 2 * hlf; c32 < 2 * hlf + 2; ++c32) {
          float v[32];
          tld32(tq + 128 + 32 * c32, v);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(sm + OFF_V + (4 * c32 + q) * 2048 + key * 16) =
                make_uint4(Y::pack(sv * v[8 * q], sv * v[8 * q + 1]), Y::pack(sv * v[8 * q + 2], sv * v[8 * q + 3]),
                           Y::pack(sv * v[8 * q + 4], sv * v[8 * q + 5]), Y::pack(sv * v[8 * q + 6], sv * v[8 * q + 7]));
        }
      }
      sync_ops();
    }
    // ---- S = Q K~^T (TMEM columns 256) -------------------------------------------------
    if (tid == 0 && !bad) {
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks)
        umma(tbase + 256, umma_desc(sQ + ks * 4096, 2048, 128), umma_desc(sKo + ks * 4096, 2048, 128), ID_S,
             ks > 0 ? 1u : 0u);
      umma_commit(barA);
    }
    wait_mma();
    // ---- online softmax: thread = (query row, half of the tile's keys) ---------------------
    {
      // keys kk <= kmax are kept: the causal rule on a cold tile (consecutive positions) is
      // one threshold per row; hot tiles and additive masks take the general path
      int kmax = nk - 1;
      if (p.causal && cold) {
        const long long lim = qp - (p.bpos[j] + t0);
        kmax = lim < 0 ? -1 : (lim >= nk ? nk - 1 : (int)lim);
      }
      const bool general = (p.causal && !cold) || (p.mask != nullptr);
      auto logit = [&](float sraw, int kk) -> float {
        if (!general) return kk <= kmax ? sraw * sl2 : -INFINITY;
        float x = sraw * sl2;
        const bool keep = kk < nk && !(p.causal && (long long)sPos[kk] > qp);
        if (!keep) return -INFINITY;
        if (p.mask != nullptr && rowv) {
          const int64_t mo = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)qi * p.msq + kbase + kk;
          const float mv = p.mask_f32 ? reinterpret_cast<const float*>(p.mask)[mo]
                                      : Y::lo(reinterpret_cast<const uint16_t*>(p.mask)[mo]);
          x += mv * LOG2E_F;
        }
        return x;
      };
      // the half's 64 logits, kept in registers across the two passes
      float lg[64];
      {
        float v[32];
        tld32(tq + 256 + 64 * hlf, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) lg[e] = logit(v[e], 64 * hlf + e);
        tld32(tq + 256 + 64 * hlf + 32, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) lg[32 + e] = logit(v[e], 64 * hlf + 32 + e);
      }
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        m0 = fmaxf(m0, lg[e]);
        m1 = fmaxf(m1, lg[e + 1]);
      }
      s_pair[hlf][row] = fmaxf(m0, m1);
      __syncthreads();
      const float mx = fmaxf(s_pair[0][row], s_pair[1][row]);
      if (mx > m_used + RESCALE) {   // also true for the first finite maximum; same in both halves
        const float corr = exp2f(m_used - mx);   // 0 while m_used is -inf
        lsum *= corr;
        if (o_init) {
#pragma unroll 1
          for (int c32 = 2 * hlf; c32 < 2 * hlf + 2; ++c32) {
            float o[32];
            tld32(tq + 384 + 32 * c32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= corr;
            tst32(tq + 384 + 32 * c32, o);
          }
        }
        m_used = mx;
      }
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {   // 8-key chunks 8 hlf + q of the A operand
        uint32_t pw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = exp2f(lg[8 * q + 2 * e] - mu), p1 = exp2f(lg[8 * q + 2 * e + 1] - mu);
          l0 += p0;
          l1 += p1;
          pw[e] = Y::pack(p0, p1);
        }
        *reinterpret_cast<uint4*>(sm + OFF_P + (8 * hlf + q) * 2048 + row * 16) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
      }
      lsum += l0 + l1;   // this half's share of the row sum
    }
    sync_ops();
    // ---- O += P V~ (TMEM columns 384) ---------------------------------------------------
    if (tid == 0 && !bad) {
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks)
        umma(tbase + 384, umma_desc(sPo + ks * 4096, 2048, 128), umma_desc(sVo + ks * 256, 128, 2048), ID_PV,
             (o_init || ks > 0) ? 1u : 0u);
      umma_commit(barA);
    }
    o_init = true;
    wait_mma();
  }
  // ---- normalise and store: the two halves' row sums added, thread = (row, half of dims)
  s_pair[hlf][row] = lsum;
  __syncthreads();
  {
    const float inv = 1.f / (s_pair[0][row] + s_pair[1][row]);
    T* og = reinterpret_cast<T*>(p.out) + (((int64_t)b * p.Hq + hq) * p.qlen + qi) * 128;
#pragma unroll 1
    for (int c32 = 2 * hlf; c32 < 2 * hlf + 2; ++c32) {
      float o[32];
      tld32(tq + 384 + 32 * c32, o);
      if (rowv) {
        const float nanv = __int_as_float(0x7fc00000);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t hw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 8 * q + 2 * e;
            const float a = (o_init && !bad) ? o[i] * inv : nanv, c = (o_init && !bad) ? o[i + 1] * inv : nanv;
            hw[e] = Y::pack(a, c);
          }
          *reinterpret_cast<uint4*>(og + 32 * c32 + 8 * q) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, 512);
}

}  // namespace ptc

bool prefill_tc_supported(int block_size, int num_blocks) { return num_blocks == 0 || block_size % 128 == 0; }

int prefill_tc_launch(const PrefillParams& p, int dtype, cudaStream_t st) {
  const dim3 grid((p.qlen + p.QT - 1) / p.QT, p.B * p.H);
  if (dtype == SPX_F16) {
    cudaFuncSetAttribute(ptc::prefill_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, ptc::SMEM);
    ptc::prefill_tc_kernel<__half><<<grid, ptc::NT, ptc::SMEM, st>>>(p);
  } else {
    cudaFuncSetAttribute(ptc::prefill_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         ptc::SMEM);
    ptc::prefill_tc_kernel<__nv_bfloat16><<<grid, ptc::NT, ptc::SMEM, st>>>(p);
  }
  return launch_status("prefill_tc_kernel");
}

}  // namespace spx
