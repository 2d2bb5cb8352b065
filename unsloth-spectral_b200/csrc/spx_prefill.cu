// Multi-query (prefill) attention over the compressed cache: the reference's
// integration.py:292-346 path (get_kv, RoPE of the keys at their positions, softmax
// attention with the caller's additive mask), without materialising K, V or the score
// matrix.
//
// Flash-attention structure.  A CTA of 8 warps owns 128 query rows of one (sequence, KV
// head): QT = 128 / n_rep consecutive queries of each of the n_rep query heads that read
// the head, 16 rows (one head, 16 queries) per warp.  It walks the keys in cache order in
// tiles of 64 tokens -- the cold blocks, then the hot tier -- and for each tile
//   1. rebuilds the key and value tiles from their INT8 codes and the block's bases on
//      the tensor cores (mma.sync m16n8k16, f32 accumulate: K~ = scale_K codes_K B_K,
//      V~ = scale_V codes_V B_V), rotates the keys at their absolute positions in f32
//      (the half-split rotation with the first half of the tables, as the reference's
//      apply_rope), and stores both tiles in shared memory in the cache dtype (hot-tier
//      tiles are copied and rotated instead);
//   2. scores its 16 x 64 tile S = Q K~^T, scales it, applies the causal rule (key position
//      > query position -> -inf) and the additive mask, and runs the online softmax
//      (float32 row max / sum, exp2), then O += P V~ with P in the cache dtype.
// A warp's two query rows per thread are lanes g and g + 8 of the m16 fragments; the row
// statistics are reduced over the four threads of a quad.  Tiles whose first key lies
// past every query of the CTA are skipped when the causal rule is on.
//
// The rebuilt tiles cost 2 * 64 * 128 * (R_K + R_V) FLOPs per tile against
// 4 * 128 * 64 * 128 for the attention itself (about 12 % at R = 16).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "spx_common.cuh"
#include "spx_prefill.cuh"
#include "spx_sm100.cuh"

namespace spx {
namespace pfa {

using namespace sm100;

constexpr int NT = 256;      // 8 warps
constexpr int ROWS = 128;    // query rows per CTA
constexpr int KT = 64;       // keys per tile
constexpr int PITCH = 136;   // shared row pitch (elements) of the K / V / basis tiles
constexpr int RMAX = 64;
constexpr float LOG2E_F = 1.4426950408889634f;

using Params = PrefillParams;

template <typename T>
struct Ty;
template <>
struct Ty<__half> {
  __device__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static uint32_t pack_i8(int a, int b) {
    __half2 h = __halves2half2(__int2half_rn(a), __int2half_rn(b));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static float2 unpack(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <>
struct Ty<__nv_bfloat16> {
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static uint32_t pack_i8(int a, int b) { return pack((float)a, (float)b); }
  __device__ static float2 unpack(uint32_t w) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w);
    return __bfloat1622float2(h);
  }
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// shared memory (bytes)
constexpr int SZ_TILE = KT * PITCH * 2;     // K or V tile
constexpr int SZ_BASIS = RMAX * PITCH * 2;  // one basis
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + SZ_TILE;
constexpr int OFF_BK = OFF_V + SZ_TILE;
constexpr int OFF_BV = OFF_BK + SZ_BASIS;
constexpr int OFF_CK = OFF_BV + SZ_BASIS;   // key codes of the tile [64][RK]
constexpr int OFF_CV = OFF_CK + KT * RMAX;  // value codes of the tile (value-tile layout)
constexpr int OFF_POS = OFF_CV + KT * RMAX; // key positions [64] int64
constexpr int SMEM = OFF_POS + KT * 8;

__device__ __forceinline__ uint32_t ld32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <typename T>
__global__ void __launch_bounds__(NT, 1) prefill_kernel(Params p) {
  using Y = Ty<T>;
  extern __shared__ __align__(16) uint8_t sm[];
  T* sK = reinterpret_cast<T*>(sm + OFF_K);
  T* sV = reinterpret_cast<T*>(sm + OFF_V);
  T* sBK = reinterpret_cast<T*>(sm + OFF_BK);
  T* sBV = reinterpret_cast<T*>(sm + OFF_BV);
  int8_t* cK = reinterpret_cast<int8_t*>(sm + OFF_CK);
  int8_t* cV = reinterpret_cast<int8_t*>(sm + OFF_CV);
  int64_t* sPos = reinterpret_cast<int64_t*>(sm + OFF_POS);
  __shared__ float s_scale[2];
  __shared__ long long s_qmax[8];

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
  const int h = blockIdx.y % p.H, b = blockIdx.y / p.H;
  const int64_t u = (int64_t)b * p.H + h;   // (sequence, KV head)
  // this warp's 16 rows: query head hq, queries qa .. qa + 15; this thread's rows qa+g, qa+g+8
  const int row0 = 16 * w;
  const int hq = h * p.nrep + row0 / p.QT;
  const int qa = blockIdx.x * p.QT + row0 % p.QT;
  const int qr[2] = {qa + g, qa + g + 8};
  const bool qv[2] = {qr[0] < p.qlen, qr[1] < p.qlen};
  long long qp[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) qp[i] = qv[i] ? (long long)p.qpos[qr[i]] : -1;
  {
    long long mq = qp[0] > qp[1] ? qp[0] : qp[1];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long x = __shfl_xor_sync(0xffffffffu, mq, o);
      mq = x > mq ? x : mq;
    }
    if (lane == 0) s_qmax[w] = mq;
  }
  // query fragments (A operand, 8 k-steps of 16 dims)
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)(b * p.Hq + hq) * p.qlen * 128;
  uint32_t qf[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d0 = 16 * ks + 2 * tig;
    qf[ks][0] = qv[0] ? ld32(qb + (int64_t)qr[0] * 128 + d0) : 0u;
    qf[ks][1] = qv[1] ? ld32(qb + (int64_t)qr[1] * 128 + d0) : 0u;
    qf[ks][2] = qv[0] ? ld32(qb + (int64_t)qr[0] * 128 + d0 + 8) : 0u;
    qf[ks][3] = qv[1] ? ld32(qb + (int64_t)qr[1] * 128 + d0 + 8) : 0u;
  }
  __syncthreads();
  long long qmax = s_qmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) qmax = s_qmax[i] > qmax ? s_qmax[i] : qmax;

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E_F;
  const int tpb = p.T / KT;   // tiles per block
  const int ncold = p.nblk * tpb, nhot = (p.hot + KT - 1) / KT;
  const int mt = w & 3, hh = w >> 2;   // rebuild roles: keys 16 mt .., dims 32 hh .. (+64)
  const uint32_t sK0 = smem_u32(sK), sV0 = smem_u32(sV), sBK0 = smem_u32(sBK), sBV0 = smem_u32(sBV);
  int cur = -1;

  for (int it = 0; it < ncold + nhot; ++it) {
    const bool cold = it < ncold;
    const int j = cold ? it / tpb : 0;
    const int t0 = cold ? (it - j * tpb) * KT : (it - ncold) * KT;
    const int nk = cold ? KT : min(KT, p.hot - t0);
    if (p.causal && cold && p.bpos[j] + t0 > qmax) continue;   // every key of the tile is in the future
    const int64_t kbase = cold ? (int64_t)j * p.T + t0 : (int64_t)p.nblk * p.T + t0;   // cache-order index
    // ---- stage: bases (on a new block), codes, positions
    if (cold) {
      const int64_t ub = u * p.nbc + j;
      if (j != cur) {
        const T* bk = reinterpret_cast<const T*>(p.bk) + ub * p.RK * 128;
        const T* bv = reinterpret_cast<const T*>(p.bv) + ub * p.RV * 128;
        for (int e = tid; e < p.RK * 16; e += NT)
          *reinterpret_cast<uint4*>(sBK + (e >> 4) * PITCH + (e & 15) * 8) =
              *reinterpret_cast<const uint4*>(bk + (e >> 4) * 128 + (e & 15) * 8);
        for (int e = tid; e < p.RV * 16; e += NT)
          *reinterpret_cast<uint4*>(sBV + (e >> 4) * PITCH + (e & 15) * 8) =
              *reinterpret_cast<const uint4*>(bv + (e >> 4) * 128 + (e & 15) * 8);
        if (tid == 0) {
          s_scale[0] = p.sk[ub];
          s_scale[1] = p.sv[ub];
        }
        cur = j;
      }
      const int8_t* ck = p.ck + (ub * p.T + t0) * p.RK;
      const int8_t* cv = p.cv + ub * (int64_t)p.RV * p.T + (int64_t)(t0 >> 4) * p.RV * 16;
      if (tid < 4 * p.RK) *reinterpret_cast<uint4*>(cK + 16 * tid) = *reinterpret_cast<const uint4*>(ck + 16 * tid);
      if (tid < 4 * p.RV) *reinterpret_cast<uint4*>(cV + 16 * tid) = *reinterpret_cast<const uint4*>(cv + 16 * tid);
      if (tid < KT) sPos[tid] = p.bpos[j] + t0 + tid;
    } else if (tid < KT) {
      sPos[tid] = tid < nk ? p.hpos[t0 + tid] : 0;
    }
    __syncthreads();
    // ---- rebuild the key and value tiles
    if (cold) {
      float acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      for (int ks = 0; ks < p.RK / 16; ++ks) {
        const int8_t* r0 = cK + (16 * mt + g) * p.RK + 16 * ks + 2 * tig;
        const int8_t* r1 = r0 + 8 * p.RK;
        const uint32_t a[4] = {Y::pack_i8(r0[0], r0[1]), Y::pack_i8(r1[0], r1[1]), Y::pack_i8(r0[8], r0[9]),
                               Y::pack_i8(r1[8], r1[9])};
#pragma unroll
        for (int nb = 0; nb < 4; ++nb) {
          const int nd = (nb < 2 ? 0 : 64) + 32 * hh + 16 * (nb & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sBK0 + ((16 * ks + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH + nd + (lane >> 4) * 8) * 2,
                    b0, b1, b2, b3);
          Y::mma(acc[2 * nb], a, b0, b1);
          Y::mma(acc[2 * nb + 1], a, b2, b3);
        }
      }
      // scale, rotate (pairs d, d + 64 are acc[i], acc[i + 4]) and store
      const float sc = s_scale[0];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int key = 16 * mt + g + 8 * rr;
        long long kp = sPos[key];
        kp = kp < 0 ? 0 : (kp >= p.rope_len ? p.rope_len - 1 : kp);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = 32 * hh + 8 * i + 2 * tig;
          const float2 c = *reinterpret_cast<const float2*>(p.cosT + kp * 128 + d);
          const float2 sn = *reinterpret_cast<const float2*>(p.sinT + kp * 128 + d);
          const float x0 = sc * acc[i][2 * rr], x1 = sc * acc[i][2 * rr + 1];
          const float y0 = sc * acc[i + 4][2 * rr], y1 = sc * acc[i + 4][2 * rr + 1];
          *reinterpret_cast<uint32_t*>(sK + key * PITCH + d) = Y::pack(x0 * c.x - y0 * sn.x, x1 * c.y - y1 * sn.y);
          *reinterpret_cast<uint32_t*>(sK + key * PITCH + d + 64) =
              Y::pack(y0 * c.x + x0 * sn.x, y1 * c.y + x1 * sn.y);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      const int tA = t0 + 16 * mt + g, tB = tA + 8, vb = (t0 >> 4) * p.RV * 16;
      for (int ks = 0; ks < p.RV / 16; ++ks) {
        const int r = 16 * ks + 2 * tig;
        const uint32_t a[4] = {
            Y::pack_i8(cV[vtile_offset(r, tA, p.RV) - vb], cV[vtile_offset(r + 1, tA, p.RV) - vb]),
            Y::pack_i8(cV[vtile_offset(r, tB, p.RV) - vb], cV[vtile_offset(r + 1, tB, p.RV) - vb]),
            Y::pack_i8(cV[vtile_offset(r + 8, tA, p.RV) - vb], cV[vtile_offset(r + 9, tA, p.RV) - vb]),
            Y::pack_i8(cV[vtile_offset(r + 8, tB, p.RV) - vb], cV[vtile_offset(r + 9, tB, p.RV) - vb])};
#pragma unroll
        for (int nb = 0; nb < 4; ++nb) {
          const int nd = (nb < 2 ? 0 : 64) + 32 * hh + 16 * (nb & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sBV0 + ((16 * ks + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH + nd + (lane >> 4) * 8) * 2,
                    b0, b1, b2, b3);
          Y::mma(acc[2 * nb], a, b0, b1);
          Y::mma(acc[2 * nb + 1], a, b2, b3);
        }
      }
      const float sv = s_scale[1];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int key = 16 * mt + g + 8 * rr;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int d = (i < 4 ? 0 : 64) + 32 * hh + 8 * (i & 3) + 2 * tig;
          *reinterpret_cast<uint32_t*>(sV + key * PITCH + d) = Y::pack(sv * acc[i][2 * rr], sv * acc[i][2 * rr + 1]);
        }
      }
    } else {
      // hot tier: copy, rotating the keys at their positions; keys past hot_len are zero
      const T* hk = reinterpret_cast<const T*>(p.hk) + (u * p.HC + t0) * 128;
      const T* hv = reinterpret_cast<const T*>(p.hv) + (u * p.HC + t0) * 128;
      for (int e = tid; e < KT * 32; e += NT) {
        const int key = e >> 5, d = 2 * (e & 31);
        uint32_t klo = 0u, khi = 0u, vlo = 0u, vhi = 0u;
        if (key < nk) {
          long long kp = sPos[key];
          kp = kp < 0 ? 0 : (kp >= p.rope_len ? p.rope_len - 1 : kp);
          const float2 x = Y::unpack(ld32(hk + key * 128 + d)), y = Y::unpack(ld32(hk + key * 128 + d + 64));
          const float2 c = *reinterpret_cast<const float2*>(p.cosT + kp * 128 + d);
          const float2 sn = *reinterpret_cast<const float2*>(p.sinT + kp * 128 + d);
          klo = Y::pack(x.x * c.x - y.x * sn.x, x.y * c.y - y.y * sn.y);
          khi = Y::pack(y.x * c.x + x.x * sn.x, y.y * c.y + x.y * sn.y);
          vlo = ld32(hv + key * 128 + d);
          vhi = ld32(hv + key * 128 + d + 64);
        }
        *reinterpret_cast<uint32_t*>(sK + key * PITCH + d) = klo;
        *reinterpret_cast<uint32_t*>(sK + key * PITCH + d + 64) = khi;
        *reinterpret_cast<uint32_t*>(sV + key * PITCH + d) = vlo;
        *reinterpret_cast<uint32_t*>(sV + key * PITCH + d + 64) = vhi;
      }
    }
    __syncthreads();
    // ---- scores of this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK0 + ((16 * np + (lane & 7) + (lane >> 4) * 8) * PITCH + 16 * ks + ((lane >> 3) & 1) * 8) * 2, b0, b1,
                b2, b3);
        Y::mma(s[2 * np], qf[ks], b0, b1);
        Y::mma(s[2 * np + 1], qf[ks], b2, b3);
      }
    }
    // scale (log2 units), causal rule, additive mask; online softmax
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kk = 8 * n + 2 * tig + (e & 1), rr = e >> 1;
        float x = s[n][e] * sl2;
        const bool keep = kk < nk && !(p.causal && (long long)sPos[kk] > qp[rr]);
        if (!keep) {
          x = -INFINITY;
        } else if (p.mask != nullptr && qv[rr]) {
          const int64_t mo = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)qr[rr] * p.msq + kbase + kk;
          const float mv = p.mask_f32 ? reinterpret_cast<const float*>(p.mask)[mo]
                                      : Y::unpack((uint32_t)reinterpret_cast<const uint16_t*>(p.mask)[mo]).x;
          x += mv * LOG2E_F;
        }
        s[n][e] = x;
        mx[rr] = fmaxf(mx[rr], x);
      }
    float corr[2], mu[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
      const float mn = fmaxf(m[rr], mx[rr]);
      mu[rr] = mn == -INFINITY ? 0.f : mn;
      corr[rr] = exp2f(m[rr] - mu[rr]);
      m[rr] = mn;
      l[rr] *= corr[rr];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = exp2f(s[n][e] - mu[e >> 1]);
        s[n][e] = pv;
        l[e >> 1] += pv;
      }
    // ---- O += P V~
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {Y::pack(s[2 * kk][0], s[2 * kk][1]), Y::pack(s[2 * kk][2], s[2 * kk][3]),
                             Y::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]), Y::pack(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV0 + ((16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH + 16 * nd + (lane >> 4) * 8) * 2, b0,
                  b1, b2, b3);
        Y::mma(o[2 * nd], a, b0, b1);
        Y::mma(o[2 * nd + 1], a, b2, b3);
      }
    }
    __syncthreads();   // the tiles are rewritten by the next iteration
  }
  // ---- normalise and store
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
  }
  T* ob = reinterpret_cast<T*>(p.out) + (int64_t)(b * p.Hq + hq) * p.qlen * 128;
  const float i0 = 1.f / l[0], i1 = 1.f / l[1];
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = 8 * n + 2 * tig;
    if (qv[0]) *reinterpret_cast<uint32_t*>(ob + (int64_t)qr[0] * 128 + d) = Y::pack(o[n][0] * i0, o[n][1] * i0);
    if (qv[1]) *reinterpret_cast<uint32_t*>(ob + (int64_t)qr[1] * 128 + d) = Y::pack(o[n][2] * i1, o[n][3] * i1);
  }
}

}  // namespace pfa
}  // namespace spx

using namespace spx;

extern "C" {

int spx_prefill_attn(const spx_prefill_args* a, void* stream) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->head_dim == 128, SPX_ERR_UNSUPPORTED, "prefill attention needs head_dim 128, got %d", a->head_dim);
  SPX_REQUIRE(a->dtype == SPX_F16 || a->dtype == SPX_BF16, SPX_ERR_UNSUPPORTED, "prefill attention needs f16 or bf16");
  SPX_REQUIRE(a->batch >= 1 && a->num_kv_heads >= 1 && a->q_len >= 0, SPX_ERR_SHAPE, "bad batch / heads / q_len");
  SPX_REQUIRE(a->num_q_heads % a->num_kv_heads == 0, SPX_ERR_SHAPE, "num_q_heads must be a multiple of num_kv_heads");
  const int nrep = a->num_q_heads / a->num_kv_heads;
  SPX_REQUIRE(nrep == 1 || nrep == 2 || nrep == 4 || nrep == 8, SPX_ERR_UNSUPPORTED, "n_rep %d not in {1,2,4,8}", nrep);
  SPX_REQUIRE(a->num_blocks >= 0 && a->num_blocks <= a->block_capacity, SPX_ERR_SHAPE, "num_blocks outside [0, capacity]");
  SPX_REQUIRE(a->hot_len >= 0 && a->hot_len <= a->hot_capacity, SPX_ERR_SHAPE, "hot_len outside [0, hot_capacity]");
  SPX_REQUIRE(a->num_blocks > 0 || a->hot_len > 0, SPX_ERR_EMPTY, "Empty cache - no keys available");
  if (a->num_blocks > 0) {
    SPX_REQUIRE(a->block_size % 64 == 0 && a->block_size >= 64, SPX_ERR_UNSUPPORTED, "block_size must be a multiple of 64");
    SPX_REQUIRE(a->rank_k % 16 == 0 && a->rank_k >= 16 && a->rank_k <= 64 && a->rank_v % 16 == 0 && a->rank_v >= 16 &&
                    a->rank_v <= 64,
                SPX_ERR_UNSUPPORTED, "ranks must be 16, 32, 48 or 64");
    SPX_REQUIRE(a->codes_k && a->codes_v && a->scale_k && a->scale_v && a->basis_k && a->basis_v && a->block_pos,
                SPX_ERR_NULL, "cold-tier pointers are required when num_blocks > 0");
  }
  if (a->hot_len > 0) SPX_REQUIRE(a->hot_k && a->hot_v && a->hot_pos, SPX_ERR_NULL, "hot-tier pointers are required");
  SPX_REQUIRE(a->q && a->q_pos && a->out && a->cos_table && a->sin_table, SPX_ERR_NULL, "q, q_pos, out and tables are required");
  SPX_REQUIRE(a->rope_len >= 1, SPX_ERR_SHAPE, "rope_len must be positive");
  SPX_REQUIRE(!a->mask || a->mask_dtype == SPX_F32 || a->mask_dtype == a->dtype, SPX_ERR_UNSUPPORTED,
              "mask dtype must be f32 or the attention dtype");
  SPX_REQUIRE(aligned16(a->codes_k) && aligned16(a->codes_v) && aligned16(a->basis_k) && aligned16(a->basis_v) &&
                  (reinterpret_cast<uintptr_t>(a->q) & 3u) == 0 && (reinterpret_cast<uintptr_t>(a->out) & 3u) == 0 &&
                  (reinterpret_cast<uintptr_t>(a->hot_k) & 3u) == 0 && (reinterpret_cast<uintptr_t>(a->hot_v) & 3u) == 0 &&
                  (reinterpret_cast<uintptr_t>(a->cos_table) & 7u) == 0 && (reinterpret_cast<uintptr_t>(a->sin_table) & 7u) == 0,
              SPX_ERR_ALIGN, "codes and bases need 16-byte, q / out / hot tier 4-byte, tables 8-byte alignment");
  if (a->q_len == 0) return SPX_OK;
  pfa::Params p;
  p.B = a->batch;
  p.Hq = a->num_q_heads;
  p.H = a->num_kv_heads;
  p.nrep = nrep;
  p.QT = pfa::ROWS / nrep;
  p.qlen = a->q_len;
  p.T = a->block_size;
  p.nblk = a->num_blocks;
  p.nbc = a->block_capacity;
  p.RK = a->rank_k;
  p.RV = a->rank_v;
  p.hot = a->hot_len;
  p.HC = a->hot_capacity;
  p.causal = a->causal != 0;
  p.mask_f32 = a->mask_dtype == SPX_F32;
  p.rope_len = a->rope_len;
  p.scale = a->scale;
  p.q = a->q;
  p.qpos = a->q_pos;
  p.ck = a->codes_k;
  p.cv = a->codes_v;
  p.sk = a->scale_k;
  p.sv = a->scale_v;
  p.bk = a->basis_k;
  p.bv = a->basis_v;
  p.bpos = a->block_pos;
  p.hk = a->hot_k;
  p.hv = a->hot_v;
  p.hpos = a->hot_pos;
  p.cosT = a->cos_table;
  p.sinT = a->sin_table;
  p.mask = a->mask;
  p.msb = a->mask_stride_b;
  p.msh = a->mask_stride_h;
  p.msq = a->mask_stride_q;
  p.out = a->out;
  const dim3 grid((a->q_len + p.QT - 1) / p.QT, a->batch * a->num_kv_heads);
  SPX_REQUIRE(grid.y <= 65535u, SPX_ERR_SHAPE, "batch * num_kv_heads above 65535");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // SPX_PREFILL_PATH=tc selects the tcgen05 kernel (spx_prefill_tc.cu; blocks of a
  // multiple of 128 tokens); the default is the mma.sync kernel below, measured faster
  // (8.6 against 11.3 ms per layer at config 4's prompt: the tcgen05 kernel runs its tile
  // phases one after another on one CTA per SM)
  const char* path = getenv("SPX_PREFILL_PATH");
  const bool tc = path && strcmp(path, "tc") == 0 && prefill_tc_supported(a->block_size, a->num_blocks);
  if (tc) {
    SPX_REQUIRE(aligned16(a->q) && aligned16(a->out) && aligned16(a->cos_table) && aligned16(a->sin_table) &&
                    (a->hot_len == 0 || (aligned16(a->hot_k) && aligned16(a->hot_v))),
                SPX_ERR_ALIGN, "q, out, the tables and the hot tier need 16-byte alignment");
    return prefill_tc_launch(p, a->dtype, st);
  }
  if (a->dtype == SPX_F16) {
    cudaFuncSetAttribute(pfa::prefill_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, pfa::SMEM);
    pfa::prefill_kernel<__half><<<grid, pfa::NT, pfa::SMEM, st>>>(p);
  } else {
    cudaFuncSetAttribute(pfa::prefill_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, pfa::SMEM);
    pfa::prefill_kernel<__nv_bfloat16><<<grid, pfa::NT, pfa::SMEM, st>>>(p);
  }
  return launch_status("prefill_kernel");
}

}  // extern "C"
