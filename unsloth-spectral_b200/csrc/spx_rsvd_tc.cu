// Tensor-core sketch and power-iteration GEMMs of the batched rSVD (sm_100a):
//   mode 0:  Y = M X      (M: [m][128] 16-bit, X: f32 [128][r], Y: f32 [m][r])
//   mode 1:  Z = M^T Y    (Y: f32 [m][r], Z: f32 [128][r])
// the products of unsloth_spectral/rsvd.py:99-140 (Y = A @ Omega, A^T @ Q, A @ Z).
//
// One CTA (4 warps) per matrix.  M streams through shared memory in 128 x 128 tiles
// (cp.async, double-buffered).  Every tile is stored as 16-byte chunks at
//     chunk (row t, column chunk c) -> c * 2048 + (t / 8) * 128 + (t % 8) * 16,
// which is at once the K-major no-swizzle UMMA layout of M (LBO 2048 along K, SBO 128
// along M) for mode 0 and the MN-major layout of M^T (LBO 128 along K = tokens, SBO 2048
// along M = dims) for mode 1.  The f32 right-hand side is split into 16-bit hi + lo
// halves (x = hi + lo to ~2^-22 relative; hi in the input's type, so that A and B have
// one type as kind::f16 requires) and both halves accumulate into one f32 TMEM
// accumulator: the products keep float32 accuracy at tensor-core speed.  X in mode 0 is
// scaled by a power of two so that its largest magnitude is below 1 (no 16-bit overflow
// for any sketch); mode 1's right-hand side is an orthonormal basis.
//
// Lane 0 of warp 0 issues tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = r rounded up
// to 16, K = 16) and commits each tile to an mbarrier that frees its shared-memory stage.
// The epilogue reads the accumulator with tcgen05.ld.32x32b (thread = row).  Waits are
// bounded in time; an expired wait makes the CTA write NaN, never hang.
#include <math.h>

#include "spx_common.cuh"
#include "spx_rsvd.cuh"

namespace spx {
namespace rtc {

constexpr int NTH = 128;
constexpr int TILE = 128 * 128 * 2;   // one 128 x 128 16-bit tile of M
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(cnt) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity), "n"(100000)
      : "memory");
  return ok != 0;
}
// Bounded wait: false once kWaitNs passed without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity) {
  if (mbar_test(a, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_test(a, parity))
    if (gtimer() - t0 > kWaitNs) return false;
  return true;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Shared-memory matrix descriptor, no swizzle: start address, leading-dimension byte
// offset (along K) and stride-dimension byte offset (along M or N), all >> 4; version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 16 consecutive f32 columns of this warp's 32 lanes (one row per thread), with the wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int u = 0; u < 16; ++u) v[u] = __uint_as_float(r[u]);
}

template <typename T>
struct Half16;
template <>
struct Half16<__half> {
  static constexpr uint32_t kFmt = 0;   // instruction-descriptor operand format: f16
  __device__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ static float back(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <>
struct Half16<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;   // bf16
  __device__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ static float back(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
};

// Instruction descriptor: D f32, A/B 16-bit of format fmt, A K-major (mode 0) or MN-major
// (mode 1), B K-major, N = rp, M = 128.
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int a_mn, int rp) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)(rp >> 3) << 17) |
         ((128u >> 4) << 24);
}

template <typename T, int MODE>
__global__ void __launch_bounds__(NTH) tc_gemm_kernel(const T* __restrict__ M, int64_t ms,
                                                      const float* __restrict__ X, float* __restrict__ Y, int m,
                                                      int r, int rp, int ncols) {
  using H = Half16<T>;
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int NBS = MODE == 0 ? 1 : 2;   // right-hand-side stages
  const int nt = m / 128;                  // 128-row tiles of M
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int64_t mat = blockIdx.x;
  const T* Mi = M + mat * ms;
  const float* Xi = X + mat * (int64_t)(MODE == 0 ? 128 : m) * r;
  float* Yi = Y + mat * (int64_t)(MODE == 0 ? m : 128) * r;
  const int LB = rp * 16;    // K-direction stride of the right-hand side (8 K rows x rp / 8 groups)
  const int BSZ = 128 * rp * 2;
  uint8_t* sA = sm;
  uint8_t* sB = sm + 2 * TILE;
  const uint32_t bar = smem_u32(sB + NBS * 2 * BSZ);   // mdone[2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sB + NBS * 2 * BSZ + 16);
  float* sred = reinterpret_cast<float*>(sB + NBS * 2 * BSZ + 32);
  volatile int* sbad = reinterpret_cast<volatile int*>(sB + NBS * 2 * BSZ + 64);

  if (w == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 8, 1);
    *sbad = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // 128 x 128 tile tt of M -> A stage s (chunk layout above); 16 cp.async per thread.
  // A warp covers 8 rows x 4 chunks: 64 contiguous bytes per row, conflict-free stores.
  auto stage_a = [&](int tt, int s) {
    const uint32_t dst0 = smem_u32(sA + s * TILE);
    const T* src0 = Mi + (int64_t)tt * 128 * 128;
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
      const int e = tid + NTH * it, q = e >> 5, l = e & 31;
      const int t = (q & 15) * 8 + (l & 7), c = (q >> 4) * 4 + (l >> 3);
      cp_async16(dst0 + c * 2048 + (t >> 3) * 128 + (t & 7) * 16, src0 + (int64_t)t * 128 + c * 8);
    }
  };
  // 128 rows x r columns of f32 (row stride r, r % 4 == 0) -> hi / lo K-major B tiles of
  // rp columns: element (k, j) at (k / 8) * LB + (j / 8) * 128 + (j % 8) * 16 + (k % 8) * 2.
  // Item (k-chunk kc, column quad jq) of a thread: 8 rows x float4, loaded in one go
  // (load_b) and converted / stored once the destination stage is free (store_b).
  const int nq = rp / 4, nitem = 16 * nq;   // <= 256 items: at most 2 per thread
  auto load_b = [&](const float* src, float4 (&v)[2][8]) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = tid + NTH * q, kc = e / nq, jq = e - kc * nq;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[q][u] = (e < nitem && 4 * jq < r) ? __ldg(reinterpret_cast<const float4*>(src + (int64_t)(8 * kc + u) * r) + jq)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_b = [&](const float4 (&v)[2][8], uint8_t* dst, float scale) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = tid + NTH * q, kc = e / nq, jq = e - kc * nq;
      if (e >= nitem) continue;
#pragma unroll
      for (int i0 = 0; i0 < 4; ++i0) {
        const int i = (i0 + jq) & 3;   // rotated order: fewer bank conflicts between threads
        const int j = 4 * jq + i;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int u = 0; u < 8; u += 2) {
          const float x0 = (i == 0 ? v[q][u].x : i == 1 ? v[q][u].y : i == 2 ? v[q][u].z : v[q][u].w) * scale;
          const float x1 =
              (i == 0 ? v[q][u + 1].x : i == 1 ? v[q][u + 1].y : i == 2 ? v[q][u + 1].z : v[q][u + 1].w) * scale;
          const uint16_t h0 = H::bits(x0), h1 = H::bits(x1);
          const uint16_t l0 = H::bits(x0 - H::back(h0)), l1 = H::bits(x1 - H::back(h1));
          hi[u >> 1] = (uint32_t)h0 | ((uint32_t)h1 << 16);
          lo[u >> 1] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
        const int off = kc * LB + (j >> 3) * 128 + (j & 7) * 16;
        *reinterpret_cast<uint4*>(dst + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(dst + BSZ + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
  };

  const uint32_t id = idesc(H::kFmt, MODE, rp);
  float4 vb[2][8];
  stage_a(0, 0);
  cp_async_commit();
  load_b(Xi, vb);   // mode 0: X; mode 1: rows 0..127 of Y
  // power-of-two scale of the right-hand side (mode 0): max |x| * sc < 1, from the
  // registers just loaded (the items cover X once)
  float sc = 1.f, inv = 1.f;
  if (MODE == 0) {
    float mx = 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int u = 0; u < 8; ++u)
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(vb[q][u].x), fabsf(vb[q][u].y)), fmaxf(fabsf(vb[q][u].z), fabsf(vb[q][u].w))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) sred[w] = mx;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (MODE == 0) {
    const float mx = fmaxf(fmaxf(sred[0], sred[1]), fmaxf(sred[2], sred[3]));
    int e2 = 0;
    if (mx > 0.f && isfinite(mx)) frexpf(mx, &e2);   // mx = f 2^e2, 0.5 <= f < 1
    sc = ldexpf(1.f, -e2);
    inv = ldexpf(1.f, e2);
  }
  store_b(vb, sB, sc);
  bool ok = true;
  for (int tt = 0; tt < nt; ++tt) {
    const int s = tt & 1;
    if (tt + 1 < nt) {
      if (MODE == 1) load_b(Xi + (int64_t)(tt + 1) * 128 * r, vb);   // in flight across the wait
      // stage (tt + 1) & 1 was read by the MMAs of tile tt - 1
      if (tt >= 1) ok = mbar_wait(bar + 8 * ((tt + 1) & 1), (uint32_t)(((tt - 1) >> 1) & 1)) && ok;
      stage_a(tt + 1, (tt + 1) & 1);
      cp_async_commit();
      if (MODE == 1) store_b(vb, sB + ((tt + 1) & 1) * 2 * BSZ, 1.f);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + s * TILE);
      const uint32_t b0 = smem_u32(sB + (MODE == 1 ? s * 2 * BSZ : 0));
      const uint32_t d = tbase + (MODE == 0 ? (uint32_t)(tt * rp) : 0u);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a = MODE == 0 ? umma_desc(a0 + ks * 4096, 2048, 128) : umma_desc(a0 + ks * 256, 128, 2048);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const uint64_t b = umma_desc(b0 + part * BSZ + ks * 2 * LB, LB, 128);
          umma(d, a, b, id, (MODE == 0 ? (ks | part) : (tt | ks | part)) != 0 ? 1u : 0u);
        }
      }
      umma_commit(bar + 8 * s);
    }
    __syncwarp();
  }
  ok = mbar_wait(bar + 8 * ((nt - 1) & 1), (uint32_t)(((nt - 1) >> 1) & 1)) && ok;
  if (!ok) *sbad = 1;
  tc_fence_after();
  __syncthreads();
  const bool bad = *sbad != 0;

  // epilogue: thread = accumulator row (TMEM lane 32 w + lane).  A tile's 128 output
  // rows are one contiguous [128][r] block of global memory: rows go to shared memory
  // (the A stages are free now) at pitch r + 4 (conflict-free float4 writes), then the
  // block is copied out with coalesced float4 stores.
  const int row = 32 * w + lane;
  const uint32_t tl = tbase + ((uint32_t)(32 * w) << 16);
  const int sp = r + 4, nq4 = r / 4;
  float* stg = reinterpret_cast<float*>(sA);
  for (int tt = 0; tt < (MODE == 0 ? nt : 1); ++tt) {
    float* srow = stg + row * sp;
    for (int cb = 0; cb < rp; cb += 16) {
      float v[16];
      tmem_ld16(tl + (uint32_t)(MODE == 0 ? tt * rp + cb : cb), v);
#pragma unroll
      for (int u = 0; u < 16; u += 4)
        if (cb + u < r) {
          float4 o = make_float4(v[u] * inv, v[u + 1] * inv, v[u + 2] * inv, v[u + 3] * inv);
          if (bad) o = make_float4(__int_as_float(0x7fc00000), 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(srow + cb + u) = o;
        }
    }
    __syncthreads();
    float4* dst4 = reinterpret_cast<float4*>(Yi + (int64_t)(MODE == 0 ? tt * 128 : 0) * r);
    for (int g = tid; g < 128 * nq4; g += NTH) {
      const int rr = g / nq4, c4 = g - rr * nq4;
      dst4[g] = *reinterpret_cast<const float4*>(stg + rr * sp + 4 * c4);
    }
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(ncols) : "memory");
}

template <typename T>
static int launch(int mode, const T* M, int64_t ms, const float* X, float* Y, int Nb, int m, int r,
                  cudaStream_t st) {
  const int rp = (r + 15) / 16 * 16;
  const int BSZ = 128 * rp * 2;
  const int need = mode == 0 ? (m / 128) * rp : rp;
  int ncols = 32;
  while (ncols < need) ncols <<= 1;
  const size_t smem = 2 * TILE + (size_t)(mode == 0 ? 1 : 2) * 2 * BSZ + 128;
  if (mode == 0) {
    cudaFuncSetAttribute(tc_gemm_kernel<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tc_gemm_kernel<T, 0><<<Nb, NTH, smem, st>>>(M, ms, X, Y, m, r, rp, ncols);
  } else {
    cudaFuncSetAttribute(tc_gemm_kernel<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tc_gemm_kernel<T, 1><<<Nb, NTH, smem, st>>>(M, ms, X, Y, m, r, rp, ncols);
  }
  return SPX_OK;
}

}  // namespace rtc

bool rsvd_tc_supported(int dtype, const void* M, int64_t ms, int m, int n, int r) {
  if (dtype != SPX_F16 && dtype != SPX_BF16) return false;
  if (n != 128 || m % 128 != 0 || m > 1024 || r > 64 || r % 4 != 0) return false;
  if ((m / 128) * ((r + 15) / 16 * 16) > 512) return false;   // TMEM columns of mode 0
  return (reinterpret_cast<uintptr_t>(M) & 15u) == 0 && (ms * 2) % 16 == 0;
}

int rsvd_tc_gemm(int mode, int dtype, const void* M, int64_t ms, const float* X, float* Y, int Nb, int m, int r,
                 cudaStream_t st) {
  if (dtype == SPX_F16)
    return rtc::launch<__half>(mode, reinterpret_cast<const __half*>(M), ms, X, Y, Nb, m, r, st);
  return rtc::launch<__nv_bfloat16>(mode, reinterpret_cast<const __nv_bfloat16*>(M), ms, X, Y, Nb, m, r, st);
}

}  // namespace spx
