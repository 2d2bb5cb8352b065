// sm_100a device helpers shared by the decode kernels: mbarrier waits bounded in time,
// bulk async copies, tensor-memory allocation, UMMA descriptors, warp-level MMA and
// ldmatrix wrappers, INT8 -> f16 conversion, and the persistent work-plan walk.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

namespace spx {
namespace sm100 {

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr uint64_t kWaitNs = 2000000000ull;   // 2 s: every wait gives up after this
constexpr int GMAX = 32;                       // units per work item at most

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Named barrier over n threads, non-aligned form: threads of a warp may arrive separately.
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// ------------------------------------------------------------------ mbarrier / TMA --
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(cnt) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
// Test of a phase (the common, already-completed case of every wait).  try_wait without
// a suspend hint returns at once on a completed phase and may hold the thread in
// hardware for a short, system-defined time otherwise; on a completed phase it measured
// faster than test_wait under load (3 % of the decode kernel).
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
// The same test, but the thread may sleep in hardware (up to kSuspendNs) until the phase
// completes instead of spinning on issue slots the working warps need.
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Two independent phase tests in one statement, so that their latencies overlap.
__device__ __forceinline__ void mbar_test2(uint32_t a, uint32_t pa, uint32_t b, uint32_t pb, bool& ra, bool& rb) {
  uint32_t x, y;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%2], %3;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q, [%4], %5;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "selp.u32 %1, 1, 0, q;\n\t}"
      : "=r"(x), "=r"(y)
      : "r"(a), "r"(pa), "r"(b), "r"(pb)
      : "memory");
  ra = x != 0;
  rb = y != 0;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Streaming copies are marked evict-first in L2 so that the data reused across CTAs
// (query rows, packed RoPE words, partial records) stays resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

struct Abort {
  volatile int* flag;   // shared: set once any wait of the CTA expired
  int* err;             // workspace error word
};

// Single-thread bounded wait.  Returns false when aborted (now or earlier).
__device__ __forceinline__ bool wait1(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  for (;;) {
    if (*ab.flag) return false;
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (gtimer() - t0 > kWaitNs) {
      *ab.flag = 1;
      atomicExch(ab.err, 1);
      return false;
    }
  }
}
// Slow path of waitw: lane 0 sleeps on the barrier (bounded), then every lane observes
// the completed phase itself (acquire); the warp is reconverged before returning.
__device__ __forceinline__ bool waitw_slow(uint32_t bar, uint32_t parity, const Abort& ab) {
  int r = 0;
  if ((threadIdx.x & 31) == 0) r = wait1(bar, parity, ab) ? 1 : 0;
  r = __shfl_sync(0xffffffffu, r, 0);
  if (r) {
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity) && gtimer() - t0 < kWaitNs) {
    }
  }
  __syncwarp();
  return r != 0;
}
// Warp-wide bounded wait with a warp-uniform result (all 32 lanes call it).  The common
// case - the phase has already completed - costs one barrier test per lane.
__device__ __forceinline__ bool waitw(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return waitw_slow(bar, parity, ab);
}

// After an abort: let the copies of the last `issued` iterations of a ring land (bounded)
// before the shared memory goes away.
template <int STAGES>
__device__ __forceinline__ void drain(uint32_t full0, int issued) {
  for (int k = (issued > STAGES ? issued - STAGES : 0); k < issued; ++k) {
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait_sleep(full0 + 8 * (k % STAGES), (uint32_t)((k / STAGES) & 1)) && gtimer() - t0 < kWaitNs) {
    }
  }
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

// ------------------------------------------------------------------- tcgen05.mma ----
// Shared-memory matrix descriptor, no swizzle: start address, leading-dimension byte
// offset and stride-dimension byte offset (all >> 4), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
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

// Launch-wide item geometry (kernel parameters, uniform across the CTA).
struct Items {
  int G, JR, ngroups, nitems, nblk, units;
};

// The CTA's walk over its items: for j in range: for u in group.
struct Seq {
  int x;          // item id
  int j0, jn, u0, un;
  int jj, uu;     // position inside the item
  __device__ __forceinline__ void load_item(const Items& I) {
    const int jr = x / I.ngroups, ug = x - jr * I.ngroups;
    j0 = jr * I.JR;
    jn = min(I.JR, I.nblk - j0);
    u0 = ug * I.G;
    un = min(I.G, I.units - u0);
    jj = 0;
    uu = 0;
  }
  __device__ __forceinline__ bool valid(const Items& I) const { return x < I.nitems; }
  __device__ __forceinline__ void next(const Items& I) {
    if (++uu < un) return;
    uu = 0;
    if (++jj < jn) return;
    x += gridDim.x;
    if (x < I.nitems) load_item(I);
  }
  __device__ __forceinline__ int j() const { return j0 + jj; }
  __device__ __forceinline__ int unit() const { return u0 + uu; }
};

static int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Items of G units x JR blocks: pick the split whose slowest CTA does the least work:
// rounds of items x item size in unit-blocks, plus the partial records - one per (unit,
// block range), written by this kernel and read back by the merge kernel, each about
// 1/12 of a unit-block's bytes - spread over the SMs, plus one RoPE reload (about 1.5
// unit-blocks of stall) each time a CTA moves to a new block.
struct Plan {
  int G, JR, ngroups, nranges, nitems, grid;
};
static Plan make_plan(int units, int nblk, int G, int JR, int sms) {
  const int Gu = G < units ? G : units;
  const int ngroups = (units + Gu - 1) / Gu;
  const int nranges = (nblk + JR - 1) / JR;
  const int items = ngroups * nranges;
  return Plan{Gu, JR, ngroups, nranges, items, items < sms ? items : sms};
}
// SPX_FAST_PLAN="G,JR,CTAS" fixes units per item (<= 32), blocks per range and the
// persistent grid (a tuning knob; the tests use it to drive several items and block
// ranges through one CTA on small inputs).
static bool plan_override(int units, int nblk, Plan* out) {
  const char* e = getenv("SPX_FAST_PLAN");
  int G = 0, JR = 0, ctas = 0;
  if (!e || sscanf(e, "%d,%d,%d", &G, &JR, &ctas) != 3) return false;
  if (G < 1 || G > GMAX || JR < 1 || ctas < 1) return false;
  *out = make_plan(units, nblk, G, JR < nblk ? JR : nblk, ctas);
  return true;
}
static Plan plan(int units, int nblk, int sms) {
  Plan best{};
  if (plan_override(units, nblk, &best)) return best;
  long best_cost = -1;
  for (int G : {32, 16, 8, 4, 2, 1}) {   // small groups matter when units are few (one layer, small batch)
    const int Gu = G < units ? G : units;
    const int ngroups = (units + Gu - 1) / Gu;
    for (int nr = 1; nr <= nblk; ++nr) {
      const int JR = (nblk + nr - 1) / nr;
      const int nranges = (nblk + JR - 1) / JR;
      if (nranges != nr) continue;
      const long items = (long)ngroups * nranges;
      const long rounds = (items + sms - 1) / sms;
      const long cost = 12 * rounds * Gu * JR + ((long)units * nranges + sms - 1) / sms + 18 * rounds * JR;
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best = make_plan(units, nblk, Gu, JR, sms);
      }
    }
  }
  return best;
}

}  // namespace sm100
}  // namespace spx
