// Spectral decode attention over the three-tier cache (host entry + generic kernels).
//
// Semantics follow unsloth_spectral/spectral_attention.py:117-349 (DISTANCE mode) and
// unsloth_spectral/kernels/spectral_attention.py:684-857 (ABSOLUTE mode).  Both rotate
// the query per key token; here the rotation is moved onto the reconstructed key, which
// is the same number:
//   score_t = Q . R^-1_{a_t}-rotated ... = sum_i Q1_i (c1 K1 - s2 K2) + Q2_i (s1 K1 + c2 K2)
// with K~_t = scale_k * codes_t @ B_k, (c1, s1) = (cos, sin)[a_t, i], (c2, s2) the same
// at i + D/2 (DISTANCE mode uses the first half for both, like apply_rope at
// spectral_attention.py:80-114).  Hot keys are RoPE'd at their absolute positions.
//
// Pipeline: one partial (running max m, sum l, un-normalised output o[D]) per cold
// block and (layer, sequence, KV head, q-head), written to the workspace, then one
// kernel per (layer, sequence, KV head) that scores the hot tier and merges every
// partial with the log-sum-exp rule into the output.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "spx_common.cuh"
#include "spx_decode.cuh"

namespace spx {

constexpr int kMaxRep = 16;
constexpr size_t kMaxSmem = 227 * 1024;

// ------------------------------------------------------------------ cold, generic ---
template <typename T, int RKT>
__global__ void __launch_bounds__(256) cold_generic_kernel(DecodeParams p) {
  const int j = blockIdx.x, g = blockIdx.y, lb = blockIdx.z;
  const int b = lb % p.B;
  const int D = p.D, half = D / 2, Tb = p.Tb, RV = p.RV, nrep = p.nrep;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* sbk = sm;                  // [RKT][D]
  float* sbv = sbk + RKT * D;       // [RV][D]
  float* sq = sbv + RV * D;         // [nrep][D]
  float* ssc = sq + nrep * D;       // [nrep][Tb]
  float* svl = ssc + nrep * Tb;     // [nrep][RV]
  float* sml = svl + nrep * RV;     // [nrep][2]
  const int64_t lbg = (int64_t)lb * p.H + g;
  const int64_t slot = lbg * p.NBc + j;
  const T* bk = reinterpret_cast<const T*>(p.bk) + slot * RKT * D;
  const T* bv = reinterpret_cast<const T*>(p.bv) + slot * (int64_t)RV * D;
  const T* q = reinterpret_cast<const T*>(p.q) + ((int64_t)lb * p.Hq + (int64_t)g * nrep) * D;
  for (int i = tid; i < RKT * D; i += blockDim.x) sbk[i] = to_f(bk[i]);
  for (int i = tid; i < RV * D; i += blockDim.x) sbv[i] = to_f(bv[i]);
  for (int i = tid; i < nrep * D; i += blockDim.x) sq[i] = to_f(q[i]);
  __syncthreads();
  const float sK = p.sk[slot] * p.scale, sV = p.sv[slot];
  const int64_t p0 = p.bpos[j];
  const bool second_half = (p.mode == SPX_ROPE_ABSOLUTE) && !p.tied;
  for (int t = tid; t < Tb; t += blockDim.x) {
    float c[RKT];
    const int4* crow = reinterpret_cast<const int4*>(p.ck + (slot * Tb + t) * RKT);
#pragma unroll
    for (int v = 0; v < RKT / 16; ++v) {
      const int4 w = crow[v];
      const int ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) c[v * 16 + u * 4 + bb] = (float)(int8_t)((ws[u] >> (8 * bb)) & 0xff);
    }
    const int64_t kp = p0 + t;
    int64_t a = p.mode == SPX_ROPE_DISTANCE ? (p.qpos - kp > 0 ? p.qpos - kp : 0) : kp;
    a = a < 0 ? 0 : (a >= p.rope_len ? p.rope_len - 1 : a);
    const float* cr = p.cosT + a * D;
    const float* sr = p.sinT + a * D;
    float s[kMaxRep];
#pragma unroll
    for (int h = 0; h < kMaxRep; ++h) s[h] = 0.f;
    for (int i = 0; i < half; ++i) {
      float k1 = 0.f, k2 = 0.f;
#pragma unroll
      for (int r = 0; r < RKT; ++r) {
        k1 = fmaf(c[r], sbk[r * D + i], k1);
        k2 = fmaf(c[r], sbk[r * D + i + half], k2);
      }
      const float c1 = cr[i], s1 = sr[i];
      const float c2 = second_half ? cr[i + half] : c1;
      const float s2 = second_half ? sr[i + half] : s1;
      const float kp1 = c1 * k1 - s2 * k2;
      const float kp2 = s1 * k1 + c2 * k2;
#pragma unroll
      for (int h = 0; h < kMaxRep; ++h)
        if (h < nrep) s[h] = fmaf(sq[h * D + i], kp1, fmaf(sq[h * D + i + half], kp2, s[h]));
    }
#pragma unroll
    for (int h = 0; h < kMaxRep; ++h) {
      if (h < nrep) {
        float v = s[h] * sK;
        if (p.mask && p.mask[((int64_t)b * p.Hq + g * nrep + h) * p.mask_stride + (int64_t)j * Tb + t] == 0)
          v = -INFINITY;
        ssc[h * Tb + t] = v;
      }
    }
  }
  __syncthreads();
  for (int h = warp; h < nrep; h += nwarps) {
    float m = -INFINITY;
    for (int t = lane; t < Tb; t += 32) m = fmaxf(m, ssc[h * Tb + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < Tb; t += 32) {
      const float e = m == -INFINITY ? 0.f : __expf(ssc[h * Tb + t] - m);
      ssc[h * Tb + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sml[2 * h] = m;
      sml[2 * h + 1] = l;
    }
  }
  __syncthreads();
  const int8_t* cvb = p.cv + slot * (int64_t)RV * Tb;
  for (int pr = warp; pr < nrep * RV; pr += nwarps) {
    const int h = pr / RV, r = pr - h * RV;
    float acc = 0.f;
    for (int t = lane; t < Tb; t += 32) acc = fmaf(ssc[h * Tb + t], (float)cvb[vtile_offset(r, t, RV)], acc);
    acc = warp_sum(acc);
    if (lane == 0) svl[pr] = acc;
  }
  __syncthreads();
  float* rec = p.ws + ((lbg * p.nparts + j) * nrep) * (int64_t)(D + 4);
  for (int e = tid; e < nrep * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    float acc = 0.f;
    for (int r = 0; r < RV; ++r) acc = fmaf(svl[h * RV + r], sbv[r * D + d], acc);
    rec[(int64_t)h * (D + 4) + 4 + d] = acc * sV;
  }
  if (tid < nrep) {
    rec[(int64_t)tid * (D + 4) + 0] = sml[2 * tid];
    rec[(int64_t)tid * (D + 4) + 1] = sml[2 * tid + 1];
  }
}

// ------------------------------------------------------------- hot tier + merge ---
// Shared memory of hot_merge_kernel before the staged copies (floats; a multiple of 4,
// so the staged region starts 16-byte aligned): q, scores, (weight, 1/L), merge weights,
// partial value sums of 256 / D slices, clamped table rows.
__host__ __device__ inline size_t hot_merge_base_floats(const DecodeParams& p) {
  const size_t f = (size_t)p.nrep * p.D + (size_t)p.nrep * p.hot + 2 * p.nrep + (size_t)p.nrep * (p.nblk + 1) +
                   (size_t)(256 / p.D) * p.nrep * p.D + (size_t)p.hot;
  return (f + 3) & ~(size_t)3;
}

template <typename T, bool STAGE, int NREP>
__global__ void __launch_bounds__(256) hot_merge_kernel(DecodeParams p) {
  // STAGE: the hot K and V rows and the cold partial records are first copied to shared
  // memory with 16-byte asynchronous copies, all in flight at once, instead of being
  // read in many dependent rounds of global loads.  NREP: the query heads per KV head
  // when it is one of the compiled counts (the per-head loops then carry no tests), 0
  // for any other count (loops over kMaxRep heads, tested against p.nrep).
  constexpr int RR = NREP > 0 ? NREP : kMaxRep;
  const int g = blockIdx.x, lb = blockIdx.y;
  const int b = lb % p.B;
  const int D = p.D, half = D / 2, nrep = NREP > 0 ? NREP : p.nrep, nb = p.nblk, nc = p.ncold;
  // shared-memory layout by the launch bound p.hot; tokens used: the run-time length
  const int hmax = p.hot;
  int hot = hmax;
  if (p.hot_dev) {
    const int hd = *p.hot_dev;
    hot = hd < 0 ? 0 : (hd < hmax ? hd : hmax);
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* sq = sm;                   // [nrep][D]
  float* ssc = sq + nrep * D;       // [nrep][hmax]
  float* sml = ssc + nrep * hmax;   // [nrep][2]
  float* swt = sml + 2 * nrep;      // [nrep][nc + 1] merge weights, then 1/L
  float* sred = swt + nrep * (nc + 1);   // [slices][nrep][D] partial value sums
  int* spos = reinterpret_cast<int*>(sred + (blockDim.x / D) * nrep * D);   // [hot] clamped table rows
  const int64_t lbg = (int64_t)lb * p.H + g;
  // staged copies (STAGE): K rows [hot][D], V rows [hot][D] (T), records [nc][nrep][D + 4] f32
  uint8_t* stg = reinterpret_cast<uint8_t*>(sm) + hot_merge_base_floats(p) * sizeof(float);
  T* sK = reinterpret_cast<T*>(stg);
  T* sV = sK + (size_t)hmax * D;
  float* sR = reinterpret_cast<float*>(sV + (size_t)hmax * D);
  if (STAGE) {
    const uint8_t* gk = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.hk) + lbg * p.HC * D);
    const uint8_t* gv = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.hv) + lbg * p.HC * D);
    const uint8_t* gr = reinterpret_cast<const uint8_t*>(p.ws + (lbg * p.nparts) * nrep * (int64_t)(D + 4));
    const int nkv = hot * D * (int)sizeof(T) / 16, nr = nc * nrep * (D + 4) * 4 / 16;
    const uint32_t dk = (uint32_t)__cvta_generic_to_shared(sK), dv = (uint32_t)__cvta_generic_to_shared(sV),
                   dr = (uint32_t)__cvta_generic_to_shared(sR);
    for (int e = tid; e < nkv; e += blockDim.x) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk + 16 * e), "l"(gk + 16 * e) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv + 16 * e), "l"(gv + 16 * e) : "memory");
    }
    for (int e = tid; e < nr; e += blockDim.x)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dr + 16 * e), "l"(gr + 16 * e) : "memory");
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  }
  const T* q = reinterpret_cast<const T*>(p.q) + ((int64_t)lb * p.Hq + (int64_t)g * nrep) * D;
  for (int i = tid; i < nrep * D; i += blockDim.x) sq[i] = to_f(q[i]);
  for (int t = tid; t < hot; t += blockDim.x) {
    const int64_t a = p.hpos[t];
    spos[t] = (int)(a < 0 ? 0 : (a >= p.rope_len ? p.rope_len - 1 : a));
  }
  // a cold-tier kernel that gave up waiting marks the workspace header: report NaN
  const bool cold_failed = nb > 0 && reinterpret_cast<const int*>(p.ws)[-64] != 0;
  __syncthreads();
  const T* hk = STAGE ? sK : reinterpret_cast<const T*>(p.hk) + lbg * p.HC * D;
  const T* hv = STAGE ? sV : reinterpret_cast<const T*>(p.hv) + lbg * p.HC * D;
  const bool second_half = (p.mode == SPX_ROPE_ABSOLUTE) && !p.tied;
  // scores: one warp per hot token, lanes over the rotation pairs (coalesced rows)
#pragma unroll 2
  for (int t = warp; t < hot; t += nwarps) {
    const int64_t a = spos[t];
    const float* cr = p.cosT + a * D;
    const float* sr = p.sinT + a * D;
    const T* krow = hk + (int64_t)t * D;
    float s[RR];
#pragma unroll
    for (int h = 0; h < RR; ++h) s[h] = 0.f;
    for (int i = lane; i < half; i += 32) {
      const float k1 = to_f(krow[i]), k2 = to_f(krow[i + half]);
      const float c1 = cr[i], s1 = sr[i];
      const float c2 = second_half ? cr[i + half] : c1;
      const float s2 = second_half ? sr[i + half] : s1;
      const float kp1 = k1 * c1 - k2 * s1;   // apply_rope: x1*cos1 - x2*sin1
      const float kp2 = k2 * c2 + k1 * s2;   //             x2*cos2 + x1*sin2
#pragma unroll
      for (int h = 0; h < RR; ++h)
        if (NREP > 0 || h < nrep) s[h] = fmaf(sq[h * D + i], kp1, fmaf(sq[h * D + i + half], kp2, s[h]));
    }
#pragma unroll
    for (int h = 0; h < RR; ++h) {
      if (NREP > 0 || h < nrep) {
        float v = warp_sum(s[h]) * p.scale;
        if (p.mask && p.mask[((int64_t)b * p.Hq + g * nrep + h) * p.mask_stride + (int64_t)nb * p.Tb + t] == 0)
          v = -INFINITY;
        if (lane == 0) ssc[h * hmax + t] = v;
      }
    }
  }
  __syncthreads();
  for (int h = warp; h < nrep; h += nwarps) {
    float m = -INFINITY;
    for (int t = lane; t < hot; t += 32) m = fmaxf(m, ssc[h * hmax + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < hot; t += 32) {
      const float e = m == -INFINITY ? 0.f : __expf(ssc[h * hmax + t] - m);
      ssc[h * hmax + t] = e;
      l += e;
    }
    l = warp_sum(l);
    // merge weights over the cold partials and the hot partial
    const float* recs = STAGE ? sR : p.ws + (lbg * p.nparts) * nrep * (int64_t)(D + 4);
    float M = m;
    for (int jj = lane; jj < nc; jj += 32) M = fmaxf(M, recs[((int64_t)jj * nrep + h) * (D + 4)]);
    M = warp_max(M);
    float L = 0.f;
    for (int jj = lane; jj < nc; jj += 32) {
      const float* r = recs + ((int64_t)jj * nrep + h) * (D + 4);
      const float w = M == -INFINITY ? 0.f : __expf(r[0] - M);
      swt[h * (nc + 1) + jj] = w;
      L += w * r[1];
    }
    L = warp_sum(L);
    if (lane == 0) {
      const float wh = M == -INFINITY ? 0.f : __expf(m - M);
      L += wh * l;
      sml[2 * h] = wh;
      sml[2 * h + 1] = (M == -INFINITY || L == 0.f) ? NAN : 1.f / L;  // fully masked -> NaN
    }
  }
  __syncthreads();
  T* out = reinterpret_cast<T*>(p.out) + ((int64_t)lb * p.Hq + (int64_t)g * nrep) * D;
  const float* recs = STAGE ? sR : p.ws + (lbg * p.nparts) * nrep * (int64_t)(D + 4);
  // hot values: thread (slice, d) reads each V element once for every head of the group
  {
    const int slices = blockDim.x / D;
    const int sl = tid / D, d = tid - sl * D;
    if (sl < slices) {
      float acc[RR];
#pragma unroll
      for (int h = 0; h < RR; ++h) acc[h] = 0.f;
#pragma unroll 4
      for (int t = sl; t < hot; t += slices) {
        const float v = to_f(hv[(int64_t)t * D + d]);
#pragma unroll
        for (int h = 0; h < RR; ++h)
          if (NREP > 0 || h < nrep) acc[h] = fmaf(ssc[h * hmax + t], v, acc[h]);
      }
#pragma unroll
      for (int h = 0; h < RR; ++h)
        if (NREP > 0 || h < nrep) sred[(sl * nrep + h) * D + d] = acc[h];
    }
  }
  __syncthreads();
  for (int e = tid; e < nrep * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    float acc = 0.f;
    for (int sl = 0; sl < (int)(blockDim.x / D); ++sl) acc += sred[(sl * nrep + h) * D + d];
    acc *= sml[2 * h];
    for (int jj = 0; jj < nc; ++jj) acc = fmaf(swt[h * (nc + 1) + jj], recs[((int64_t)jj * nrep + h) * (D + 4) + 4 + d], acc);
    out[(int64_t)h * D + d] = from_f<T>(cold_failed ? NAN : acc * sml[2 * h + 1]);
  }
}

template <typename T, int RKT>
static int launch_cold_generic(const DecodeParams& p, cudaStream_t st) {
  const size_t smem = ((size_t)RKT * p.D + (size_t)p.RV * p.D + (size_t)p.nrep * p.D + (size_t)p.nrep * p.Tb +
                       (size_t)p.nrep * p.RV + 2 * p.nrep) * sizeof(float);
  SPX_REQUIRE(smem <= kMaxSmem, SPX_ERR_UNSUPPORTED, "cold tier needs %zu bytes of shared memory", smem);
  cudaFuncSetAttribute(cold_generic_kernel<T, RKT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(p.nblk, p.H, p.L * p.B);
  cold_generic_kernel<T, RKT><<<grid, 256, smem, st>>>(p);
  return launch_status("cold_generic_kernel");
}

template <typename T>
static int launch_cold(const DecodeParams& p, cudaStream_t st) {
  switch (p.RK) {
    case 16: return launch_cold_generic<T, 16>(p, st);
    case 32: return launch_cold_generic<T, 32>(p, st);
    case 48: return launch_cold_generic<T, 48>(p, st);
    case 64: return launch_cold_generic<T, 64>(p, st);
    default: set_error("rank_k %d not in {16,32,48,64}", p.RK); return SPX_ERR_UNSUPPORTED;
  }
}

template <typename T>
static int launch_hot_merge(const DecodeParams& p, cudaStream_t st) {
  const size_t smem = hot_merge_base_floats(p) * sizeof(float);
  SPX_REQUIRE(smem <= kMaxSmem, SPX_ERR_UNSUPPORTED,
              "hot tier of %d tokens with %d blocks needs %zu bytes of shared memory", p.hot, p.nblk, smem);
  // staging when it fits in a modest footprint (several CTAs per SM) and every copy is
  // whole, aligned 16-byte chunks
  const size_t stage = 2 * (size_t)p.hot * p.D * sizeof(T) + (size_t)p.ncold * p.nrep * (p.D + 4) * sizeof(float);
  const bool aligned = ((reinterpret_cast<uintptr_t>(p.hk) | reinterpret_cast<uintptr_t>(p.hv) |
                         reinterpret_cast<uintptr_t>(p.ws)) & 15u) == 0 &&
                       ((size_t)p.HC * p.D * sizeof(T)) % 16 == 0 && ((size_t)p.hot * p.D * sizeof(T)) % 16 == 0;
  dim3 grid(p.H, p.L * p.B);
  auto go = [&](auto stage_tag, auto nrep_tag) {
    constexpr bool S = decltype(stage_tag)::value;
    constexpr int R = decltype(nrep_tag)::value;
    const size_t bytes = S ? smem + stage : smem;
    cudaFuncSetAttribute(hot_merge_kernel<T, S, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    hot_merge_kernel<T, S, R><<<grid, 256, bytes, st>>>(p);
  };
  auto by_nrep = [&](auto stage_tag) {
    switch (p.nrep) {
      case 1: go(stage_tag, std::integral_constant<int, 1>()); break;
      case 2: go(stage_tag, std::integral_constant<int, 2>()); break;
      case 4: go(stage_tag, std::integral_constant<int, 4>()); break;
      case 8: go(stage_tag, std::integral_constant<int, 8>()); break;
      case 16: go(stage_tag, std::integral_constant<int, 16>()); break;
      default: go(stage_tag, std::integral_constant<int, 0>()); break;
    }
  };
  if (aligned && smem + stage <= 64 * 1024) by_nrep(std::true_type());
  else by_nrep(std::false_type());
  return launch_status("hot_merge_kernel");
}

// ------------------------------------------------------------------- host side ---
static size_t partial_bytes(const DecodeParams& p) {
  return (size_t)p.L * p.B * p.H * p.nparts * p.nrep * (p.D + 4) * sizeof(float);
}


void decode_set_workspace(DecodeParams* p, void* base) {
  p->ws = base ? reinterpret_cast<float*>(reinterpret_cast<char*>(base) + kWsHeader) : nullptr;
  p->rope = base ? reinterpret_cast<char*>(base) + kWsHeader + partial_bytes(*p) : nullptr;
}

// SPX_DECODE_PATH selects the cold-tier kernel: "generic" (FP32, any shape), "fast"
// (reconstruct-rotate) or "proj" (projection, which needs the RoPE frequencies); the
// default takes the reconstruct-rotate kernel when it covers the configuration, else
// the projection kernel, else the generic one.  Forcing a path that does not cover the
// configuration falls back the same way.  The tests use it to cross-check the kernels
// on identical inputs.
static void choose_path(DecodeParams* p) {
  const char* e = getenv("SPX_DECODE_PATH");
  const bool want_generic = e && strcmp(e, "generic") == 0;
  const bool want_proj = e && strcmp(e, "proj") == 0;
  p->path = PATH_GENERIC;
  p->nparts = p->nblk > 0 ? p->nblk : 1;
  p->ncold = p->nblk;
  if (p->nblk <= 0 || want_generic) return;
  if ((want_proj || !decode_fast_supported(*p)) && decode_proj_supported(*p)) {
    p->path = PATH_PROJ;
    p->nparts = p->ncold = decode_proj_ncold(*p);
  } else if (decode_fast_supported(*p)) {
    p->path = PATH_FAST;
    p->nparts = p->ncold = decode_fast_ncold(*p);
  }
}

static int make_params(const spx_decode_args* a, DecodeParams* p) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->num_layers >= 1 && a->batch >= 1 && a->num_kv_heads >= 1 && a->num_q_heads >= 1,
              SPX_ERR_SHAPE, "layers, batch and head counts must be >= 1");
  SPX_REQUIRE(a->num_q_heads % a->num_kv_heads == 0, SPX_ERR_SHAPE, "num_q_heads %% num_kv_heads != 0");
  const int nrep = a->num_q_heads / a->num_kv_heads;
  SPX_REQUIRE(nrep <= kMaxRep, SPX_ERR_UNSUPPORTED, "GQA group %d > %d", nrep, kMaxRep);
  SPX_REQUIRE(a->head_dim >= 16 && a->head_dim <= 256 && a->head_dim % 16 == 0, SPX_ERR_SHAPE,
              "head_dim %d must be a multiple of 16 in [16, 256]", a->head_dim);
  SPX_REQUIRE(dtype_ok(a->dtype), SPX_ERR_UNSUPPORTED, "bad dtype %d", a->dtype);
  SPX_REQUIRE(a->rope_mode == SPX_ROPE_DISTANCE || a->rope_mode == SPX_ROPE_ABSOLUTE, SPX_ERR_SHAPE,
              "bad rope_mode");
  SPX_REQUIRE(a->num_blocks >= 0 && a->num_blocks <= a->block_capacity, SPX_ERR_SHAPE,
              "num_blocks %d outside [0, block_capacity %d]", a->num_blocks, a->block_capacity);
  SPX_REQUIRE(a->hot_len >= 0 && a->hot_len <= a->hot_capacity, SPX_ERR_SHAPE, "hot_len outside [0, hot_capacity]");
  SPX_REQUIRE(a->num_blocks > 0 || a->hot_len > 0, SPX_ERR_EMPTY, "Empty cache - no keys available");
  SPX_REQUIRE(a->q && a->out && a->cos_table && a->sin_table, SPX_ERR_NULL, "q, out, cos and sin are required");
  SPX_REQUIRE(a->rope_len >= 1, SPX_ERR_SHAPE, "rope_len must be >= 1");
  if (a->num_blocks > 0) {
    SPX_REQUIRE(a->block_size >= 16 && a->block_size <= 1024 && a->block_size % 16 == 0, SPX_ERR_SHAPE,
                "block_size %d must be a multiple of 16 in [16, 1024]", a->block_size);
    SPX_REQUIRE(a->rank_k % 16 == 0 && a->rank_k >= 16 && a->rank_k <= 64 && a->rank_v % 16 == 0 &&
                    a->rank_v >= 16 && a->rank_v <= 64,
                SPX_ERR_UNSUPPORTED, "stored ranks must be 16, 32, 48 or 64");
    SPX_REQUIRE(a->codes_k && a->codes_v && a->scale_k && a->scale_v && a->basis_k && a->basis_v && a->block_pos,
                SPX_ERR_NULL, "cold-tier pointers are required when num_blocks > 0");
    SPX_REQUIRE(aligned16(a->codes_k) && aligned16(a->codes_v) && aligned16(a->basis_k) && aligned16(a->basis_v),
                SPX_ERR_ALIGN, "cold-tier tensors must be 16-byte aligned");
  }
  if (a->hot_len > 0)
    SPX_REQUIRE(a->hot_k && a->hot_v && a->hot_pos, SPX_ERR_NULL, "hot-tier pointers are required when hot_len > 0");
  if (a->mask)
    SPX_REQUIRE(a->mask_stride >= a->num_blocks * a->block_size + a->hot_len, SPX_ERR_SHAPE,
                "mask_stride shorter than the key count");
  p->L = a->num_layers;
  p->B = a->batch;
  p->Hq = a->num_q_heads;
  p->H = a->num_kv_heads;
  p->D = a->head_dim;
  p->Tb = a->num_blocks > 0 ? a->block_size : 0;
  p->nblk = a->num_blocks;
  p->NBc = a->block_capacity;
  p->RK = a->rank_k;
  p->RV = a->rank_v;
  p->hot = a->hot_len;
  p->HC = a->hot_capacity;
  p->nrep = nrep;
  p->mode = a->rope_mode;
  p->tied = a->rope_tied ? 1 : 0;
  p->rope_len = a->rope_len;
  p->mask_stride = a->mask_stride;
  p->freq = a->rope_freq;
  p->hot_dev = a->hot_len_device;
  p->nparts = a->num_blocks > 0 ? a->num_blocks : 1;
  p->ncold = a->num_blocks;
  p->qpos = a->query_position;
  p->scale = a->scale;
  p->q = a->q;
  p->ck = a->codes_k;
  p->cv = a->codes_v;
  p->sk = a->scale_k;
  p->sv = a->scale_v;
  p->bk = a->basis_k;
  p->bv = a->basis_v;
  p->bpos = a->block_pos;
  p->hk = a->hot_k;
  p->hv = a->hot_v;
  p->hpos = a->hot_pos;
  p->cosT = a->cos_table;
  p->sinT = a->sin_table;
  p->mask = a->mask;
  p->out = a->out;
  p->dtype = a->dtype;
  choose_path(p);
  decode_set_workspace(p, a->workspace);
  return SPX_OK;
}

static size_t path_scratch_bytes(const DecodeParams& p) {
  if (p.path == PATH_FAST) return (size_t)p.nblk * p.Tb * 256;
  if (p.path == PATH_PROJ) return decode_proj_scratch_bytes(p);
  return 0;
}

size_t decode_workspace_bytes(const DecodeParams& p) {
  return kWsHeader + partial_bytes(p) + path_scratch_bytes(p);
}

int decode_dispatch(const DecodeParams& p, cudaStream_t st) {
  int rc = SPX_OK;
  if (p.nblk > 0) {
    SPX_REQUIRE(p.ws && (p.path == PATH_GENERIC || p.rope), SPX_ERR_WORKSPACE,
                "decode workspace pointers are not set");
    const cudaError_t e = cudaMemsetAsync(reinterpret_cast<char*>(p.ws) - kWsHeader, 0, sizeof(int), st);
    SPX_REQUIRE(e == cudaSuccess, SPX_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    if (p.path == PATH_PROJ) rc = decode_proj_cold(p, st);
    else if (p.path == PATH_FAST) rc = decode_fast_cold(p, st);
    else rc = SPX_DISPATCH_DTYPE(p.dtype, T, [&] { return launch_cold<T>(p, st); });
    if (rc != SPX_OK) return rc;
  }
  return SPX_DISPATCH_DTYPE(p.dtype, T, [&] { return launch_hot_merge<T>(p, st); });
}

int decode_params(const spx_decode_args* a, DecodeParams* p) { return make_params(a, p); }

}  // namespace spx

using namespace spx;

extern "C" {

size_t spx_decode_workspace_size(const spx_decode_args* a) {
  DecodeParams p;
  if (make_params(a, &p) != SPX_OK) return 0;
  return decode_workspace_bytes(p);
}

int spx_decode_path(const spx_decode_args* a) {
  DecodeParams p;
  const int rc = make_params(a, &p);
  return rc != SPX_OK ? -rc : p.path;
}

int spx_decode_attn(const spx_decode_args* a, void* stream) {
  DecodeParams p;
  int rc = make_params(a, &p);
  if (rc != SPX_OK) return rc;
  const size_t need = decode_workspace_bytes(p);
  if (p.nblk > 0) {
    SPX_REQUIRE(a->workspace && a->workspace_bytes >= need, SPX_ERR_WORKSPACE,
                "workspace of %zu bytes required, %zu given", need, a->workspace_bytes);
    SPX_REQUIRE((reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0, SPX_ERR_ALIGN,
                "workspace must be 256-byte aligned");
  }
  return decode_dispatch(p, (cudaStream_t)stream);
}

}  // extern "C"
