// Parameters shared by the decode kernels (generic and fast paths).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace spx {

struct DecodeParams {
  int L, B, Hq, H, D, Tb, nblk, NBc, RK, RV, hot, HC, nrep, mode, tied, rope_len, mask_stride, nparts, dtype;
  int ncold;  // cold partial records per unit that the merge kernel reads (<= nparts)
  int64_t qpos;
  float scale;
  const void* q;
  const int8_t* ck;
  const int8_t* cv;
  const float* sk;
  const float* sv;
  const void* bk;
  const void* bv;
  const int64_t* bpos;
  const void* hk;
  const void* hv;
  const int64_t* hpos;
  const float* cosT;
  const float* sinT;
  const uint8_t* mask;
  void* out;
  float* ws;  // cold partials [L*B*H][nparts][nrep][D + 4] = (m, l, -, -, o[D]), after the header
  void* rope; // path scratch after the partials: packed RoPE words [nblk][Tb/16][32][32] u32
              // (reconstruct path) or ProjScratch (projection path)
  const float* freq;  // HOST copy of the RoPE frequencies theta_i [D/2], or nullptr
  const int* hot_dev; // DEVICE hot-tier length (tokens used: min(*hot_dev, hot)), or nullptr
  int path;           // DecodePath
};

// Cold-tier kernels: generic FP32 kernel, reconstruct-rotate kernel, projection kernel.
enum DecodePath { PATH_GENERIC = 0, PATH_FAST = 1, PATH_PROJ = 2 };

// Scratch of the projection path (inside the workspace, after the partials).
struct ProjScratch {
  float2* rot;      // [nblk][64] block rotation factors (complex)
  int* clamp;       // [nblk] first token past the query (DISTANCE mode), else T
  __half* atab;     // [T][KF] token-feature table
  float* coef;      // [16][64] Chebyshev coefficients
  long long* trace; // event timeline (SPX_PROJ_TRACE builds only)
};
__host__ __device__ inline size_t proj_align(size_t x) { return (x + 255) / 256 * 256; }
// Builds with -DSPX_PROJ_TRACE=1 (diagnostics only) append an event-timeline buffer of
// 64 iterations x 64 events of clock64 values, written by the first CTA.
#ifdef SPX_PROJ_TRACE
constexpr size_t kProjTraceBytes = 64 * 64 * 8;
#else
constexpr size_t kProjTraceBytes = 0;
#endif
__host__ __device__ inline size_t proj_scratch_bytes(int nblk, int T, int kfmax) {
  return proj_align((size_t)nblk * 64 * 8) + proj_align((size_t)nblk * 4) + proj_align((size_t)T * kfmax * 2) +
         proj_align(16 * 64 * 4) + kProjTraceBytes;
}
__host__ __device__ inline ProjScratch proj_scratch(const DecodeParams& p, int /*kf*/) {
  char* b = reinterpret_cast<char*>(p.rope);
  ProjScratch s;
  s.rot = reinterpret_cast<float2*>(b);
  b += proj_align((size_t)p.nblk * 64 * 8);
  s.clamp = reinterpret_cast<int*>(b);
  b += proj_align((size_t)p.nblk * 4);
  s.atab = reinterpret_cast<__half*>(b);
  b += proj_align((size_t)p.Tb * 128 * 2);
  s.coef = reinterpret_cast<float*>(b);
  b += proj_align(16 * 64 * 4);
  s.trace = reinterpret_cast<long long*>(b);
  return s;
}

// The workspace starts with a 256-byte header (word 0: set to 1 by a cold-tier kernel
// whose bounded wait expired); the cold partials follow it.
constexpr size_t kWsHeader = 256;

size_t decode_workspace_bytes(const DecodeParams& p);
// Point ws (partials) and rope (packed RoPE words) into a workspace starting at base.
void decode_set_workspace(DecodeParams* p, void* base);
int decode_dispatch(const DecodeParams& p, cudaStream_t st);

// Reconstruct-rotate cold-tier path (spx_decode_fast.cu): true when the configuration is covered.
bool decode_fast_supported(const DecodeParams& p);
int decode_fast_ncold(const DecodeParams& p);   // partial records per unit it writes
int decode_fast_cold(const DecodeParams& p, cudaStream_t st);

// Projection cold-tier path (spx_decode_proj.cu): needs the RoPE frequencies.
bool decode_proj_supported(const DecodeParams& p);
int decode_proj_ncold(const DecodeParams& p);
size_t decode_proj_scratch_bytes(const DecodeParams& p);
int decode_proj_cold(const DecodeParams& p, cudaStream_t st);

}  // namespace spx
