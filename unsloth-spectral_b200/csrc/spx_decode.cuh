// Parameters shared by the decode kernels (generic and fast paths).
#pragma once
#include <cuda_runtime.h>
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
  void* rope; // fast path: packed RoPE words [nblk][Tb/16][32][32] u32, after the partials
};

// The workspace starts with a 256-byte header (word 0: set to 1 by a cold-tier kernel
// whose bounded wait expired); the cold partials follow it.
constexpr size_t kWsHeader = 256;

size_t decode_workspace_bytes(const DecodeParams& p);
// Point ws (partials) and rope (packed RoPE words) into a workspace starting at base.
void decode_set_workspace(DecodeParams* p, void* base);
int decode_dispatch(const DecodeParams& p, cudaStream_t st);

// Fast cold-tier path (spx_decode_fast.cu): true when the configuration is covered.
bool decode_fast_supported(const DecodeParams& p);
int decode_fast_ncold(const DecodeParams& p);   // partial records per unit it writes
int decode_fast_cold(const DecodeParams& p, cudaStream_t st);

}  // namespace spx
